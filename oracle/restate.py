"""Numpy restatement of the RFSN compressed-KV decode path (CPU oracle).

TEST INFRASTRUCTURE ONLY — see ``oracle/__init__.py``.  Every function
follows the reference line by line and cites it as ``file:line`` (paths are
relative to the reference project root).  Float16 cast points are kept where
the reference has them:

* PQ residual cast to the input dtype          quantization.py:142
* RVQ correction summed in fp32, cast to fp16   quantization.py:266-272
* hybrid decode ``base + correction`` in fp16   quantization.py:319
* attention output cast to q.dtype              attention.py:105

Extensions with no reference counterpart (parity for them is *unpinned*: they
are checked only for self-consistency and against reference-expressible
special cases):

* ``num_kv_heads`` (GQA): query head h reads KV head ``h // (Hq // Hkv)``;
  equivalent to the reference after ``_repeat_kv`` (llama32_adapter.py:380-386).
* batch of independent sequences (the reference cache is batch-1).
* ``hot_policy="recent"``: hot = newest tokens, older tokens spill to warm,
  warm spills whole chunks to cold (the reference keeps hot = first tokens,
  cache.py:103-118, which is ``hot_policy="prefix"``).
* ``sparse_topk`` S: after PQ+RVQ, the S coordinates with the largest
  ``|x - decode(x)|`` (fp32; ties to the lower index) keep their error as an
  fp16 value; decode adds it in fp32 and rounds once to fp16.
* dense RVQ: ``rvq_sparsity_threshold < 0`` makes every token active, which
  the reference already expresses (norm > negative threshold).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

F16 = np.float16
F32 = np.float32
MASK_FILL_VALUE = np.float32(-1e30)  # storage.py:16


# ---------------------------------------------------------------------------
# Config (storage.py:19-59)
# ---------------------------------------------------------------------------

@dataclass
class OracleConfig:
    hidden_dim: int = 4096
    num_heads: int = 32
    head_dim: int = 128
    num_subspaces: int = 8
    pq_bits: int = 8
    subspace_dim: int = 16
    num_rvq_layers: int = 4
    rvq_codebook_size: int = 4096
    rvq_sparsity_threshold: float = 0.005
    hot_capacity: int = 8192
    warm_capacity: int = 65536
    block_size_seq: int = 128
    # extensions
    num_kv_heads: Optional[int] = None
    sparse_topk: int = 0
    hot_policy: str = "prefix"
    cold_chunk_tokens: Optional[int] = None

    def __post_init__(self):
        if self.num_subspaces * self.subspace_dim != self.head_dim:  # storage.py:53-59
            raise ValueError("head_dim must equal num_subspaces * subspace_dim")
        if self.num_kv_heads is None:
            self.num_kv_heads = self.num_heads

    @property
    def chunk_tokens(self) -> int:
        return self.cold_chunk_tokens or max(1, self.block_size_seq)


# ---------------------------------------------------------------------------
# Quantization (quantization.py:92-402)
# ---------------------------------------------------------------------------

def squared_l2_distance(lhs: np.ndarray, rhs: np.ndarray) -> np.ndarray:
    """quantization.py:92-96 — fp32 ``|x|^2 - 2 x.C^T + |C|^2``."""
    lhs = lhs.astype(F32, copy=False)
    rhs = rhs.astype(F32, copy=False)
    lhs_sq = np.sum(lhs * lhs, axis=1, keepdims=True, dtype=F32)
    rhs_sq = np.sum(rhs * rhs, axis=1, keepdims=True, dtype=F32).T
    cross = lhs @ rhs.T
    return (lhs_sq - (F32(2.0) * cross) + rhs_sq).astype(F32, copy=False)


def pq_quantize(vectors: np.ndarray, codebooks: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """quantization.py:124-144 — per-subspace argmin; residual cast to input dtype.

    vectors fp16 [N, D]; codebooks fp16 [M, K, ds] -> (codes u8 [N, M], residual fp16 [N, D]).
    """
    n, d = vectors.shape
    m_sub, _, ds = codebooks.shape
    if d != m_sub * ds:
        raise ValueError(f"Expected vectors with dim {m_sub * ds}, got {d}")
    codes = np.zeros((n, m_sub), dtype=np.uint8)
    residual = np.zeros_like(vectors)
    for m in range(m_sub):
        sub = vectors[:, m * ds:(m + 1) * ds].astype(F32)
        cb = codebooks[m].astype(F32)
        dists = squared_l2_distance(sub, cb)
        idx = np.argmin(dists, axis=1)  # first minimum, like mx.argmin
        codes[:, m] = idx.astype(np.uint8)
        residual[:, m * ds:(m + 1) * ds] = (sub - cb[idx]).astype(vectors.dtype)
    return codes, residual


def pq_decode(codes: np.ndarray, codebooks: np.ndarray) -> np.ndarray:
    """quantization.py:146-157 — fp16 gather per subspace."""
    m_sub, _, ds = codebooks.shape
    out = np.zeros((codes.shape[0], m_sub * ds), dtype=F16)
    for m in range(m_sub):
        out[:, m * ds:(m + 1) * ds] = codebooks[m][codes[:, m].astype(np.int64)]
    return out


def rvq_encode(residuals: np.ndarray, codebooks: np.ndarray, threshold: float
               ) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """quantization.py:206-252 — norm-gated greedy RVQ.

    residuals fp16 [N, D]; codebooks fp16 [L, Kr, D] ->
    (codes u16 [A, L], mask bool [N], offsets int32 [A]).
    """
    n, d = residuals.shape
    n_layers, kr, _ = codebooks.shape
    r32 = residuals.astype(F32)
    norms = np.sqrt(np.sum(r32 ** 2, axis=1, dtype=F32))
    mask = norms > F32(threshold) if np.isfinite(threshold) else norms > threshold
    active = np.flatnonzero(mask)
    if active.size == 0 or n_layers == 0:
        return (np.zeros((0, n_layers), dtype=np.uint16), mask,
                np.zeros((0,), dtype=np.int32)) if active.size == 0 else (
                np.zeros((active.size, 0), dtype=np.uint16), mask, active.astype(np.int32))
    running = r32[active]
    codes = np.zeros((active.size, n_layers), dtype=np.uint16)
    chunk = min(512, kr)
    for layer in range(n_layers):
        cb = codebooks[layer].astype(F32)
        best_d = np.full((active.size,), np.inf, dtype=F32)
        best_i = np.zeros((active.size,), dtype=np.int64)
        for start in range(0, kr, chunk):
            end = min(start + chunk, kr)
            dists = squared_l2_distance(running, cb[start:end])
            local_i = np.argmin(dists, axis=1)
            local_b = dists[np.arange(dists.shape[0]), local_i]
            upd = local_b < best_d  # strict <: ties keep the earlier chunk
            best_d = np.where(upd, local_b, best_d)
            best_i = np.where(upd, local_i + start, best_i)
        codes[:, layer] = best_i.astype(np.uint16)
        running = running - cb[best_i]
    return codes, mask, active.astype(np.int32)


def rvq_correction_rows(codes: np.ndarray, codebooks: np.ndarray) -> np.ndarray:
    """quantization.py:266-272 — fp32 sum over layers (left to right), cast to fp16."""
    total = np.zeros((codes.shape[0], codebooks.shape[2]), dtype=F32)
    for layer in range(codebooks.shape[0]):
        total = total + codebooks[layer].astype(F32)[codes[:, layer].astype(np.int64)]
    return total.astype(F16)


def rvq_decode_correction(codes, mask, offsets, codebooks) -> np.ndarray:
    """quantization.py:254-275 — corrections scattered to active rows, zero elsewhere."""
    corr = np.zeros((mask.shape[0], codebooks.shape[2]), dtype=F16)
    if codes.shape[0] == 0:
        return corr
    corr[offsets.astype(np.int64)] = rvq_correction_rows(codes, codebooks)
    return corr


def sparse_topk_encode(vectors: np.ndarray, recon: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """Extension (no reference counterpart): keep the k largest |x - recon| errors.

    Order: descending |err| (fp32), ties to the lower coordinate.  Returns
    (idx u8 [N, k], val fp16 [N, k]) with val = fp16(x - recon) at idx.
    """
    n, d = vectors.shape
    if k == 0:
        return np.zeros((n, 0), np.uint8), np.zeros((n, 0), F16)
    err = vectors.astype(F32) - recon.astype(F32)
    order = np.argsort(-np.abs(err), axis=1, kind="stable")[:, :k]
    vals = np.take_along_axis(err, order, axis=1).astype(F16)
    return order.astype(np.uint8), vals


def sparse_apply(recon: np.ndarray, idx: np.ndarray, val: np.ndarray) -> np.ndarray:
    """Extension: fp32 decode ``recon + sparse`` (returned in fp32, no rounding)."""
    out = recon.astype(F32)
    if idx.shape[1]:
        rows = np.arange(out.shape[0])[:, None]
        np.add.at(out, (rows, idx.astype(np.int64)), val.astype(F32))
    return out


@dataclass
class Codes:
    """Dense per-token code layout used by the B200 build for one [T, H] store.

    pq u8 [T, H, M]; rvq u16 [T, H, L] (zero where inactive); mask bool [T, H];
    sp_idx u8 [T, H, S]; sp_val fp16 [T, H, S].  The reference's sparse
    (codes, offsets) form is ``rvq[mask]`` / ``flatnonzero(mask)``.
    """
    pq: np.ndarray
    rvq: np.ndarray
    mask: np.ndarray
    sp_idx: np.ndarray
    sp_val: np.ndarray

    @property
    def num_tokens(self) -> int:
        return self.pq.shape[0]

    def slice(self, a: int, b: int) -> "Codes":
        return Codes(self.pq[a:b], self.rvq[a:b], self.mask[a:b], self.sp_idx[a:b], self.sp_val[a:b])

    @staticmethod
    def concat(parts: Sequence["Codes"]) -> "Codes":
        return Codes(*(np.concatenate([getattr(p, f) for p in parts], axis=0)
                       for f in ("pq", "rvq", "mask", "sp_idx", "sp_val")))


@dataclass
class Quantizer:
    """HybridQuantizerMLX (quantization.py:296-319) with explicit codebooks."""
    pq_codebooks: np.ndarray            # fp16 [M, K, ds]
    rvq_codebooks: np.ndarray           # fp16 [L, Kr, D]
    rvq_threshold: float
    sparse_topk: int = 0

    @property
    def head_dim(self) -> int:
        return self.pq_codebooks.shape[0] * self.pq_codebooks.shape[2]

    def encode_flat(self, vectors: np.ndarray):
        """quantization.py:305-308 (+ sparse extension) on [N, D] fp16."""
        pq_codes, residual = pq_quantize(vectors, self.pq_codebooks)
        rvq_codes, mask, offsets = rvq_encode(residual, self.rvq_codebooks, self.rvq_threshold)
        recon = self.decode_flat(pq_codes, rvq_codes, mask, offsets)
        sp_idx, sp_val = sparse_topk_encode(vectors, recon, self.sparse_topk)
        return pq_codes, rvq_codes, mask, offsets, sp_idx, sp_val

    def decode_flat(self, pq_codes, rvq_codes, mask, offsets) -> np.ndarray:
        """quantization.py:310-319 — fp16 ``base + correction``."""
        base = pq_decode(pq_codes, self.pq_codebooks)
        corr = rvq_decode_correction(rvq_codes, mask, offsets, self.rvq_codebooks)
        return (base + corr).astype(F16)

    def compress(self, tensor: np.ndarray) -> Codes:
        """quantization.py:330-343 — [T, H, D] flattened to [T*H, D] and encoded."""
        t, h, d = tensor.shape
        pq_codes, rvq_codes, mask, offsets, sp_idx, sp_val = self.encode_flat(tensor.reshape(t * h, d))
        n_layers = self.rvq_codebooks.shape[0]
        dense_rvq = np.zeros((t * h, n_layers), dtype=np.uint16)
        if offsets.size:
            dense_rvq[offsets] = rvq_codes
        return Codes(pq_codes.reshape(t, h, -1), dense_rvq.reshape(t, h, n_layers),
                     mask.reshape(t, h), sp_idx.reshape(t, h, -1), sp_val.reshape(t, h, -1))

    def decode_f32(self, codes: Codes) -> np.ndarray:
        """quantization.py:394-402 decode (+ sparse in fp32).  Returns fp32 [T, H, D]."""
        t, h = codes.pq.shape[:2]
        flat_mask = codes.mask.reshape(t * h)
        offsets = np.flatnonzero(flat_mask).astype(np.int32)
        rvq = codes.rvq.reshape(t * h, -1)[offsets]
        recon = self.decode_flat(codes.pq.reshape(t * h, -1), rvq, flat_mask, offsets)
        out = sparse_apply(recon, codes.sp_idx.reshape(t * h, -1), codes.sp_val.reshape(t * h, -1))
        return out.reshape(t, h, -1)

    def decode(self, codes: Codes) -> np.ndarray:
        """Dense fp16 reconstruction (single rounding of the sparse-corrected value)."""
        if codes.num_tokens == 0:
            return np.zeros((0, codes.pq.shape[1], self.head_dim), dtype=F16)
        return self.decode_f32(codes).astype(F16)


# ---------------------------------------------------------------------------
# Attention (attention.py:16-138)
# ---------------------------------------------------------------------------

def normalize_query_positions(query_positions, batch_size: int, num_heads: int, default_position: int) -> np.ndarray:
    """attention.py:16-36 — None | [B] | [B, H] -> int32 [B, H]."""
    if query_positions is None:
        return np.full((batch_size, num_heads), default_position, dtype=np.int32)
    pos = np.asarray(query_positions, dtype=np.int32)
    if pos.ndim == 1:
        if pos.shape[0] != batch_size:
            raise ValueError("query_positions length must equal batch size")
        return np.broadcast_to(pos.reshape(batch_size, 1), (batch_size, num_heads)).astype(np.int32)
    if pos.shape == (batch_size, num_heads):
        return pos.astype(np.int32)
    raise ValueError("query_positions must have shape [B] or [B, H]")


def blockwise_exact_attention(q: np.ndarray, keys: np.ndarray, values: np.ndarray, scale: float,
                              block_size: int, causal: bool = False, query_positions=None) -> np.ndarray:
    """attention.py:39-105 — fp32 online softmax over key blocks.

    q [Q, Hq, D]; keys/values [W, Hkv, D] (Hkv divides Hq; Hkv == Hq is the
    reference case).  Returns q.dtype [Q, Hq, D].
    """
    nq, hq, d = q.shape
    w = keys.shape[0]
    if w == 0:
        return np.zeros((nq, hq, d), dtype=q.dtype)
    hkv = keys.shape[1]
    group = hq // hkv
    q32 = q.astype(F32)
    running_max = np.full((nq, hq), MASK_FILL_VALUE, dtype=F32)
    running_sum = np.zeros((nq, hq), dtype=F32)
    out = np.zeros((nq, hq, d), dtype=F32)
    pos = normalize_query_positions(query_positions, nq, hq, w - 1)
    scale32 = F32(scale)
    for start in range(0, w, block_size):
        end = min(start + block_size, w)
        kb = keys[start:end].astype(F32)
        vb = values[start:end].astype(F32)
        if group > 1:
            kb = np.repeat(kb, group, axis=1)
            vb = np.repeat(vb, group, axis=1)
        scores = np.sum(q32[:, :, None, :] * np.swapaxes(kb, 0, 1)[None], axis=-1, dtype=F32) * scale32
        if causal:
            positions = np.arange(start, end, dtype=np.int32)
            allowed = positions[None, None, :] <= pos[:, :, None]
            scores = np.where(allowed, scores, MASK_FILL_VALUE).astype(F32)
        else:
            allowed = None
        block_max = np.max(scores, axis=-1)
        new_max = np.maximum(running_max, block_max)
        prev_rescale = np.exp(running_max - new_max).astype(F32)
        running_sum = running_sum * prev_rescale
        out = out * prev_rescale[:, :, None]
        exp_scores = np.exp(scores - new_max[:, :, None]).astype(F32)
        if allowed is not None:
            exp_scores = exp_scores * allowed.astype(F32)
        running_sum = running_sum + np.sum(exp_scores, axis=-1, dtype=F32)
        out = out + np.sum(exp_scores[:, :, :, None] * np.swapaxes(vb, 0, 1)[None], axis=2, dtype=F32)
        running_max = new_max
    safe = np.where(running_sum > 0, running_sum, np.ones_like(running_sum))
    return (out / safe[:, :, None]).astype(q.dtype)


def dense_exact_attention(q: np.ndarray, keys: np.ndarray, values: np.ndarray, scale: float,
                          causal: bool = True) -> np.ndarray:
    """attention.py:108-134 — full-softmax attention for [B, S, H, D] (prefill)."""
    q32, k32, v32 = q.astype(F32), keys.astype(F32), values.astype(F32)
    hq, hkv = q.shape[2], keys.shape[2]
    if hq != hkv:
        k32 = np.repeat(k32, hq // hkv, axis=2)
        v32 = np.repeat(v32, hq // hkv, axis=2)
    scores = np.einsum("bqhd,bkhd->bhqk", q32, k32).astype(F32) * F32(scale)
    if causal:
        qp = np.arange(q.shape[1])
        kp = np.arange(keys.shape[1])
        mask = kp[None, :] <= qp[:, None]
        scores = np.where(mask[None, None], scores, MASK_FILL_VALUE).astype(F32)
    scores = scores - scores.max(axis=-1, keepdims=True)
    probs = np.exp(scores)
    probs = probs / probs.sum(axis=-1, keepdims=True)
    ctx = np.einsum("bhqk,bkhd->bqhd", probs.astype(F32), v32)
    return ctx.astype(q.dtype)


def gelu(x: np.ndarray) -> np.ndarray:
    """attention.py:137-138 — tanh approximation (computed in the input dtype)."""
    return (0.5 * x * (1.0 + np.tanh(0.7978845608 * (x + 0.044715 * (x ** 3))))).astype(x.dtype)


# ---------------------------------------------------------------------------
# Tiered cache (cache.py:33-440) — batch of independent sequences
# ---------------------------------------------------------------------------

def _empty_stats() -> Dict[str, int]:
    """cache.py:59-76 — the 15 access-stat keys."""
    return {k: 0 for k in (
        "window_start", "window_end", "window_tokens", "context_window", "query_tokens",
        "used_router", "hot_tokens_materialized", "warm_tokens_materialized",
        "cold_tokens_materialized", "reconstructed_tokens", "warm_chunk_decodes",
        "cold_chunk_decodes", "cold_chunks_touched", "cold_chunk_cache_hits",
        "cold_chunk_cache_misses")} | {"context_window": -1}


def window_bounds(total: int, query_positions, context_window, current_position):
    """cache.py:199-241 — returns (start, end, adjusted int32 | None)."""
    def to_arr(v):
        return None if v is None else np.asarray(v, dtype=np.int32)
    if total == 0:
        return 0, 0, to_arr(query_positions)
    if query_positions is not None:
        max_query = int(np.max(np.asarray(query_positions, dtype=np.int64)))
    elif current_position is not None:
        max_query = current_position
    else:
        max_query = max(total - 1, 0)
    end = min(max_query + 1, total)
    start = 0 if context_window is None else max(0, end - context_window)
    if query_positions is None:
        return start, end, None
    adjusted = np.maximum(to_arr(query_positions) - start, -1).astype(np.int32)
    return start, end, adjusted


def _overlap(a, b, s, e):
    """cache.py:243-248."""
    lo, hi = max(a, s), min(b, e)
    return None if lo >= hi else (lo, hi)


class OracleCache:
    """RFSNv10KVCacheMLX (cache.py:33-440) on numpy, batch of B sequences.

    Tensors are [B, T, Hkv, D].  ``hot_policy="prefix"`` reproduces the
    reference tiering exactly (hot = first ``hot_capacity`` tokens, then warm,
    then cold chunks of ``block_size_seq`` with chunk id = start // chunk,
    cache.py:103-118, 144-191).  ``"recent"`` (extension) keeps the newest
    tokens hot and spills older ones to warm, and whole chunks from warm to
    cold.  Cold chunks live in host memory here (the reference writes NPZ
    files, storage.py:117-135); their content is the same codes.
    """

    def __init__(self, config: OracleConfig, quantizer: Quantizer, batch: int = 1):
        self.cfg = config
        self.q = quantizer
        self.batch = batch
        self.h = config.num_kv_heads
        self.d = config.head_dim
        self.tokens_k: List[np.ndarray] = []  # raw appended K [B, n, H, D] fp16 (for spills)
        self.hot_k = np.zeros((batch, 0, self.h, self.d), F16)
        self.hot_v = np.zeros_like(self.hot_k)
        self.hot_start = 0  # global position of hot token 0
        self.warm_k: List[Codes] = [self._empty_codes() for _ in range(batch)]
        self.warm_v: List[Codes] = [self._empty_codes() for _ in range(batch)]
        self.warm_start = 0
        self.cold: List[dict] = []  # {"chunk_id", "start_token", "end_token", "k": [Codes]*B, "v": [...]}
        self.num_hot = self.num_warm = self.num_cold = self.total_tokens = 0
        self.last_access_stats = _empty_stats()

    def _empty_codes(self) -> Codes:
        m = self.q.pq_codebooks.shape[0]
        L = self.q.rvq_codebooks.shape[0]
        s = self.q.sparse_topk
        return Codes(np.zeros((0, self.h, m), np.uint8), np.zeros((0, self.h, L), np.uint16),
                     np.zeros((0, self.h), bool), np.zeros((0, self.h, s), np.uint8),
                     np.zeros((0, self.h, s), F16))

    # -- update -------------------------------------------------------------
    def update(self, k: np.ndarray, v: np.ndarray) -> None:
        """cache.py:89-120 (prefix) / recent-hot extension.  k, v fp16 [B, n, H, D]."""
        if k.shape != v.shape:
            raise ValueError("new_keys and new_values must have identical shapes")
        if self.cfg.hot_policy == "prefix":
            self._update_prefix(k, v)
        else:
            self._update_recent(k, v)
        self.total_tokens += k.shape[1]

    def _compress_rows(self, x: np.ndarray) -> List[Codes]:
        return [self.q.compress(x[b]) for b in range(self.batch)]

    def _update_prefix(self, k, v):
        n = k.shape[1]
        off = 0
        hot_space = max(self.cfg.hot_capacity - self.num_hot, 0)
        if hot_space and off < n:
            take = min(hot_space, n - off)
            self.hot_k = np.concatenate([self.hot_k, k[:, off:off + take]], 1)
            self.hot_v = np.concatenate([self.hot_v, v[:, off:off + take]], 1)
            self.num_hot += take
            off += take
        warm_space = max(self.cfg.warm_capacity - self.num_warm, 0)
        if warm_space and off < n:
            take = min(warm_space, n - off)
            ck, cv = self._compress_rows(k[:, off:off + take]), self._compress_rows(v[:, off:off + take])
            self.warm_k = [Codes.concat([a, b]) for a, b in zip(self.warm_k, ck)]
            self.warm_v = [Codes.concat([a, b]) for a, b in zip(self.warm_v, cv)]
            self.num_warm += take
            off += take
        if off < n:
            self._add_to_cold(k[:, off:], v[:, off:], self.num_hot + self.num_warm + self.num_cold)

    def _add_to_cold(self, k, v, start_token):
        """cache.py:134-191 — chunk id = start // chunk, contiguous merge of partial chunks."""
        ct = self.cfg.chunk_tokens
        n = k.shape[1]
        for off in range(0, n, ct):
            end = min(off + ct, n)
            cstart = start_token + off
            cid = cstart // ct
            ck, cv = self._compress_rows(k[:, off:end]), self._compress_rows(v[:, off:end])
            meta = next((m for m in self.cold if m["chunk_id"] == cid), None)
            if meta is not None:
                if cstart != meta["end_token"]:
                    raise ValueError("Cold chunk append must be contiguous with existing metadata")
                meta["k"] = [Codes.concat([a, b]) for a, b in zip(meta["k"], ck)]
                meta["v"] = [Codes.concat([a, b]) for a, b in zip(meta["v"], cv)]
                meta["end_token"] += end - off
                meta["num_tokens"] += end - off
            else:
                self.cold.append({"chunk_id": cid, "start_token": cstart, "end_token": cstart + end - off,
                                  "num_tokens": end - off, "k": ck, "v": cv})
        self.num_cold += n

    def _update_recent(self, k, v):
        cap_h, cap_w, ct = self.cfg.hot_capacity, self.cfg.warm_capacity, self.cfg.chunk_tokens
        self.hot_k = np.concatenate([self.hot_k, k], 1)
        self.hot_v = np.concatenate([self.hot_v, v], 1)
        over = self.hot_k.shape[1] - cap_h
        if over > 0:
            sk, sv = self.hot_k[:, :over], self.hot_v[:, :over]
            self.hot_k, self.hot_v = self.hot_k[:, over:], self.hot_v[:, over:]
            self.hot_start += over
            ck, cv = self._compress_rows(sk), self._compress_rows(sv)
            self.warm_k = [Codes.concat([a, b]) for a, b in zip(self.warm_k, ck)]
            self.warm_v = [Codes.concat([a, b]) for a, b in zip(self.warm_v, cv)]
        n_w = self.warm_k[0].num_tokens
        if n_w > cap_w:
            evict = ((n_w - cap_w + ct - 1) // ct) * ct
            for off in range(0, evict, ct):
                cstart = self.warm_start + off
                self.cold.append({"chunk_id": cstart // ct, "start_token": cstart, "end_token": cstart + ct,
                                  "num_tokens": ct,
                                  "k": [c.slice(off, off + ct) for c in self.warm_k],
                                  "v": [c.slice(off, off + ct) for c in self.warm_v]})
            self.warm_k = [c.slice(evict, c.num_tokens) for c in self.warm_k]
            self.warm_v = [c.slice(evict, c.num_tokens) for c in self.warm_v]
            self.warm_start += evict
        self.num_hot = self.hot_k.shape[1]
        self.num_warm = self.warm_k[0].num_tokens
        self.num_cold = sum(m["num_tokens"] for m in self.cold)

    # -- spans -----------------------------------------------------------------
    def spans(self):
        """(kind, global_start, global_end) for hot/warm in global position order."""
        if self.cfg.hot_policy == "prefix":
            return [("hot", 0, self.num_hot), ("warm", self.num_hot, self.num_hot + self.num_warm)]
        return [("warm", self.warm_start, self.warm_start + self.num_warm),
                ("hot", self.hot_start, self.hot_start + self.num_hot)]

    # -- materialize ------------------------------------------------------------
    def chunk_centroids(self) -> Tuple[List[int], np.ndarray]:
        """Centroid routing (extension): (cold chunk ids, fp32 [C, B * Hkv, D] mean decoded key of
        each chunk per row, row = b * Hkv + h)."""
        ids, cents = [], []
        for meta in self.cold:
            dec = np.stack([self.q.decode(c) for c in meta["k"]])  # [B, n, Hkv, D] fp16
            cents.append(dec.astype(F32).mean(axis=1).reshape(self.batch * self.h, self.d))
            ids.append(meta["chunk_id"])
        return ids, (np.stack(cents).astype(F32) if cents else np.zeros((0, self.batch * self.h, self.d), F32))

    def materialize_window(self, query_positions=None, context_window=None, current_position=None,
                           cold_hits: Optional[set] = None, used_router: bool = False,
                           routed_chunks: Optional[Sequence[int]] = None):
        """cache.py:344-393 — dense fp16 window [B, W, H, D] in position order + stats.

        Sparse residuals (an extension) are added in fp32 and the sum is rounded
        to fp16 once, so attention sees exactly the materialised values."""
        dec = self.q.decode
        start, end, adjusted = window_bounds(self.total_tokens, query_positions, context_window, current_position)
        stats = _empty_stats()
        stats["window_start"], stats["window_end"] = start, end
        stats["window_tokens"] = max(0, end - start)
        stats["context_window"] = -1 if context_window is None else context_window
        stats["used_router"] = int(used_router)
        pieces_k: List[Tuple[int, np.ndarray]] = []
        pieces_v: List[Tuple[int, np.ndarray]] = []
        bs = max(1, self.cfg.block_size_seq)
        for kind, s, e in self.spans():
            ov = _overlap(start, end, s, e)
            if ov is None:
                continue
            a, b = ov[0] - s, ov[1] - s
            if kind == "hot":  # cache.py:250-261
                stats["hot_tokens_materialized"] += b - a
                pieces_k.append((ov[0], self.hot_k[:, a:b]))
                pieces_v.append((ov[0], self.hot_v[:, a:b]))
            else:  # cache.py:263-291 — decoded in block_size_seq chunks from the overlap start
                for cs in range(a, b, bs):
                    ce = min(cs + bs, b)
                    pieces_k.append((s + cs, np.stack([dec(c.slice(cs, ce)) for c in self.warm_k])))
                    pieces_v.append((s + cs, np.stack([dec(c.slice(cs, ce)) for c in self.warm_v])))
                    stats["warm_tokens_materialized"] += ce - cs
                    stats["reconstructed_tokens"] += ce - cs
                    stats["warm_chunk_decodes"] += 1
        for meta in self.cold:  # cache.py:293-342
            ov = _overlap(start, end, meta["start_token"], meta["end_token"])
            if ov is None or (routed_chunks is not None and meta["chunk_id"] not in routed_chunks):
                continue
            if used_router:
                if cold_hits is not None and meta["chunk_id"] in cold_hits:
                    stats["cold_chunk_cache_hits"] += 1
                else:
                    stats["cold_chunk_cache_misses"] += 1
            a, b = ov[0] - meta["start_token"], ov[1] - meta["start_token"]
            pieces_k.append((ov[0], np.stack([dec(c.slice(a, b)) for c in meta["k"]])))
            pieces_v.append((ov[0], np.stack([dec(c.slice(a, b)) for c in meta["v"]])))
            stats["cold_tokens_materialized"] += b - a
            stats["reconstructed_tokens"] += b - a
            stats["cold_chunk_decodes"] += 1
            stats["cold_chunks_touched"] += 1
        self.last_access_stats = dict(stats)
        if not pieces_k:
            empty = np.zeros((self.batch, 0, self.h, self.d), F16)
            return empty, empty, adjusted
        if self.cfg.hot_policy == "prefix":
            # reference concatenation order: hot, warm chunks, cold chunks (cache.py:378-391)
            keys = np.concatenate([p for _, p in pieces_k], 1)
            vals = np.concatenate([p for _, p in pieces_v], 1)
        else:
            order = np.argsort([s for s, _ in pieces_k], kind="stable")
            keys = np.concatenate([pieces_k[i][1] for i in order], 1)
            vals = np.concatenate([pieces_v[i][1] for i in order], 1)
        return keys, vals, adjusted

    def attention_forward(self, q: np.ndarray, causal=True, query_positions=None, context_window=None,
                          current_position=None, routed_chunks: Optional[Sequence[int]] = None) -> np.ndarray:
        """cache.py:395-428 — q [B, Q, Hq, D] (one query set per sequence).  routed_chunks
        (centroid routing, extension): only these cold chunks enter the window."""
        keys, vals, adjusted = self.materialize_window(query_positions, context_window, current_position,
                                                       routed_chunks=routed_chunks)
        self.last_access_stats["query_tokens"] = int(q.shape[1])
        if keys.shape[1] == 0:
            return np.zeros_like(q)
        out = np.stack([blockwise_exact_attention(q[b], keys[b], vals[b], self.d ** -0.5,
                                                  self.cfg.block_size_seq, causal, adjusted)
                        for b in range(self.batch)])
        return out


# ---------------------------------------------------------------------------
# Router (storage.py:154-237)
# ---------------------------------------------------------------------------

def router_candidates(existing_chunk_ids: Sequence[int], current_position: int, context_window: int,
                      chunk_size: int, top_k: int) -> List[int]:
    """storage.py:166-182 — existing ids in [(p-w)//cs, (p+w)//cs] sorted by |id*cs - p|."""
    cs = max(chunk_size, 1)
    start_chunk = max(0, (current_position - context_window) // cs)
    end_chunk = max(start_chunk, (current_position + context_window) // cs)
    existing = set(int(c) for c in existing_chunk_ids)
    cands = [c for c in range(start_chunk, end_chunk + 1) if c in existing]
    cands.sort(key=lambda c: abs(c * cs - current_position))
    return cands[:top_k]


def route_topk(q: np.ndarray, centroids: np.ndarray, kv_heads: int, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """Centroid routing (extension, rfsn_route_topk): q [B, Q, Hq, D], centroids fp32 [C, B * Hkv, D].
    score[c] = max over (b, i, h) of q[b, i, h] . centroids[c, b * Hkv + h // G] in fp32; returns
    (the k highest-scoring chunk indices, descending, ties to the lower index; scores [C])."""
    b_, nq, hq, d = q.shape
    g = hq // kv_heads
    cent = centroids.astype(F32).reshape(centroids.shape[0], b_, kv_heads, d)
    cent = np.repeat(cent, g, axis=2)                                  # [C, B, Hq, D]
    dots = np.einsum("bihd,cbhd->cbih", q.astype(F32), cent)           # [C, B, Q, Hq]
    scores = dots.reshape(centroids.shape[0], -1).max(axis=1).astype(F32)
    order = np.lexsort((np.arange(scores.shape[0]), -scores))          # descending, ties to lower index
    return order[:k], scores


def centroid_router_scores(q: np.ndarray, chunk_centroids: np.ndarray) -> np.ndarray:
    """Extension: score of each cold chunk = max over query heads of q_h . mean_k(chunk)."""
    # q [Hq, D]; chunk_centroids [C, Hkv, D] -> [C]
    hq, d = q.shape
    hkv = chunk_centroids.shape[1]
    cent = np.repeat(chunk_centroids.astype(F32), hq // hkv, axis=1)
    return np.max(np.einsum("hd,chd->ch", q.astype(F32), cent), axis=1)


# ---------------------------------------------------------------------------
# Calibration (rfsn_v10_mlx_ane_complete.py:175-225)
# ---------------------------------------------------------------------------

def calibrate_pq(vectors: np.ndarray, num_subspaces: int, codebook_size: int, iterations: int,
                 sample_idx: np.ndarray) -> Tuple[np.ndarray, List[float]]:
    """k-means: init from ``sample_idx`` rows (one index array per subspace, [M, K]),
    Lloyd updates, empty clusters keep their centroid (rfsn_v10_mlx_ane_complete.py:185-209).
    Returns (codebooks fp16 [M, K, ds], avg distortion per iteration)."""
    n, d = vectors.shape
    ds = d // num_subspaces
    cbs = np.stack([vectors[sample_idx[m], m * ds:(m + 1) * ds] for m in range(num_subspaces)]).astype(F16)
    x32 = vectors.astype(F32)
    distortion = []
    for _ in range(iterations):
        codes, _ = pq_quantize(vectors, cbs)
        new = cbs.astype(F32).copy()
        for m in range(num_subspaces):
            sub = x32[:, m * ds:(m + 1) * ds]
            c = codes[:, m].astype(np.int64)
            for centroid in range(codebook_size):  # rfsn_v10_mlx_ane_complete.py:203-206
                members = np.where(c == centroid)[0]
                if members.size:
                    new[m][centroid] = sub[members].mean(axis=0)
        cbs = new.astype(F16)
        recon = pq_decode(codes, cbs)
        distortion.append(float(np.mean((x32 - recon.astype(F32)) ** 2)))
    return cbs, distortion


# ---------------------------------------------------------------------------
# Decoder layer (rfsn_v10_mlx_ane_complete.py:55-172)
# ---------------------------------------------------------------------------

def rms_norm(x: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """mlx.nn.RMSNorm with unit weight: fp32 x * rsqrt(mean(x^2) + eps), back to x's dtype."""
    xf = x.astype(F32)
    y = xf * (F32(1.0) / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True, dtype=F32) + F32(eps)))
    return y.astype(x.dtype)


def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """mlx.nn.Linear without bias: W cast to x's dtype (fp16), products summed in fp32."""
    return (x.astype(F32) @ w.astype(x.dtype).astype(F32).T).astype(x.dtype)


class OracleDecoderLayer:
    """RFSNDecoderLayerMLX restated: RMSNorm -> q/k/v -> cache update -> cache attention (or
    dense causal attention) -> o_proj + residual -> RMSNorm -> GELU FFN (2x) + residual.
    Weights are fp16 [out, in]; batch 1 as in the reference's cache path."""

    def __init__(self, config: OracleConfig, quantizer: Quantizer, weights: Dict[str, np.ndarray]):
        self.cfg = config
        self.w = weights
        self.h = config.num_heads
        self.hkv = config.num_kv_heads
        self.d = config.head_dim
        self.cache = OracleCache(config, quantizer, batch=1)

    def _heads(self, y: np.ndarray, heads: int) -> np.ndarray:
        b, s, _ = y.shape
        return y.reshape(b, s, heads, self.d).astype(F16)

    def prefill_cache(self, x: np.ndarray) -> None:
        """rfsn_v10_mlx_ane_complete.py:90-104."""
        a = rms_norm(x.astype(F16))
        self.cache.update(self._heads(linear(a, self.w["k_proj"]), self.hkv),
                          self._heads(linear(a, self.w["v_proj"]), self.hkv))

    def __call__(self, x: np.ndarray, use_cache: bool = False, context_window: Optional[int] = None) -> np.ndarray:
        """rfsn_v10_mlx_ane_complete.py:114-172."""
        residual = x.astype(F16)
        a = rms_norm(residual)
        q = self._heads(linear(a, self.w["q_proj"]), self.h)
        k = self._heads(linear(a, self.w["k_proj"]), self.hkv)
        v = self._heads(linear(a, self.w["v_proj"]), self.hkv)
        b, s = x.shape[:2]
        if use_cache:
            self.cache.update(k, v)
            total = self.cache.total_tokens
            win = context_window if context_window is not None else \
                max(self.cfg.block_size_seq, min(total, self.cfg.warm_capacity))
            att = self.cache.attention_forward(q[:, :1], causal=True, query_positions=[total - 1],
                                               current_position=total - 1, context_window=win)
            att = att.reshape(b, 1, self.h, self.d)
        else:
            att = dense_exact_attention(q, k, v, self.d ** -0.5, causal=True)
        hidden = residual + linear(att.reshape(b, s, self.h * self.d).astype(F16), self.w["o_proj"])
        f = rms_norm(hidden)
        return hidden + linear(gelu(linear(f, self.w["ffn_up"])), self.w["ffn_down"])


# ---------------------------------------------------------------------------
# Llama adapter layer (llama32_adapter.py:374-386, 417-662)
# ---------------------------------------------------------------------------

def llama_rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """llama32_adapter.py:497-500 — fp32 x / sqrt(mean(x^2) + eps) * weight, to fp16."""
    xf = x.astype(F32)
    var = np.mean(xf ** 2, axis=-1, keepdims=True, dtype=F32)
    return ((xf / np.sqrt(var + F32(eps))) * weight.astype(F32)).astype(F16)


def llama_linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """llama32_adapter.py:492-494 — fp32 matmul of fp16 operands, to fp16."""
    return (x.astype(F32) @ w.astype(F32).T).astype(F16)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """llama32_adapter.py:375-377."""
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def apply_rope(q: np.ndarray, k: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """llama32_adapter.py:555-568 — tables fp16 [1, S, D] (as _normalize_position_component
    leaves them), x * cos + rotate_half(x) * sin in fp32, to fp16."""
    c = cos.astype(F16).astype(F32)[:, :, None, :]
    s = sin.astype(F16).astype(F32)[:, :, None, :]
    q32, k32 = q.astype(F32), k.astype(F32)
    return ((q32 * c + rotate_half(q32) * s).astype(F16), (k32 * c + rotate_half(k32) * s).astype(F16))


def silu(x: np.ndarray) -> np.ndarray:
    """llama32_adapter.py:502-504 — fp32 x * sigmoid(x), to fp16."""
    xf = x.astype(F32)
    return (xf * (F32(1.0) / (F32(1.0) + np.exp(-xf)))).astype(F16)


class OracleLlamaLayer:
    """Llama32DecoderLayerMLX restated for batch 1 (the reference's limit): RMSNorm with a
    weight, q/k/v projections, RoPE from given tables, the RFSN cache (GQA heads stored once,
    which equals the reference's cache over _repeat_kv'd heads), o_proj + residual, RMSNorm,
    SwiGLU MLP + residual.  weights: fp16 [out, in] projections and fp16 norm weights."""

    def __init__(self, config: OracleConfig, quantizer: Quantizer, weights: Dict[str, np.ndarray], kv_heads: int,
                 eps: float):
        self.cfg = replace(config, num_kv_heads=kv_heads)
        self.w = weights
        self.h, self.hkv, self.d, self.eps = config.num_heads, kv_heads, config.head_dim, eps
        self.cache = OracleCache(self.cfg, quantizer, batch=1)

    def _qkv(self, x: np.ndarray, cos: np.ndarray, sin: np.ndarray):
        """llama32_adapter.py:570-582 (without the repeat: the cache keeps the KV heads)."""
        b, s, _ = x.shape
        a = llama_rms_norm(x, self.w["input_layernorm"], self.eps)
        q = llama_linear(a, self.w["q_proj"]).reshape(b, s, self.h, self.d)
        k = llama_linear(a, self.w["k_proj"]).reshape(b, s, self.hkv, self.d)
        v = llama_linear(a, self.w["v_proj"]).reshape(b, s, self.hkv, self.d)
        q, k = apply_rope(q, k, cos, sin)
        return q, k, v

    def prefill_cache(self, x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> None:
        """llama32_adapter.py:591-614."""
        _, k, v = self._qkv(x.astype(F16), cos, sin)
        self.cache.update(k, v)

    def __call__(self, x: np.ndarray, cos: np.ndarray, sin: np.ndarray, use_cache: bool = False,
                 context_window: Optional[int] = None) -> np.ndarray:
        """llama32_adapter.py:616-662."""
        residual = x.astype(F16)
        q, k, v = self._qkv(residual, cos, sin)
        b, s = x.shape[:2]
        if use_cache:
            self.cache.update(k, v)
            total = self.cache.total_tokens
            att = self.cache.attention_forward(q[:, :1], causal=True, query_positions=[total - 1],
                                               current_position=total - 1, context_window=context_window)
            att = att.reshape(b, 1, self.h, self.d)
        else:
            att = dense_exact_attention(q, k, v, self.d ** -0.5, causal=True)
        hidden = residual + llama_linear(att.reshape(b, s, self.h * self.d).astype(F16), self.w["o_proj"])
        m = llama_rms_norm(hidden, self.w["post_attention_layernorm"], self.eps)
        act = silu(llama_linear(m, self.w["gate_proj"])) * llama_linear(m, self.w["up_proj"])
        return hidden + llama_linear(act.astype(F16), self.w["down_proj"])


# ---------------------------------------------------------------------------
# Affine codebook quantization (quantization.py:36-89; MLX 0.29.3 mx.quantize, affine mode)
# ---------------------------------------------------------------------------

def affine_quantize(w: np.ndarray, bits: int, group: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """The published affine scheme of mx.quantize / mx.dequantize, per group of `group`
    consecutive elements of a row (fp32): scale = (max - min) / (2^bits - 1), bias = min,
    q = clip(round_half_even((w - bias) / scale), 0, 2^bits - 1), w' = q * scale + bias.
    A constant group has scale 0, codes 0 and w' = bias.  MLX is not installed here, so this
    restatement is not pinned to MLX's own output.  Returns (q uint8, scales, biases, w')."""
    w32 = np.asarray(w, F32)
    rows, cols = w32.shape
    g = w32.reshape(rows, cols // group, group)
    mx_, mn = g.max(-1), g.min(-1)
    nbins = F32((1 << bits) - 1)
    scale = ((mx_ - mn) / nbins).astype(F32)
    safe = np.where(scale > 0, scale, F32(1)).astype(F32)
    q = np.where(scale[..., None] > 0, np.clip(np.rint((g - mn[..., None]) / safe[..., None]), 0, nbins), 0).astype(F32)
    deq = (q * scale[..., None]).astype(F32) + mn[..., None]
    return q.astype(np.uint8).reshape(rows, cols), scale, mn.astype(F32), deq.astype(F32).reshape(rows, cols)
