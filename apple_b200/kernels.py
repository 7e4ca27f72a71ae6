"""Tensor-level wrappers over the C ABI (include/rfsn_b200.h).

Every function takes CUDA tensors, checks dtype/device/layout, builds the
ABI structs and calls the library on the current torch stream.  Storage
classes here own the device buffers of one code store or one quantizer.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import AttnArgs, CodeStore, DenseStore, Quantizer, Segment, call, lib

STORE_HOT, STORE_WARM, STORE_COLD = 0, 1, 2


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device_index: Optional[int] = None) -> int:
    """Handle of the current torch CUDA stream (of ``device_index``, default the current device)."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(torch.cuda.current_device() if device_index is None else device_index)
    return torch.cuda.current_stream().cuda_stream


def align16(n: int) -> int:
    return (n + 15) // 16 * 16


def _need_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the RFSN B200 path has no CPU fallback)")


@dataclass
class QuantizerBuffers:
    """Device codebooks of one HybridQuantizer plus the fields of ``rfsn_quantizer``."""
    pq_codebooks: torch.Tensor           # fp16 [M, K, ds]
    rvq_codebooks: Optional[torch.Tensor]  # fp16 [L, Kr, D] or None
    threshold: float
    sparse_topk: int = 0

    def __post_init__(self):
        _need_cuda(self.pq_codebooks, "pq_codebooks")
        self.pq_codebooks = self.pq_codebooks.to(torch.float16).contiguous()
        if self.rvq_codebooks is not None and self.rvq_codebooks.shape[0] == 0:
            self.rvq_codebooks = None
        if self.rvq_codebooks is not None:
            self.rvq_codebooks = self.rvq_codebooks.to(torch.float16).contiguous()

    @property
    def M(self) -> int:
        return self.pq_codebooks.shape[0]

    @property
    def K(self) -> int:
        return self.pq_codebooks.shape[1]

    @property
    def ds(self) -> int:
        return self.pq_codebooks.shape[2]

    @property
    def D(self) -> int:
        return self.M * self.ds

    @property
    def L(self) -> int:
        return 0 if self.rvq_codebooks is None else self.rvq_codebooks.shape[0]

    @property
    def Kr(self) -> int:
        return 0 if self.rvq_codebooks is None else self.rvq_codebooks.shape[1]

    @property
    def rvq_code_dtype(self) -> torch.dtype:
        return torch.uint8 if self.Kr <= 256 else torch.int16

    def struct(self) -> Quantizer:
        q = Quantizer()
        q.pq_codebooks = _ptr(self.pq_codebooks)
        q.rvq_codebooks = _ptr(self.rvq_codebooks)
        q.head_dim, q.num_subspaces, q.subspace_dim, q.pq_codebook_size = self.D, self.M, self.ds, self.K
        q.rvq_layers, q.rvq_codebook_size = self.L, self.Kr
        q.rvq_threshold = float(self.threshold)
        q.sparse_topk = int(self.sparse_topk)
        return q


BLOCK_TOKENS = 16
FIELD_NAMES = ("pq", "rvq", "active", "sp_idx", "sp_val")


def block_layout(qz: "QuantizerBuffers"):
    """Byte layout of one 16-token block (mirrors apple_b200/csrc/rfsn_layout.h).

    Returns (offsets[10], bytes_per_token[5], block_bytes); field f = kv*5 + k with
    k in (pq, rvq, active, sp_idx, sp_val)."""
    cs = 2 if qz.Kr > 256 else 1
    bpt = [qz.M, qz.L * cs, 1 if qz.L > 0 else 0, qz.sparse_topk, 2 * qz.sparse_topk]
    off, pos = [], 0
    for f in range(10):
        off.append(pos)
        pos += BLOCK_TOKENS * bpt[f % 5]
    return off, bpt, pos


class CodeStoreBuffers:
    """Device (or pinned host) ``rfsn_code_store``: K and V codes of [slots, rows, cap]
    tokens in 16-token blocks that interleave every field (one contiguous range per
    token run, so a tile is one bulk copy)."""

    def __init__(self, qz: QuantizerBuffers, rows: int, cap: int, slots: int = 1,
                 device: Optional[torch.device] = None, pin_memory: bool = False):
        cap = align16(max(cap, 16))
        dev = device if device is not None else qz.pq_codebooks.device
        self.qz = qz
        self.rows, self.cap, self.slots = rows, cap, slots
        self.off, self.bpt, self.block_bytes = block_layout(qz)
        shape = (slots, rows, cap // BLOCK_TOKENS, self.block_bytes)
        if pin_memory:
            self.data = torch.zeros(shape, dtype=torch.uint8, device="cpu", pin_memory=True)
        else:
            self.data = torch.zeros(shape, dtype=torch.uint8, device=dev)

    def struct(self) -> CodeStore:
        s = CodeStore()
        s.data = _ptr(self.data)
        s.cap, s.rows, s.slots = self.cap, self.rows, self.slots
        return s

    def field(self, kv: int, name: str) -> Optional[torch.Tensor]:
        """Strided view [slots, rows, cap/16, 16, width] of one field (None if absent).

        dtypes: pq/active/sp_idx uint8; rvq uint8 (Kr <= 256) or int16; sp_val fp16."""
        k = FIELD_NAMES.index(name)
        w = self.bpt[k]
        if w == 0:
            return None
        f = kv * 5 + k
        v = self.data[..., self.off[f]: self.off[f] + BLOCK_TOKENS * w]
        v = v.unflatten(-1, (BLOCK_TOKENS, w))
        if name == "sp_val":
            v = v.view(torch.float16)
        elif name == "rvq" and self.qz.Kr > 256:
            v = v.view(torch.int16)
        return v

    def read(self, kv: int, name: str, slot: int, row: int, first: int, count: int) -> Optional[torch.Tensor]:
        """Copy of a field for tokens [first, first+count) of one row: [count, width]."""
        v = self.field(kv, name)
        if v is None:
            return None
        t = torch.arange(first, first + count, device=v.device)
        return v[slot, row, t // BLOCK_TOKENS, t % BLOCK_TOKENS]

    def write(self, kv: int, name: str, slot: int, row: int, first: int, values: torch.Tensor) -> None:
        """Scatter [count, width] values into tokens [first, first+count) of one row."""
        v = self.field(kv, name)
        if v is None:
            return
        t = torch.arange(first, first + values.shape[0], device=v.device)
        v[slot, row, t // BLOCK_TOKENS, t % BLOCK_TOKENS] = values.to(device=v.device, dtype=v.dtype)

    def read_rows(self, kv: int, name: str, slot: int, first: int, count: int,
                  rows: Optional[int] = None) -> Optional[torch.Tensor]:
        """Copy of a field for tokens [first, first+count) of rows [0, rows): [rows, count, width]."""
        v = self.field(kv, name)
        if v is None:
            return None
        t = torch.arange(first, first + count, device=v.device)
        return v[slot, : (self.rows if rows is None else rows)][:, t // BLOCK_TOKENS, t % BLOCK_TOKENS]

    def write_rows(self, kv: int, name: str, slot: int, first: int, values: torch.Tensor) -> None:
        """Scatter [rows, count, width] values into tokens [first, first+count) of rows [0, rows)."""
        v = self.field(kv, name)
        if v is None:
            return
        t = torch.arange(first, first + values.shape[1], device=v.device)
        v[slot, : values.shape[0]][:, t // BLOCK_TOKENS, t % BLOCK_TOKENS] = values.to(device=v.device,
                                                                                   dtype=v.dtype)

    def put(self, kv: int, name: str, slot: int, row: int, tokens: torch.Tensor, values: torch.Tensor) -> None:
        """Scatter [n, width] values into the given token indices of one row."""
        v = self.field(kv, name)
        if v is None:
            return
        t = tokens.to(device=v.device, dtype=torch.long)
        v[slot, row, t // BLOCK_TOKENS, t % BLOCK_TOKENS] = values.to(device=v.device, dtype=v.dtype)

    def nbytes_per_slot(self) -> int:
        return self.data[0].numel()

    def grow(self, qz: QuantizerBuffers, new_cap: int) -> "CodeStoreBuffers":
        new = CodeStoreBuffers(qz, self.rows, new_cap, self.slots, device=self.data.device)
        nb = self.cap // BLOCK_TOKENS
        new.data[:, :, :nb].copy_(self.data)
        return new


def encode(qz: QuantizerBuffers, x: torch.Tensor, store: CodeStoreBuffers, slot: int, first: int,
           residual_out: Optional[torch.Tensor] = None, kv: int = 0) -> None:
    """Encode fp16 vectors x [B, T, H, D] (D contiguous) into the K (kv=0) or V (kv=1)
    fields of rows b*H+h, tokens first..first+T."""
    _need_cuda(x, "x")
    if x.dtype != torch.float16 or x.dim() != 4 or x.shape[-1] != qz.D or x.stride(-1) != 1:
        raise ValueError("x must be fp16 [B, T, H, D] with a contiguous last dim")
    B, T, H, _ = x.shape
    if residual_out is not None and residual_out.stride() != x.stride():
        raise ValueError("residual_out must have the same strides as x")
    q = qz.struct()
    s = store.struct()
    call("rfsn_encode", C.byref(q), _ptr(x), B, T, H, x.stride(0), x.stride(1), x.stride(2), C.byref(s),
         kv, slot, first, _ptr(residual_out), _stream())


def encode_kv(qz: QuantizerBuffers, k: torch.Tensor, v: torch.Tensor, store: CodeStoreBuffers, slot: int,
              first: int) -> None:
    """Encode K and V [B, T, H, D] (same shape and strides) into tokens first..first+T of a
    store in one launch (rfsn_encode_kv)."""
    _need_cuda(k, "k")
    _need_cuda(v, "v")
    if k.shape != v.shape or k.stride() != v.stride():
        raise ValueError("k and v must have the same shape and strides")
    if k.dtype != torch.float16 or v.dtype != torch.float16 or k.dim() != 4 or k.shape[-1] != qz.D or k.stride(-1) != 1:
        raise ValueError("k and v must be fp16 [B, T, H, D] with a contiguous last dim")
    B, T, H, _ = k.shape
    q = qz.struct()
    s = store.struct()
    call("rfsn_encode_kv", C.byref(q), _ptr(k), _ptr(v), B, T, H, k.stride(0), k.stride(1), k.stride(2), C.byref(s),
         slot, first, _stream())


def decode_codes(qz: QuantizerBuffers, store: CodeStoreBuffers, slot: int, first: int, count: int,
                 out: torch.Tensor, kv: int = 0) -> torch.Tensor:
    """Exact fp16 decode of K (kv=0) or V (kv=1) tokens [first, first+count) into
    out [B, count, H, D] (D contiguous)."""
    _need_cuda(out, "out")
    if out.dtype != torch.float16 or out.dim() != 4 or out.shape[1] != count or out.stride(-1) != 1:
        raise ValueError("out must be fp16 [B, count, H, D]")
    B, _, H, _ = out.shape
    q = qz.struct()
    s = store.struct()
    call("rfsn_decode_codes", C.byref(q), C.byref(s), kv, slot, first, count, B, H, _ptr(out), out.stride(0),
         out.stride(1), out.stride(2), _stream())
    return out


_WORKSPACE: dict = {}


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Per-device scratch buffer for the split-K partials (grown on demand).  It starts
    zeroed: its leading launch counter and row tickets are then kept by the library."""
    key = (device.type, device.index)
    buf = _WORKSPACE.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACE[key] = buf
    return buf


class _AttnCall:
    """Argument structs of one decode-attention call shape, kept for reuse: a
    decode loop calls with the same stores, window and shapes step after step,
    so only the tensor pointers are rewritten."""

    __slots__ = ("args", "segs", "qs", "ws", "src")

    def __init__(self, args, segs, qs, ws):
        self.args, self.segs, self.qs, self.ws = args, segs, qs, ws
        self.src = None  # the segment list last written into segs (patch_segments)


_ATTN_CALLS: "dict" = {}


def queries_packed(q: torch.Tensor) -> bool:
    """[B, Q, Hq, D] with each sequence's queries packed and any batch stride the kernel takes."""
    B, Qn, Hq, D = q.shape
    inner = q.stride(3) == 1 and (Hq == 1 or q.stride(2) == D) and (Qn == 1 or q.stride(1) == Hq * D)
    return inner and (B == 1 or (q.stride(0) % 8 == 0 and q.stride(0) >= Qn * Hq * D)) and q.data_ptr() % 16 == 0


def _qz_key(qz: QuantizerBuffers) -> tuple:
    return (_ptr(qz.pq_codebooks), _ptr(qz.rvq_codebooks), qz.M, qz.K, qz.ds, qz.L, qz.Kr, float(qz.threshold),
            int(qz.sparse_topk))


def _store_key(st: Optional[CodeStoreBuffers]) -> Optional[tuple]:
    return None if st is None else (_ptr(st.data), st.cap, st.rows, st.slots)


def decode_attention(qz: QuantizerBuffers, q: torch.Tensor, out: torch.Tensor, segments: Sequence[Tuple],
                     kv_heads: int, qpos: Optional[torch.Tensor] = None, causal: bool = True, scale: Optional[float] = None,
                     hot: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                     warm: Optional[CodeStoreBuffers] = None,
                     cold: Optional[CodeStoreBuffers] = None,
                     num_ctas: int = 0, device_status: Optional[torch.Tensor] = None, gather=None) -> torch.Tensor:
    """Fused decode attention.  q/out fp16 [B, Q, Hq, D]; qpos int32 [B, Q, Hq] (global positions).

    hot: (k, v) fp16 [rows, cap, D]; warm/cold: code stores (K and V fields).
    segments: (store, slot, first, count, pos0) tuples in window order.
    gather: a sharding.PeerGather; the whole batch's output then also lands in gather.full.
    """
    entry = attention_call(qz, q, out, segments, kv_heads, qpos=qpos, causal=causal, scale=scale, hot=hot, warm=warm,
                           cold=cold, num_ctas=num_ctas, gather=gather)
    run_attention(entry, q, out, qpos if causal else None, device_status)
    return out


def run_attention(entry: "_AttnCall", q: torch.Tensor, out: torch.Tensor, qpos: Optional[torch.Tensor] = None,
                  device_status: Optional[torch.Tensor] = None) -> None:
    """Launch a prepared call (attention_call) with this step's q / out / qpos.  The caller
    guarantees they have the shapes, strides and causal setting the call was prepared for.
    A call whose segments were patched (patch_segments) may need more split-K workspace
    than it was prepared with: the library then refuses the launch, and it is sized again."""
    a = entry.args
    a.q, a.out = q.data_ptr(), out.data_ptr()
    a.qpos = qpos.data_ptr() if qpos is not None else None
    a.device_status = _ptr(device_status)
    stream = _stream(q.device.index)
    status = lib().rfsn_decode_attention(C.byref(a), C.byref(entry.qs), stream)
    if status == _lib.RFSN_ERR_WORKSPACE_TOO_SMALL:
        _size_workspace(entry, q.device)
        status = lib().rfsn_decode_attention(C.byref(a), C.byref(entry.qs), stream)
    _lib.check("rfsn_decode_attention", status)


def run_attention_host(entry: "_AttnCall", q_host: torch.Tensor, stage: torch.Tensor, out: torch.Tensor,
                       qpos: Optional[torch.Tensor] = None, synchronize: bool = True) -> None:
    """Launch a prepared call with the query in pinned host memory (rfsn_decode_attention_host):
    the library copies q_host into `stage` (a contiguous device tensor shaped like the prepared
    call's q) on the stream and runs the attention; with synchronize it returns once the stream
    has finished, so a pinned host `out`, which the kernel writes over the bus, holds the result."""
    a = entry.args
    a.out = out.data_ptr()
    a.qpos = qpos.data_ptr() if qpos is not None else None
    a.device_status = None
    stream = _stream(stage.device.index)
    args = (C.byref(a), C.byref(entry.qs), q_host.data_ptr(), stage.data_ptr(), int(bool(synchronize)), stream)
    status = lib().rfsn_decode_attention_host(*args)
    if status == _lib.RFSN_ERR_WORKSPACE_TOO_SMALL:
        _size_workspace(entry, stage.device)
        status = lib().rfsn_decode_attention_host(*args)
    _lib.check("rfsn_decode_attention_host", status)


def _size_workspace(entry: "_AttnCall", device: torch.device) -> None:
    a = entry.args
    nbytes = C.c_size_t(0)
    call("rfsn_attention_workspace_size", C.byref(a), C.byref(entry.qs), C.byref(nbytes))
    ws = workspace(nbytes.value, device)
    a.workspace, a.workspace_bytes = _ptr(ws), ws.numel()
    entry.ws = ws


def patch_segments(entry: "_AttnCall", segments: Sequence[Tuple]) -> None:
    """Point a prepared call (attention_call with memo=False) at new token ranges: the
    segments keep their count, stores and slots, and take new first / count / pos0.  A
    decode loop over a growing or sliding window patches its call each step instead of
    preparing a new one.  Passing the same list object as the last patch is a no-op."""
    if segments is entry.src:
        return
    segs = entry.segs
    if len(segments) != entry.args.num_segments:
        raise ValueError("patch_segments keeps the number of segments")
    for i, (st, slot, first, count, pos0) in enumerate(segments):
        sg = segs[i]
        if sg.store != st or sg.slot != slot:
            raise ValueError("patch_segments keeps each segment's store and slot")
        sg.first, sg.count, sg.pos0 = first, count, pos0
    entry.src = segments


def attention_call(qz: QuantizerBuffers, q: torch.Tensor, out: torch.Tensor, segments: Sequence[Tuple],
                   kv_heads: int, qpos: Optional[torch.Tensor] = None, causal: bool = True,
                   scale: Optional[float] = None, hot: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                   warm: Optional[CodeStoreBuffers] = None, cold: Optional[CodeStoreBuffers] = None,
                   num_ctas: int = 0, memo: bool = True, gather=None) -> "_AttnCall":
    """Validate the arguments and return the prepared call for them: memoised by its exact
    arguments, or (memo=False) a private one that the caller may patch_segments.  gather: a
    sharding.PeerGather, to fuse the output all-gather over peer memory into the launch."""
    _need_cuda(q, "q")
    if q.dtype != torch.float16 or q.dim() != 4 or not queries_packed(q):
        raise ValueError("q must be fp16 [B, Q, Hq, D], packed within a sequence (batch stride a multiple of 8)")
    if out.shape != q.shape or out.dtype != torch.float16 or not out.is_contiguous():
        raise ValueError("out must be contiguous fp16 like q")
    B, Qn, Hq, D = q.shape
    if len(segments) > _lib.RFSN_MAX_SEGMENTS:
        raise ValueError(f"at most {_lib.RFSN_MAX_SEGMENTS} segments per call")
    if causal and (qpos is None or qpos.dtype != torch.int32 or tuple(qpos.shape) != (B, Qn, Hq)
                   or not qpos.is_contiguous()):
        raise ValueError("causal attention needs contiguous int32 qpos [B, Q, Hq]")
    scale = float(D ** -0.5 if scale is None else scale)
    hot_key = None if hot is None else (_ptr(hot[0]), _ptr(hot[1]), hot[0].shape[1], hot[0].shape[0])
    key = (q.device.index, B, Qn, Hq, D, kv_heads, bool(causal), scale, num_ctas, tuple(map(tuple, segments)),
           hot_key, _store_key(warm), _store_key(cold), _qz_key(qz), q.stride(0) if B > 1 else 0,
           None if gather is None else id(gather))
    entry = _ATTN_CALLS.get(key) if memo else None
    if entry is None:
        a = AttnArgs()
        a.batch, a.queries, a.q_heads, a.kv_heads = B, Qn, Hq, kv_heads
        if hot is not None:
            a.hot = DenseStore(*hot_key)
        if warm is not None:
            a.warm = warm.struct()
        if cold is not None:
            a.cold = cold.struct()
        a.head_dim = D
        a.causal = int(bool(causal))
        a.scale = scale
        segs = (Segment * max(1, len(segments)))()
        for i, (st, slot, first, count, pos0) in enumerate(segments):
            segs[i].store, segs[i].slot, segs[i].first, segs[i].count, segs[i].pos0 = st, slot, first, count, pos0
        a.segments = segs
        a.num_segments = len(segments)
        a.num_ctas = num_ctas
        a.q_batch_stride = q.stride(0) if B > 1 else 0  # one sequence: no stride to follow
        if gather is not None:
            a.gather = gather.pointer
        qs = qz.struct()
        a.q, a.out, a.qpos = _ptr(q), _ptr(out), _ptr(qpos) if causal else None
        entry = _AttnCall(a, segs, qs, None)
        _size_workspace(entry, q.device)
        if memo:
            if len(_ATTN_CALLS) >= 256:
                _ATTN_CALLS.clear()
            _ATTN_CALLS[key] = entry
    return entry


def route_topk(q: torch.Tensor, centroids: torch.Tensor, kv_heads: int, k: int,
               scores: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Centroid routing (rfsn_route_topk): q fp16 [B, Q, Hq, D] (packed per sequence),
    centroids fp32 [C, B * kv_heads, D] -> (ids int32 [k] on the device, descending score,
    ties to the lower index; scores fp32 [C])."""
    _need_cuda(q, "q")
    _need_cuda(centroids, "centroids")
    if q.dtype != torch.float16 or q.dim() != 4 or not queries_packed(q):
        raise ValueError("q must be fp16 [B, Q, Hq, D], packed within a sequence")
    B, Qn, Hq, D = q.shape
    C = centroids.shape[0]
    if centroids.dtype != torch.float32 or not centroids.is_contiguous() or \
            tuple(centroids.shape[1:]) != (B * kv_heads, D):
        raise ValueError(f"centroids must be contiguous fp32 [C, {B * kv_heads}, {D}]")
    if not 0 <= k <= min(C, 64):
        raise ValueError("route_topk: 0 <= k <= min(num_chunks, 64)")
    if scores is None or scores.numel() < C:
        scores = torch.empty(max(C, 1), dtype=torch.float32, device=q.device)
    ids = torch.empty(max(k, 1), dtype=torch.int32, device=q.device)
    scratch = torch.empty(max(C, 1), dtype=torch.uint8, device=q.device)
    call("rfsn_route_topk", _ptr(q), q.stride(0) if B > 1 else 0, B, Qn, Hq, kv_heads, D, _ptr(centroids), C, k,
         _ptr(scores), _ptr(ids), _ptr(scratch), _stream(q.device.index))
    return ids[:k], scores[:C]


_LIN_WORKSPACE: dict = {}
LINEAR_NONE, LINEAR_RESIDUAL, LINEAR_GELU = 0, 1, 2


# Whether the decoder layers run their decode-sized projections on rfsn_linear_f16 (with the
# residual add and the GELU fused into its epilogue) instead of cuBLAS.  Off: at the config-3
# layer shapes (M = 32, 8-23 MB weights) the kernel measures 9.6-12.8 us per launch inside CUDA
# graphs against cuBLAS's 5.2-9.9 us, because the cross-CTA reduction of its split-K tiles
# costs about 5 us per launch; the 22-layer step is faster on cuBLAS (2.08 ms against 2.64 ms).
LAYER_LINEAR = False


def use_linear(x: torch.Tensor, w: torch.Tensor) -> bool:
    """True when a layer should call linear() for x @ w^T: LAYER_LINEAR and a supported shape."""
    return LAYER_LINEAR and linear_supported(x, w)


def linear_supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Shapes the weight-streaming kernel takes: fp16, M <= 32 rows, N % 64 == 0, K % 128 == 0."""
    M = x.numel() // x.shape[-1] if x.shape[-1] else 0
    return (x.is_cuda and x.dtype == torch.float16 and w.dtype == torch.float16 and w.dim() == 2
            and 0 < M <= 32 and w.shape[0] % 64 == 0 and w.shape[1] % 128 == 0 and x.shape[-1] == w.shape[1])


def linear(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None, gelu: bool = False,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ w^T (rfsn_linear_f16): fp16 x [..., K] with at most 32 rows, fp16 w [N, K];
    residual: y = fp16(fp16(acc) + residual); gelu: y = the layer's fp16 tanh-GELU of fp16(acc)."""
    _need_cuda(x, "x")
    K = x.shape[-1]
    N = w.shape[0]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    w = w if w.is_contiguous() else w.contiguous()
    y = out if out is not None else torch.empty((M, N), dtype=torch.float16, device=x.device)
    y2 = y.reshape(M, N)
    r2 = None
    if residual is not None:
        r2 = residual.reshape(M, N)
        if r2.stride(-1) != 1:
            r2 = r2.contiguous()
    nbytes = C.c_size_t(0)
    call("rfsn_linear_workspace_size", M, N, K, C.byref(nbytes))
    key = (x.device.index,)
    ws = _LIN_WORKSPACE.get(key)
    if ws is None or ws.numel() < nbytes.value:
        ws = torch.zeros(max(nbytes.value, 1 << 20), dtype=torch.uint8, device=x.device)
        _LIN_WORKSPACE[key] = ws
    mode = LINEAR_RESIDUAL if residual is not None else (LINEAR_GELU if gelu else LINEAR_NONE)
    call("rfsn_linear_f16", _ptr(x2), x2.stride(0), _ptr(w), w.stride(0), _ptr(r2), r2.stride(0) if r2 is not None else N,
         _ptr(y2), y2.stride(0), M, N, K, mode, _ptr(ws), ws.numel(), None, _stream(x.device.index))
    return y.reshape(*x.shape[:-1], N) if out is None else y


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """fp16 RMSNorm over the last dim in one launch (fp32 math, fp32 weight)."""
    _need_cuda(x, "x")
    if x.dtype != torch.float16 or weight.dtype != torch.float32 or weight.numel() != x.shape[-1]:
        raise ValueError("rms_norm expects fp16 x [..., dim] and an fp32 weight of dim")
    x = x.contiguous()
    w = weight.contiguous()
    y = torch.empty_like(x)
    dim = int(x.shape[-1])
    call("rfsn_rmsnorm_f16", _ptr(x), _ptr(w), _ptr(y), x.numel() // dim if dim else 0, dim, float(eps),
         _stream(x.device.index))
    return y


def add_rms_norm(x: torch.Tensor, b: torch.Tensor, weight: torch.Tensor,
                 eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """(x + b, rms_norm(x + b)) for fp16 x, b of the same shape, in one launch."""
    _need_cuda(x, "x")
    if x.dtype != torch.float16 or b.dtype != torch.float16 or b.shape != x.shape or weight.dtype != torch.float32 \
            or weight.numel() != x.shape[-1]:
        raise ValueError("add_rms_norm expects fp16 x and b of one shape [..., dim] and an fp32 weight of dim")
    x = x.contiguous()
    b = b.contiguous()
    w = weight.contiguous()
    s = torch.empty_like(x)
    y = torch.empty_like(x)
    dim = int(x.shape[-1])
    call("rfsn_add_rmsnorm_f16", _ptr(x), _ptr(b), _ptr(s), _ptr(w), _ptr(y), x.numel() // dim if dim else 0, dim,
         float(eps), _stream(x.device.index))
    return s, y


def llama_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
                   residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """The Llama adapter's RMSNorm (rfsn_llama_rmsnorm_f16): fp16 x [..., dim] and an fp16 weight.
    With ``residual``, normalises s = fp16(x + residual) and returns (y, s); else (y, None)."""
    _need_cuda(x, "x")
    if x.dtype != torch.float16 or weight.dtype != torch.float16 or weight.numel() != x.shape[-1]:
        raise ValueError("llama_rms_norm expects fp16 x [..., dim] and an fp16 weight of dim")
    x = x.contiguous()
    w = weight.contiguous()
    y = torch.empty_like(x)
    s = None
    if residual is not None:
        if residual.shape != x.shape or residual.dtype != torch.float16:
            raise ValueError("residual must be fp16 like x")
        residual = residual.contiguous()
        s = torch.empty_like(x)
    dim = int(x.shape[-1])
    call("rfsn_llama_rmsnorm_f16", _ptr(x), _ptr(residual), _ptr(s), _ptr(w), _ptr(y), x.numel() // dim, dim,
         float(eps), _stream(x.device.index))
    return y, s


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotary embedding of fp16 x [B, S, H, D] (any strides, D contiguous) with fp16 tables [S, D]
    (rfsn_rope_f16); out defaults to a new contiguous tensor (it may be x itself)."""
    _need_cuda(x, "x")
    B, S, H, D = x.shape
    if x.dtype != torch.float16 or x.stride(-1) != 1:
        raise ValueError("rope expects fp16 [B, S, H, D] with a contiguous last dim")
    cos = cos.to(device=x.device, dtype=torch.float16).reshape(S, D).contiguous()
    sin = sin.to(device=x.device, dtype=torch.float16).reshape(S, D).contiguous()
    y = torch.empty((B, S, H, D), dtype=torch.float16, device=x.device) if out is None else out
    if y.shape != x.shape or y.stride(-1) != 1 or y.dtype != torch.float16:
        raise ValueError("out must be fp16 like x with a contiguous last dim")
    call("rfsn_rope_f16", _ptr(x), x.stride(0), x.stride(1), x.stride(2), _ptr(y), y.stride(0), y.stride(1),
         y.stride(2), _ptr(cos), _ptr(sin), B, S, H, D, _stream(x.device.index))
    return y


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """fp16(fp16(g * sigmoid(g)) * up) in one launch (rfsn_silu_mul_f16)."""
    _need_cuda(gate, "gate")
    if gate.dtype != torch.float16 or up.dtype != torch.float16 or gate.shape != up.shape:
        raise ValueError("silu_mul expects fp16 gate and up of one shape")
    gate, up = gate.contiguous(), up.contiguous()
    y = torch.empty_like(gate)
    call("rfsn_silu_mul_f16", _ptr(gate), _ptr(up), _ptr(y), gate.numel(), _stream(gate.device.index))
    return y


def affine_quantize(w: torch.Tensor, bits: int, group: int):
    """Affine quantization of fp32 w [rows, cols] in groups along the last dim
    (rfsn_affine_quantize_f32) -> (q uint8 [rows, cols], scales, biases fp32 [rows, cols/group],
    dequantized fp32 [rows, cols])."""
    _need_cuda(w, "w")
    w = w.to(torch.float32).contiguous()
    rows, cols = w.shape
    q = torch.empty((rows, cols), dtype=torch.uint8, device=w.device)
    sc = torch.empty((rows, cols // group), dtype=torch.float32, device=w.device)
    bi = torch.empty_like(sc)
    deq = torch.empty_like(w)
    call("rfsn_affine_quantize_f32", _ptr(w), rows, cols, group, bits, _ptr(q), _ptr(sc), _ptr(bi), _ptr(deq),
         _stream(w.device.index))
    return q, sc, bi, deq


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """Tanh-approximate GELU of fp16 x in one launch, rounded to fp16 after every operation."""
    _need_cuda(x, "x")
    if x.dtype != torch.float16:
        raise ValueError("gelu_tanh expects fp16 input")
    x = x.contiguous()
    y = torch.empty_like(x)
    call("rfsn_gelu_tanh_f16", _ptr(x), _ptr(y), x.numel(), _stream(x.device.index))
    return y


def version() -> int:
    return lib().rfsn_version()
