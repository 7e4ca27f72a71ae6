"""Tiered KV cache on B200 (cache.py of the reference, cache.py:33-440).

``RFSNv10KVCacheMLX`` keeps the reference's API and tiering but stores every
tier in preallocated device / pinned-host buffers (no O(T) concatenation per
append, cache.py:106-107) and answers ``attention_forward`` with one fused
kernel over the codes (no dense window is materialised, cache.py:390-391).

Tier policies
  "prefix" (reference, cache.py:103-118): hot = first ``hot_capacity`` tokens,
     then ``warm_capacity`` warm tokens, then cold chunks of ``chunk_tokens``
     with chunk id = start // chunk_tokens and partial-chunk merges
     (cache.py:144-191).  Tokens never move between tiers.
  "recent" (extension): hot = the newest ``hot_capacity`` tokens in a ring;
     older tokens are encoded into a warm ring; when warm exceeds
     ``warm_capacity``, whole chunks of the oldest warm codes move to the cold
     tier (a device->pinned-host copy; no re-encoding).

Shapes follow the reference for ``batch_size == 1`` ([T, H, D] updates, q
[Q, H, D] with positions [Q] or [Q, H]); with ``batch_size = B > 1`` updates
are [B, T, H, D] and q is [B, Hq, D] (one query per sequence) or
[B, Q, Hq, D].  ``num_kv_heads < num_heads`` enables GQA (query head h reads
KV head h // (num_heads // num_kv_heads)).
"""
from __future__ import annotations

import logging
import math
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import kernels as K
from .quantization import HybridQuantizerMLX
from .storage import (AsyncHierarchicalRouterMLX, ColdTier, RFSNConfig, chunk_file_path, register_cold_tier,
                      unregister_cold_tier)

logger = logging.getLogger("RFSN_CACHE")

STAT_KEYS = ("window_start", "window_end", "window_tokens", "context_window", "query_tokens", "used_router",
             "hot_tokens_materialized", "warm_tokens_materialized", "cold_tokens_materialized",
             "reconstructed_tokens", "warm_chunk_decodes", "cold_chunk_decodes", "cold_chunks_touched",
             "cold_chunk_cache_hits", "cold_chunk_cache_misses")


def _ceil_to(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class RFSNv10KVCacheMLX:
    """Tiered KV cache with exact hot storage and compressed warm/cold storage."""

    def __init__(self, config: RFSNConfig, layer_idx: int = 0):
        self.config = config
        self.layer_idx = layer_idx
        self.hot_capacity = config.hot_capacity
        self.warm_capacity = config.warm_capacity
        self.batch = config.batch_size
        self.heads = config.kv_heads
        self.rows = self.batch * self.heads
        self.head_dim = config.head_dim
        self.device = torch.device(config.device)
        self.policy = config.hot_policy
        self.chunk_tokens = config.chunk_tokens

        self.num_hot = 0
        self.num_warm = 0
        self.num_cold = 0
        self.total_tokens = 0
        self.quantizer: Optional[HybridQuantizerMLX] = None
        self.cold_chunk_paths: List[Path] = []
        self.cold_chunk_paths_by_id: Dict[int, Path] = {}
        self.cold_chunk_metadata: List[dict] = []
        self.last_access_stats = self._empty_access_stats()

        self._qz: Optional[K.QuantizerBuffers] = None
        self._hot_k: Optional[torch.Tensor] = None  # [rows, cap, D]
        self._hot_v: Optional[torch.Tensor] = None
        self._hot_start = 0  # global position of the oldest hot token
        self._hot_ring = max(1, self.hot_capacity)
        self._warm: Optional[K.CodeStoreBuffers] = None  # K and V codes, rows x cap
        self._warm_start = 0  # global position of the oldest warm token
        self._warm_ring = 0
        self._cold: Optional[ColdTier] = None
        self._cold_root: Optional[Path] = None
        self._plan_cache: Dict[Tuple, Tuple[List, Dict[str, int], Tuple]] = {}
        self._q_stage: Dict[Tuple, torch.Tensor] = {}  # device staging buffers of host queries, by shape
        self._host_memo: Optional[Tuple] = None  # the last host call: its key and what it reuses
        # prepared attention calls for cached plans; _store_epoch changes whenever a store
        # buffer or the quantizer is replaced, which retires the calls that point at them
        self._attn_calls: Dict[Tuple, Any] = {}
        self._store_epoch = 0
        self.last_routed_chunks: List[int] = []  # centroid routing: the cold chunks the last call attended

    # ------------------------------------------------------------------ stats
    def _empty_access_stats(self) -> Dict[str, int]:
        """cache.py:59-76."""
        s = {k: 0 for k in STAT_KEYS}
        s["context_window"] = -1
        return s

    def get_last_access_stats(self) -> Dict[str, int]:
        return dict(self.last_access_stats)

    @property
    def current_tier(self) -> str:
        """cache.py:81-87."""
        if self.total_tokens < self.hot_capacity:
            return "hot"
        if self.total_tokens < self.hot_capacity + self.warm_capacity:
            return "warm"
        return "cold"

    # ------------------------------------------------------------ reference views
    @property
    def hot_keys(self) -> torch.Tensor:
        return self._hot_view(self._hot_k)

    @property
    def hot_values(self) -> torch.Tensor:
        return self._hot_view(self._hot_v)

    def _hot_view(self, buf) -> torch.Tensor:
        D = self.head_dim
        if buf is None or self.num_hot == 0:
            shape = (0, self.heads, D) if self.batch == 1 else (self.batch, 0, self.heads, D)
            return torch.zeros(shape, dtype=torch.float16, device=self.device)
        idx = self._hot_index(self._hot_pos0(), self.num_hot)
        x = buf[:, idx].reshape(self.batch, self.heads, self.num_hot, D).permute(0, 2, 1, 3)
        return x[0] if self.batch == 1 else x

    @property
    def warm_keys(self):
        return self._warm_view(0)

    @property
    def warm_values(self):
        return self._warm_view(1)

    def _warm_view(self, kv: int):
        """Warm codes of sequence 0 in position order as a CompressedTensorMLX [T, H, ...]."""
        from .storage import CompressedTensorMLX
        if self._warm is None or self.num_warm == 0:
            return CompressedTensorMLX.empty(self.config, self.heads)
        parts = [CompressedTensorMLX.from_store(self._warm, kv, 0, idx, cnt, self.heads)
                 for idx, cnt, _ in self._warm_runs(self._warm_pos0(), self.num_warm)]
        if len(parts) == 1:
            return parts[0]
        return CompressedTensorMLX(*(torch.cat([getattr(p, f) for p in parts], 0)
                                     for f in ("pq_codes", "rvq", "rvq_mask", "sp_idx", "sp_val")), self.heads)

    # ------------------------------------------------------------ layout helpers
    def _hot_pos0(self) -> int:
        return 0 if self.policy == "prefix" else self._hot_start

    def _warm_pos0(self) -> int:
        return self.num_hot if self.policy == "prefix" else self._warm_start

    def _hot_index(self, pos0: int, n: int) -> torch.Tensor:
        if self.policy == "prefix":
            return torch.arange(pos0, pos0 + n, device=self.device)
        return torch.arange(pos0, pos0 + n, device=self.device) % self._hot_ring

    def _warm_index(self, pos0: int, n: int) -> torch.Tensor:
        base = self._warm_pos0()
        if self.policy == "prefix":
            return torch.arange(pos0 - base, pos0 - base + n, device=self.device)
        return torch.arange(pos0, pos0 + n, device=self.device) % self._warm_ring

    def _ring_runs(self, pos0: int, n: int, ring: int, offset: int = 0) -> List[Tuple[int, int, int]]:
        """Split positions [pos0, pos0+n) into (storage_index, count, pos) runs of a ring."""
        runs = []
        p = pos0
        while n > 0:
            i = (p - offset) % ring if ring else p - offset
            c = min(n, ring - i) if ring else n
            runs.append((i, c, p))
            p += c
            n -= c
        return runs

    def _hot_runs(self, pos0: int, n: int):
        if self.policy == "prefix":
            return [(pos0, n, pos0)] if n > 0 else []
        return self._ring_runs(pos0, n, self._hot_ring)

    def _warm_runs(self, pos0: int, n: int):
        if self.policy == "prefix":
            return [(pos0 - self.num_hot, n, pos0)] if n > 0 else []
        return self._ring_runs(pos0, n, self._warm_ring)

    # ------------------------------------------------------------ allocation
    def _ensure_quantizer(self, quantizer: HybridQuantizerMLX) -> None:
        self.quantizer = quantizer
        qz = quantizer.buffers()
        if self._qz is not None and self._qz is not qz and self.total_tokens:
            if (qz.M, qz.K, qz.ds, qz.L, qz.Kr, qz.sparse_topk) != (self._qz.M, self._qz.K, self._qz.ds, self._qz.L,
                                                                     self._qz.Kr, self._qz.sparse_topk):
                raise ValueError("quantizer layout changed after tokens were cached")
        if qz is not self._qz:
            self._store_epoch += 1
        self._qz = qz

    def _ensure_hot(self, need: int) -> None:
        D = self.head_dim
        if self.policy == "recent":
            cap = K.align16(self._hot_ring)
        else:
            cap = K.align16(min(self.hot_capacity, max(need, 16)))
            if self._hot_k is not None and self._hot_k.shape[1] >= need:
                return
            if self._hot_k is not None:
                cap = K.align16(min(self.hot_capacity, max(need, 2 * self._hot_k.shape[1])))
        if self._hot_k is not None and self._hot_k.shape[1] >= cap:
            return
        new_k = torch.zeros((self.rows, cap, D), dtype=torch.float16, device=self.device)
        new_v = torch.zeros_like(new_k)
        if self._hot_k is not None:
            n = self._hot_k.shape[1]
            new_k[:, :n] = self._hot_k
            new_v[:, :n] = self._hot_v
        self._hot_k, self._hot_v = new_k, new_v
        self._store_epoch += 1

    def _ensure_warm(self, need: int) -> None:
        qz = self._qz
        if self.policy == "recent":
            if self._warm is None:
                self._warm_ring = _ceil_to(max(self.warm_capacity, 1), self.chunk_tokens) + self.chunk_tokens
                self._warm = K.CodeStoreBuffers(qz, self.rows, self._warm_ring, device=self.device)
                self._store_epoch += 1
            return
        if self._warm is not None and self._warm.cap >= need:
            return
        cap = min(K.align16(self.warm_capacity), K.align16(max(need, 64, 2 * (self._warm.cap if self._warm else 0))))
        cap = max(cap, K.align16(need))
        if self._warm is None:
            self._warm = K.CodeStoreBuffers(qz, self.rows, cap, device=self.device)
        else:
            self._warm = self._warm.grow(qz, cap)
        self._store_epoch += 1

    def _ensure_cold(self, disk_dir: Optional[Path]) -> ColdTier:
        root = Path(self.config.disk_cache_dir) if disk_dir is None else Path(disk_dir)
        if self._cold is None:
            # the reference's merges can make a prefix-policy chunk up to 2 * chunk_tokens - 1 long
            cap = 2 * self.chunk_tokens if self.policy == "prefix" else self.chunk_tokens
            self._cold = ColdTier(self._qz, self.rows, self.chunk_tokens, self.config.cold_pool_chunks, self.device,
                                  spill_dir=root, layer_idx=self.layer_idx, host_chunks=self.config.cold_host_chunks,
                                  capacity=cap)
            self._cold.track_centroids = self.config.cold_routing == "centroid"
            self._cold_root = root
            register_cold_tier(root, self.layer_idx, self._cold)
        return self._cold

    # ------------------------------------------------------------ update
    def _as_batched(self, x: torch.Tensor) -> torch.Tensor:
        if not isinstance(x, torch.Tensor):
            x = torch.as_tensor(np.asarray(x))
        x = x.to(device=self.device, dtype=torch.float16)
        if self.batch == 1 and x.dim() == 3:
            x = x.unsqueeze(0)
        if x.dim() != 4 or x.shape[0] != self.batch or x.shape[2] != self.heads or x.shape[3] != self.head_dim:
            raise ValueError(f"expected keys/values shaped [T, {self.heads}, {self.head_dim}] (batch 1) or "
                             f"[{self.batch}, T, {self.heads}, {self.head_dim}], got {tuple(x.shape)}")
        return x

    def update(self, new_keys, new_values, quantizer: HybridQuantizerMLX, disk_dir: Optional[Path] = None) -> None:
        """cache.py:89-120."""
        if tuple(new_keys.shape) != tuple(new_values.shape):
            raise ValueError("new_keys and new_values must have identical shapes")
        k = self._as_batched(new_keys)
        v = self._as_batched(new_values)
        self._ensure_quantizer(quantizer)
        n = k.shape[1]
        if n == 0:
            return
        if self.policy == "prefix":
            self._update_prefix(k, v, disk_dir)
        else:
            for a in range(0, n, self.chunk_tokens):
                b = min(n, a + self.chunk_tokens)
                self._update_recent(k[:, a:b], v[:, a:b], disk_dir)
        self.total_tokens += n

    def _write_hot(self, k, v, pos0: int) -> None:
        for idx, cnt, p in self._hot_runs(pos0, k.shape[1]):
            off = p - pos0
            self._hot_k[:, idx:idx + cnt] = k[:, off:off + cnt].permute(0, 2, 1, 3).reshape(self.rows, cnt, -1)
            self._hot_v[:, idx:idx + cnt] = v[:, off:off + cnt].permute(0, 2, 1, 3).reshape(self.rows, cnt, -1)

    def _encode_kv(self, k: torch.Tensor, v: torch.Tensor, store: K.CodeStoreBuffers, slot: int, first: int) -> None:
        """Spill encoder: K and V tokens [B, T, H, D] into tokens [first, first+T) of a store
        (one launch when their layouts match, as projections of one input give)."""
        if k.stride() == v.stride():
            K.encode_kv(self._qz, k, v, store, slot, first)
        else:
            K.encode(self._qz, k, store, slot, first, kv=0)
            K.encode(self._qz, v, store, slot, first, kv=1)

    def _update_prefix(self, k, v, disk_dir) -> None:
        n = k.shape[1]
        off = 0
        hot_space = max(self.hot_capacity - self.num_hot, 0)
        if hot_space > 0 and off < n:
            take = min(hot_space, n - off)
            self._ensure_hot(self.num_hot + take)
            self._write_hot(k[:, off:off + take], v[:, off:off + take], self.num_hot)
            self.num_hot += take
            off += take
        warm_space = max(self.warm_capacity - self.num_warm, 0)
        if warm_space > 0 and off < n:
            take = min(warm_space, n - off)
            self._ensure_warm(self.num_warm + take)
            self._encode_kv(k[:, off:off + take], v[:, off:off + take], self._warm, 0, self.num_warm)
            self.num_warm += take
            off += take
        if off < n:
            self._add_to_cold(k[:, off:], v[:, off:], disk_dir)

    def _record_chunk_meta(self, chunk_id: int, start: int, n: int) -> None:
        root = self._cold_root
        path = chunk_file_path(root, self.layer_idx, chunk_id)
        meta = next((m for m in self.cold_chunk_metadata if m["chunk_id"] == chunk_id), None)
        if meta is None:
            self.cold_chunk_paths.append(path)
            self.cold_chunk_paths_by_id[chunk_id] = path
            self.cold_chunk_metadata.append({"chunk_id": chunk_id, "start_token": start, "end_token": start + n,
                                             "num_tokens": n, "path": str(path)})
        else:
            meta["end_token"] += n
            meta["num_tokens"] += n

    def _add_to_cold(self, k, v, disk_dir) -> None:
        """cache.py:134-191: the appended tokens in pieces of chunk_tokens from the update's start;
        a piece's chunk id = its start // chunk_tokens, and a piece whose id exists is merged onto
        that chunk (which must end where the piece starts)."""
        tier = self._ensure_cold(disk_dir)
        ct = self.chunk_tokens
        start_token = self.num_hot + self.num_warm + self.num_cold
        stream = torch.cuda.current_stream()
        n = k.shape[1]
        off = 0
        while off < n:
            pos = start_token + off
            cid = pos // ct
            chunk = tier.chunks.get(cid)
            if chunk is not None and pos != chunk.end_token:
                raise ValueError("Cold chunk append must be contiguous with existing metadata: "
                                 f"chunk_id={cid} start={pos} expected={chunk.end_token}")
            take = min(n - off, ct)  # the reference's piece (cache.py:146-149)
            if chunk is None:
                chunk = tier.new_chunk(cid, pos)
                within = 0
            else:
                within = chunk.end_token - chunk.start_token
                if within + take > tier.capacity:
                    raise ValueError(f"cold chunk {cid} would hold {within + take} tokens (capacity {tier.capacity})")
                tier.load_stage(chunk, stream)  # keep the chunk's earlier tokens in the image
            self._encode_kv(k[:, off:off + take], v[:, off:off + take], tier.stage, 0, within)
            tier.store_stage(chunk, stream, num_tokens=within + take)
            chunk.end_token += take
            self._record_chunk_meta(cid, pos, take)
            off += take
        self.num_cold += n

    def _update_recent(self, k, v, disk_dir) -> None:
        n = k.shape[1]
        self._ensure_hot(self._hot_ring)
        cap_h = self.hot_capacity
        spill_hot = min(self.num_hot, max(0, self.num_hot + n - cap_h))
        spill_new = max(0, n - cap_h)
        if spill_hot or spill_new:
            self._ensure_warm(0)
        warm_end = self._warm_start + self.num_warm
        # oldest hot tokens -> warm (encoded straight from the hot ring)
        for idx, cnt, p in self._hot_runs(self._hot_start, spill_hot):
            self._spill_to_warm(self._as_bthd(self._hot_k[:, idx:idx + cnt]), self._as_bthd(self._hot_v[:, idx:idx + cnt]),
                                p)
        self._hot_start += spill_hot
        self.num_hot -= spill_hot
        if spill_new:
            self._spill_to_warm(k[:, :spill_new], v[:, :spill_new], warm_end + spill_hot)
            self._hot_start += spill_new
        keep_k, keep_v = k[:, spill_new:], v[:, spill_new:]
        if self.num_hot == 0 and spill_new == 0 and spill_hot == 0 and self.total_tokens == 0:
            self._hot_start = 0
        self._write_hot(keep_k, keep_v, self._hot_start + self.num_hot)
        self.num_hot += keep_k.shape[1]
        self.num_warm += spill_hot + spill_new
        self._evict_warm_chunks(disk_dir)

    def _as_bthd(self, rows_view: torch.Tensor) -> torch.Tensor:
        """[rows, cnt, D] slice of a ring -> strided [B, cnt, H, D] view."""
        B, H = self.batch, self.heads
        cnt, D = rows_view.shape[1], rows_view.shape[2]
        st = rows_view.stride()
        return rows_view.as_strided((B, cnt, H, D), (H * st[0], st[1], st[0], st[2]))

    def _spill_to_warm(self, k, v, pos0: int) -> None:
        for idx, cnt, p in self._warm_runs(pos0, k.shape[1]):
            off = p - pos0
            self._encode_kv(k[:, off:off + cnt], v[:, off:off + cnt], self._warm, 0, idx)

    def _evict_warm_chunks(self, disk_dir) -> None:
        ct = self.chunk_tokens
        if self.num_warm <= self.warm_capacity:
            return
        evict = _ceil_to(self.num_warm - self.warm_capacity, ct)
        tier = self._ensure_cold(disk_dir)
        stream = torch.cuda.current_stream()
        for off in range(0, evict, ct):
            pos = self._warm_start + off
            cid = pos // ct
            chunk = tier.new_chunk(cid, pos)
            b0 = (pos % self._warm_ring) // K.BLOCK_TOKENS  # chunk-aligned, so whole blocks
            nb = ct // K.BLOCK_TOKENS
            with torch.cuda.stream(stream):
                tier.stage.data[0].copy_(self._warm.data[0, :, b0:b0 + nb])
            tier.store_stage(chunk, stream, num_tokens=ct)
            chunk.end_token = pos + ct
            self._record_chunk_meta(cid, pos, ct)
        self._warm_start += evict
        self.num_warm -= evict
        self.num_cold += evict

    # ------------------------------------------------------------ windows
    def _max_query_position(self, query_positions, current_position) -> int:
        if query_positions is not None:
            return int(np.max(_host_ints(query_positions)))
        if current_position is not None:
            return int(current_position)
        return max(self.total_tokens - 1, 0)

    def _window_bounds(self, query_positions, context_window, current_position, adjusted: bool = True):
        """cache.py:210-241 -> (start, end, adjusted or None); adjusted=False skips the third."""
        if self.total_tokens == 0:
            return 0, 0, None if query_positions is None else _host_ints(query_positions).astype(np.int32)
        ints = _int_list(query_positions)
        max_query = max(ints) if ints else self._max_query_position(query_positions, current_position)
        end = min(max_query + 1, self.total_tokens)
        start = 0 if context_window is None else max(0, end - context_window)
        if query_positions is None or not adjusted:
            return start, end, None
        adjusted = np.maximum(_host_ints(query_positions) - start, -1).astype(np.int32)
        return start, end, adjusted

    def _spans(self):
        if self.policy == "prefix":
            return [("hot", 0, self.num_hot), ("warm", self.num_hot, self.num_hot + self.num_warm)]
        return [("warm", self._warm_start, self._warm_start + self.num_warm),
                ("hot", self._hot_start, self._hot_start + self.num_hot)]

    def _plan(self, start: int, end: int, router, current_position, context_window, stats,
              routed: Optional[Tuple[List[int], set]] = None) -> List[Tuple]:
        """Segments of the window [start, end) in position order + reference stats (cache.py:250-342).

        routed (centroid routing): (chosen cold chunk ids, ids resident before the choice);
        only the chosen cold chunks enter the window, and they count as router hits or misses."""
        segs: List[Tuple[int, Tuple]] = []
        bs = max(1, self.config.block_size_seq)
        for kind, s, e in self._spans():
            a, b = max(start, s), min(end, e)
            if a >= b:
                continue
            if kind == "hot":
                stats["hot_tokens_materialized"] += b - a
                for idx, cnt, p in self._hot_runs(a, b - a):
                    segs.append((p, (K.STORE_HOT, 0, idx, cnt, p)))
            else:
                stats["warm_tokens_materialized"] += b - a
                stats["reconstructed_tokens"] += b - a
                stats["warm_chunk_decodes"] += (b - a + bs - 1) // bs
                for idx, cnt, p in self._warm_runs(a, b - a):
                    segs.append((p, (K.STORE_WARM, 0, idx, cnt, p)))
        tier = self._cold
        if tier is not None and self.cold_chunk_metadata and routed is not None:
            chosen, hits = routed
            keep = set(chosen)
            stream = torch.cuda.current_stream()
            for meta in self.cold_chunk_metadata:
                a, b = max(start, meta["start_token"]), min(end, meta["end_token"])
                cid = meta["chunk_id"]
                if a >= b or cid not in keep:
                    continue
                stats["cold_chunk_cache_hits" if cid in hits else "cold_chunk_cache_misses"] += 1
                stats["cold_tokens_materialized"] += b - a
                stats["reconstructed_tokens"] += b - a
                stats["cold_chunk_decodes"] += 1
                stats["cold_chunks_touched"] += 1
                slot = tier.ensure_resident(cid, stream, keep)
                tier.wait_ready(slot, stream)
                segs.append((a, (K.STORE_COLD, slot, a - meta["start_token"], b - a, a)))
        elif tier is not None and self.cold_chunk_metadata:
            if router is not None and current_position is not None and context_window is not None:
                ct = self.chunk_tokens
                router.prefetch_sync(current_position=current_position, context_window=context_window,
                                     top_k=max(1, (context_window + ct - 1) // ct))
            needed = []
            for meta in self.cold_chunk_metadata:
                a, b = max(start, meta["start_token"]), min(end, meta["end_token"])
                if a >= b:
                    continue
                cid = meta["chunk_id"]
                if router is not None:
                    if router.get_chunk(cid) is not None:
                        stats["cold_chunk_cache_hits"] += 1
                    else:
                        stats["cold_chunk_cache_misses"] += 1
                needed.append((cid, a, b, meta["start_token"]))
                stats["cold_tokens_materialized"] += b - a
                stats["reconstructed_tokens"] += b - a
                stats["cold_chunk_decodes"] += 1
                stats["cold_chunks_touched"] += 1
            keep = {c for c, *_ in needed}
            stream = torch.cuda.current_stream()
            for cid, a, b, cstart in needed:
                slot = tier.ensure_resident(cid, stream, keep)
                tier.wait_ready(slot, stream)
                segs.append((a, (K.STORE_COLD, slot, a - cstart, b - a, a)))
        segs.sort(key=lambda x: x[0])
        return [s for _, s in segs]

    def _begin_stats(self, start, end, context_window, router) -> Dict[str, int]:
        stats = self._empty_access_stats()
        stats["window_start"], stats["window_end"] = start, end
        stats["window_tokens"] = max(0, end - start)
        stats["context_window"] = -1 if context_window is None else context_window
        stats["used_router"] = int(router is not None)
        return stats

    def materialize_window(self, query_positions=None, context_window: Optional[int] = None,
                           router: Optional[AsyncHierarchicalRouterMLX] = None,
                           current_position: Optional[int] = None):
        """cache.py:344-393 -> (keys fp16, values fp16, adjusted positions int32 | None).

        keys/values are [W, H, D] for batch_size 1, else [B, W, H, D]; warm and
        cold tokens are decoded bit-exactly as the reference decodes them."""
        if self.quantizer is None:
            raise RuntimeError("Cache cannot materialize values before update() provides a quantizer")
        start, end, adjusted = self._window_bounds(query_positions, context_window, current_position)
        stats = self._begin_stats(start, end, context_window, router)
        segs = self._plan(start, end, router, current_position, context_window, stats)
        W = max(0, end - start)
        B, H, D = self.batch, self.heads, self.head_dim
        keys = torch.empty((B, W, H, D), dtype=torch.float16, device=self.device)
        values = torch.empty_like(keys)
        for store, slot, first, count, pos in segs:
            w0 = pos - start
            if store == K.STORE_HOT:
                for buf, out in ((self._hot_k, keys), (self._hot_v, values)):
                    out[:, w0:w0 + count] = buf[:, first:first + count].reshape(B, H, count, D).permute(0, 2, 1, 3)
            else:
                st = self._warm if store == K.STORE_WARM else self._cold.pool
                K.decode_codes(self._qz, st, slot, first, count, keys[:, w0:w0 + count], kv=0)
                K.decode_codes(self._qz, st, slot, first, count, values[:, w0:w0 + count], kv=1)
        self.last_access_stats = dict(stats)
        if B == 1:
            keys, values = keys[0], values[0]
        return keys, values, (None if adjusted is None else torch.as_tensor(adjusted, device=self.device))

    def _queries(self, q: torch.Tensor) -> Tuple[torch.Tensor, bool]:
        # a pinned host query is uploaded asynchronously on the current stream (ordered
        # before the attention kernel); keep it unchanged until the call's result is read
        uploaded = not q.is_cuda
        if uploaded or q.dtype != torch.float16 or self.device.index is None or q.get_device() != self.device.index:
            q = q.to(device=self.device, dtype=torch.float16, non_blocking=bool(uploaded and q.is_pinned()))
        # a view whose sequences are each packed (e.g. the query heads of a wider projection
        # output) is read in place through the kernel's batch stride; a contiguous upload is a
        # fresh allocation, packed and aligned by construction
        check = not (uploaded and q.is_contiguous())
        if self.batch == 1 and q.dim() == 3:
            qb, squeeze = q.unsqueeze(0), True                # [1, Q, Hq, D]
        elif q.dim() == 3 and q.shape[0] == self.batch:
            qb, squeeze = q.unsqueeze(1), False               # [B, 1, Hq, D]
        elif q.dim() == 4 and q.shape[0] == self.batch:
            qb, squeeze = q, False
        else:
            raise ValueError(f"q must be [Q, H, D] (batch 1), [B, H, D] or [B, Q, H, D]; got {tuple(q.shape)}")
        if check and not K.queries_packed(qb):
            qb = qb.contiguous()
        return qb, squeeze

    def _staged_queries(self, q: torch.Tensor) -> Tuple[torch.Tensor, bool]:
        """The device staging buffer a host query is copied into, shaped as _queries shapes an
        upload ([1, Q, Hq, D], [B, 1, Hq, D] or [B, Q, Hq, D]); its contents are written by the
        library call that uses it, on the stream, after every earlier call's kernels."""
        if self.batch == 1 and q.dim() == 3:
            shape, squeeze = (1,) + tuple(q.shape), True
        elif q.dim() == 3 and q.shape[0] == self.batch:
            shape, squeeze = (q.shape[0], 1) + tuple(q.shape[1:]), False
        elif q.dim() == 4 and q.shape[0] == self.batch:
            shape, squeeze = tuple(q.shape), False
        else:
            raise ValueError(f"q must be [Q, H, D] (batch 1), [B, H, D] or [B, Q, H, D]; got {tuple(q.shape)}")
        stage = self._q_stage.get(shape)
        if stage is None:
            stage = torch.empty(shape, dtype=torch.float16, device=self.device)
            self._q_stage[shape] = stage
        return stage, squeeze

    def _qpos(self, query_positions, start, end, qb: torch.Tensor) -> Optional[torch.Tensor]:
        """Per-query last visible positions [B, Q, Hq] int32, or None when every query sits at
        the window's last position end - 1: then causal masking hides no key of the window
        [start, end), and the kernel runs unmasked with no position tensor."""
        B, Qn, Hq, _ = qb.shape
        if query_positions is None:
            return None
        ints = _int_list(query_positions)
        if ints and len(ints) == (Qn if self.batch == 1 else B) and min(ints) >= end - 1:
            return None  # one position per query or sequence, each at the window's end
        pos = _host_ints(query_positions)
        pos = np.maximum(pos - start, -1) + start
        if self.batch == 1:
            if pos.ndim == 1:
                if pos.shape[0] != Qn:
                    raise ValueError("query_positions length must equal batch size")
                pos = np.broadcast_to(pos[:, None], (Qn, Hq))
            elif pos.shape != (Qn, Hq):
                raise ValueError("query_positions must have shape [B] or [B, H]")
            pos = pos[None]
        else:
            if pos.ndim == 1:
                pos = np.broadcast_to(pos[:, None, None], (B, Qn, Hq))
            elif pos.ndim == 2:
                pos = np.broadcast_to(pos[:, None, :], (B, Qn, Hq))
            elif pos.shape != (B, Qn, Hq):
                raise ValueError("query_positions must be [B], [B, H] or [B, Q, H]")
        if pos.size and bool((pos >= end - 1).all()):
            return None  # the decode case: every query sees the whole window
        return torch.as_tensor(np.ascontiguousarray(pos, dtype=np.int32)).to(self.device, non_blocking=True)

    def attention_forward(self, q: torch.Tensor, pq_codebook=None, rvq_codebook=None, causal: bool = True,
                          query_positions=None, router: Optional[AsyncHierarchicalRouterMLX] = None,
                          current_position: Optional[int] = None, context_window: Optional[int] = None,
                          out: Optional[torch.Tensor] = None, gather=None) -> torch.Tensor:
        """cache.py:395-428 — fused decode attention over hot/warm/cold without a dense window.

        gather (extension, multi-GPU): a sharding.PeerGather whose ranks each hold an equal batch
        shard; the kernel then also all-gathers the outputs over peer memory and the call returns
        the whole batch's output (gather.full, [total, Q, Hq, D], as [total, Hq, D] for one query).

        out (extension): a contiguous fp16 tensor with q's element count to write the result to.
        A pinned host tensor is written by the kernel itself over the bus (no separate copy), and
        the call then waits for the stream, so the host holds the result when it returns."""
        del pq_codebook, rvq_codebook  # ignored by the reference too (cache.py:406)
        if self.quantizer is None:
            raise RuntimeError("Cache cannot run attention before update() provides a quantizer")
        # pinned host query and pinned host output: one library call uploads the query into a
        # device staging buffer, runs the attention, whose kernel stores the result straight into
        # the host buffer, and waits for the stream (rfsn_decode_attention_host)
        host_call = (out is not None and gather is None and not q.is_cuda and not out.is_cuda
                     and q.dtype == torch.float16 and q.is_contiguous() and q.is_pinned() and out.is_pinned())
        # a decode loop that calls again from the same host buffers against an unchanged cache
        # (the same window, tiers and stores) reuses the last host call's plan, prepared
        # arguments, staging buffer, positions and statistics
        memo_key = None
        if host_call and router is None and not self.cold_chunk_metadata:
            qp = None if query_positions is None else _int_list(query_positions)
            if query_positions is None or qp is not None:
                memo_key = (q.data_ptr(), tuple(q.shape), out.data_ptr(), tuple(out.shape), bool(causal),
                            None if qp is None else tuple(qp), context_window, current_position, self.total_tokens,
                            self.num_hot, self.num_warm, self._hot_start, self._warm_start, self._store_epoch)
                memo = self._host_memo
                if memo is not None and memo[0] == memo_key:
                    _, entry, stage, qpos, stats, ret = memo
                    self.last_access_stats = dict(stats)
                    K.run_attention_host(entry, q, stage, out, qpos, synchronize=True)
                    return ret
        qb, squeeze = self._staged_queries(q) if host_call else self._queries(q)
        start, end, _ = self._window_bounds(query_positions, context_window, current_position, adjusted=False)
        # without a cold tier or router the plan depends only on the window and the tier
        # layout, so a decode loop that reads the same window reuses it
        key = None
        if router is None and not self.cold_chunk_metadata:
            key = (start, end, context_window, self.total_tokens, self.num_hot, self.num_warm, self._hot_start,
                   self._warm_start)
        cached = self._plan_cache.get(key) if key is not None else None
        routed = None
        if self.config.cold_routing == "centroid" and router is not None and self._cold is not None:
            eligible = [m["chunk_id"] for m in self.cold_chunk_metadata
                        if m["start_token"] < end and m["end_token"] > start]
            routed = router.route_centroids(qb, self.heads, self.config.cold_route_top_k, eligible)
            self.last_routed_chunks = list(routed[0])
        if cached is not None:
            segs, stats, shape = cached[0], dict(cached[1]), cached[2]
        else:
            stats = self._begin_stats(start, end, context_window, router)
            segs = self._plan(start, end, router, current_position, context_window, stats, routed)
            shape = tuple((sg[0], sg[1]) for sg in segs)  # the stores and slots, in order
            if key is not None:
                if len(self._plan_cache) > 32:
                    self._plan_cache.clear()
                self._plan_cache[key] = (segs, dict(stats), shape)
        stats["query_tokens"] = int(qb.shape[1])  # queries per sequence (q.shape[0] for one sequence)
        self.last_access_stats = stats
        host_out = out is not None and not out.is_cuda
        if host_out and not out.is_pinned():
            raise ValueError("a host out must be pinned memory: the kernel writes it over the bus")
        if out is None:
            out = torch.empty(qb.shape, dtype=torch.float16, device=qb.device)
        elif out.shape != qb.shape:
            if out.numel() != qb.numel() or not out.is_contiguous():
                raise ValueError(f"out must be contiguous with {qb.numel()} elements; got {tuple(out.shape)}")
            out = out.view(qb.shape)
        qpos = self._qpos(query_positions, start, end, qb) if causal else None
        # without a cold tier or router, a prepared call is reused across steps: its key is
        # the segments' stores and slots plus the shapes and buffers, and each step patches
        # the token ranges (a decode loop's window grows or slides by one token per step)
        ck = entry = None
        if key is not None:
            ck = (shape, qb.shape, qb.stride(0), qpos is not None,
                  self._store_epoch, self._cold is not None, None if gather is None else id(gather))
            entry = self._attn_calls.get(ck)
            if entry is not None:
                K.patch_segments(entry, segs)
        if entry is None:
            entry = K.attention_call(self._qz, qb, out, segs, kv_heads=self.heads, qpos=qpos,
                                     causal=qpos is not None, scale=self.head_dim ** -0.5,
                                     hot=(self._hot_k, self._hot_v) if self._hot_k is not None else None,
                                     warm=self._warm, cold=self._cold.pool if self._cold is not None else None,
                                     memo=ck is None, gather=gather)
            if ck is not None:
                if len(self._attn_calls) > 32:
                    self._attn_calls.clear()
                self._attn_calls[ck] = entry
        if host_call:
            K.run_attention_host(entry, q, qb, out, qpos, synchronize=True)
        else:
            K.run_attention(entry, qb, out, qpos)
            if host_out:  # the kernel's stores to host memory are complete and visible
                torch.cuda.current_stream(qb.device).synchronize()
        if gather is not None:
            full = gather.full
            return full[:, 0] if (q.dim() == 3 and not squeeze) else full
        ret = out[0] if squeeze else (out.reshape(q.shape) if q.dim() == 3 else out)
        if memo_key is not None and ck is not None:
            self._host_memo = (memo_key, entry, qb, qpos, dict(stats), ret)
        return ret

    def memory_usage_bytes(self) -> Dict[str, int]:
        """cache.py:430-440 (same formulas: hot K+V fp16, PQ 2 bytes per code, RVQ 2 bytes per code)."""
        c = self.config
        hot_bytes = self.num_hot * self.rows * c.head_dim * 2 * 2
        warm_pq_bytes = self.num_warm * self.rows * c.num_subspaces * 2
        active = 0
        if self._warm is not None and self._qz.L and self.num_warm:
            for kv in (0, 1):
                for idx, cnt, _ in self._warm_runs(self._warm_pos0(), self.num_warm):
                    act = self._warm.read_rows(kv, "active", 0, idx, cnt)
                    active += int(act.sum().item()) if self._qz.threshold >= 0 else act.numel()
        return {"hot_bytes": hot_bytes, "warm_pq_bytes": warm_pq_bytes,
                "warm_rvq_bytes": active * c.num_rvq_layers * 2,
                "cold_chunks": len(self.cold_chunk_paths), "cold_tokens": self.num_cold}

    def load_cold_chunk(self, chunk_id: int) -> Dict[str, np.ndarray]:
        """cache.py:193-194: the chunk's codes by id, as the arrays of its chunk file
        (storage.py:117-135, apple_b200/chunk_io.py); KeyError for unknown ids."""
        from .chunk_io import _arrays, load_compressed_chunk
        from .storage import CompressedTensorMLX
        if self._cold is None or chunk_id not in self._cold.chunks:
            raise KeyError(chunk_id)
        c = self._cold.chunks[chunk_id]
        if c.store is None:
            return load_compressed_chunk(c.spill_path)
        if c.ready is not None:
            c.ready.synchronize()
        n = c.num_tokens
        keys = CompressedTensorMLX.from_store(c.store, 0, 0, 0, n, self.rows)
        values = CompressedTensorMLX.from_store(c.store, 1, 0, 0, n, self.rows)
        return {"num_tokens": np.array([n], np.int32), "num_heads": np.array([self.rows], np.int32),
                **_arrays(keys, "key"), **_arrays(values, "value")}

    def close(self) -> None:
        if self._cold_root is not None:
            unregister_cold_tier(self._cold_root, self.layer_idx)


def _int_list(values):
    """values itself when it is a flat list or tuple of Python ints, else None."""
    if type(values) in (list, tuple) and set(map(type, values)) <= {int}:
        return values
    return None


def _host_ints(values) -> np.ndarray:
    if isinstance(values, torch.Tensor):
        values = values.detach().cpu().numpy()
    return np.asarray(values, dtype=np.int64)
