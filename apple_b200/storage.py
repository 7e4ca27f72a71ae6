"""Config, compressed-tensor container, pinned-host cold tier and the async router.

Mirrors storage.py of the reference (RFSNConfig storage.py:19-59,
CompressedTensorMLX :75-98, chunk IO :113-151, AsyncHierarchicalRouterMLX
:154-237).  The cold tier moves from zlib NPZ files on disk to pinned host
memory: each chunk is a pinned code store (same codes the reference writes to
``layer{L}_chunk{id}.npz``), copied into a device-resident chunk pool with
``rfsn_cold_prefetch`` (cudaMemcpyAsync) — by the router on its side stream
ahead of time, or by the cache on the compute stream on a miss.  A chunk is
one packed code-store image (K and V fields of every row, 16-token blocks), so
moving it either way is a single contiguous copy.
"""
from __future__ import annotations

import asyncio
import logging
import threading
from collections import OrderedDict
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import kernels as K

logger = logging.getLogger("RFSN_STORAGE")

SUPPORTED_GROUP_SIZES = (128, 64, 32)
MASK_FILL_VALUE = -1e30


@dataclass
class RFSNConfig:
    """Hyperparameters (storage.py:19-59) plus the B200 build's extensions.

    Extensions (all default to the reference behaviour):
      num_kv_heads      KV heads (GQA); None = num_heads.
      batch_size        independent sequences per cache (reference: 1).
      hot_policy        "prefix" (reference: hot = first tokens) or "recent"
                        (hot = newest tokens; older tokens spill hot->warm->cold).
      sparse_topk       top-S |error| fp16 residual entries per token (0 = off).
      cold_chunk_tokens cold chunk length (None = block_size_seq, as cache.py:144).
      cold_pool_chunks  device-resident cold chunk slots (LRU).
      cold_routing      "exact" (reference: attention reads every cold chunk the window
                        overlaps, cache.py:293-342) or "centroid": with a router, attention
                        reads only the cold_route_top_k chunks whose mean key scores highest
                        against the step's queries (rfsn_route_topk).
      cold_route_top_k  chunks a centroid-routed step attends (at most 64).
      cold_host_chunks  chunk images kept in pinned host memory (None = all); beyond it the
                        least recently used chunks spill to layer{L}_chunk{id}.npz files in
                        the reference's format under disk_cache_dir and come back on use.
      device            CUDA device of the cache and quantizer.
    """

    hidden_dim: int = 4096
    num_heads: int = 32
    head_dim: int = 128
    num_layers: int = 32

    num_subspaces: int = 8
    pq_bits: int = 8
    subspace_dim: int = 16
    pq_codebook_dtype: str = "float16"

    num_rvq_layers: int = 4
    rvq_codebook_size: int = 4096
    rvq_sparsity_threshold: float = 0.005
    max_rvq_sparse: int = 64

    hot_capacity: int = 8192
    warm_capacity: int = 65536
    cold_capacity: int = 2_000_000

    block_size_seq: int = 128

    ane_quant_bits: int = 6
    ane_group_size: int = 128

    disk_cache_dir: str = "./rfsn_disk_cache"
    max_open_files: int = 8
    prefetch_throttle_s: float = 0.5

    cpu_threads: int = 4

    num_kv_heads: Optional[int] = None
    batch_size: int = 1
    hot_policy: str = "prefix"
    sparse_topk: int = 0
    cold_chunk_tokens: Optional[int] = None
    cold_pool_chunks: int = 32
    cold_routing: str = "exact"
    cold_route_top_k: int = 8
    cold_host_chunks: Optional[int] = None
    device: str = "cuda"

    def __post_init__(self) -> None:
        expected = self.num_subspaces * self.subspace_dim
        if expected != self.head_dim:
            raise ValueError(
                "head_dim must equal num_subspaces * subspace_dim: "
                f"{self.head_dim} != {expected}"
            )
        if self.hot_policy not in ("prefix", "recent"):
            raise ValueError("hot_policy must be 'prefix' or 'recent'")
        if self.cold_routing not in ("exact", "centroid"):
            raise ValueError("cold_routing must be 'exact' or 'centroid'")
        if not 1 <= self.cold_route_top_k <= 64:
            raise ValueError("cold_route_top_k must be in [1, 64]")
        if self.cold_host_chunks is not None and self.cold_host_chunks < 1:
            raise ValueError("cold_host_chunks must be at least 1 (or None: every chunk stays in host memory)")
        if self.num_kv_heads is not None and self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        if self.hot_policy == "recent" and self.chunk_tokens % 16:
            raise ValueError("hot_policy 'recent' moves whole 16-token blocks to the cold tier: "
                             "cold_chunk_tokens (or block_size_seq) must be a multiple of 16")

    @property
    def kv_heads(self) -> int:
        return self.num_kv_heads or self.num_heads

    @property
    def chunk_tokens(self) -> int:
        return max(1, self.cold_chunk_tokens or self.block_size_seq)


@dataclass
class QuantizedMatrix:
    """Affine-quantised 2-D tensor (storage.py:62-72).  weights holds one code per byte (uint8,
    the B200 build's layout; MLX packs them into uint32 words); scales and biases are fp32 per
    group; dequantized caches q * scale + bias (fp32, in the original orientation)."""
    weights: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    bits: int
    group_size: int
    transposed: bool
    original_shape: Tuple[int, ...]
    dequantized: Optional[torch.Tensor] = None


class CompressedTensorMLX:
    """Compressed [T, H, D] tensor (storage.py:75-98) in the device layout.

    Fields: pq_codes uint8 [T, H, M]; rvq uint8/int16 [T, H, L] for every token
    (zero when inactive); rvq_mask bool [T, H]; sp_idx uint8 [T, H, S];
    sp_val fp16 [T, H, S].  ``rvq_codes`` / ``rvq_offsets`` give the
    reference's sparse (codes [A, L], flat offsets t*H+h [A]) form.
    """

    def __init__(self, pq_codes, rvq, rvq_mask, sp_idx, sp_val, num_heads: int):
        self.pq_codes = pq_codes
        self.rvq = rvq
        self.rvq_mask = rvq_mask
        self.sp_idx = sp_idx
        self.sp_val = sp_val
        self.num_heads = num_heads

    @property
    def num_tokens(self) -> int:
        return int(self.pq_codes.shape[0])

    @property
    def rvq_offsets(self) -> torch.Tensor:
        return torch.nonzero(self.rvq_mask.reshape(-1), as_tuple=False).reshape(-1).to(torch.int32)

    @property
    def rvq_codes(self) -> torch.Tensor:
        L = self.rvq.shape[-1]
        flat = self.rvq.reshape(-1, L)
        return flat[self.rvq_mask.reshape(-1)].to(torch.int32) & 0xFFFF

    @classmethod
    def empty(cls, config: RFSNConfig, num_heads: Optional[int] = None) -> "CompressedTensorMLX":
        heads = config.num_heads if num_heads is None else num_heads
        dev = torch.device(config.device)
        code_dtype = torch.uint8 if config.rvq_codebook_size <= 256 else torch.int16
        return cls(torch.zeros((0, heads, config.num_subspaces), dtype=torch.uint8, device=dev),
                   torch.zeros((0, heads, config.num_rvq_layers), dtype=code_dtype, device=dev),
                   torch.zeros((0, heads), dtype=torch.bool, device=dev),
                   torch.zeros((0, heads, config.sparse_topk), dtype=torch.uint8, device=dev),
                   torch.zeros((0, heads, config.sparse_topk), dtype=torch.float16, device=dev), heads)

    def to_store(self, qz: K.QuantizerBuffers, kv: int = 0,
                 store: Optional[K.CodeStoreBuffers] = None) -> K.CodeStoreBuffers:
        """Write into the K (kv=0) or V (kv=1) fields of a one-slot code store with
        rows = heads (allocated when ``store`` is None)."""
        T, H = self.num_tokens, self.num_heads
        st = store if store is not None else K.CodeStoreBuffers(qz, rows=H, cap=max(T, 16),
                                                                device=self.pq_codes.device)
        if T:
            st.write_rows(kv, "pq", 0, 0, self.pq_codes.transpose(0, 1))
            if qz.L:
                st.write_rows(kv, "rvq", 0, 0, self.rvq.transpose(0, 1))
                st.write_rows(kv, "active", 0, 0, self.rvq_mask.transpose(0, 1).to(torch.uint8).unsqueeze(-1))
            if qz.sparse_topk:
                st.write_rows(kv, "sp_idx", 0, 0, self.sp_idx.transpose(0, 1))
                st.write_rows(kv, "sp_val", 0, 0, self.sp_val.transpose(0, 1))
        return st

    @classmethod
    def from_store(cls, st: K.CodeStoreBuffers, kv: int, slot: int, first: int, count: int, rows: int,
                   device: Optional[torch.device] = None) -> "CompressedTensorMLX":
        """Tokens [first, first+count) of rows [0, rows) of a store as a [T, H, ...] tensor."""
        qz = st.qz
        dev = device if device is not None else st.data.device

        def grab(name, empty_w, dtype):
            v = st.read_rows(kv, name, slot, first, count, rows)
            if v is None:
                return torch.zeros((count, rows, empty_w), dtype=dtype, device=dev)
            return v.transpose(0, 1).contiguous().to(dev)

        pq = grab("pq", 0, torch.uint8)
        rvq = grab("rvq", 0, qz.rvq_code_dtype)
        act = st.read_rows(kv, "active", slot, first, count, rows)
        mask = (act[..., 0].transpose(0, 1).bool().contiguous().to(dev) if act is not None
                else torch.zeros((count, rows), dtype=torch.bool, device=dev))
        if qz.L and qz.threshold < 0:
            mask = torch.ones_like(mask)
        return cls(pq, rvq, mask, grab("sp_idx", 0, torch.uint8), grab("sp_val", 0, torch.float16), rows)


def _concat0(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    """storage.py:101-106."""
    if lhs.shape[0] == 0:
        return rhs
    if rhs.shape[0] == 0:
        return lhs
    return torch.cat([lhs, rhs], dim=0)


def _numpy_ints(values) -> np.ndarray:
    """storage.py:109-110."""
    if isinstance(values, torch.Tensor):
        values = values.detach().cpu().numpy()
    return np.asarray(values, dtype=np.int64)


def chunk_file_path(root: Path, layer_idx: int, chunk_id: int) -> Path:
    """storage.py:113-114 — name of a cold chunk (also its key in the pinned tier)."""
    return Path(root) / f"layer{layer_idx}_chunk{chunk_id}.npz"


# ---------------------------------------------------------------------------
# Pinned-host cold tier
# ---------------------------------------------------------------------------

@dataclass
class ColdChunk:
    chunk_id: int
    start_token: int
    end_token: int
    store: Optional[K.CodeStoreBuffers]  # pinned host, one slot: K and V codes of every row (None: spilled)
    ready: Optional[torch.cuda.Event] = None  # device-to-host writes into `store` done
    version: int = 0
    spill_path: Optional[Path] = None  # set while the chunk lives only in its NPZ file

    @property
    def num_tokens(self) -> int:
        return self.end_token - self.start_token


class ColdTier:
    """Cold chunks in pinned host memory plus a device-resident LRU chunk pool.

    ``chunks`` maps chunk id -> ColdChunk (codes for every row of the cache).
    ``pool`` is a device code store with ``slots`` chunk slots; a chunk is
    resident when ``slot_of[chunk_id]`` exists and its version matches.
    Chunk images move with one cudaMemcpyAsync each way through the C ABI
    (rfsn_cold_prefetch / rfsn_cold_evict).
    """

    def __init__(self, qz: K.QuantizerBuffers, rows: int, chunk_tokens: int, slots: int, device,
                 spill_dir: Optional[Path] = None, layer_idx: int = 0, host_chunks: Optional[int] = None,
                 capacity: Optional[int] = None):
        self.qz = qz
        # tokens one chunk image holds: chunk_tokens, or more where the reference's merges of a
        # partial chunk with a whole piece make longer chunks (cache.py:144-176)
        self.capacity = K.align16(max(chunk_tokens, capacity or chunk_tokens))
        self.spill_dir = None if spill_dir is None else Path(spill_dir)
        self.layer_idx = layer_idx
        self.host_chunks = host_chunks
        self.host_lru: "OrderedDict[int, None]" = OrderedDict()  # chunks with a pinned image, LRU first
        self.spills = 0
        self.unspills = 0
        self.rows = rows
        self.chunk_tokens = chunk_tokens
        self.device = torch.device(device)
        self.chunks: "OrderedDict[int, ColdChunk]" = OrderedDict()
        self.slots = max(1, slots)
        self.pool = K.CodeStoreBuffers(qz, rows, self.capacity, self.slots, device=self.device)
        self.stage = K.CodeStoreBuffers(qz, rows, self.capacity, 1, device=self.device)
        self.slot_of: "OrderedDict[int, int]" = OrderedDict()  # chunk id -> slot (LRU order)
        self.slot_version: Dict[int, int] = {}
        self.slot_ready: Dict[int, torch.cuda.Event] = {}
        self.pinned_by_router: set = set()
        self.lock = threading.Lock()
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        # centroid routing: mean decoded key of every chunk per row, fp32 [capacity, rows, D]
        self.track_centroids = False
        self.centroids: Optional[torch.Tensor] = None
        self.centroid_ids: List[int] = []          # table index -> chunk id
        self.centroid_index: Dict[int, int] = {}   # chunk id -> table index

    @property
    def image_bytes(self) -> int:
        return self.stage.nbytes_per_slot()

    # -- host side -------------------------------------------------------
    def _pinned_store(self) -> K.CodeStoreBuffers:
        return K.CodeStoreBuffers(self.qz, self.rows, self.capacity, 1, pin_memory=True)

    def new_chunk(self, chunk_id: int, start: int) -> ColdChunk:
        c = ColdChunk(chunk_id, start, start, self._pinned_store())
        self.chunks[chunk_id] = c
        self.host_lru[chunk_id] = None
        return c

    # -- NPZ spill below the pinned tier ----------------------------------
    def _spill_one(self, keep: set) -> bool:
        """Write the least recently used pinned image (not in keep) to its NPZ file and free it."""
        from .chunk_io import store_to_npz
        for cid in self.host_lru:
            if cid in keep:
                continue
            c = self.chunks[cid]
            if c.ready is not None:
                c.ready.synchronize()  # the image's device-to-host copy is complete
            path = chunk_file_path(self.spill_dir, self.layer_idx, cid)
            store_to_npz(c.store, c.num_tokens, path)
            c.store = None
            c.spill_path = path
            del self.host_lru[cid]
            self.spills += 1
            return True
        return False

    def enforce_host_limit(self, keep: set = frozenset()) -> None:
        if self.host_chunks is None or self.spill_dir is None:
            return
        while len(self.host_lru) > self.host_chunks and self._spill_one(set(keep)):
            pass

    def host_image(self, chunk: ColdChunk, keep: set = frozenset()) -> K.CodeStoreBuffers:
        """The chunk's pinned image, read back from its NPZ file if it was spilled."""
        if chunk.store is None:
            from .chunk_io import npz_to_store
            st = self._pinned_store()
            n = npz_to_store(chunk.spill_path, st)
            if n != chunk.num_tokens:
                raise ValueError(f"{chunk.spill_path}: {n} tokens, the chunk has {chunk.num_tokens}")
            chunk.store = st
            chunk.spill_path = None
            chunk.ready = None
            self.unspills += 1
            self.host_lru[chunk.chunk_id] = None
            self.enforce_host_limit(set(keep) | {chunk.chunk_id})
        else:
            self.host_lru.move_to_end(chunk.chunk_id)
        return chunk.store

    def load_stage(self, chunk: ColdChunk, stream: torch.cuda.Stream) -> K.CodeStoreBuffers:
        """Bring a chunk's current image into the device stage (for a partial-chunk append)."""
        self.host_image(chunk)
        if chunk.ready is not None:
            stream.wait_event(chunk.ready)
        K.call("rfsn_cold_prefetch", self.stage.data.data_ptr(), chunk.store.data.data_ptr(), self.image_bytes,
               stream.cuda_stream, None)
        self.h2d_bytes += self.image_bytes
        return self.stage

    def store_stage(self, chunk: ColdChunk, stream: torch.cuda.Stream, num_tokens: Optional[int] = None) -> None:
        """Write the device stage back as the chunk's image (device -> pinned host); with
        centroid routing, also record the mean decoded key of its ``num_tokens`` tokens."""
        if self.track_centroids and num_tokens:
            self.set_centroid(chunk.chunk_id, num_tokens, stream)
        K.call("rfsn_cold_evict", chunk.store.data.data_ptr(), self.stage.data.data_ptr(), self.image_bytes,
               stream.cuda_stream)
        self.d2h_bytes += self.image_bytes
        ev = torch.cuda.Event()
        ev.record(stream)
        chunk.ready = ev
        chunk.version += 1
        self.invalidate(chunk.chunk_id)
        self.host_lru.move_to_end(chunk.chunk_id)
        self.enforce_host_limit({chunk.chunk_id})

    def set_centroid(self, chunk_id: int, num_tokens: int, stream: torch.cuda.Stream) -> None:
        """Mean of the stage's decoded keys over its first num_tokens tokens, per row, in fp32."""
        D = self.qz.D
        with torch.cuda.stream(stream):
            keys = torch.empty((1, num_tokens, self.rows, D), dtype=torch.float16, device=self.device)
            K.decode_codes(self.qz, self.stage, 0, 0, num_tokens, keys, kv=0)
            idx = self.centroid_index.get(chunk_id)
            if idx is None:
                idx = len(self.centroid_ids)
                if self.centroids is None or idx >= self.centroids.shape[0]:
                    grown = torch.zeros((max(64, 2 * idx), self.rows, D), dtype=torch.float32, device=self.device)
                    if self.centroids is not None:
                        grown[:idx].copy_(self.centroids[:idx])
                    self.centroids = grown
                self.centroid_ids.append(chunk_id)
                self.centroid_index[chunk_id] = idx
            self.centroids[idx].copy_(keys[0].float().mean(dim=0))

    def invalidate(self, chunk_id: int) -> None:
        slot = self.slot_of.pop(chunk_id, None)
        if slot is not None:
            self.slot_version.pop(slot, None)
            self.slot_ready.pop(slot, None)
        self.pinned_by_router.discard(chunk_id)

    # -- device pool ------------------------------------------------------
    def _grow(self, need: int) -> None:
        new_slots = max(need, self.slots * 2)
        new = K.CodeStoreBuffers(self.qz, self.rows, self.capacity, new_slots, device=self.device)
        new.data[: self.slots].copy_(self.pool.data)
        self.pool = new
        self.slots = new_slots

    def _free_slot(self, keep: set) -> int:
        used = set(self.slot_of.values())
        for s in range(self.slots):
            if s not in used:
                return s
        for cid, s in self.slot_of.items():  # LRU order
            if cid not in keep and cid not in self.pinned_by_router:
                self.invalidate(cid)
                return s
        for cid, s in self.slot_of.items():
            if cid not in keep:
                self.invalidate(cid)
                return s
        self._grow(self.slots + 1)
        return self._free_slot(keep)

    def resident(self, chunk_id: int) -> bool:
        c = self.chunks.get(chunk_id)
        s = self.slot_of.get(chunk_id)
        return c is not None and s is not None and self.slot_version.get(s) == c.version

    def ensure_resident(self, chunk_id: int, stream: torch.cuda.Stream, keep: set = frozenset()) -> int:
        """Make chunk resident (one H2D copy on `stream` if needed); return its slot."""
        with self.lock:
            if self.resident(chunk_id):
                self.slot_of.move_to_end(chunk_id)
                return self.slot_of[chunk_id]
            chunk = self.chunks[chunk_id]
            self.host_image(chunk, set(keep) | {chunk_id})
            slot = self._free_slot(set(keep) | {chunk_id})
            if chunk.ready is not None:
                stream.wait_event(chunk.ready)
            K.call("rfsn_cold_prefetch", self.pool.data[slot].data_ptr(), chunk.store.data.data_ptr(),
                   self.image_bytes, stream.cuda_stream, None)
            self.h2d_bytes += self.image_bytes
            ev = torch.cuda.Event()
            ev.record(stream)
            self.slot_of[chunk_id] = slot
            self.slot_version[slot] = chunk.version
            self.slot_ready[slot] = ev
            return slot

    def wait_ready(self, slot: int, stream: torch.cuda.Stream) -> None:
        """Order `stream` after the copy into `slot`.  The compute stream is the only reader of
        pool slots, so once it has waited the event is dropped: later work on the stream
        is already ordered after the copy."""
        ev = self.slot_ready.pop(slot, None)
        if ev is not None:
            stream.wait_event(ev)


_COLD_REGISTRY: Dict[Tuple[str, int], ColdTier] = {}


def register_cold_tier(root: Path, layer_idx: int, tier: ColdTier) -> None:
    _COLD_REGISTRY[cold_tier_key(root, layer_idx)] = tier


def cold_tier_key(root: Path, layer_idx: int) -> Tuple[str, int]:
    return str(Path(root).resolve()), int(layer_idx)


def lookup_cold_tier(root: Path, layer_idx: int) -> Optional[ColdTier]:
    return _COLD_REGISTRY.get(cold_tier_key(root, layer_idx))


def unregister_cold_tier(root: Path, layer_idx: int) -> None:
    _COLD_REGISTRY.pop(cold_tier_key(root, layer_idx), None)


class AsyncHierarchicalRouterMLX:
    """Cold-chunk prefetcher (storage.py:154-237) for the pinned-host tier.

    Candidate selection is the reference's (storage.py:166-182): chunk ids in
    [(p - w) // cs, (p + w) // cs] that exist, nearest first by |id*cs - p|,
    the first ``top_k`` loaded.  "Loading" copies the chunk's codes into the
    device pool with cudaMemcpyAsync on the router's own CUDA stream (the
    reference reads an NPZ file in an executor thread); the cache's attention
    waits on the copy's event before reading the slot.  The router keeps at
    most 16 chunks (FIFO, storage.py:186-188), which the pool does not evict.
    """

    def __init__(self, config: RFSNConfig, layer_idx: int = 0):
        self.config = config
        self.layer_idx = layer_idx
        self.disk_dir = Path(config.disk_cache_dir)
        # resolved once: a per-lookup Path.resolve() costs filesystem calls on every candidate
        self._tier_key = cold_tier_key(self.disk_dir, layer_idx)
        self.throttle = config.prefetch_throttle_s
        self._cache: "OrderedDict[int, Dict[str, object]]" = OrderedDict()
        self._max_cache_size = 16
        self._pending_prefetch: set = set()
        self._stream: Optional[torch.cuda.Stream] = None

    def _tier(self) -> Optional[ColdTier]:
        return _COLD_REGISTRY.get(self._tier_key)

    @property
    def stream(self) -> torch.cuda.Stream:
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=torch.device(self.config.device))
        return self._stream

    def candidates(self, current_position: int, context_window: int, top_k: int) -> List[int]:
        tier = self._tier()
        if tier is None:
            return []
        cs = max(self.config.chunk_tokens, 1)
        start_chunk = max(0, (current_position - context_window) // cs)
        end_chunk = max(start_chunk, (current_position + context_window) // cs)
        cands = [c for c in range(start_chunk, end_chunk + 1) if c in tier.chunks]
        cands.sort(key=lambda cid: abs(cid * cs - current_position))
        return cands[:top_k]

    async def predict_and_prefetch(self, current_position: int, context_window: int, top_k: int = 2) -> List[int]:
        loaded: List[int] = []
        tier = self._tier()
        for chunk_id in self.candidates(current_position, context_window, top_k):
            entry = self._cache.get(chunk_id)
            if entry is not None and tier is not None and tier.resident(chunk_id):
                loaded.append(chunk_id)
                continue
            if chunk_id in self._pending_prefetch:
                continue
            self._pending_prefetch.add(chunk_id)
            await self._load_chunk(chunk_id)
            self._pending_prefetch.discard(chunk_id)
            loaded.append(chunk_id)
            if self.throttle > 0:
                await asyncio.sleep(self.throttle)
        while len(self._cache) > self._max_cache_size:
            old, _ = self._cache.popitem(last=False)
            if tier is not None:
                tier.pinned_by_router.discard(old)
        return loaded

    def prefetch_sync(self, current_position: int, context_window: int, top_k: int = 2) -> List[int]:
        coro = self.predict_and_prefetch(current_position, context_window, top_k)
        if self.throttle <= 0:
            # With no throttle sleep the coroutine has no suspension point (chunk copies are
            # queued on the router's CUDA stream, not awaited), so one send() runs it to the end
            # without building an event loop per decode step.
            try:
                coro.send(None)
            except StopIteration as done:
                return done.value
            coro.close()
            raise RuntimeError("router prefetch suspended with throttle disabled")
        try:
            return asyncio.run(coro)
        except RuntimeError:
            coro.close()
            loop = asyncio.new_event_loop()
            try:
                return loop.run_until_complete(self.predict_and_prefetch(current_position, context_window, top_k))
            finally:
                loop.close()

    async def _load_chunk(self, chunk_id: int) -> None:
        self._cache[chunk_id] = self._load_chunk_sync(chunk_id)

    def _load_chunk_sync(self, chunk_id: int) -> Dict[str, object]:
        tier = self._tier()
        if tier is None or chunk_id not in tier.chunks:
            return {}
        slot = tier.ensure_resident(chunk_id, self.stream)
        tier.pinned_by_router.add(chunk_id)
        c = tier.chunks[chunk_id]
        return {"chunk_id": chunk_id, "slot": slot, "num_tokens": c.num_tokens, "start_token": c.start_token}

    def route_centroids(self, q: torch.Tensor, kv_heads: int, top_k: int, eligible: List[int]) -> Tuple[List[int], set]:
        """Centroid routing (extension): the top_k of the ``eligible`` cold chunk ids by the
        score of rfsn_route_topk for queries q fp16 [B, Q, Hq, D], prefetched into the device
        pool on the router's side stream (the reference's router orders by distance from the
        position instead, storage.py:166-182).  Returns (chunk ids in score order, ids that
        were already resident before this call)."""
        tier = self._tier()
        if tier is None or tier.centroids is None or not eligible:
            return [], set()
        idx = [tier.centroid_index[c] for c in eligible]
        n = len(tier.centroid_ids)
        if idx == list(range(n)):
            cent = tier.centroids[:n]
        else:
            cent = tier.centroids.index_select(0, torch.as_tensor(idx, device=tier.centroids.device))
        k = min(top_k, len(idx))
        # the scores read q on the compute stream; the chunk copies go on the router's stream
        ids_dev, _ = K.route_topk(q, cent, kv_heads, k)
        chosen = [eligible[i] for i in ids_dev.tolist()]
        hits = {c for c in chosen if tier.resident(c)}
        for cid in chosen:
            if cid not in hits or cid not in self._cache:
                self._cache[cid] = self._load_chunk_sync(cid)
            self._cache.move_to_end(cid)
        while len(self._cache) > max(self._max_cache_size, top_k):
            old, _ = self._cache.popitem(last=False)
            tier.pinned_by_router.discard(old)
        return chosen, hits

    def get_chunk(self, chunk_id: int) -> Optional[Dict[str, object]]:
        entry = self._cache.get(chunk_id)
        if entry is None:
            return None
        tier = self._tier()
        if tier is None or not tier.resident(chunk_id):
            return None
        return entry
