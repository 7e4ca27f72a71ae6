"""Cold chunks as NPZ files: the reference's on-disk chunk format (storage.py:113-151).

The B200 cold tier keeps chunk images in pinned host memory.  Below it, a
chunk can be spilled to ``layer{L}_chunk{id}.npz`` in the reference's format,
so the cold tier can outgrow host memory and chunk files move between the two
implementations:

  num_tokens            int32 [1]
  num_heads             int32 [1]
  {key,value}_pq_codes  uint8 [T, H, M]
  {key,value}_rvq_codes uint16 [A, L]   codes of the active (t, h) pairs only
  {key,value}_rvq_mask  bool [T, H]
  {key,value}_rvq_offsets int32 [A]     flat offsets t * H + h of the active pairs

(save_compressed_chunk, storage.py:117-135; the reference's loader,
storage.py:138-151, reads these ten arrays).  The B200 build's extensions add
arrays the reference's loader never reads: ``{key,value}_sp_idx`` uint8 [T, H, S]
and ``{key,value}_sp_val`` float16 [T, H, S] for the top-S sparse residual.  A
cache with batch B and KV heads Hkv writes its B * Hkv rows as H = B * Hkv
heads (row b * Hkv + h), which is the reference's layout when B = 1.
"""
from __future__ import annotations

from pathlib import Path
from typing import Dict, Optional

import numpy as np
import torch

from . import kernels as K
from .storage import CompressedTensorMLX

ARRAYS = ("pq_codes", "rvq_codes", "rvq_mask", "rvq_offsets")


def _arrays(t: CompressedTensorMLX, prefix: str) -> Dict[str, np.ndarray]:
    mask = t.rvq_mask.detach().cpu().numpy().astype(bool)
    L = t.rvq.shape[-1]
    dense = t.rvq.detach().cpu().numpy().reshape(-1, L).astype(np.int64) & 0xFFFF
    flat = mask.reshape(-1)
    out = {f"{prefix}_pq_codes": t.pq_codes.detach().cpu().numpy().astype(np.uint8),
           f"{prefix}_rvq_codes": dense[flat].astype(np.uint16),
           f"{prefix}_rvq_mask": mask,
           f"{prefix}_rvq_offsets": np.flatnonzero(flat).astype(np.int32)}
    if t.sp_idx.shape[-1]:
        out[f"{prefix}_sp_idx"] = t.sp_idx.detach().cpu().numpy().astype(np.uint8)
        out[f"{prefix}_sp_val"] = t.sp_val.detach().cpu().numpy().astype(np.float16)
    return out


def save_compressed_chunk(chunk_path: Path, keys: CompressedTensorMLX, values: CompressedTensorMLX) -> None:
    """storage.py:117-135: zlib NPZ of the chunk's codes (plus the sparse extension arrays)."""
    chunk_path = Path(chunk_path)
    chunk_path.parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(chunk_path, num_tokens=np.array([keys.num_tokens], dtype=np.int32),
                        num_heads=np.array([keys.num_heads], dtype=np.int32), **_arrays(keys, "key"),
                        **_arrays(values, "value"))


def load_compressed_chunk(chunk_path: Path) -> Dict[str, np.ndarray]:
    """storage.py:138-140: every array of the file."""
    with np.load(Path(chunk_path)) as data:
        return {k: data[k] for k in data.files}


def compressed_tensor_from_loaded(loaded: Dict[str, np.ndarray], prefix: str, num_rvq_layers: Optional[int] = None,
                                  sparse_topk: int = 0, rvq_code_dtype=torch.uint8) -> CompressedTensorMLX:
    """storage.py:143-151 into the device layout (host tensors): dense per-token RVQ codes,
    zero where inactive; the sparse arrays when the file has them (else an error when the
    cache needs them)."""
    H = int(np.asarray(loaded["num_heads"]).reshape(-1)[0])
    pq = np.asarray(loaded[f"{prefix}_pq_codes"])
    T = pq.shape[0]
    pq = pq.reshape(T, H, -1)
    codes = np.asarray(loaded[f"{prefix}_rvq_codes"])
    L = codes.shape[1] if codes.ndim == 2 else 0
    if num_rvq_layers is not None and L != num_rvq_layers and codes.shape[0]:
        raise ValueError(f"chunk has {L} RVQ layers, the quantizer {num_rvq_layers}")
    L = num_rvq_layers if num_rvq_layers is not None else L
    mask = np.asarray(loaded[f"{prefix}_rvq_mask"]).astype(bool).reshape(T, H)
    dense = np.zeros((T * H, L), np.int64)
    if codes.shape[0]:
        dense[np.asarray(loaded[f"{prefix}_rvq_offsets"]).astype(np.int64)] = codes.astype(np.int64)
    rvq = torch.from_numpy(dense.reshape(T, H, L))
    rvq = rvq.to(torch.uint8) if rvq_code_dtype == torch.uint8 else rvq.to(torch.int16)
    if sparse_topk:
        if f"{prefix}_sp_idx" not in loaded:
            raise ValueError(f"chunk file has no sparse residual; the cache keeps top-{sparse_topk}")
        spi = torch.from_numpy(np.asarray(loaded[f"{prefix}_sp_idx"]).astype(np.uint8).reshape(T, H, -1))
        spv = torch.from_numpy(np.asarray(loaded[f"{prefix}_sp_val"]).astype(np.float16).reshape(T, H, -1))
    else:
        spi = torch.zeros((T, H, 0), dtype=torch.uint8)
        spv = torch.zeros((T, H, 0), dtype=torch.float16)
    return CompressedTensorMLX(torch.from_numpy(np.ascontiguousarray(pq)), rvq, torch.from_numpy(mask), spi, spv, H)


def store_to_npz(store: K.CodeStoreBuffers, num_tokens: int, chunk_path: Path) -> None:
    """Write the first num_tokens tokens of a one-slot (host) code store as a chunk file."""
    keys = CompressedTensorMLX.from_store(store, 0, 0, 0, num_tokens, store.rows)
    values = CompressedTensorMLX.from_store(store, 1, 0, 0, num_tokens, store.rows)
    save_compressed_chunk(chunk_path, keys, values)


def npz_to_store(chunk_path: Path, store: K.CodeStoreBuffers) -> int:
    """Read a chunk file into a one-slot (host) code store; returns its token count."""
    loaded = load_compressed_chunk(chunk_path)
    qz = store.qz
    n = int(np.asarray(loaded["num_tokens"]).reshape(-1)[0])
    if int(np.asarray(loaded["num_heads"]).reshape(-1)[0]) != store.rows or n > store.cap:
        raise ValueError(f"{chunk_path}: chunk of {n} tokens x {int(loaded['num_heads'][0])} heads does not fit a "
                         f"store of {store.cap} tokens x {store.rows} rows")
    store.data.zero_()
    for kv, prefix in ((0, "key"), (1, "value")):
        t = compressed_tensor_from_loaded(loaded, prefix, qz.L, qz.sparse_topk, qz.rvq_code_dtype)
        if qz.L and qz.threshold < 0:
            t.rvq_mask = torch.ones_like(t.rvq_mask)
        t.to_store(qz, kv, store)
    return n
