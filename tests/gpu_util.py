"""Helpers shared by the GPU tests: move oracle (numpy) codes into device code stores."""
from __future__ import annotations

import numpy as np
import torch

from apple_b200 import kernels as K


def codes_to_store(qz: K.QuantizerBuffers, codes_per_row, cap: int, store: K.CodeStoreBuffers = None,
                   slot: int = 0, first: int = 0):
    """codes_per_row: list (one per row) of oracle ``Codes`` with [T, 1, ...] or [T, ...] arrays."""
    rows = len(codes_per_row)
    if store is None:
        store = K.CodeStoreBuffers(qz, rows, cap)
    dev = store.pq.device
    for r, c in enumerate(codes_per_row):
        T = c.pq.shape[0]
        sl = slice(first, first + T)
        store.pq[slot, r, sl] = torch.from_numpy(c.pq.reshape(T, -1)).to(dev)
        if store.rvq is not None:
            rv = c.rvq.reshape(T, -1).astype(np.int64)
            store.rvq[slot, r, sl] = torch.from_numpy(rv).to(dev).to(store.rvq.dtype)
            store.mask[slot, r, sl] = torch.from_numpy(c.mask.reshape(T).astype(np.uint8)).to(dev)
        if store.sp_idx is not None:
            store.sp_idx[slot, r, sl] = torch.from_numpy(c.sp_idx.reshape(T, -1)).to(dev)
            store.sp_val[slot, r, sl] = torch.from_numpy(c.sp_val.reshape(T, -1)).to(dev)
    return store


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)
