"""Helpers shared by the GPU tests: move oracle (numpy) codes into device code stores."""
from __future__ import annotations

import numpy as np
import torch

from apple_b200 import kernels as K


def codes_to_store(qz: K.QuantizerBuffers, codes_per_row, cap: int, store: K.CodeStoreBuffers = None,
                   slot: int = 0, first: int = 0, kv: int = 0, slots: int = 1):
    """Write oracle ``Codes`` (one per row, arrays [T, ...]) into the K (kv=0) or V (kv=1)
    fields of a packed code store, tokens [first, first+T) of each row."""
    rows = len(codes_per_row)
    if store is None:
        store = K.CodeStoreBuffers(qz, rows, cap, slots=slots)
    for r, c in enumerate(codes_per_row):
        T = c.pq.shape[0]
        store.write(kv, "pq", slot, r, first, torch.from_numpy(np.ascontiguousarray(c.pq.reshape(T, -1))))
        if qz.L:
            rv = torch.from_numpy(c.rvq.reshape(T, -1).astype(np.int64))
            store.write(kv, "rvq", slot, r, first, rv)
            store.write(kv, "active", slot, r, first, torch.from_numpy(c.mask.reshape(T, 1).astype(np.uint8)))
        if qz.sparse_topk:
            store.write(kv, "sp_idx", slot, r, first, torch.from_numpy(np.ascontiguousarray(c.sp_idx.reshape(T, -1))))
            store.write(kv, "sp_val", slot, r, first, torch.from_numpy(np.ascontiguousarray(c.sp_val.reshape(T, -1))))
    return store


def kv_to_store(qz, kcodes, vcodes, cap, store=None, slot=0, first=0, slots=1):
    store = codes_to_store(qz, kcodes, cap, store=store, slot=slot, first=first, kv=0, slots=slots)
    return codes_to_store(qz, vcodes, cap, store=store, slot=slot, first=first, kv=1)


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)
