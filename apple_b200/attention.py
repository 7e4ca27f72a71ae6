"""Attention entry points of the reference (attention.py:16-170) on B200.

* ``_blockwise_exact_attention`` (attention.py:39-105) and
  ``RFSNHybridAttentionMLX`` (attention.py:141-170) run the fused decode
  kernel (librfsn_b200.so): dense K/V become a hot (exact fp16) segment,
  compressed stores become code segments decoded inside the kernel.  The
  softmax is fp32 with online rescaling like the reference; ``block_size`` only
  changed the reference's summation blocking and is accepted for API parity.
* ``_dense_exact_attention`` (attention.py:108-134) is the prefill path of the
  decoder layer (use_cache=False); it is a plain fp32 softmax over [B, S, H, D]
  written with torch tensor ops on the GPU.
"""
from __future__ import annotations

import logging
from typing import Optional, Sequence

import numpy as np
import torch

from . import kernels as K
from .quantization import HybridQuantizerMLX, _decode_compressed_tensor
from .storage import MASK_FILL_VALUE, CompressedTensorMLX, RFSNConfig

logger = logging.getLogger("RFSN_ATTENTION")


def _normalize_query_positions(query_positions, batch_size: int, num_heads: int, default_position: int
                               ) -> torch.Tensor:
    """attention.py:16-36 -> int32 [B, H] (host-validated, returned on the CPU)."""
    if query_positions is None:
        return torch.full((batch_size, num_heads), default_position, dtype=torch.int32)
    pos = query_positions.detach().cpu() if isinstance(query_positions, torch.Tensor) else \
        torch.as_tensor(np.asarray(query_positions))
    pos = pos.to(torch.int32)
    if pos.dim() == 1:
        if pos.shape[0] != batch_size:
            raise ValueError("query_positions length must equal batch size")
        return pos.reshape(batch_size, 1).expand(batch_size, num_heads).contiguous()
    if tuple(pos.shape) == (batch_size, num_heads):
        return pos.contiguous()
    raise ValueError("query_positions must have shape [B] or [B, H]")


def _blockwise_exact_attention(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, scale: float,
                               block_size: int, causal: bool = False, query_positions=None,
                               quantizer: Optional[HybridQuantizerMLX] = None) -> torch.Tensor:
    """attention.py:39-105 over dense fp16 K/V [W, Hkv, D]; q [Q, Hq, D] (Q queries, one sequence)."""
    del block_size
    nq, hq, d = q.shape
    w = int(keys.shape[0])
    dev = q.device if q.is_cuda else torch.device("cuda")
    if w == 0:
        return torch.zeros((nq, hq, d), dtype=q.dtype, device=dev)
    hkv = int(keys.shape[1])
    cap = K.align16(w)
    kr = torch.zeros((hkv, cap, d), dtype=torch.float16, device=dev)
    vr = torch.zeros_like(kr)
    kr[:, :w] = keys.to(device=dev, dtype=torch.float16).transpose(0, 1)
    vr[:, :w] = values.to(device=dev, dtype=torch.float16).transpose(0, 1)
    qb = q.to(device=dev, dtype=torch.float16).reshape(1, nq, hq, d).contiguous()
    out = torch.empty_like(qb)
    qpos = None
    if causal:
        pos = _normalize_query_positions(query_positions, nq, hq, w - 1)
        qpos = torch.clamp(pos, min=-1).reshape(1, nq, hq).to(dev)
    qz = _dense_only_quantizer(d, dev)
    K.decode_attention(qz, qb, out, [(K.STORE_HOT, 0, 0, w, 0)], kv_heads=hkv, qpos=qpos, causal=causal,
                       scale=scale, hot=(kr, vr))
    return out[0].to(q.dtype)


_DENSE_QZ = {}


def _dense_only_quantizer(d: int, dev: torch.device) -> K.QuantizerBuffers:
    key = (d, dev.index)
    if key not in _DENSE_QZ:
        _DENSE_QZ[key] = K.QuantizerBuffers(torch.zeros((d // 8, 1, 8), dtype=torch.float16, device=dev), None, 0.0)
    return _DENSE_QZ[key]


def _dense_exact_attention(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, scale: float,
                           causal: bool = True) -> torch.Tensor:
    """attention.py:108-134 — [B, S, H, D] prefill attention in fp32 (GQA-aware)."""
    qf, kf, vf = q.float(), keys.float(), values.float()
    hq, hkv = q.shape[2], keys.shape[2]
    if hq != hkv:
        kf = kf.repeat_interleave(hq // hkv, dim=2)
        vf = vf.repeat_interleave(hq // hkv, dim=2)
    scores = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale
    if causal:
        qp = torch.arange(q.shape[1], device=q.device)
        kp = torch.arange(keys.shape[1], device=q.device)
        mask = kp[None, :] <= qp[:, None]
        scores = torch.where(mask[None, None], scores, torch.full_like(scores, MASK_FILL_VALUE))
    probs = torch.softmax(scores, dim=-1)
    ctx = torch.einsum("bhqk,bkhd->bqhd", probs, vf)
    return ctx.to(q.dtype)


def _gelu(x: torch.Tensor) -> torch.Tensor:
    """attention.py:137-138 — tanh approximation."""
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608 * (x + 0.044715 * (x ** 3))))


class RFSNHybridAttentionMLX:
    """Attention over compressed key/value stores (attention.py:141-170), fused: the
    stores are decoded inside the kernel instead of being materialised first."""

    def __init__(self, config: RFSNConfig):
        self.config = config
        self.scale = config.head_dim ** -0.5
        self.block_size = config.block_size_seq

    def __call__(self, q: torch.Tensor, key_store: CompressedTensorMLX, value_store: CompressedTensorMLX,
                 quantizer: HybridQuantizerMLX, causal: bool = False, query_positions=None) -> torch.Tensor:
        if key_store.num_tokens != value_store.num_tokens:
            raise ValueError("Key/value stores must have the same token count")
        T, H = key_store.num_tokens, key_store.num_heads
        nq, hq, d = q.shape
        qz = quantizer.buffers()
        dev = qz.pq_codebooks.device
        if T == 0:
            return torch.zeros((nq, hq, d), dtype=q.dtype, device=dev)
        st = key_store.to_store(qz, kv=0)
        value_store.to_store(qz, kv=1, store=st)
        qb = q.to(device=dev, dtype=torch.float16).reshape(1, nq, hq, d).contiguous()
        out = torch.empty_like(qb)
        qpos = None
        if causal:
            qpos = torch.clamp(_normalize_query_positions(query_positions, nq, hq, T - 1), min=-1)
            qpos = qpos.reshape(1, nq, hq).to(dev)
        K.decode_attention(qz, qb, out, [(K.STORE_WARM, 0, 0, T, 0)], kv_heads=H, qpos=qpos, causal=causal,
                           scale=self.scale, warm=st)
        return out[0].to(q.dtype)


__all__ = ["_normalize_query_positions", "_blockwise_exact_attention", "_dense_exact_attention", "_gelu",
           "RFSNHybridAttentionMLX", "_decode_compressed_tensor"]
