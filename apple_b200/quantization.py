"""PQ / RVQ quantizers and compressed-tensor helpers (quantization.py of the reference).

Same class and function names as the reference (quantization.py:99-402);
arrays are CUDA torch tensors and all encode/decode arithmetic runs in
librfsn_b200.so:

* ``ProductQuantizerMLX.quantize`` / ``HybridQuantizerMLX.encode`` ->
  ``rfsn_encode`` (fp32 distances, first arg-min, fp16 residual, norm-gated
  greedy RVQ — quantization.py:124-144, 206-252).
* ``decode`` / ``decode_correction`` / ``_decode_compressed_tensor`` ->
  ``rfsn_decode_codes`` (fp16 centroids + fp16(fp32 sum of RVQ rows), fp16 add —
  quantization.py:146-157, 254-275, 310-319), bit-identical to the reference.

RVQ-only calls reuse the same kernels with a one-centroid all-zero PQ
codebook: its residual is the input itself (x - 0 is exact) and its decode
contributes +0, so the RVQ arithmetic is unchanged.
"""
from __future__ import annotations

import logging
from typing import Dict, List, Optional, Tuple

import torch

from . import kernels as K
from .storage import CompressedTensorMLX, QuantizedMatrix, RFSNConfig, SUPPORTED_GROUP_SIZES, _concat0, _numpy_ints

logger = logging.getLogger("RFSN_QUANT")

_GEN: Dict[str, torch.Generator] = {}


def _generator(seed: Optional[int] = None) -> torch.Generator:
    g = _GEN.get("default")
    if g is None:
        g = torch.Generator().manual_seed(0)
        _GEN["default"] = g
    if seed is not None:
        g.manual_seed(int(seed))
    return g


def seed(value: int) -> None:
    """Seed the generator used for codebook initialisation (mx.random.seed analogue)."""
    _generator(value)


def _device(config: RFSNConfig) -> torch.device:
    return torch.device(config.device)


def _as_half_cuda(x: torch.Tensor, device: torch.device) -> torch.Tensor:
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    return x.to(device=device, dtype=torch.float16)


def _zero_pq(D: int, device: torch.device) -> torch.Tensor:
    return torch.zeros((D // 8, 1, 8), dtype=torch.float16, device=device)


def _code_values(codes: torch.Tensor, qz: K.QuantizerBuffers, dev: torch.device) -> torch.Tensor:
    """RVQ codes (int32 holding uint16 values) as the store's code dtype, [A, L]."""
    c = codes.to(device=dev, dtype=torch.int32).reshape(-1, qz.L)
    if qz.Kr > 256:
        c = torch.where(c > 32767, c - 65536, c)  # uint16 values stored in int16
    return c.to(qz.rvq_code_dtype)


def _choose_group_size(last_dim: int, preferred: int) -> Optional[int]:
    """quantization.py:23-33 (kept for API parity)."""
    cands: List[int] = [preferred] if preferred in SUPPORTED_GROUP_SIZES else []
    cands += [s for s in SUPPORTED_GROUP_SIZES if s not in cands]
    for size in cands:
        if last_dim % size == 0:
            return size
    return None


def _quantize_matrix(matrix: torch.Tensor, bits: int, preferred_group_size: int) -> Optional[QuantizedMatrix]:
    """quantization.py:36-76: affine quantization of a 2-D codebook in groups along its last
    dim (the first of the preferred, 128, 64, 32 sizes that divides it; else along the other
    dim, transposed), by rfsn_affine_quantize_f32.  None when no group size fits."""
    if matrix.dim() != 2:
        return None
    shape = tuple(int(d) for d in matrix.shape)
    cand = matrix.to(torch.float32)
    transposed = False
    group = _choose_group_size(int(cand.shape[-1]), preferred_group_size)
    if group is None:
        cand = cand.transpose(0, 1)
        group = _choose_group_size(int(cand.shape[-1]), preferred_group_size)
        if group is None:
            return None
        transposed = True
    q, scales, biases, deq = K.affine_quantize(cand.contiguous(), bits, group)
    return QuantizedMatrix(q, scales, biases, bits, group, transposed, shape,
                           deq.transpose(0, 1).contiguous() if transposed else deq)


def _dequantize_matrix(matrix: QuantizedMatrix, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """quantization.py:79-89: q * scale + bias in the original orientation, as dtype."""
    return matrix.dequantized.to(dtype)


class ProductQuantizerMLX:
    """Product quantizer (quantization.py:99-175): codebooks fp16 [M, 2^pq_bits, ds]."""

    def __init__(self, config: RFSNConfig):
        self.config = config
        self.num_subspaces = config.num_subspaces
        self.subspace_dim = config.subspace_dim
        self.codebook_size = 1 << config.pq_bits
        scale = (2.0 / self.subspace_dim) ** 0.5
        cb = torch.randn((self.num_subspaces, self.codebook_size, self.subspace_dim), generator=_generator(),
                         dtype=torch.float32) * scale
        self.codebooks = cb.to(torch.float16).to(_device(config))
        self._ane_codebooks: List[Optional[QuantizedMatrix]] = [None] * self.num_subspaces

    def effective_codebooks(self) -> torch.Tensor:
        """The codebooks the kernels read: the dequantized affine codebook of every subspace that
        quantize_codebooks_for_ane quantized (quantization.py:118-122), the fp16 codebook
        elsewhere.  The B200 path carries codebooks in fp16, so the dequantized values are
        rounded to fp16 for encoding as well as decoding (the reference encodes with them in
        fp32)."""
        if not any(m is not None for m in self._ane_codebooks):
            return self.codebooks
        parts = [_dequantize_matrix(m, torch.float16) if m is not None else self.codebooks[i].to(torch.float16)
                 for i, m in enumerate(self._ane_codebooks)]
        return torch.stack(parts).contiguous()

    def _buffers(self) -> K.QuantizerBuffers:
        return K.QuantizerBuffers(_as_half_cuda(self.effective_codebooks(), _device(self.config)), None,
                                  float("inf"), 0)

    def quantize(self, vectors: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """quantization.py:124-144 -> (codes uint8 [N, M], residual fp16 [N, D])."""
        n, d = vectors.shape
        if d != self.num_subspaces * self.subspace_dim:
            raise ValueError(f"Expected vectors with dim {self.num_subspaces * self.subspace_dim}, got {d}")
        qz = self._buffers()
        x = _as_half_cuda(vectors, qz.pq_codebooks.device).contiguous()
        store = K.CodeStoreBuffers(qz, rows=1, cap=max(n, 1))
        residual = torch.empty_like(x)
        if n == 0:
            return torch.zeros((0, self.num_subspaces), dtype=torch.uint8, device=x.device), residual
        K.encode(qz, x.view(1, n, 1, d), store, 0, 0, residual_out=residual.view(1, n, 1, d))
        return store.read_rows(0, "pq", 0, 0, n)[0], residual

    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        """quantization.py:146-157 -> fp16 [N, D]."""
        qz = self._buffers()
        n = int(codes.shape[0])
        out = torch.empty((1, n, 1, qz.D), dtype=torch.float16, device=qz.pq_codebooks.device)
        if n:
            store = K.CodeStoreBuffers(qz, rows=1, cap=n)
            store.write(0, "pq", 0, 0, 0, codes.to(dtype=torch.uint8))
            K.decode_codes(qz, store, 0, 0, n, out)
        return out.view(n, qz.D)

    def quantize_codebooks_for_ane(self) -> Dict[str, int]:
        """quantization.py:159-175: affine ane_quant_bits-bit codebooks (group ane_group_size)."""
        quantized = 0
        for m in range(self.num_subspaces):
            packed = _quantize_matrix(self.codebooks[m], self.config.ane_quant_bits, self.config.ane_group_size)
            self._ane_codebooks[m] = packed
            quantized += packed is not None
        logger.info("PQ codebook fast path prepared for %d/%d subspaces", quantized, self.num_subspaces)
        return {"quantized_subspaces": quantized, "total_subspaces": self.num_subspaces}


class ResidualVQMLX:
    """Norm-gated residual VQ (quantization.py:178-293): codebooks fp16 [L, Kr, D], row 0 zeroed."""

    def __init__(self, config: RFSNConfig):
        self.config = config
        self.num_layers = config.num_rvq_layers
        self.codebook_size = config.rvq_codebook_size
        self.head_dim = config.head_dim
        self.sparsity_threshold = config.rvq_sparsity_threshold
        scale = (2.0 / self.head_dim) ** 0.5
        cb = torch.randn((self.num_layers, self.codebook_size, self.head_dim), generator=_generator(),
                         dtype=torch.float32) * scale
        cb = cb.to(torch.float16)
        if self.num_layers:
            cb[:, 0] = 0  # quantization.py:196-197
        self.codebooks = cb.to(_device(config))
        self._ane_codebooks: List[Optional[QuantizedMatrix]] = [None] * self.num_layers

    def effective_codebooks(self) -> torch.Tensor:
        """As ProductQuantizerMLX.effective_codebooks, per RVQ layer (quantization.py:200-204)."""
        if not any(m is not None for m in self._ane_codebooks):
            return self.codebooks
        parts = [_dequantize_matrix(m, torch.float16) if m is not None else self.codebooks[i].to(torch.float16)
                 for i, m in enumerate(self._ane_codebooks)]
        return torch.stack(parts).contiguous()

    def _buffers(self) -> K.QuantizerBuffers:
        dev = _device(self.config)
        return K.QuantizerBuffers(_zero_pq(self.head_dim, dev), _as_half_cuda(self.effective_codebooks(), dev),
                                  float(self.sparsity_threshold), 0)

    def encode(self, residuals: torch.Tensor, base_codes: Optional[torch.Tensor] = None
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """quantization.py:206-252 -> (codes int32 [A, L] (uint16 values), mask bool [N], offsets int32 [A])."""
        del base_codes
        n, d = residuals.shape
        if d != self.head_dim:
            raise ValueError(f"Expected residual dim {self.head_dim}, got {d}")
        qz = self._buffers()
        x = _as_half_cuda(residuals, qz.pq_codebooks.device).contiguous()
        store = K.CodeStoreBuffers(qz, rows=1, cap=max(n, 1))
        if n and qz.L:
            K.encode(qz, x.view(1, n, 1, d), store, 0, 0)
        if not qz.L:
            mask = torch.zeros(n, dtype=torch.bool, device=x.device)
            return torch.zeros((0, 0), dtype=torch.int32, device=x.device), mask, torch.zeros(0, dtype=torch.int32,
                                                                                             device=x.device)
        if n == 0:
            return (torch.zeros((0, qz.L), dtype=torch.int32, device=x.device),
                    torch.zeros(0, dtype=torch.bool, device=x.device), torch.zeros(0, dtype=torch.int32, device=x.device))
        mask = store.read_rows(0, "active", 0, 0, n)[0, :, 0].bool()
        offsets = torch.nonzero(mask, as_tuple=False).reshape(-1).to(torch.int32)
        codes = (store.read_rows(0, "rvq", 0, 0, n)[0][mask].to(torch.int32) & 0xFFFF)
        return codes, mask, offsets

    def decode_correction(self, rvq_codes: torch.Tensor, rvq_mask: torch.Tensor, rvq_offsets: torch.Tensor
                          ) -> torch.Tensor:
        """quantization.py:254-275 -> fp16 [N, D], zero rows where inactive."""
        qz = self._buffers()
        dev = qz.pq_codebooks.device
        n = int(rvq_mask.shape[0])
        out = torch.zeros((1, n, 1, self.head_dim), dtype=torch.float16, device=dev)
        if n == 0 or int(rvq_codes.shape[0]) == 0 or not qz.L:
            return out.view(n, self.head_dim)
        store = K.CodeStoreBuffers(qz, rows=1, cap=n)
        offs = rvq_offsets.to(device=dev, dtype=torch.long)
        store.put(0, "rvq", 0, 0, offs, _code_values(rvq_codes, qz, dev))
        store.put(0, "active", 0, 0, offs, torch.ones((offs.numel(), 1), dtype=torch.uint8, device=dev))
        K.decode_codes(qz, store, 0, 0, n, out)
        return out.view(n, self.head_dim)

    def quantize_codebooks_for_ane(self) -> Dict[str, int]:
        """quantization.py:277-293."""
        quantized = 0
        for layer in range(self.num_layers):
            packed = _quantize_matrix(self.codebooks[layer], self.config.ane_quant_bits, self.config.ane_group_size)
            self._ane_codebooks[layer] = packed
            quantized += packed is not None
        logger.info("RVQ codebook fast path prepared for %d/%d layers", quantized, self.num_layers)
        return {"quantized_layers": quantized, "total_layers": self.num_layers}


class HybridQuantizerMLX:
    """PQ base + sparse RVQ refinement (quantization.py:296-327), plus the top-S
    sparse residual extension when ``config.sparse_topk > 0``."""

    def __init__(self, config: RFSNConfig):
        self.config = config
        self.pq = ProductQuantizerMLX(config)
        self.rvq = ResidualVQMLX(config)
        self._cache_key = None
        self._cache_val: Optional[K.QuantizerBuffers] = None

    def buffers(self) -> K.QuantizerBuffers:
        """Device description of the current codebooks (rebuilt when they change)."""
        pq, rvq = self.pq.codebooks, self.rvq.codebooks
        key = (id(pq), getattr(pq, "_version", 0), id(rvq), getattr(rvq, "_version", 0),
               self.config.rvq_sparsity_threshold, self.config.sparse_topk,
               tuple(id(m) for m in self.pq._ane_codebooks), tuple(id(m) for m in self.rvq._ane_codebooks))
        if key != self._cache_key:
            dev = _device(self.config)
            pq, rvq = self.pq.effective_codebooks(), self.rvq.effective_codebooks()
            self._cache_val = K.QuantizerBuffers(_as_half_cuda(pq, dev),
                                                 _as_half_cuda(rvq, dev) if self.config.num_rvq_layers else None,
                                                 float(self.config.rvq_sparsity_threshold),
                                                 int(self.config.sparse_topk))
            self._cache_key = key
        return self._cache_val

    def encode(self, vectors: torch.Tensor):
        """quantization.py:305-308 -> (pq_codes, rvq_codes, rvq_mask, rvq_offsets)."""
        ct = _compress_tensor_sequence(vectors.reshape(vectors.shape[0], 1, -1), self)
        return ct.pq_codes[:, 0], ct.rvq_codes, ct.rvq_mask[:, 0], ct.rvq_offsets

    def decode(self, pq_codes: torch.Tensor, rvq_codes: torch.Tensor, rvq_mask: torch.Tensor,
               rvq_offsets: torch.Tensor) -> torch.Tensor:
        """quantization.py:310-319 -> fp16 [N, D] = fp16(pq_decode + correction)."""
        qz = self.buffers()
        n = int(pq_codes.shape[0])
        dev = qz.pq_codebooks.device
        out = torch.empty((1, n, 1, qz.D), dtype=torch.float16, device=dev)
        if n == 0:
            return out.view(0, qz.D)
        q0 = K.QuantizerBuffers(qz.pq_codebooks, qz.rvq_codebooks, qz.threshold, 0)
        store = K.CodeStoreBuffers(q0, rows=1, cap=n)
        store.write(0, "pq", 0, 0, 0, pq_codes.to(dtype=torch.uint8))
        if q0.L and int(rvq_codes.shape[0]):
            offs = rvq_offsets.to(device=dev, dtype=torch.long)
            store.put(0, "rvq", 0, 0, offs, _code_values(rvq_codes, q0, dev))
            store.put(0, "active", 0, 0, offs, torch.ones((offs.numel(), 1), dtype=torch.uint8, device=dev))
        K.decode_codes(q0, store, 0, 0, n, out)
        return out.view(n, qz.D)

    def quantize_codebooks_for_ane(self) -> Dict[str, int]:
        """quantization.py:321-327."""
        pq_report = self.pq.quantize_codebooks_for_ane()
        rvq_report = self.rvq.quantize_codebooks_for_ane()
        return {"pq_quantized": pq_report["quantized_subspaces"], "rvq_quantized": rvq_report["quantized_layers"]}


def _compress_tensor_sequence(tensor: torch.Tensor, quantizer: HybridQuantizerMLX) -> CompressedTensorMLX:
    """quantization.py:330-343 — encode [T, H, D] token-major (rows = heads)."""
    num_tokens, num_heads, head_dim = tensor.shape
    qz = quantizer.buffers()
    dev = qz.pq_codebooks.device
    x = _as_half_cuda(tensor, dev).contiguous()
    store = K.CodeStoreBuffers(qz, rows=num_heads, cap=max(num_tokens, 1))
    if num_tokens:
        K.encode(qz, x.view(1, num_tokens, num_heads, head_dim), store, 0, 0)
    return CompressedTensorMLX.from_store(store, 0, 0, 0, num_tokens, num_heads)


def _append_compressed_tensor(base: CompressedTensorMLX, addition: CompressedTensorMLX) -> CompressedTensorMLX:
    """quantization.py:346-361 (dense layout: offsets shift implicitly)."""
    if base.num_heads != addition.num_heads:
        raise ValueError("Compressed tensors must have the same number of heads")
    return CompressedTensorMLX(_concat0(base.pq_codes, addition.pq_codes), _concat0(base.rvq, addition.rvq),
                               _concat0(base.rvq_mask, addition.rvq_mask), _concat0(base.sp_idx, addition.sp_idx),
                               _concat0(base.sp_val, addition.sp_val), base.num_heads)


def _slice_compressed_tensor(tensor: CompressedTensorMLX, start: int, end: int) -> CompressedTensorMLX:
    """quantization.py:364-391."""
    if start < 0 or end < start or end > tensor.num_tokens:
        raise ValueError("Invalid slice for compressed tensor")
    return CompressedTensorMLX(tensor.pq_codes[start:end], tensor.rvq[start:end], tensor.rvq_mask[start:end],
                               tensor.sp_idx[start:end], tensor.sp_val[start:end], tensor.num_heads)


def _decode_compressed_tensor(tensor: CompressedTensorMLX, quantizer: HybridQuantizerMLX) -> torch.Tensor:
    """quantization.py:394-402 -> fp16 [T, H, D] (sparse residual added in fp32, rounded once)."""
    qz = quantizer.buffers()
    dev = qz.pq_codebooks.device
    T, H = tensor.num_tokens, tensor.num_heads
    out = torch.empty((1, T, H, qz.D), dtype=torch.float16, device=dev)
    if T == 0:
        return out.view(0, H, qz.D)
    store = tensor.to_store(qz)
    K.decode_codes(qz, store, 0, 0, T, out)
    return out.view(T, H, qz.D)


__all__ = ["ProductQuantizerMLX", "ResidualVQMLX", "HybridQuantizerMLX", "_compress_tensor_sequence",
           "_append_compressed_tensor", "_slice_compressed_tensor", "_decode_compressed_tensor",
           "_choose_group_size", "seed", "_numpy_ints"]
