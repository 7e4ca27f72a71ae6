"""Decoder layer and PQ calibration (rfsn_v10_mlx_ane_complete.py:55-225 of the reference).

``RFSNDecoderLayerMLX`` keeps the reference's structure and API: RMSNorm ->
q/k/v projections -> cache update -> cache-backed fused decode attention (or
dense causal attention without a cache) -> o_proj + residual -> RMSNorm ->
GELU FFN (2x) + residual.  Decode-sized projections (at most 32 rows) stream
their weights with rfsn_linear_f16, the FFN's GELU and residual add fused
into its epilogues; larger ones (prefill) are cuBLAS GEMMs.  The attention,
every quantizer operation and the RMSNorms run in librfsn_b200.so too.  Extensions:
``num_kv_heads`` (GQA) and ``batch_size`` > 1 sequences per cache.
"""
from __future__ import annotations

import logging
import math
import shutil
from pathlib import Path
from typing import Dict, List, Optional

import torch

from . import kernels as K
from .attention import _dense_exact_attention, _gelu
from .cache import RFSNv10KVCacheMLX
from .quantization import HybridQuantizerMLX
from .storage import AsyncHierarchicalRouterMLX, RFSNConfig

logger = logging.getLogger("RFSN_MLX_APPLE")


def _as(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """t in dtype (t itself when it already is: a decode step makes many such calls)."""
    return t if t.dtype == dtype else t.to(dtype)


class _Linear:
    """y = x @ W^T (no bias); W ~ U(-1/sqrt(in), 1/sqrt(in)) like mlx.nn.Linear, or N(0, 1/in).
    The product runs in the activations' dtype, as mlx.nn.Linear casts W to x's dtype."""

    def __init__(self, in_dim: int, out_dim: int, device, dtype, gen: torch.Generator, init: str):
        if init == "normal":
            w = torch.randn((out_dim, in_dim), generator=gen) / math.sqrt(in_dim)
        else:
            w = (torch.rand((out_dim, in_dim), generator=gen) * 2 - 1) / math.sqrt(in_dim)
        self.weight = w.to(device=device, dtype=dtype)
        self._cast = None  # weight in the activations' dtype, refreshed when the weight is replaced
        self._src = None

    def cast(self, dtype: torch.dtype) -> torch.Tensor:
        """The weight in the activations' dtype (mlx.nn.Linear casts it to x's dtype), cached."""
        if self._cast is None or self._cast.dtype != dtype or self._src is not self.weight:
            self._cast, self._src = self.weight.to(dtype).contiguous(), self.weight
        return self._cast

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None, gelu: bool = False) -> torch.Tensor:
        """x @ W^T; decode-sized fp16 products (at most 32 rows) stream W with rfsn_linear_f16, which
        also fuses the residual add (fp16(fp16(y) + residual)) or the layer's fp16 tanh-GELU; other
        shapes run the GEMM in cuBLAS and the epilogue separately."""
        w = self.cast(x.dtype)
        if K.use_linear(x, w):
            return K.linear(x, w, residual=residual, gelu=gelu)
        y = torch.nn.functional.linear(x, w)
        if gelu:
            y = K.gelu_tanh(y) if y.dtype == torch.float16 and y.is_cuda else _gelu(y)
        if residual is not None:
            y = residual + y
        return y


class _RMSNorm:
    """RMSNorm with an fp32 weight (mlx.nn.RMSNorm).  fp16 inputs, which are what the layer
    passes, run as one kernel (rfsn_rmsnorm_f16) with the same operation order."""

    def __init__(self, dims: int, device, eps: float = 1e-5):
        self.weight = torch.ones(dims, device=device)
        self.eps = eps

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype == torch.float16 and x.is_cuda:
            return K.rms_norm(x, self.weight, self.eps)
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight).to(x.dtype)


class RFSNDecoderLayerMLX:
    """Decoder layer that owns its projections, quantizer, and cache-backed decode path."""

    def __init__(self, config: RFSNConfig, layer_idx: int = 0, ffn_multiplier: int = 2,
                 weight_dtype: torch.dtype = torch.float32, init: str = "uniform", seed: int = 0):
        self.config = config
        self.layer_idx = layer_idx
        self.num_heads = config.num_heads
        self.num_kv_heads = config.kv_heads
        self.head_dim = config.head_dim
        self.model_dim = config.hidden_dim
        self.ffn_hidden_dim = max(config.hidden_dim * ffn_multiplier, config.hidden_dim)
        self.scale = config.head_dim ** -0.5
        dev = torch.device(config.device)
        self._device = dev
        g = torch.Generator().manual_seed(seed + 1000 * layer_idx)
        mk = lambda i, o: _Linear(i, o, dev, weight_dtype, g, init)  # noqa: E731
        self.attn_norm = _RMSNorm(config.hidden_dim, dev)
        self.ffn_norm = _RMSNorm(config.hidden_dim, dev)
        self.q_proj = mk(config.hidden_dim, config.num_heads * config.head_dim)
        self.k_proj = mk(config.hidden_dim, self.num_kv_heads * config.head_dim)
        self.v_proj = mk(config.hidden_dim, self.num_kv_heads * config.head_dim)
        self.o_proj = mk(config.num_heads * config.head_dim, config.hidden_dim)
        self.ffn_up = mk(config.hidden_dim, self.ffn_hidden_dim)
        self.ffn_down = mk(self.ffn_hidden_dim, config.hidden_dim)
        self._qkv_w: Optional[torch.Tensor] = None  # q/k/v weights concatenated in the activations' dtype
        self._qkv_src: tuple = ()
        self.quantizer = HybridQuantizerMLX(config)
        self.disk_cache_dir = Path(config.disk_cache_dir) / f"decoder_layer_{layer_idx}"
        self.cache = RFSNv10KVCacheMLX(config, layer_idx=layer_idx)

    @property
    def cache_tokens(self) -> int:
        return self.cache.total_tokens

    def reset_cache(self, remove_disk: bool = True) -> None:
        """rfsn_v10_mlx_ane_complete.py:85-88."""
        if remove_disk and self.disk_cache_dir.exists():
            shutil.rmtree(self.disk_cache_dir)
        self.cache.close()
        self.cache = RFSNv10KVCacheMLX(self.config, layer_idx=self.layer_idx)

    def _qkv(self, a: torch.Tensor):
        """q, k and v projections of the same input as one GEMM over the concatenated weights
        (rebuilt when a projection's weight is replaced); returns views of the one product."""
        ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        src = self._qkv_src
        if (self._qkv_w is None or self._qkv_w.dtype != a.dtype or len(src) != 3
                or src[0] is not ws[0] or src[1] is not ws[1] or src[2] is not ws[2]):
            self._qkv_w = torch.cat([w.to(a.dtype) for w in ws], 0)
            self._qkv_src = ws
        y = K.linear(a, self._qkv_w) if K.use_linear(a, self._qkv_w) else \
            torch.nn.functional.linear(a, self._qkv_w)
        nq = self.num_heads * self.head_dim
        nk = self.num_kv_heads * self.head_dim
        return y[..., :nq], y[..., nq:nq + nk], y[..., nq + nk:]

    def _project_heads(self, projected: torch.Tensor, heads: int) -> torch.Tensor:
        b, s, _ = projected.shape
        return _as(projected.reshape(b, s, heads, self.head_dim), torch.float16)

    def prefill_cache(self, x: torch.Tensor, reset: bool = True) -> None:
        """rfsn_v10_mlx_ane_complete.py:90-104 ([B, S, hidden] with B = config.batch_size)."""
        if x.dim() != 3 or int(x.shape[0]) != self.config.batch_size:
            raise ValueError("prefill_cache expects input shape [1, seq_len, hidden_dim]"
                             if self.config.batch_size == 1 else
                             f"prefill_cache expects input shape [{self.config.batch_size}, seq_len, hidden_dim]")
        if reset:
            self.reset_cache(remove_disk=True)
        attn_input = self.attn_norm(x.to(torch.float16))
        keys = self._project_heads(self.k_proj(attn_input), self.num_kv_heads)
        values = self._project_heads(self.v_proj(attn_input), self.num_kv_heads)
        if self.config.batch_size == 1:
            keys, values = keys[0], values[0]
        self.cache.update(keys, values, self.quantizer, disk_dir=self.disk_cache_dir)

    def __call__(self, x: torch.Tensor, use_cache: bool = False,
                 router: Optional[AsyncHierarchicalRouterMLX] = None,
                 context_window: Optional[int] = None) -> torch.Tensor:
        """rfsn_v10_mlx_ane_complete.py:114-172."""
        if x.dim() != 3:
            raise ValueError("Decoder layer expects input shape [batch, seq_len, hidden_dim]")
        if int(x.shape[-1]) != self.model_dim:
            raise ValueError(f"Expected hidden_dim {self.model_dim}, got {int(x.shape[-1])}")
        x = x.to(device=self._device)
        residual = _as(x, torch.float16)
        attn_input = _as(self.attn_norm(residual), torch.float16)
        q_p, k_p, v_p = self._qkv(attn_input)
        q_heads = self._project_heads(q_p, self.num_heads)
        k_heads = self._project_heads(k_p, self.num_kv_heads)
        v_heads = self._project_heads(v_p, self.num_kv_heads)
        B = int(x.shape[0])
        if use_cache:
            if tuple(x.shape[:2]) != (self.config.batch_size, 1):
                raise ValueError("cache-backed decoding currently supports input shape "
                                 f"[{self.config.batch_size}, 1, hidden_dim]; use prefill_cache() for longer prompts")
            k_new = k_heads[0] if self.config.batch_size == 1 else k_heads
            v_new = v_heads[0] if self.config.batch_size == 1 else v_heads
            self.cache.update(k_new, v_new, self.quantizer, disk_dir=self.disk_cache_dir)
            total = self.cache.total_tokens
            window = context_window
            if window is None:
                window = max(self.config.block_size_seq, min(total, self.config.warm_capacity))
            qpos = [total - 1] if self.config.batch_size == 1 else [total - 1] * B
            attended = self.cache.attention_forward(q_heads[:, 0], causal=True, query_positions=qpos,
                                                    router=router, current_position=total - 1,
                                                    context_window=window)
            attended = attended.reshape(B, 1, self.num_heads, self.head_dim)
        else:
            attended = _dense_exact_attention(q_heads, k_heads, v_heads, self.scale, causal=True)
        attn_out = _as(self.o_proj(attended.reshape(B, -1, self.num_heads * self.head_dim)), residual.dtype)
        if residual.is_cuda and residual.dtype == torch.float16 and attn_out.dtype == torch.float16:
            # residual add and FFN RMSNorm in one launch (same roundings)
            hidden, ffn_input = K.add_rms_norm(residual, attn_out, self.ffn_norm.weight, self.ffn_norm.eps)
        else:
            hidden = residual + attn_out
            ffn_input = self.ffn_norm(hidden).to(torch.float16)
        act = self.ffn_up(ffn_input, gelu=True)  # GELU fused into the projection's epilogue
        return self.ffn_down(act, residual=hidden)  # residual add fused likewise


def calibrate_quantizer(quantizer: HybridQuantizerMLX, calibration_vectors: torch.Tensor, num_iterations: int = 20,
                        sample_idx: Optional[torch.Tensor] = None, generator: Optional[torch.Generator] = None
                        ) -> Dict[str, List[float]]:
    """k-means PQ calibration (rfsn_v10_mlx_ane_complete.py:175-225) on the GPU.

    Initial centroids are rows ``sample_idx[m]`` (shape [M, K]) of each
    subspace, drawn uniformly when not given; each Lloyd iteration assigns
    with the PQ encoder kernel and moves every non-empty centroid to the mean
    of its members (empty clusters keep their centroid)."""
    cfg = quantizer.config
    dev = torch.device(cfg.device)
    x = calibration_vectors.to(device=dev, dtype=torch.float16)
    n = int(x.shape[0])
    K = quantizer.pq.codebook_size
    M, ds = cfg.num_subspaces, cfg.subspace_dim
    if sample_idx is None:
        g = generator or torch.Generator().manual_seed(0)
        sample_idx = torch.randint(0, n, (M, K), generator=g)
    sample_idx = sample_idx.to(dev).long()
    quantizer.pq.codebooks = torch.stack([x[sample_idx[m], m * ds:(m + 1) * ds] for m in range(M)]).contiguous()
    metrics: Dict[str, List[float]] = {"avg_distortion": [], "sparsity_fraction": []}
    x32 = x.float()
    for it in range(num_iterations):
        codes, residuals = quantizer.pq.quantize(x)
        codes = codes.long()
        new = quantizer.pq.codebooks.float().clone()
        for m in range(M):
            sub = x32[:, m * ds:(m + 1) * ds]
            sums = torch.zeros((K, ds), device=dev).index_add_(0, codes[:, m], sub)
            cnt = torch.bincount(codes[:, m], minlength=K)
            nz = cnt > 0
            new[m][nz] = sums[nz] / cnt[nz, None].float()
        quantizer.pq.codebooks = new.to(torch.float16)
        recon = quantizer.pq.decode(codes)
        distortion = float(((x32 - recon.float()) ** 2).mean())
        norms = torch.sqrt((residuals.float() ** 2).sum(1))
        sparsity = float((norms < cfg.rvq_sparsity_threshold).float().mean())
        metrics["avg_distortion"].append(distortion)
        metrics["sparsity_fraction"].append(sparsity)
    return metrics
