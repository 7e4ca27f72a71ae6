"""Llama adapter decoder layer (llama32_adapter.py:374-662 of the reference) on the B200 path.

``Llama32DecoderLayerMLX`` keeps the reference's constructor, ``from_hf_layer``,
``prefill_cache``, ``reset_cache`` and ``__call__``: RMSNorm with a weight ->
q/k/v projections -> RoPE from given position tables (or a rotary module) ->
the RFSN cache (cache-backed decode) or dense causal attention -> o_proj +
residual -> RMSNorm -> SwiGLU MLP + residual.

On this path the RMSNorms (with the residual add folded into the second),
RoPE and the SwiGLU product are one librfsn_b200.so launch each, in the
adapter's operation order and rounding points; the q/k/v and gate/up
projections are one product each over concatenated weights (the weight-
streaming rfsn_linear_f16 at decode sizes, with the final residual add fused
into the down projection; cuBLAS otherwise); decode attention is the fused
compressed-KV kernel.  The cache stores the KV heads
once (GQA) instead of the reference's _repeat_kv'd copies (llama32_adapter.py:
380-386, 580-581): attention reads KV head h // group for query head h, the
same values.  Batch > 1 is an extension (the reference adapter takes batch 1).
"""
from __future__ import annotations

import shutil
from dataclasses import replace
from pathlib import Path
from typing import Any, Optional, Tuple

import numpy as np
import torch

from . import kernels as K
from .attention import _dense_exact_attention
from .cache import RFSNv10KVCacheMLX
from .quantization import HybridQuantizerMLX
from .storage import AsyncHierarchicalRouterMLX, RFSNConfig


def _tensor(value: Any, device, dtype=torch.float16) -> torch.Tensor:
    if isinstance(value, torch.Tensor):
        return value.detach().to(device=device, dtype=dtype).contiguous()
    return torch.as_tensor(np.asarray(value)).to(device=device, dtype=dtype).contiguous()


def _position_table(component: Any, seq_len: int, head_dim: int, device) -> torch.Tensor:
    """llama32_adapter.py:389-405: a cos or sin table as fp16 [seq_len, head_dim] ([D], [S, D] or
    [1, S, D] accepted)."""
    t = component.detach() if isinstance(component, torch.Tensor) else torch.as_tensor(np.asarray(component))
    t = t.squeeze()
    if t.dim() == 1:
        t = t.reshape(1, -1)
    elif t.dim() == 3:
        if t.shape[0] != 1:
            raise ValueError("Only batch size 1 is supported for the Llama adapter")
        t = t[0]
    elif t.dim() != 2:
        raise ValueError(f"Unsupported rotary embedding rank {t.dim()}")
    if t.shape[0] != seq_len:
        raise ValueError(f"Expected {seq_len} position rows, got {t.shape[0]}")
    if t.shape[1] != head_dim:
        raise ValueError(f"Expected rotary head dim {head_dim}, got {t.shape[1]}")
    return t.to(device=device, dtype=torch.float16).contiguous()


def _linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """llama32_adapter.py:492-494: decode-sized products stream W with rfsn_linear_f16, others cuBLAS."""
    return K.linear(x, w) if K.use_linear(x, w) else torch.nn.functional.linear(x, w)


class Llama32DecoderLayerMLX:
    """Llama-3.2 decoder layer with the RFSN compressed KV cache (llama32_adapter.py:417-662)."""

    def __init__(self, config: RFSNConfig, layer_idx: int, num_key_value_heads: int, rms_norm_eps: float,
                 input_layernorm_weight, post_attention_layernorm_weight, q_proj_weight, k_proj_weight,
                 v_proj_weight, o_proj_weight, gate_proj_weight, up_proj_weight, down_proj_weight,
                 rotary_module: Optional[torch.nn.Module] = None):
        if config.num_heads % num_key_value_heads:
            raise ValueError("num_heads must be a multiple of num_key_value_heads")
        # the cache keeps the KV heads (GQA); queries of head h read KV head h // group
        self.config = replace(config, num_kv_heads=num_key_value_heads)
        self.layer_idx = layer_idx
        self.hidden_dim = config.hidden_dim
        self.num_heads = config.num_heads
        self.num_key_value_heads = num_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.head_dim = config.head_dim
        self.scale = self.head_dim ** -0.5
        self.rms_norm_eps = rms_norm_eps
        dev = torch.device(self.config.device)
        self._device = dev
        self.input_layernorm_weight = _tensor(input_layernorm_weight, dev)
        self.post_attention_layernorm_weight = _tensor(post_attention_layernorm_weight, dev)
        self.q_proj_weight = _tensor(q_proj_weight, dev)
        self.k_proj_weight = _tensor(k_proj_weight, dev)
        self.v_proj_weight = _tensor(v_proj_weight, dev)
        self.o_proj_weight = _tensor(o_proj_weight, dev)
        self.gate_proj_weight = _tensor(gate_proj_weight, dev)
        self.up_proj_weight = _tensor(up_proj_weight, dev)
        self.down_proj_weight = _tensor(down_proj_weight, dev)
        nq, nk = self.num_heads * self.head_dim, self.num_key_value_heads * self.head_dim
        for name, w, shape in (("q_proj", self.q_proj_weight, (nq, self.hidden_dim)),
                               ("k_proj", self.k_proj_weight, (nk, self.hidden_dim)),
                               ("v_proj", self.v_proj_weight, (nk, self.hidden_dim)),
                               ("o_proj", self.o_proj_weight, (self.hidden_dim, nq))):
            if tuple(w.shape) != shape:
                raise ValueError(f"{name} weight must be {shape}, got {tuple(w.shape)}")
        # one GEMM for q/k/v and one for gate/up (the same products as separate projections)
        self._qkv_w = torch.cat([self.q_proj_weight, self.k_proj_weight, self.v_proj_weight], 0).contiguous()
        self._gate_up_w = torch.cat([self.gate_proj_weight, self.up_proj_weight], 0).contiguous()
        self.quantizer = HybridQuantizerMLX(self.config)
        self.disk_cache_dir = Path(self.config.disk_cache_dir)
        self.cache = RFSNv10KVCacheMLX(self.config, layer_idx=layer_idx)
        self.rotary_module = rotary_module

    @classmethod
    def from_hf_layer(cls, hf_layer: torch.nn.Module, hf_config: Any, rfsn_config: RFSNConfig, layer_idx: int,
                      rotary_module: Optional[torch.nn.Module] = None) -> "Llama32DecoderLayerMLX":
        """llama32_adapter.py:459-485: the weights of a Hugging Face LlamaDecoderLayer."""
        kvh = int(getattr(hf_config, "num_key_value_heads", hf_config.num_attention_heads))
        return cls(config=rfsn_config, layer_idx=layer_idx, num_key_value_heads=kvh,
                   rms_norm_eps=float(getattr(hf_config, "rms_norm_eps", 1e-5)),
                   input_layernorm_weight=hf_layer.input_layernorm.weight,
                   post_attention_layernorm_weight=hf_layer.post_attention_layernorm.weight,
                   q_proj_weight=hf_layer.self_attn.q_proj.weight, k_proj_weight=hf_layer.self_attn.k_proj.weight,
                   v_proj_weight=hf_layer.self_attn.v_proj.weight, o_proj_weight=hf_layer.self_attn.o_proj.weight,
                   gate_proj_weight=hf_layer.mlp.gate_proj.weight, up_proj_weight=hf_layer.mlp.up_proj.weight,
                   down_proj_weight=hf_layer.mlp.down_proj.weight, rotary_module=rotary_module)

    def reset_cache(self, remove_disk: bool = True) -> None:
        """llama32_adapter.py:487-490."""
        if remove_disk and self.disk_cache_dir.exists():
            shutil.rmtree(self.disk_cache_dir)
        self.cache.close()
        self.cache = RFSNv10KVCacheMLX(self.config, layer_idx=self.layer_idx)

    def _positions(self, seq_len: int, position_embeddings, position_ids) -> Tuple[torch.Tensor, torch.Tensor]:
        """llama32_adapter.py:516-553: given (cos, sin), or recomputed with the rotary module."""
        if position_embeddings is not None:
            return (_position_table(position_embeddings[0], seq_len, self.head_dim, self._device),
                    _position_table(position_embeddings[1], seq_len, self.head_dim, self._device))
        if self.rotary_module is None:
            raise RuntimeError("No position embeddings were captured and no rotary embedding module is available to "
                               "recompute them.")
        ids = position_ids if position_ids is not None else torch.arange(seq_len, dtype=torch.long).unsqueeze(0)
        buf = next(self.rotary_module.buffers(), None)
        dev = buf.device if buf is not None else ids.device
        ids = ids.to(dev)
        with torch.no_grad():
            try:
                cos, sin = self.rotary_module(torch.zeros((1, seq_len, self.hidden_dim), device=dev), ids)
            except TypeError:
                cos, sin = self.rotary_module(ids)
        return (_position_table(cos, seq_len, self.head_dim, self._device),
                _position_table(sin, seq_len, self.head_dim, self._device))

    def _project_qkv(self, hidden: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """llama32_adapter.py:570-582 (KV heads kept, not repeated)."""
        B, S, _ = hidden.shape
        normed, _ = K.llama_rms_norm(hidden, self.input_layernorm_weight, self.rms_norm_eps)
        y = _linear(normed, self._qkv_w)
        nq, nk = self.num_heads * self.head_dim, self.num_key_value_heads * self.head_dim
        q = K.rope(y[..., :nq].unflatten(-1, (self.num_heads, self.head_dim)), cos, sin)
        k = K.rope(y[..., nq:nq + nk].unflatten(-1, (self.num_key_value_heads, self.head_dim)), cos, sin)
        v = y[..., nq + nk:].unflatten(-1, (self.num_key_value_heads, self.head_dim)).contiguous()
        return q, k, v

    def _check_input(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 3 or int(x.shape[-1]) != self.hidden_dim:
            raise ValueError(f"expected hidden states [batch, seq_len, {self.hidden_dim}], got {tuple(x.shape)}")
        if int(x.shape[0]) != self.config.batch_size:
            raise ValueError("The Llama adapter currently supports batch size 1 only" if self.config.batch_size == 1
                             else f"expected batch size {self.config.batch_size}")
        return x.to(device=self._device, dtype=torch.float16)

    def prefill_cache(self, hidden_states, position_embeddings=None, position_ids=None, reset: bool = True) -> None:
        """llama32_adapter.py:591-614."""
        x = self._check_input(torch.as_tensor(hidden_states) if not isinstance(hidden_states, torch.Tensor)
                              else hidden_states)
        S = int(x.shape[1])
        if reset:
            self.reset_cache(remove_disk=True)
        if S == 0:
            return
        cos, sin = self._positions(S, position_embeddings, position_ids)
        _, k, v = self._project_qkv(x, cos, sin)
        if self.config.batch_size == 1:
            k, v = k[0], v[0]
        self.cache.update(k, v, self.quantizer, disk_dir=self.disk_cache_dir)

    def __call__(self, hidden_states, position_embeddings=None, position_ids=None, use_cache: bool = False,
                 router: Optional[AsyncHierarchicalRouterMLX] = None,
                 context_window: Optional[int] = None) -> torch.Tensor:
        """llama32_adapter.py:616-662."""
        x = self._check_input(torch.as_tensor(hidden_states) if not isinstance(hidden_states, torch.Tensor)
                              else hidden_states)
        B, S = int(x.shape[0]), int(x.shape[1])
        cos, sin = self._positions(S, position_embeddings, position_ids)
        residual = x
        q, k, v = self._project_qkv(residual, cos, sin)
        if use_cache:
            if S != 1:
                raise ValueError("cache-backed decode expects input shape [1, 1, hidden_dim]")
            if B == 1:
                self.cache.update(k[0], v[0], self.quantizer, disk_dir=self.disk_cache_dir)
            else:
                self.cache.update(k, v, self.quantizer, disk_dir=self.disk_cache_dir)
            total = self.cache.total_tokens
            attended = self.cache.attention_forward(q[:, 0], causal=True, query_positions=[total - 1] * B,
                                                    router=router, current_position=total - 1,
                                                    context_window=context_window)
            attended = attended.reshape(B, 1, self.num_heads * self.head_dim)
        else:
            attended = _dense_exact_attention(q, k, v, self.scale, causal=True).reshape(B, S, -1)
        attn_out = _linear(attended.to(torch.float16), self.o_proj_weight)
        # hidden = residual + attn_out and the post-attention RMSNorm in one launch
        mlp_in, hidden = K.llama_rms_norm(attn_out, self.post_attention_layernorm_weight, self.rms_norm_eps,
                                          residual=residual)
        gu = _linear(mlp_in, self._gate_up_w)
        inter = self.gate_proj_weight.shape[0]
        act = K.silu_mul(gu[..., :inter], gu[..., inter:])
        if K.use_linear(act, self.down_proj_weight):  # residual add fused into the epilogue
            return K.linear(act, self.down_proj_weight, residual=hidden)
        return hidden + torch.nn.functional.linear(act, self.down_proj_weight)
