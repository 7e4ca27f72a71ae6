"""Torch-CPU stand-in for the subset of ``mlx.nn`` the RFSN reference uses.

TEST INFRASTRUCTURE ONLY (see ``mlx/core.py``).  ``Module`` is a plain
attribute container; ``Linear`` computes ``x @ W.T`` with W ~ U(-1/sqrt(in),
1/sqrt(in)) (MLX's default init) drawn from the shim's seeded generator;
``RMSNorm`` computes ``x * rsqrt(mean(x^2) + eps) * weight`` in float32 and
returns the input dtype, as MLX's ``fast.rms_norm`` does.
"""
from __future__ import annotations

import math

import torch as _torch

from . import core as mx


class Module:
    def __init__(self):
        pass

    def __call__(self, *args, **kwargs):
        raise NotImplementedError


class Linear(Module):
    def __init__(self, input_dims: int, output_dims: int, bias: bool = True):
        super().__init__()
        scale = math.sqrt(1.0 / input_dims)
        w = (_torch.rand((output_dims, input_dims), generator=mx.random.gen) * 2 - 1) * scale
        self.weight = mx._wrap(w, mx.float32)
        self.bias = mx._wrap(_torch.zeros(output_dims), mx.float32) if bias else None

    def __call__(self, x: mx.array) -> mx.array:
        w = self.weight._t.to(x._t.dtype)
        y = x._t @ w.T
        if self.bias is not None:
            y = y + self.bias._t.to(y.dtype)
        return mx._wrap(y)


class RMSNorm(Module):
    def __init__(self, dims: int, eps: float = 1e-5):
        super().__init__()
        self.weight = mx._wrap(_torch.ones(dims), mx.float32)
        self.eps = eps

    def __call__(self, x: mx.array) -> mx.array:
        xf = x._t.float()
        y = xf * _torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps) * self.weight._t
        return mx._wrap(y.to(x._t.dtype))
