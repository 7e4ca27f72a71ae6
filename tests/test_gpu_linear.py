"""Weight-streaming projection (rfsn_linear_f16) against a torch fp32 reference.

y = fp16(x32 @ w32^T) (+ the fused epilogues: residual add, tanh-GELU in fp16
steps).  The kernel sums in a different order than the reference, so an
element may differ where the fp32 value sits on an fp16 rounding boundary: at
most one fp16 step, and equal in most elements.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from apple_b200 import kernels as K


def _ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    ai = a.view(torch.int16).int()
    bi = b.view(torch.int16).int()
    ai = torch.where(ai < 0, -32768 - ai, ai)
    bi = torch.where(bi < 0, -32768 - bi, bi)
    return (ai - bi).abs()


def _gelu_chain(h: torch.Tensor) -> torch.Tensor:
    # the layer's fp16 expression, every operation rounded to fp16 (float64 in between)
    r = lambda v: v.to(torch.float16).to(torch.float64)  # noqa: E731
    x = h.to(torch.float64)
    x3 = r(x * x * x)
    inner = r(x + r(0.044715 * x3))
    t = r(torch.tanh(r(0.7978845608 * inner)))
    return (r(0.5 * x) * r(1.0 + t)).to(torch.float16)


@pytest.mark.parametrize("M,N,K", [(1, 64, 256), (7, 192, 512), (32, 2560, 2048), (32, 2048, 4096), (17, 4096, 768)])
@pytest.mark.parametrize("mode", ["none", "residual", "gelu"])
def test_linear_vs_fp32_reference(M, N, K, mode):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    wide = torch.randn((M, K + 64), generator=g, device="cuda").half()
    x = wide[:, 32:32 + K]  # strided rows: the layer passes views of wider activations
    w = (torch.randn((N, K), generator=g, device="cuda") / K ** 0.5).half()
    r = torch.randn((M, N), generator=g, device="cuda").half()
    y = K.linear(x, w, residual=r if mode == "residual" else None, gelu=mode == "gelu")
    ref = (x.float() @ w.float().T).half()
    if mode == "residual":
        ref = (ref.float() + r.float()).half()
    elif mode == "gelu":
        ref = _gelu_chain(ref)
    torch.cuda.synchronize()
    d = _ulps(y, ref)
    assert int(d.max()) <= 1 if mode != "gelu" else int(d.max()) <= 2, (int(d.max()), mode)
    assert float((d == 0).float().mean()) > 0.95


def test_linear_rejects_unsupported_shapes():
    x = torch.zeros((40, 256), dtype=torch.float16, device="cuda")
    w = torch.zeros((64, 256), dtype=torch.float16, device="cuda")
    from apple_b200 import RFSNError
    with pytest.raises(RFSNError):
        K.linear(x, w)  # more than 32 rows
    with pytest.raises(RFSNError):
        K.linear(x[:4, :200].contiguous(), w[:, :200].contiguous())  # K not a multiple of 256
