"""Weight-streaming projection (rfsn_linear_f16) against a torch fp32 reference.

y = fp16(x32 @ w32^T).  The kernel sums in its own fixed order (per-chunk MMA
sums, then the K-chunk shares in order), so it is compared with the float64
product through the error bound of fp32 summation: |y - ref| <= 2^-11 |ref| (the
fp16 rounding) + K 2^-24 sum|x||w| (fp32 accumulation of K products).  Most
elements round to the same fp16 value as the float64 product.  The fused
epilogues are checked exactly against the kernel's own plain product: residual
y = fp16(fp16(acc) + r), and the layer's fp16 tanh-GELU chain within one fp16
step (tanhf's last bit).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from apple_b200 import kernels as kern

SHAPES = [(1, 64, 128), (7, 192, 512), (32, 2560, 2048), (32, 2048, 4096), (17, 4096, 768), (32, 2048, 5632),
          (32, 5632, 2048), (3, 128, 384)]


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


def _inputs(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    wide = torch.randn((M, K + 64), generator=g, device="cuda").half()
    x = wide[:, 32:32 + K]  # strided rows: the layer passes views of wider activations
    w = (torch.randn((N, K), generator=g, device="cuda") / K ** 0.5).half()
    r = torch.randn((M, N), generator=g, device="cuda").half()
    return x, w, r


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_vs_fp32_reference(M, N, K):
    x, w, r = _inputs(M, N, K, M * 7 + N + K)
    y = kern.linear(x, w)
    ref = x.double() @ w.double().T
    bound = 2.0 ** -11 * ref.abs() + K * 2.0 ** -24 * (x.double().abs() @ w.double().abs().T)
    err = (y.double() - ref).abs()
    assert bool((err <= bound).all()), float((err / bound).max())
    assert float((y == ref.half()).float().mean()) > 0.9
    # fused epilogues on the same sums
    y_res = kern.linear(x, w, residual=r)
    assert torch.equal(y_res, (y.float() + r.float()).half())
    y_gelu = kern.linear(x, w, gelu=True)
    dg = _ulps(y_gelu, _gelu_chain(y))
    assert int(dg.max()) <= 1 and int((dg != 0).sum()) <= max(2, dg.numel() // 1000), (int(dg.max()), int((dg != 0).sum()))
    # the sum order is fixed: a second call is bit-identical
    assert torch.equal(kern.linear(x, w), y)


def test_linear_chain_in_graph_replays():
    """Two projections back to back on one stream (the second starts early under programmatic
    dependent launch and shares the workspace), captured once and replayed on new inputs."""
    M, H, F = 32, 2048, 5632
    g = torch.Generator(device="cuda").manual_seed(5)
    w1 = (torch.randn((F, H), generator=g, device="cuda") / H ** 0.5).half()
    w2 = (torch.randn((H, F), generator=g, device="cuda") / F ** 0.5).half()
    x = torch.randn((M, H), generator=g, device="cuda").half()
    res = torch.randn((M, H), generator=g, device="cuda").half()

    def chain():
        a = kern.linear(x, w1, gelu=True)
        return kern.linear(a, w2, residual=res)

    for _ in range(2):
        chain()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        out = chain()
    for i in range(4):
        x.copy_(torch.randn((M, H), generator=g, device="cuda").half())
        res.copy_(torch.randn((M, H), generator=g, device="cuda").half())
        out.fill_(float("nan"))
        graph.replay()
        want = chain()
        torch.cuda.synchronize()
        assert torch.equal(out, want), i
    del graph


def test_linear_rejects_unsupported_shapes():
    x = torch.zeros((40, 256), dtype=torch.float16, device="cuda")
    w = torch.zeros((64, 256), dtype=torch.float16, device="cuda")
    from apple_b200 import RFSNError
    with pytest.raises(RFSNError):
        kern.linear(x, w)  # more than 32 rows
    with pytest.raises(RFSNError):
        kern.linear(x[:4, :200].contiguous(), w[:, :200].contiguous())  # K not a multiple of 128
