"""Decode attention replayed from a CUDA graph with new inputs on every replay.

A captured launch keeps its kernel parameters, so every replay of one decode
step runs with the same host call number.  The split-K row merge must still
happen inside every replay: each replay here writes new queries into the
captured input buffer, fills the output with NaN, replays, and compares with an
eager call (and the oracle) on those queries.  Tolerance as the other attention
tests: |out - ref| <= 2e-3 |ref| + 2e-3 rms(ref).
"""
import numpy as np
import pytest
import torch

from oracle import restate as R

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from apple_b200 import kernels as K
    from tests.gpu_util import kv_to_store, to_dev


def _close(out, ref, what):
    out = np.asarray(out, np.float32)
    ref = np.asarray(ref, np.float32)
    assert np.isfinite(out).all(), f"{what}: output not written"
    rms = float(np.sqrt(np.mean(ref ** 2)))
    err = np.abs(out - ref)
    bad = err > 2e-3 * np.abs(ref) + 2e-3 * rms
    assert not bad.any(), f"{what}: {int(bad.sum())} off, max err {err.max():.3e}"


@pytest.mark.parametrize("num_ctas", [0, 7])
def test_attention_graph_replays_track_new_queries(num_ctas):
    rng = np.random.default_rng(21 + num_ctas)
    B, Hkv, G, D, ds, S, T_hot, T_warm = 2, 8, 4, 64, 4, 8, 160, 1800
    M = D // ds
    pq_cb = (rng.standard_normal((M, 256, ds)) * 0.7).astype(np.float16)
    rvq_cb = (rng.standard_normal((1, 256, D)) * 0.2).astype(np.float16)
    oq = R.Quantizer(pq_cb, rvq_cb, -1.0, sparse_topk=S)
    qz = K.QuantizerBuffers(to_dev(pq_cb), to_dev(rvq_cb), -1.0, S)
    k = rng.standard_normal((B, T_hot + T_warm, Hkv, D)).astype(np.float16)
    v = rng.standard_normal((B, T_hot + T_warm, Hkv, D)).astype(np.float16)
    kc = [oq.compress(k[b, :T_warm]) for b in range(B)]
    vc = [oq.compress(v[b, :T_warm]) for b in range(B)]

    def rows(cs):
        return [R.Codes(c.pq[:, h], c.rvq[:, h], c.mask[:, h], c.sp_idx[:, h], c.sp_val[:, h])
                for c in cs for h in range(Hkv)]

    warm = kv_to_store(qz, rows(kc), rows(vc), cap=T_warm)
    hot = (to_dev(np.ascontiguousarray(k[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D))),
           to_dev(np.ascontiguousarray(v[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D))))
    segs = [(K.STORE_WARM, 0, 0, T_warm, 0), (K.STORE_HOT, 0, 0, T_hot, T_warm)]
    Hq = Hkv * G
    T = T_hot + T_warm
    qpos = torch.full((B, 1, Hq), T - 1, dtype=torch.int32, device="cuda")
    q_in = torch.zeros((B, 1, Hq, D), dtype=torch.float16, device="cuda")
    out = torch.empty_like(q_in)
    entry = K.attention_call(qz, q_in, out, segs, kv_heads=Hkv, qpos=qpos, hot=hot, warm=warm, num_ctas=num_ctas,
                             memo=False)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        K.run_attention(entry, q_in, out, qpos, status)
    kw = [np.concatenate([oq.decode(kc[b]), k[b, T_warm:]], 0) for b in range(B)]
    vw = [np.concatenate([oq.decode(vc[b]), v[b, T_warm:]], 0) for b in range(B)]
    for rep in range(4):
        qn = rng.standard_normal((B, 1, Hq, D)).astype(np.float16)
        q_in.copy_(to_dev(qn))
        out.fill_(float("nan"))
        graph.replay()
        eager = torch.empty_like(out)
        K.decode_attention(qz, q_in, eager, segs, kv_heads=Hkv, qpos=qpos, hot=hot, warm=warm, num_ctas=num_ctas)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        got = out.cpu().numpy()
        _close(got, eager.cpu().numpy(), f"replay {rep} vs eager")
        b = rep % B
        ref = R.blockwise_exact_attention(qn[b].reshape(1, Hq, D), kw[b], vw[b], D ** -0.5, 128, True,
                                          np.full((1, Hq), T - 1, np.int32))
        _close(got[b], ref, f"replay {rep} vs oracle")
    del graph
