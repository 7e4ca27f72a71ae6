"""rfsn_decode_attention_noalloc (library-internal fixed scratch) against rfsn_decode_attention.

The allocation-free entry point has no counterpart in the reference; it must
give the same outputs as the workspace entry point, call after call, and
reject calls whose partials do not fit its fixed buffer.  Both entry points
are called through the C ABI with hand-built argument structs.  This file is
collected last so it also runs after every other GPU test in one process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import restate as R

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from apple_b200 import _lib
    from apple_b200 import kernels as K
    from tests.gpu_util import kv_to_store, to_dev

NOALLOC_BYTES = 4 << 20


def _close(out, ref, what):
    out = np.asarray(out, np.float32)
    ref = np.asarray(ref, np.float32)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    tol = 2e-3 * np.abs(ref) + 2e-3 * rms
    err = np.abs(out - ref)
    assert (err <= tol).all(), f"{what}: max err {err.max():.3e}"


def _args(qz, q, out, qpos, segs, kv_heads, hot=None, warm=None, num_ctas=0):
    B, Qn, Hq, D = q.shape
    a = _lib.AttnArgs()
    a.q, a.out, a.qpos = q.data_ptr(), out.data_ptr(), qpos.data_ptr()
    a.batch, a.queries, a.q_heads, a.kv_heads, a.head_dim = B, Qn, Hq, kv_heads, D
    a.causal, a.scale = 1, float(D ** -0.5)
    if hot is not None:
        a.hot = _lib.DenseStore(hot[0].data_ptr(), hot[1].data_ptr(), hot[0].shape[1], hot[0].shape[0])
    if warm is not None:
        a.warm = warm.struct()
    arr = (_lib.Segment * len(segs))()
    for i, (st, slot, first, count, pos0) in enumerate(segs):
        arr[i].store, arr[i].slot, arr[i].first, arr[i].count, arr[i].pos0 = st, slot, first, count, pos0
    a.segments, a.num_segments, a.num_ctas = arr, len(segs), num_ctas
    a._keep = arr  # keep the segment array alive with the struct
    return a


def _run(fn, a, qz):
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.call(fn, C.byref(a), C.byref(qz.struct()), stream)


def _workspace(a, qz):
    n = C.c_size_t(0)
    _lib.call("rfsn_attention_workspace_size", C.byref(a), C.byref(qz.struct()), C.byref(n))
    return n.value


def test_noalloc_matches_workspace_entry_point_twice():
    rng = np.random.default_rng(7)
    B, Hkv, G, D, ds, S, T_hot, T_warm = 2, 8, 4, 64, 4, 8, 96, 1500
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
    for call in range(2):  # two calls in a row, different queries each time
        q = torch.randn((B, 1, Hq, D), device="cuda").half()
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        a_ref = _args(qz, q, ref, qpos, segs, Hkv, hot=hot, warm=warm)
        ws = torch.zeros(_workspace(a_ref, qz), dtype=torch.uint8, device="cuda")
        a_ref.workspace, a_ref.workspace_bytes = ws.data_ptr(), ws.numel()
        _run("rfsn_decode_attention", a_ref, qz)
        _run("rfsn_decode_attention_noalloc", _args(qz, q, got, qpos, segs, Hkv, hot=hot, warm=warm), qz)
        torch.cuda.synchronize()
        _close(got.cpu().numpy(), ref.cpu().numpy(), f"call {call}")


def test_noalloc_rejects_oversized_call():
    rng = np.random.default_rng(3)
    qz = K.QuantizerBuffers(to_dev(rng.standard_normal((8, 256, 8)).astype(np.float16)), None, 0.0)
    B, Hkv, G, D, T = 64, 8, 8, 64, 64
    q = torch.zeros((B, 1, Hkv * G, D), dtype=torch.float16, device="cuda")
    out = torch.empty_like(q)
    qpos = torch.full((B, 1, Hkv * G), T - 1, dtype=torch.int32, device="cuda")
    hot = (torch.zeros((B * Hkv, T, D), dtype=torch.float16, device="cuda"),
           torch.zeros((B * Hkv, T, D), dtype=torch.float16, device="cuda"))
    a = _args(qz, q, out, qpos, [(K.STORE_HOT, 0, 0, T, 0)], Hkv, hot=hot, num_ctas=2048)
    assert _workspace(a, qz) > NOALLOC_BYTES
    with pytest.raises(_lib.RFSNError) as e:
        _run("rfsn_decode_attention_noalloc", a, qz)
    assert e.value.status == -4
