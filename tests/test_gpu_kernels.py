"""GPU parity of the C-ABI kernels against the CPU oracle and the reference's golden fixtures.

Tolerances:
* PQ/RVQ/sparse codes: bit-exact, except where the two best candidates tie to
  fp32 rounding, proven per mismatch in float64 against the rounding bound of
  the reference's distance formula (tests/parity.py); RVQ codes are compared on
  vectors whose PQ codes agree, sparse codes where PQ and RVQ agree.
* decoded K/V (rfsn_decode_codes): bit-exact fp16 (well inside 1e-3 absolute).
* attention outputs: |out - ref| <= 2e-3 * |ref| + 2e-3 * rms(ref) element-wise
  (fp32 accumulation; keys and values are the materialised fp16 window, so
  only the summation order differs from the oracle).
"""
import numpy as np
import pytest
import torch

from oracle import restate as R
from tests.conftest import GOLDEN
from tests.parity import prove_ties, rvq_ties_ok

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from apple_b200 import kernels as K
    from tests.gpu_util import codes_to_store, kv_to_store, to_dev

QUANT_CASES = ["quant_d128_m8x16_rvq3", "quant_d64_m16x4_rvq1_dense", "quant_d64_m8x8_rvq1", "quant_d64_m8x8_pqonly"]


def assert_attn_close(out, ref, what=""):
    out = np.asarray(out, np.float32)
    ref = np.asarray(ref, np.float32)
    rms = float(np.sqrt(np.mean(ref ** 2))) if ref.size else 0.0
    err = np.abs(out - ref)
    tol = 2e-3 * np.abs(ref) + 2e-3 * rms
    bad = err > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} elements off, max err {err.max():.3e} (rms ref {rms:.3e})"


def quantizer_from(g, sparse=0):
    return K.QuantizerBuffers(to_dev(g["pq_codebooks"]), to_dev(g["rvq_codebooks"]), float(g["threshold"]), sparse)


def pq_tie_ok(x, cb, got, want):
    """Every PQ code mismatch is a proven fp32 distance tie."""
    ds = cb.shape[2]
    n, m = np.nonzero(got != want)
    if n.size:
        sub = x.reshape(x.shape[0], -1, ds)[n, m].astype(np.float64)
        ok = prove_ties(sub, cb[m, got[n, m]].astype(np.float64), cb[m, want[n, m]].astype(np.float64))
        assert ok.all(), f"{int((~ok).sum())} PQ code mismatches are not fp32 ties"


@pytest.mark.parametrize("name", QUANT_CASES)
def test_encode_matches_reference_codes(name):
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    qz = quantizer_from(g)
    x = to_dev(g["x"])
    N, D = x.shape
    store = K.CodeStoreBuffers(qz, rows=1, cap=N)
    res = torch.empty_like(x)
    K.encode(qz, x.view(1, N, 1, D), store, 0, 0, residual_out=res.view(1, N, 1, D))
    torch.cuda.synchronize()
    pq = store.read(0, "pq", 0, 0, 0, N).cpu().numpy()
    pq_tie_ok(g["x"], g["pq_codebooks"], pq, g["pq_codes"])
    agree = (pq == g["pq_codes"]).all(axis=1)
    assert agree.mean() > 0.99
    np.testing.assert_array_equal(res.cpu().numpy()[agree].view(np.uint16), g["residual"][agree].view(np.uint16))
    if qz.L:
        mask = store.read(0, "active", 0, 0, 0, N)[:, 0].cpu().numpy().astype(bool)
        np.testing.assert_array_equal(mask[agree], g["rvq_mask"][agree])
        dense = np.zeros((N, qz.L), np.int64)
        dense[g["rvq_offsets"]] = g["rvq_codes"]
        got = store.read(0, "rvq", 0, 0, 0, N).cpu().numpy().astype(np.int64)
        sel = agree & g["rvq_mask"]
        if sel.any():
            rvq_ties_ok(g["residual"][sel], g["rvq_codebooks"], got[sel], dense[sel])


@pytest.mark.parametrize("name", QUANT_CASES)
def test_decode_codes_bit_exact(name):
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    qz = quantizer_from(g)
    N, D = g["x"].shape
    dense = np.zeros((N, qz.L), np.uint16)
    dense[g["rvq_offsets"]] = g["rvq_codes"]
    codes = R.Codes(g["pq_codes"][:, None], dense[:, None], g["rvq_mask"][:, None],
                    np.zeros((N, 1, 0), np.uint8), np.zeros((N, 1, 0), np.float16))
    store = codes_to_store(qz, [R.Codes(codes.pq[:, 0], codes.rvq[:, 0], codes.mask[:, 0], codes.sp_idx[:, 0],
                                        codes.sp_val[:, 0])], cap=N)
    out = torch.empty((1, N, 1, D), dtype=torch.float16, device="cuda")
    K.decode_codes(qz, store, 0, 0, N, out)
    np.testing.assert_array_equal(out.cpu().numpy()[0, :, 0].view(np.uint16), g["decoded"].view(np.uint16))


def test_sparse_encode_and_decode_match_oracle():
    g = dict(np.load(GOLDEN / "quant_d64_m16x4_rvq1_dense.npz"))
    S = 8
    qz = quantizer_from(g, sparse=S)
    oq = R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], float(g["threshold"]), sparse_topk=S)
    x = g["x"]
    N, D = x.shape
    ref = oq.compress(x[:, None])
    store = K.CodeStoreBuffers(qz, rows=1, cap=N)
    K.encode(qz, to_dev(x).view(1, N, 1, D), store, 0, 0)
    pq = store.read(0, "pq", 0, 0, 0, N).cpu().numpy()
    agree = (pq == ref.pq[:, 0]).all(axis=1)
    assert agree.mean() > 0.99
    np.testing.assert_array_equal(store.read(0, "sp_idx", 0, 0, 0, N).cpu().numpy()[agree], ref.sp_idx[agree, 0])
    np.testing.assert_array_equal(store.read(0, "sp_val", 0, 0, 0, N).cpu().numpy()[agree].view(np.uint16),
                                  ref.sp_val[agree, 0].view(np.uint16))
    # decode of the oracle's codes is bit-exact with the oracle decode
    st2 = codes_to_store(qz, [R.Codes(ref.pq[:, 0], ref.rvq[:, 0], ref.mask[:, 0], ref.sp_idx[:, 0],
                                      ref.sp_val[:, 0])], cap=N)
    out = torch.empty((1, N, 1, D), dtype=torch.float16, device="cuda")
    K.decode_codes(qz, st2, 0, 0, N, out)
    np.testing.assert_array_equal(out.cpu().numpy()[0, :, 0].view(np.uint16), oq.decode(ref)[:, 0].view(np.uint16))


def _qpos_global(adjusted, window_start, shape):
    a = np.broadcast_to(np.asarray(adjusted, np.int32).reshape(shape[0], -1), shape[:2]).astype(np.int64)
    return (np.maximum(a, -1) + window_start).astype(np.int32)


def test_hybrid_attention_golden():
    """RFSNHybridAttentionMLX case of the reference suite (rfsn_v10_mlx_ane_complete.py:418-446)."""
    g = dict(np.load(GOLDEN / "attention_hybrid.npz"))
    qz = quantizer_from(g)
    oq = R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], float(g["threshold"]))
    kc, vc = oq.compress(g["keys"]), oq.compress(g["values"])
    H, T = 4, 24
    ws = kv_to_store(qz, [R.Codes(kc.pq[:, h], kc.rvq[:, h], kc.mask[:, h], kc.sp_idx[:, h], kc.sp_val[:, h])
                          for h in range(H)],
                     [R.Codes(vc.pq[:, h], vc.rvq[:, h], vc.mask[:, h], vc.sp_idx[:, h], vc.sp_val[:, h])
                      for h in range(H)], cap=T)
    q = to_dev(g["q"]).view(1, 2, H, 128)  # two queries against one sequence
    out = torch.empty_like(q)
    seg = [(K.STORE_WARM, 0, 0, T, 0)]
    for key, causal, pos in (("out_causal", True, g["positions"]), ("out_plain", False, None),
                             ("out_bh", True, g["positions_bh"])):
        qpos = None
        if causal:
            qpos = to_dev(np.broadcast_to(np.asarray(pos, np.int32).reshape(2, -1), (2, H)).reshape(1, 2, H).copy())
        K.decode_attention(qz, q, out, seg, kv_heads=H, qpos=qpos, causal=causal, warm=ws)
        assert_attn_close(out.cpu().numpy()[0], g[key], key)


def _oracle_cache_from_golden(g):
    cfg = R.OracleConfig(hidden_dim=512, num_heads=4, head_dim=128, num_subspaces=8, subspace_dim=16,
                         num_rvq_layers=3, rvq_codebook_size=256, rvq_sparsity_threshold=0.25,
                         hot_capacity=16, warm_capacity=24, block_size_seq=16)
    oq = R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], float(g["threshold"]))
    c = R.OracleCache(cfg, oq, batch=1)
    s = int(g["update_split"])
    c.update(g["keys"][None, :s], g["values"][None, :s])
    c.update(g["keys"][None, s:], g["values"][None, s:])
    return c


@pytest.mark.parametrize("num_ctas", [0, 1, 3, 37])
def test_tiered_attention_golden(num_ctas):
    """hot + warm + two cold chunks (cache.py tiering) vs the reference's outputs, all windows."""
    g = dict(np.load(GOLDEN / "cache_tiers.npz"))
    oc = _oracle_cache_from_golden(g)
    qz = quantizer_from(g)
    H, D = 4, 128
    hot_k = to_dev(np.ascontiguousarray(g["keys"][:16].transpose(1, 0, 2)))
    hot_v = to_dev(np.ascontiguousarray(g["values"][:16].transpose(1, 0, 2)))

    def rows(c):
        return [R.Codes(c.pq[:, h], c.rvq[:, h], c.mask[:, h], c.sp_idx[:, h], c.sp_val[:, h]) for h in range(H)]

    ws = kv_to_store(qz, rows(oc.warm_k[0]), rows(oc.warm_v[0]), cap=32)
    cst = K.CodeStoreBuffers(qz, rows=H, cap=16, slots=len(oc.cold))
    for i, meta in enumerate(oc.cold):
        kv_to_store(qz, rows(meta["k"][0]), rows(meta["v"][0]), cap=16, store=cst, slot=i)
    q = to_dev(g["q"]).view(1, 1, H, D)
    out = torch.empty_like(q)
    spans = [(K.STORE_HOT, 0, 0, 16), (K.STORE_WARM, 0, 16, 24)] + \
            [(K.STORE_COLD, i, m["start_token"], m["num_tokens"]) for i, m in enumerate(oc.cold)]
    for i, (qpos, win) in enumerate(g["cases"]):
        tag = f"q{i // 3}_w{i % 3}"
        win = None if win < 0 else int(win)
        start, end, adj = R.window_bounds(60, [int(qpos)], win, None)
        segs = []
        for st, slot, s0, n in spans:
            a, b = max(start, s0), min(end, s0 + n)
            if a < b:
                segs.append((st, slot, a - s0, b - a, a))
        qp = to_dev(_qpos_global(adj, start, (1, 1)).repeat(H).reshape(1, 1, H))
        K.decode_attention(qz, q, out, segs, kv_heads=H, qpos=qp, causal=True, hot=(hot_k, hot_v),
                           warm=ws, cold=cst, num_ctas=num_ctas)
        assert_attn_close(out.cpu().numpy()[0], g[f"{tag}_out"], tag)


def _make_cfg2_like(rng, B, Hkv, G, D, T_hot, T_warm, S=8, ds=4, L=1, thr=-1.0, outliers=4):
    M = D // ds
    pq_cb = (rng.standard_normal((M, 256, ds)) * np.sqrt(2.0 / ds)).astype(np.float16)
    rvq_cb = (rng.standard_normal((L, 256, D)) * np.sqrt(2.0 / D)).astype(np.float16) if L else \
        np.zeros((0, 256, D), np.float16)
    if L:
        rvq_cb[:, 0] = 0
    T = T_hot + T_warm
    k = rng.standard_normal((B, T, Hkv, D)).astype(np.float32)
    if outliers:
        k[..., rng.choice(D, outliers, replace=False)] *= 10
    k = k.astype(np.float16)
    v = rng.standard_normal((B, T, Hkv, D)).astype(np.float16)
    return pq_cb, rvq_cb, k, v


@pytest.mark.parametrize("B,Hkv,G,Qn,D,ds,L,S,thr,T_hot,T_warm,num_ctas", [
    (2, 8, 4, 1, 64, 4, 1, 8, -1.0, 300, 2000, 0),     # config-2 shape (small T)
    (2, 8, 4, 1, 64, 4, 1, 8, -1.0, 300, 2000, 5),
    (1, 4, 2, 4, 64, 8, 2, 0, 0.5, 64, 700, 0),        # R = 8 query rows per KV head, gated RVQ
    (3, 2, 1, 1, 64, 8, 0, 0, 0.0, 128, 1000, 11),     # PQ only, no GQA
    (1, 2, 2, 1, 128, 16, 1, 4, -1.0, 50, 400, 0),     # D = 128
    (1, 4, 4, 1, 64, 4, 1, 0, 0.5, 100, 900, 7),       # PQ 16x4 + gated RVQ (masked preset)
    (2, 2, 2, 1, 64, 8, 1, 0, 0.5, 33, 777, 0),        # PQ 8x8 + gated RVQ (masked preset)
    (1, 2, 1, 2, 64, 4, 1, 4, -1.0, 17, 500, 3),       # dense RVQ, top-4 sparse (generic path)
    (1, 2, 4, 1, 64, 4, 1, 12, -1.0, 40, 300, 0),      # top-12 sparse: two entries per lane
    (1, 2, 4, 2, 64, 4, 1, 8, -1.0, 64, 600, 0),       # config-2 preset with R = 8 query rows
    (2, 2, 1, 1, 64, 4, 1, 8, -1.0, 32, 500, 3),       # config-2 preset with R = 1
    (2, 4, 8, 1, 64, 8, 0, 0, 0.0, 48, 1013, 5),       # config-3 preset (PQ 8x8, GQA 8): partial 32-token chunks
])
def test_fused_attention_vs_oracle(B, Hkv, G, Qn, D, ds, L, S, thr, T_hot, T_warm, num_ctas):
    rng = np.random.default_rng(B * 1000 + Hkv * 10 + D + L)
    pq_cb, rvq_cb, k, v = _make_cfg2_like(rng, B, Hkv, G, D, T_hot, T_warm, S=S, ds=ds, L=L, thr=thr)
    oq = R.Quantizer(pq_cb, rvq_cb, thr, sparse_topk=S)
    qz = K.QuantizerBuffers(to_dev(pq_cb), to_dev(rvq_cb) if L else None, thr, S)
    # warm = oldest tokens (encoded), hot = newest (exact), like hot_policy="recent"
    kc = [oq.compress(k[b, :T_warm]) for b in range(B)]
    vc = [oq.compress(v[b, :T_warm]) for b in range(B)]

    def rows(cs):
        return [R.Codes(c.pq[:, h], c.rvq[:, h], c.mask[:, h], c.sp_idx[:, h], c.sp_val[:, h])
                for c in cs for h in range(Hkv)]

    ws = kv_to_store(qz, rows(kc), rows(vc), cap=T_warm)
    hot_k = to_dev(np.ascontiguousarray(k[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D)))
    hot_v = to_dev(np.ascontiguousarray(v[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D)))
    Hq = Hkv * G
    q = rng.standard_normal((B, Qn, Hq, D)).astype(np.float16)
    T = T_hot + T_warm
    pos = rng.integers(T // 2, T, size=(B, Qn, Hq)).astype(np.int32)
    pos[:, 0, 0] = T - 1
    segs = [(K.STORE_WARM, 0, 0, T_warm, 0), (K.STORE_HOT, 0, 0, T_hot, T_warm)]
    out = torch.empty((B, Qn, Hq, D), dtype=torch.float16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.decode_attention(qz, to_dev(q), out, segs, kv_heads=Hkv, qpos=to_dev(pos), causal=True,
                       hot=(hot_k, hot_v), warm=ws, num_ctas=num_ctas, device_status=status)
    got = out.cpu().numpy()
    assert int(status.item()) == 0
    for b in range(B):
        kw = np.concatenate([oq.decode(kc[b]), k[b, T_warm:]], 0)
        vw = np.concatenate([oq.decode(vc[b]), v[b, T_warm:]], 0)
        ref = R.blockwise_exact_attention(q[b].reshape(Qn, Hq, D), kw, vw, D ** -0.5, 128, True, pos[b])
        assert_attn_close(got[b], ref, f"batch {b}")


def test_empty_window_writes_zeros():
    rng = np.random.default_rng(0)
    pq_cb = rng.standard_normal((8, 256, 8)).astype(np.float16)
    qz = K.QuantizerBuffers(to_dev(pq_cb), None, 0.0)
    q = torch.randn(1, 1, 4, 64, device="cuda").half()
    out = torch.full_like(q, 7.0)
    K.decode_attention(qz, q, out, [], kv_heads=4, qpos=torch.zeros(1, 1, 4, dtype=torch.int32, device="cuda"))
    assert torch.count_nonzero(out).item() == 0


def test_abi_rejects_out_of_range_segment():
    rng = np.random.default_rng(1)
    pq_cb = rng.standard_normal((8, 256, 8)).astype(np.float16)
    qz = K.QuantizerBuffers(to_dev(pq_cb), None, 0.0)
    st = K.CodeStoreBuffers(qz, rows=4, cap=32)
    q = torch.randn(1, 1, 4, 64, device="cuda").half()
    out = torch.empty_like(q)
    from apple_b200 import RFSNError
    with pytest.raises(RFSNError):
        K.decode_attention(qz, q, out, [(K.STORE_WARM, 0, 20, 20, 0)], kv_heads=4, causal=False, warm=st)


@pytest.mark.parametrize("ds,L,thr,S,T", [(8, 1, 0.5, 0, 1249), (4, 1, -1.0, 8, 1249), (8, 0, 0.0, 0, 1249),
                                          (4, 1, 0.5, 0, 1249), (8, 1, -1.0, 4, 1249),
                                          (8, 0, 0.0, 0, 37), (4, 1, -1.0, 8, 37)])
def test_tensor_core_encoder_vs_oracle(ds, L, thr, S, T):
    """Spill encoder on tensor cores (D = 64 presets) vs the oracle on strided, ragged input:
    B=2 sequences x T tokens x 2 heads (not a multiple of the 16-vector tile).  T = 1249 runs
    one warp per 16-vector group; T = 37 (a decode-sized append) runs split mode, one warp
    per PQ subspace."""
    rng = np.random.default_rng(100 * ds + 10 * L + S)
    D, M = 64, 64 // ds
    pq_cb = (rng.standard_normal((M, 256, ds)) * 0.8).astype(np.float16)
    rvq_cb = (rng.standard_normal((1, 256, D)) * 0.3).astype(np.float16)
    rvq_cb[:, 0] = 0
    big = rng.standard_normal((2, 1300, 2, D)).astype(np.float32)
    big[..., rng.choice(D, 4, replace=False)] *= 6.0
    big = big.astype(np.float16)
    T0 = 30
    x = big[:, T0:T0 + T]
    oq = R.Quantizer(pq_cb, rvq_cb if L else np.zeros((0, 256, D), np.float16), thr, sparse_topk=S)
    qz = K.QuantizerBuffers(to_dev(pq_cb), to_dev(rvq_cb) if L else None, thr, S)
    xd = to_dev(big)[:, T0:T0 + T]  # strided view: stride_t = 2*D, stride_b = 1300*2*D
    store = K.CodeStoreBuffers(qz, rows=2 * 2, cap=T + 7)
    res = torch.empty_like(to_dev(big))[:, T0:T0 + T]
    K.encode(qz, xd, store, 0, 7, residual_out=res)
    torch.cuda.synchronize()
    for b in range(2):
        ref = oq.compress(x[b])
        _, residual = R.pq_quantize(x[b].reshape(-1, D), pq_cb)
        for h in range(2):
            row = b * 2 + h
            pq = store.read(0, "pq", 0, row, 7, T).cpu().numpy()
            pq_tie_ok(x[b, :, h], pq_cb, pq, ref.pq[:, h])
            agree = (pq == ref.pq[:, h]).all(axis=1)
            assert (~agree).sum() <= max(1, T // 100)  # fp32 distance ties only (checked above)
            got_res = res[b, :, h].cpu().numpy()
            np.testing.assert_array_equal(got_res[agree].view(np.uint16),
                                          residual.reshape(T, 2, D)[agree, h].view(np.uint16))
            if L:
                act = store.read(0, "active", 0, row, 7, T)[:, 0].cpu().numpy().astype(bool)
                np.testing.assert_array_equal(act[agree], ref.mask[agree, h])
                rv = store.read(0, "rvq", 0, row, 7, T).cpu().numpy()[:, :1].astype(np.int64)
                sel = agree & ref.mask[:, h]
                rvq_ties_ok(residual.reshape(T, 2, D)[sel, h], rvq_cb, rv[sel], ref.rvq[sel, h, :1].astype(np.int64))
                sel = sel & (rv[:, 0] == ref.rvq[:, h, 0])
            else:
                sel = agree
            if S:
                np.testing.assert_array_equal(store.read(0, "sp_idx", 0, row, 7, T).cpu().numpy()[sel],
                                              ref.sp_idx[sel, h])
                np.testing.assert_array_equal(
                    store.read(0, "sp_val", 0, row, 7, T).cpu().numpy()[sel].view(np.uint16),
                    ref.sp_val[sel, h].view(np.uint16))


def _ulp_diff(a, b):
    ai = a.view(torch.int16).int()
    bi = b.view(torch.int16).int()
    # map sign-magnitude fp16 bit patterns to a monotonic integer line
    ai = torch.where(ai < 0, -32768 - ai, ai)
    bi = torch.where(bi < 0, -32768 - bi, bi)
    return (ai - bi).abs()


@pytest.mark.parametrize("rows,dim,offset", [(32, 2048, 0), (3, 1000, 0), (5, 512, 1)])
def test_fused_rmsnorm_vs_torch_chain(rows, dim, offset):
    """rfsn_rmsnorm_f16 vs the layer's tensor-op RMSNorm (fp32 math): at most one fp16 step
    apart (the sum of squares is reduced in another order), and almost all bit-exact.
    dim 1000 and a 2-byte offset view take the scalar path."""
    from apple_b200.layer import _RMSNorm
    g = torch.Generator(device="cuda").manual_seed(rows * dim)
    base = (torch.randn(rows * dim + offset, generator=g, device="cuda") * 3).half()
    x = base[offset:].view(rows, dim)
    w = torch.rand(dim, generator=g, device="cuda") + 0.5
    xf = x.float()
    ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w).half()
    got = K.rms_norm(x, w, 1e-5)
    d = _ulp_diff(got, ref)
    assert int(d.max()) <= 1
    assert float((d == 0).float().mean()) > 0.99
    norm = _RMSNorm(dim, "cuda")
    norm.weight = w
    assert torch.equal(norm(x), got)


def _gelu_chain64(x16: np.ndarray) -> np.ndarray:
    """attention.py:137-138 operation by operation: float64 math, fp16 rounding after each step."""
    r = lambda a: a.astype(np.float16).astype(np.float64)  # noqa: E731
    x = x16.astype(np.float64)
    x3 = r(x * x * x)
    inner = r(x + r(0.044715 * x3))
    t = r(np.tanh(r(0.7978845608 * inner)))
    return (r(0.5 * x) * r(1.0 + t)).astype(np.float16)


@pytest.mark.parametrize("n", [32 * 4096, 1001])
def test_fused_gelu_vs_fp16_chain(n):
    """rfsn_gelu_tanh_f16 vs the layer's fp16 expression evaluated with accurate math
    (float64, fp16 rounding after every operation): bit-exact except where tanhf's last
    fp32 bit crosses an fp16 rounding boundary, which moves the result by one fp16 step
    of itself or, near tanh = -1, by one step of tanh (2^-11) times 0.5 x.  Also close to
    the torch tensor chain the layer used before (its fp16 tanh differs in rounding)."""
    from apple_b200.attention import _gelu
    g = torch.Generator(device="cuda").manual_seed(n)
    x = (torch.randn(n, generator=g, device="cuda") * 2.5).half()
    x[:8] = torch.tensor([0.0, -0.0, 1e-4, -1e-4, 6.0, -6.0, 30.0, -30.0], device="cuda").half()
    got = K.gelu_tanh(x).cpu()
    ref = torch.from_numpy(_gelu_chain64(x.cpu().numpy()))
    err = (got.float() - ref.float()).abs()
    ulp_ref = torch.exp2(torch.floor(torch.log2(ref.float().abs().clamp_min(2.0 ** -14))) - 10)
    bound = torch.maximum(ulp_ref, 0.5 * x.cpu().float().abs() * 2.0 ** -11)
    assert bool((err <= bound * 1.0001).all()), f"max err {float(err.max())}"
    assert float((err == 0).float().mean()) > 0.999
    torch_chain = _gelu(x).cpu()
    assert float((torch_chain == got).float().mean()) > 0.99


@pytest.mark.parametrize("D,ds,L,S,T", [(64, 8, 0, 0, 1), (64, 4, 1, 8, 3), (64, 8, 1, 4, 700), (128, 16, 1, 0, 5)])
def test_encode_kv_matches_two_calls(D, ds, L, S, T):
    """rfsn_encode_kv (K and V in one launch) writes the same store bytes as rfsn_encode with
    kv = 0 and kv = 1: decode-sized appends (split mode), a large batch (one warp per group)
    and a configuration outside the tensor-core encoder (D = 128, 16-dim subspaces)."""
    rng = np.random.default_rng(D + ds + T)
    M = D // ds
    pq_cb = rng.standard_normal((M, 256, ds)).astype(np.float16)
    rvq_cb = (rng.standard_normal((1, 256, D)) * 0.3).astype(np.float16)
    rvq_cb[:, 0] = 0
    qz = K.QuantizerBuffers(to_dev(pq_cb), to_dev(rvq_cb) if L else None, 0.2, S)
    kv = torch.from_numpy(rng.standard_normal((2, 3, T, 4, D)).astype(np.float16)).cuda()
    k, v = kv[0], kv[1]
    one = K.CodeStoreBuffers(qz, rows=12, cap=K.align16(T + 5))
    two = K.CodeStoreBuffers(qz, rows=12, cap=K.align16(T + 5))
    K.encode_kv(qz, k, v, one, 0, 5)
    K.encode(qz, k, two, 0, 5, kv=0)
    K.encode(qz, v, two, 0, 5, kv=1)
    torch.cuda.synchronize()
    assert torch.equal(one.data, two.data)


@pytest.mark.parametrize("Qn", [1, 2])
def test_fused_attention_strided_queries(Qn):
    """q as a view with a batch stride (the query heads of a wider projection output) gives
    bit-identical outputs to the packed copy; a batch stride that is not a multiple of 8
    elements is refused."""
    rng = np.random.default_rng(7 + Qn)
    B, Hkv, G, D, T_hot, T_warm = 3, 2, 4, 64, 48, 160
    pq_cb, rvq_cb, k, v = _make_cfg2_like(rng, B, Hkv, G, D, T_hot, T_warm, S=8, ds=4, L=1, thr=-1.0)
    oq = R.Quantizer(pq_cb, rvq_cb, -1.0, sparse_topk=8)
    qz = K.QuantizerBuffers(to_dev(pq_cb), to_dev(rvq_cb), -1.0, 8)
    kc = [oq.compress(k[b, :T_warm]) for b in range(B)]
    vc = [oq.compress(v[b, :T_warm]) for b in range(B)]

    def rows(cs):
        return [R.Codes(c.pq[:, h], c.rvq[:, h], c.mask[:, h], c.sp_idx[:, h], c.sp_val[:, h])
                for c in cs for h in range(Hkv)]

    ws = kv_to_store(qz, rows(kc), rows(vc), cap=T_warm)
    hot_k = to_dev(np.ascontiguousarray(k[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D)))
    hot_v = to_dev(np.ascontiguousarray(v[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D)))
    Hq = Hkv * G
    wide = torch.from_numpy(rng.standard_normal((B, Qn * Hq * D + 320)).astype(np.float16)).cuda()
    qv = wide[:, :Qn * Hq * D].view(B, Qn, Hq, D)  # batch stride Qn*Hq*D + 320
    segs = [(K.STORE_WARM, 0, 0, T_warm, 0), (K.STORE_HOT, 0, 0, T_hot, T_warm)]
    out_v = torch.empty((B, Qn, Hq, D), dtype=torch.float16, device="cuda")
    out_c = torch.empty_like(out_v)
    K.decode_attention(qz, qv, out_v, segs, kv_heads=Hkv, causal=False, hot=(hot_k, hot_v), warm=ws)
    K.decode_attention(qz, qv.contiguous(), out_c, segs, kv_heads=Hkv, causal=False, hot=(hot_k, hot_v), warm=ws)
    torch.cuda.synchronize()
    assert torch.equal(out_v, out_c)
    odd = torch.zeros((B, Qn * Hq * D + 4), dtype=torch.float16, device="cuda")[:, :Qn * Hq * D].view(B, Qn, Hq, D)
    with pytest.raises(ValueError):
        K.decode_attention(qz, odd, out_v, segs, kv_heads=Hkv, causal=False, hot=(hot_k, hot_v), warm=ws)


def test_patched_call_matches_fresh_call():
    """A prepared call (attention_call with memo=False) whose segments are patched step by
    step, as a decode loop over a growing window does, gives bit-identical outputs to a
    call prepared afresh for each window; a workspace the library finds too small is sized
    again and the launch retried (the library refuses such a launch before it starts)."""
    rng = np.random.default_rng(23)
    B, Hkv, G, D, T_hot, T_warm = 3, 2, 4, 64, 48, 1600
    pq_cb, rvq_cb, k, v = _make_cfg2_like(rng, B, Hkv, G, D, T_hot, T_warm, S=8, ds=4, L=1, thr=-1.0)
    oq = R.Quantizer(pq_cb, rvq_cb, -1.0, sparse_topk=8)
    qz = K.QuantizerBuffers(to_dev(pq_cb), to_dev(rvq_cb), -1.0, 8)
    kc = [oq.compress(k[b, :T_warm]) for b in range(B)]
    vc = [oq.compress(v[b, :T_warm]) for b in range(B)]

    def rows(cs):
        return [R.Codes(c.pq[:, h], c.rvq[:, h], c.mask[:, h], c.sp_idx[:, h], c.sp_val[:, h])
                for c in cs for h in range(Hkv)]

    ws = kv_to_store(qz, rows(kc), rows(vc), cap=T_warm)
    hot_k = to_dev(np.ascontiguousarray(k[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D)))
    hot_v = to_dev(np.ascontiguousarray(v[:, T_warm:].transpose(0, 2, 1, 3).reshape(B * Hkv, T_hot, D)))
    q = to_dev(rng.standard_normal((B, 1, Hkv * G, D)).astype(np.float16))
    kw = dict(kv_heads=Hkv, causal=False, hot=(hot_k, hot_v), warm=ws)

    def segs(n):  # the newest n warm tokens, then the hot tokens
        return [(K.STORE_WARM, 0, T_warm - n, n, T_warm - n), (K.STORE_HOT, 0, 0, T_hot, T_warm)]

    out_p = torch.empty_like(q)
    out_f = torch.empty_like(q)
    entry = K.attention_call(qz, q, out_p, segs(16), memo=False, **kw)
    for step, n in enumerate([16, 17, 200, 1599, 1600, 40]):
        s = segs(n)
        K.patch_segments(entry, s)
        if step == 3:
            entry.args.workspace_bytes = 16  # refused by the library, then sized again
        K.run_attention(entry, q, out_p)
        K.decode_attention(qz, q, out_f, s, **kw)
        torch.cuda.synchronize()
        assert torch.equal(out_p, out_f), f"window of {n} warm tokens"
    import ctypes as C
    need = C.c_size_t(0)
    K.call("rfsn_attention_workspace_size", C.byref(entry.args), C.byref(entry.qs), C.byref(need))
    assert entry.args.workspace_bytes >= need.value
    with pytest.raises(ValueError):
        K.patch_segments(entry, segs(8)[:1])  # the segment count is part of the prepared call


@pytest.mark.parametrize("rows,dim,offset", [(32, 2048, 0), (3, 1000, 0)])
def test_fused_add_rmsnorm(rows, dim, offset):
    """rfsn_add_rmsnorm_f16: the sum is the fp16 tensor add bit for bit, and the normalised
    output equals rfsn_rmsnorm_f16 of that sum bit for bit (dim 1000 takes the scalar path)."""
    g = torch.Generator(device="cuda").manual_seed(rows + dim)
    x = (torch.randn((rows, dim), generator=g, device="cuda") * 2).half()
    b = (torch.randn((rows, dim), generator=g, device="cuda") * 2).half()
    w = torch.rand(dim, generator=g, device="cuda") + 0.5
    s, y = K.add_rms_norm(x, b, w, 1e-5)
    assert torch.equal(s, x + b)
    assert torch.equal(y, K.rms_norm(x + b, w, 1e-5))
