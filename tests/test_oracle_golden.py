"""Pin the numpy restatement (oracle/restate.py) to fixtures made by the reference itself.

The fixtures in tests/golden/ were produced by running the reference's own
quantization.py / attention.py / cache.py / storage.py (through the torch-CPU
mlx shim) on seeded inputs; see tests/golden/make_golden.py.  Integer outputs
(codes, masks, offsets, tier counts, stats) must match exactly; fp16 decodes
must be bit-identical; attention outputs must agree within 1e-3 absolute
(only reduction order differs: torch-CPU sums vs numpy sums).
"""
import numpy as np
import pytest

from oracle import restate as R
from tests.conftest import GOLDEN

QUANT_CASES = ["quant_d128_m8x16_rvq3", "quant_d64_m16x4_rvq1_dense", "quant_d64_m8x8_rvq1",
               "quant_d64_m8x8_pqonly"]


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


@pytest.mark.parametrize("name", QUANT_CASES)
def test_pq_codes_and_residual(name):
    g = load(name)
    codes, residual = R.pq_quantize(g["x"], g["pq_codebooks"])
    # Reference distances come from torch-CPU sgemm, ours from numpy sgemm; codes
    # may only differ where two centroids are tied to fp32 rounding.
    mism = np.argwhere(codes != g["pq_codes"])
    for n, m in mism:
        ds = g["pq_codebooks"].shape[2]
        sub = g["x"][n, m * ds:(m + 1) * ds].astype(np.float64)
        cb = g["pq_codebooks"][m].astype(np.float64)
        d = ((cb - sub) ** 2).sum(1)
        a, b = d[codes[n, m]], d[g["pq_codes"][n, m]]
        assert abs(a - b) <= 1e-5 * max(1.0, abs(a)), (n, m, a, b)
    assert len(mism) <= max(1, codes.size // 10000)
    if len(mism) == 0:
        np.testing.assert_array_equal(residual.view(np.uint16), g["residual"].view(np.uint16))


@pytest.mark.parametrize("name", QUANT_CASES)
def test_rvq_encode_and_hybrid_decode(name):
    g = load(name)
    codes, mask, offsets = R.rvq_encode(g["residual"], g["rvq_codebooks"], float(g["threshold"]))
    np.testing.assert_array_equal(mask, g["rvq_mask"])
    np.testing.assert_array_equal(offsets, g["rvq_offsets"])
    np.testing.assert_array_equal(codes, g["rvq_codes"])
    q = R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], float(g["threshold"]))
    dec = q.decode_flat(g["pq_codes"], g["rvq_codes"], g["rvq_mask"], g["rvq_offsets"])
    np.testing.assert_array_equal(dec.view(np.uint16), g["decoded"].view(np.uint16))
    np.testing.assert_array_equal(R.pq_decode(g["pq_codes"], g["pq_codebooks"]).view(np.uint16),
                                  g["pq_decoded"].view(np.uint16))


def test_hybrid_attention():
    g = load("attention_hybrid")
    q = R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], float(g["threshold"]))
    kc = q.compress(g["keys"])
    vc = q.compress(g["values"])
    np.testing.assert_array_equal(kc.pq, g["key_pq"])
    np.testing.assert_array_equal(kc.mask, g["key_mask"])
    np.testing.assert_array_equal(vc.pq, g["val_pq"])
    dk, dv = q.decode(kc), q.decode(vc)
    np.testing.assert_array_equal(dk.view(np.uint16), g["decoded_keys"].view(np.uint16))
    np.testing.assert_array_equal(dv.view(np.uint16), g["decoded_values"].view(np.uint16))
    scale = 128 ** -0.5
    out = R.blockwise_exact_attention(g["q"], dk, dv, scale, 16, True, g["positions"])
    np.testing.assert_allclose(out.astype(np.float32), g["out_causal"].astype(np.float32), atol=1e-3, rtol=0)
    out = R.blockwise_exact_attention(g["q"], dk, dv, scale, 16, False, None)
    np.testing.assert_allclose(out.astype(np.float32), g["out_plain"].astype(np.float32), atol=1e-3, rtol=0)
    out = R.blockwise_exact_attention(g["q"], dk, dv, scale, 16, True, g["positions_bh"])
    np.testing.assert_allclose(out.astype(np.float32), g["out_bh"].astype(np.float32), atol=1e-3, rtol=0)


STAT_KEYS = ("window_start", "window_end", "window_tokens", "context_window", "query_tokens", "used_router",
             "hot_tokens_materialized", "warm_tokens_materialized", "cold_tokens_materialized",
             "reconstructed_tokens", "warm_chunk_decodes", "cold_chunk_decodes", "cold_chunks_touched",
             "cold_chunk_cache_hits", "cold_chunk_cache_misses")


def build_oracle_cache(g):
    cfg = R.OracleConfig(hidden_dim=512, num_heads=4, head_dim=128, num_subspaces=8, subspace_dim=16,
                         num_rvq_layers=3, rvq_codebook_size=256, rvq_sparsity_threshold=0.25,
                         hot_capacity=16, warm_capacity=24, block_size_seq=16)
    qz = R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], float(g["threshold"]))
    cache = R.OracleCache(cfg, qz, batch=1)
    split = int(g["update_split"])
    cache.update(g["keys"][None, :split], g["values"][None, :split])
    cache.update(g["keys"][None, split:], g["values"][None, split:])
    return cache


def test_cache_tiers_materialize_and_attention():
    g = load("cache_tiers")
    cache = build_oracle_cache(g)
    assert [cache.num_hot, cache.num_warm, cache.num_cold] == list(g["tiers"])
    assert [m["chunk_id"] for m in cache.cold] == list(g["cold_chunk_ids"])
    assert [[m["start_token"], m["end_token"]] for m in cache.cold] == g["cold_chunk_bounds"].tolist()
    for i, (qpos, win) in enumerate(g["cases"]):
        qi, wi = divmod(i, 3)
        tag = f"q{qi}_w{wi}"
        win = None if win < 0 else int(win)
        out = cache.attention_forward(g["q"][None], causal=True, query_positions=[int(qpos)], context_window=win)
        stats = cache.last_access_stats
        assert [stats[k] for k in STAT_KEYS] == list(g[f"{tag}_stats"]), tag
        np.testing.assert_allclose(out[0].astype(np.float32), g[f"{tag}_out"].astype(np.float32), atol=1e-3)
        k_w, v_w, adj = cache.materialize_window([int(qpos)], win)
        np.testing.assert_array_equal(k_w[0].view(np.uint16), g[f"{tag}_keys"].view(np.uint16))
        np.testing.assert_array_equal(v_w[0].view(np.uint16), g[f"{tag}_values"].view(np.uint16))
        np.testing.assert_array_equal(adj, g[f"{tag}_adjusted"])


def test_gqa_and_batch_match_reference_loop():
    """GQA (the reference's _repeat_kv then its cache) and batch > 1 (a loop of reference caches)
    against the oracle's grouped-head, batched cache."""
    g = load("gqa_batch_cache")
    B, T, Hkv, D = g["keys"].shape
    Hq = g["q"].shape[1]
    cfg = R.OracleConfig(hidden_dim=Hq * D, num_heads=Hq, head_dim=D, num_subspaces=16, subspace_dim=4,
                         num_rvq_layers=1, rvq_codebook_size=256, rvq_sparsity_threshold=-1.0, hot_capacity=16,
                         warm_capacity=24, block_size_seq=16, num_kv_heads=Hkv)
    cache = R.OracleCache(cfg, R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], -1.0), batch=B)
    split = int(g["update_split"])
    cache.update(g["keys"][:, :split], g["values"][:, :split])
    cache.update(g["keys"][:, split:], g["values"][:, split:])
    for i, (qpos, win) in enumerate(g["cases"]):
        win = None if win < 0 else int(win)
        out = cache.attention_forward(g["q"][:, None], causal=True, query_positions=[int(qpos)], context_window=win)
        assert [cache.last_access_stats[k] for k in STAT_KEYS] == list(g["stats"][i, 0]), i
        np.testing.assert_allclose(out[:, 0].astype(np.float32), g["out"][i].astype(np.float32), atol=1e-3)


def test_router_candidate_order():
    g = load("router_order")
    for (pos, win, k), want in zip(g["queries"], g["loaded"]):
        got = R.router_candidates(g["chunk_ids"], int(pos), int(win), int(g["chunk_size"]), int(k))
        assert got == [int(x) for x in want if x >= 0]


def test_recent_policy_matches_prefix_arithmetic():
    """Extension sanity: with hot_policy='recent' the materialised window is still the
    position-ordered decode of every token; its hot part is exact fp16."""
    rng = np.random.default_rng(5)
    cfg = R.OracleConfig(hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=8, subspace_dim=8,
                         num_rvq_layers=1, rvq_codebook_size=64, rvq_sparsity_threshold=-1.0,
                         hot_capacity=8, warm_capacity=16, block_size_seq=8, num_kv_heads=2,
                         sparse_topk=4, hot_policy="recent")
    pq = rng.standard_normal((8, 256, 8)).astype(np.float16)
    rvq = (rng.standard_normal((1, 64, 64)) * 0.3).astype(np.float16)
    qz = R.Quantizer(pq, rvq, -1.0, sparse_topk=4)
    cache = R.OracleCache(cfg, qz, batch=2)
    k = rng.standard_normal((2, 40, 2, 64)).astype(np.float16)
    v = rng.standard_normal((2, 40, 2, 64)).astype(np.float16)
    cache.update(k[:, :30], v[:, :30])
    for t in range(30, 40):
        cache.update(k[:, t:t + 1], v[:, t:t + 1])
    assert cache.num_hot == 8 and cache.num_hot + cache.num_warm + cache.num_cold == 40
    assert cache.num_cold % 8 == 0 and cache.num_warm <= 16
    kw, vw, _ = cache.materialize_window()
    assert kw.shape == (2, 40, 2, 64)
    np.testing.assert_array_equal(kw[:, -8:], k[:, -8:])
    # sparse residual strictly reduces the reconstruction error versus PQ+RVQ alone
    full = qz.decode_f32(qz.compress(k[0, :8]))
    base = qz.decode_flat(*qz.encode_flat(k[0, :8].reshape(-1, 64))[:4]).reshape(8, 2, 64)
    assert np.abs(full - k[0, :8]).sum() < np.abs(base.astype(np.float32) - k[0, :8]).sum()


def test_router_candidates_api_matches_golden(tmp_path):
    """AsyncHierarchicalRouterMLX.candidates (the B200 router's selection) vs the reference's order."""
    from apple_b200.storage import AsyncHierarchicalRouterMLX, RFSNConfig, register_cold_tier, unregister_cold_tier
    g = load("router_order")
    cs = int(g["chunk_size"])

    class _Tier:  # only the chunk-id index is consulted when choosing candidates
        chunks = {int(c): None for c in g["chunk_ids"]}

    cfg = RFSNConfig(hidden_dim=512, num_heads=4, head_dim=128, block_size_seq=cs, disk_cache_dir=str(tmp_path))
    register_cold_tier(tmp_path, 7, _Tier())
    try:
        router = AsyncHierarchicalRouterMLX(cfg, layer_idx=7)
        for (pos, win, k), want in zip(g["queries"], g["loaded"]):
            assert router.candidates(int(pos), int(win), int(k)) == [int(x) for x in want if x >= 0]
    finally:
        unregister_cold_tier(tmp_path, 7)


def test_calibration_matches_reference():
    """calibrate_quantizer (rfsn_v10_mlx_ane_complete.py:175-225) from the reference's own initial samples."""
    g = load("calibration_kmeans")
    cbs, dist = R.calibrate_pq(g["vectors"], 8, 256, int(g["iters"]), g["sample_idx"])
    same = (cbs.view(np.uint16) == g["codebooks"].view(np.uint16)).mean()
    assert same > 0.999, same
    np.testing.assert_allclose(cbs.astype(np.float32), g["codebooks"].astype(np.float32), atol=2e-3, rtol=0)
    np.testing.assert_allclose(dist, g["avg_distortion"], rtol=1e-4)


def test_oracle_decoder_layer_matches_reference():
    """OracleDecoderLayer vs the reference layer's outputs (prefill, 24 cache decode steps, dense)."""
    g = load("decoder_layer")
    cfg = R.OracleConfig(hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=8, subspace_dim=8,
                         num_rvq_layers=1, rvq_codebook_size=64, rvq_sparsity_threshold=0.3, hot_capacity=16,
                         warm_capacity=24, block_size_seq=16)
    qz = R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], 0.3)
    w = {k[2:]: g[k] for k in g if k.startswith("w_")}
    layer = R.OracleDecoderLayer(cfg, qz, w)
    P = int(g["n_prefill"])
    layer.prefill_cache(g["x"][:, :P])
    outs = np.concatenate([layer(g["x"][:, t:t + 1], use_cache=True) for t in range(P, g["x"].shape[1])], 1)
    _layer_close(outs, g["decode_out"])
    assert [layer.cache.num_hot, layer.cache.num_warm, layer.cache.num_cold] == list(g["tiers"])
    assert [layer.cache.last_access_stats[k] for k in STAT_KEYS] == list(g["last_stats"])
    _layer_close(layer(g["x_dense"], use_cache=False), g["dense_out"])


def _layer_close(out, ref):
    """|out - ref| <= 2e-3 |ref| + 2e-3 rms(ref): fp16 outputs of fp16 GEMMs whose fp32 summation
    order differs from the reference's."""
    out, ref = np.asarray(out, np.float32), np.asarray(ref, np.float32)
    tol = 2e-3 * np.abs(ref) + 2e-3 * float(np.sqrt(np.mean(ref ** 2)))
    assert (np.abs(out - ref) <= tol).all(), float(np.abs(out - ref).max())


def test_oracle_llama_layer_matches_reference():
    """Llama32DecoderLayerMLX (llama32_adapter.py:417-662): prefill, 20 cache-backed decode steps
    through every tier, and the dense path, against the reference run through the shim."""
    g = load("llama_layer")
    D = 64
    hidden = g["x"].shape[-1]
    heads = g["w_q_proj"].shape[0] // D
    cfg = R.OracleConfig(hidden_dim=hidden, num_heads=heads, head_dim=D, num_subspaces=16, subspace_dim=4,
                         num_rvq_layers=1, rvq_codebook_size=256, rvq_sparsity_threshold=0.2, hot_capacity=16,
                         warm_capacity=24, block_size_seq=16)
    w = {k[2:]: v for k, v in g.items() if k.startswith("w_")}
    layer = R.OracleLlamaLayer(cfg, R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], 0.2), w, int(g["kv_heads"]),
                               float(g["eps"]))
    n = int(g["n_prefill"])
    layer.prefill_cache(g["x"][:, :n], g["cos"][:, :n], g["sin"][:, :n])
    outs = [layer(g["x"][:, t:t + 1], g["cos"][:, t:t + 1], g["sin"][:, t:t + 1], use_cache=True)
            for t in range(n, g["x"].shape[1])]
    assert [layer.cache.num_hot, layer.cache.num_warm, layer.cache.num_cold] == list(g["tiers"])
    assert [layer.cache.last_access_stats[k] for k in STAT_KEYS] == list(g["last_stats"])
    # fp16 outputs of magnitude up to ~5: one fp16 step (the fp32 matmul summation order differs)
    np.testing.assert_allclose(np.concatenate(outs, 1).astype(np.float32), g["decode_out"].astype(np.float32),
                               atol=4e-3, rtol=2e-3)
    dense = layer(g["x_dense"], g["cos_dense"], g["sin_dense"], use_cache=False)
    np.testing.assert_allclose(dense.astype(np.float32), g["dense_out"].astype(np.float32), atol=4e-3, rtol=2e-3)


def test_affine_codebook_quantization_properties():
    """The affine scheme (quantization.py:36-89 via mx.quantize): codes in range, the group's
    minimum exact, every value within half a step, a constant group exact."""
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((4, 256)) * 0.7).astype(np.float16).astype(np.float32)
    w[3, 128:] = 0.25
    q, sc, bi, deq = R.affine_quantize(w, 6, 128)
    assert q.max() <= 63 and q.dtype == np.uint8 and sc.shape == (4, 2)
    g = w.reshape(4, 2, 128)
    np.testing.assert_array_equal(bi, g.min(-1))
    assert (np.abs(deq - w).reshape(4, 2, 128) <= sc[..., None] * 0.5 * (1 + 1e-5) + 1e-7).all()
    np.testing.assert_array_equal(deq[3, 128:], w[3, 128:])
