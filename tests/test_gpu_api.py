"""GPU parity of the reference-facing Python API (cache, quantizers, attention, layer).

Mirrors the reference's own suite (rfsn_v10_mlx_ane_complete.py tests and
cache/quantization unit behaviour) on the golden fixtures generated from the
unmodified reference, and compares the extensions (batch > 1, GQA, sparse
residual, hot_policy="recent") against the CPU oracle.  Tolerances: codes and
materialised windows bit-exact; attention |out - ref| <= 2e-3 |ref| + 2e-3 rms.
"""
import numpy as np
import pytest
import torch

from oracle import restate as R
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from apple_b200.attention import RFSNHybridAttentionMLX, _blockwise_exact_attention
    from apple_b200.cache import RFSNv10KVCacheMLX
    from apple_b200.layer import RFSNDecoderLayerMLX
    from apple_b200.quantization import (HybridQuantizerMLX, _compress_tensor_sequence, _decode_compressed_tensor,
                                         _slice_compressed_tensor)
    from apple_b200.storage import AsyncHierarchicalRouterMLX, RFSNConfig

STAT_KEYS = ("window_start", "window_end", "window_tokens", "context_window", "query_tokens", "used_router",
             "hot_tokens_materialized", "warm_tokens_materialized", "cold_tokens_materialized",
             "reconstructed_tokens", "warm_chunk_decodes", "cold_chunk_decodes", "cold_chunks_touched",
             "cold_chunk_cache_hits", "cold_chunk_cache_misses")


def close(out, ref, what=""):
    out = np.asarray(out, np.float32)
    ref = np.asarray(ref, np.float32)
    rms = float(np.sqrt(np.mean(ref ** 2))) if ref.size else 0.0
    err = np.abs(out - ref)
    bad = err > 2e-3 * np.abs(ref) + 2e-3 * rms
    assert not bad.any(), f"{what}: {int(bad.sum())} off, max err {err.max():.3e}"


def u16(x):
    x = x.cpu().numpy() if isinstance(x, torch.Tensor) else x
    return np.ascontiguousarray(x).view(np.uint16)


def golden_quantizer(cfg, g):
    qz = HybridQuantizerMLX(cfg)
    qz.pq.codebooks = torch.from_numpy(g["pq_codebooks"]).cuda()
    qz.rvq.codebooks = torch.from_numpy(g["rvq_codebooks"]).cuda()
    return qz


def tiers_config(tmp_path, **kw):
    base = dict(hidden_dim=512, num_heads=4, head_dim=128, num_subspaces=8, subspace_dim=16, num_rvq_layers=3,
                rvq_codebook_size=256, rvq_sparsity_threshold=0.25, hot_capacity=16, warm_capacity=24,
                block_size_seq=16, disk_cache_dir=str(tmp_path), prefetch_throttle_s=0.0)
    base.update(kw)
    return RFSNConfig(**base)


def test_cache_tiers_golden(tmp_path):
    """cache.py tiering (hot prefix, warm, partial cold chunks) vs the reference's outputs."""
    g = dict(np.load(GOLDEN / "cache_tiers.npz"))
    cfg = tiers_config(tmp_path)
    qz = golden_quantizer(cfg, g)
    cache = RFSNv10KVCacheMLX(cfg, layer_idx=0)
    s = int(g["update_split"])
    cache.update(torch.from_numpy(g["keys"][:s]).cuda(), torch.from_numpy(g["values"][:s]).cuda(), qz)
    cache.update(torch.from_numpy(g["keys"][s:]).cuda(), torch.from_numpy(g["values"][s:]).cuda(), qz)
    assert [cache.num_hot, cache.num_warm, cache.num_cold] == list(g["tiers"])
    assert [m["chunk_id"] for m in cache.cold_chunk_metadata] == list(g["cold_chunk_ids"])
    assert [[m["start_token"], m["end_token"]] for m in cache.cold_chunk_metadata] == g["cold_chunk_bounds"].tolist()
    mem = cache.memory_usage_bytes()
    assert [mem["hot_bytes"], mem["warm_pq_bytes"], mem["warm_rvq_bytes"], mem["cold_chunks"],
            mem["cold_tokens"]] == list(g["memory"])
    q = torch.from_numpy(g["q"]).cuda()
    for i, (qpos, win) in enumerate(g["cases"]):
        tag = f"q{i // 3}_w{i % 3}"
        win = None if win < 0 else int(win)
        out = cache.attention_forward(q, causal=True, query_positions=[int(qpos)], context_window=win)
        assert [cache.last_access_stats[k] for k in STAT_KEYS] == list(g[f"{tag}_stats"]), tag
        close(out.cpu().numpy(), g[f"{tag}_out"], tag)
        # the same call from pinned host buffers (one library call: upload, attention, wait)
        hq = q.cpu().pin_memory()
        hout = torch.full(q.shape, float("nan"), dtype=torch.float16).pin_memory()
        cache.attention_forward(hq, causal=True, query_positions=[int(qpos)], context_window=win, out=hout)
        assert torch.equal(hout, out.cpu()), tag
        assert [cache.last_access_stats[k] for k in STAT_KEYS] == list(g[f"{tag}_stats"]), tag
        kw, vw, adj = cache.materialize_window([int(qpos)], win)
        np.testing.assert_array_equal(u16(kw), u16(g[f"{tag}_keys"]))
        np.testing.assert_array_equal(u16(vw), u16(g[f"{tag}_values"]))
        np.testing.assert_array_equal(adj.cpu().numpy(), g[f"{tag}_adjusted"])
    # cold chunks read back from the pinned tier equal the codes the reference stores
    chunk = cache.load_cold_chunk(int(g["cold_chunk_ids"][0]))
    assert int(chunk["num_tokens"][0]) == 16
    with pytest.raises(KeyError):
        cache.load_cold_chunk(999)
    cache.close()


def test_gqa_batch_cache_golden(tmp_path):
    """GQA and batch > 1 pinned to the reference: one batched, grouped-head cache against the
    reference's cache over _repeat_kv'd heads (llama32_adapter.py:380-386), one reference cache
    per sequence, at 3 query positions x 3 windows."""
    g = dict(np.load(GOLDEN / "gqa_batch_cache.npz"))
    B, T, Hkv, D = g["keys"].shape
    Hq = g["q"].shape[1]
    cfg = tiers_config(tmp_path, hidden_dim=Hq * D, num_heads=Hq, head_dim=D, num_subspaces=16, subspace_dim=4,
                       num_rvq_layers=1, rvq_sparsity_threshold=-1.0, num_kv_heads=Hkv, batch_size=B)
    qz = golden_quantizer(cfg, g)
    cache = RFSNv10KVCacheMLX(cfg, layer_idx=0)
    s = int(g["update_split"])
    cache.update(torch.from_numpy(g["keys"][:, :s]).cuda(), torch.from_numpy(g["values"][:, :s]).cuda(), qz)
    cache.update(torch.from_numpy(g["keys"][:, s:]).cuda(), torch.from_numpy(g["values"][:, s:]).cuda(), qz)
    q = torch.from_numpy(g["q"]).cuda()
    for i, (qpos, win) in enumerate(g["cases"]):
        win = None if win < 0 else int(win)
        out = cache.attention_forward(q, causal=True, query_positions=[int(qpos)], context_window=win)
        assert [cache.last_access_stats[k] for k in STAT_KEYS] == list(g["stats"][i, 0]), i
        close(out.cpu().numpy(), g["out"][i], f"case {i}")
        # a pinned host query in, and a pinned host output that the kernel writes itself
        hq = q.cpu().pin_memory()
        hout = torch.full(q.shape, float("nan"), dtype=torch.float16).pin_memory()
        got = cache.attention_forward(hq, causal=True, query_positions=[int(qpos)], context_window=win, out=hout)
        assert got.data_ptr() == hout.data_ptr()
        assert torch.equal(hout, out.cpu()), i
    cache.close()


def test_host_buffer_calls_repeat_and_advance(tmp_path):
    """Decode-loop use of the host-buffer path: the same pinned buffers with new query values
    each call (the cache reuses the last call's plan), then a token appended to the cache (the
    next call plans again); every output equals the device-resident call on the same query."""
    g = dict(np.load(GOLDEN / "gqa_batch_cache.npz"))
    B, T, Hkv, D = g["keys"].shape
    Hq = g["q"].shape[1]
    # hot and warm tiers hold every token (no cold tier: the case the reuse applies to)
    cfg = tiers_config(tmp_path, hidden_dim=Hq * D, num_heads=Hq, head_dim=D, num_subspaces=16, subspace_dim=4,
                       num_rvq_layers=1, rvq_sparsity_threshold=-1.0, num_kv_heads=Hkv, batch_size=B,
                       warm_capacity=int(T) + 16)
    qz = golden_quantizer(cfg, g)
    cache = RFSNv10KVCacheMLX(cfg, layer_idx=0)
    keys, values = torch.from_numpy(g["keys"]).cuda(), torch.from_numpy(g["values"]).cuda()
    cache.update(keys[:, :T - 2], values[:, :T - 2], qz)
    gen = torch.Generator().manual_seed(3)
    hq = torch.empty((B, Hq, D), dtype=torch.float16).pin_memory()
    hout = torch.empty((B, Hq, D), dtype=torch.float16).pin_memory()
    for step in range(6):
        if step == 3:
            cache.update(keys[:, T - 2:T - 1], values[:, T - 2:T - 1], qz)
        hq.copy_(torch.randn((B, Hq, D), generator=gen).half())
        hout.fill_(float("nan"))
        cache.attention_forward(hq, causal=True, out=hout)
        host_stats = dict(cache.last_access_stats)
        want = cache.attention_forward(hq.cuda(), causal=True)
        assert torch.equal(hout, want.cpu()), step
        assert host_stats == cache.last_access_stats, step
    assert cache.num_cold == 0 and cache._host_memo is not None
    cache.close()


def test_cache_tiers_with_router(tmp_path):
    """Router-driven prefetch: same outputs, hit/miss statistics as the oracle with the router's loads."""
    g = dict(np.load(GOLDEN / "cache_tiers.npz"))
    cfg = tiers_config(tmp_path)
    qz = golden_quantizer(cfg, g)
    cache = RFSNv10KVCacheMLX(cfg, layer_idx=3)
    cache.update(torch.from_numpy(g["keys"]).cuda(), torch.from_numpy(g["values"]).cuda(), qz)
    router = AsyncHierarchicalRouterMLX(cfg, layer_idx=3)
    q = torch.from_numpy(g["q"]).cuda()
    ocfg = R.OracleConfig(hidden_dim=512, num_heads=4, head_dim=128, num_subspaces=8, subspace_dim=16,
                          num_rvq_layers=3, rvq_codebook_size=256, rvq_sparsity_threshold=0.25,
                          hot_capacity=16, warm_capacity=24, block_size_seq=16)
    oc = R.OracleCache(ocfg, R.Quantizer(g["pq_codebooks"], g["rvq_codebooks"], float(g["threshold"])), batch=1)
    oc.update(g["keys"][None], g["values"][None])
    held = []  # the router's chunk cache persists across calls (FIFO of 16, storage.py:186-188)
    for pos, win in ((59, 30), (45, 16), (59, 8)):
        out = cache.attention_forward(q, causal=True, query_positions=[pos], router=router, current_position=pos,
                                      context_window=win)
        ids = [m["chunk_id"] for m in oc.cold]
        for c in R.router_candidates(ids, pos, win, 16, max(1, (win + 15) // 16)):
            if c not in held:
                held.append(c)
        held = held[-16:]
        kw, vw, adj = oc.materialize_window([pos], win, cold_hits=set(held), used_router=True)
        ref = R.blockwise_exact_attention(g["q"], kw[0], vw[0], 128 ** -0.5, 16, True, adj)
        close(out.cpu().numpy(), ref, f"pos {pos} win {win}")
        st = cache.last_access_stats
        assert st["used_router"] == 1
        assert (st["cold_chunk_cache_hits"], st["cold_chunk_cache_misses"]) == (
            oc.last_access_stats["cold_chunk_cache_hits"], oc.last_access_stats["cold_chunk_cache_misses"])
    cache.close()


@pytest.mark.parametrize("policy", ["prefix", "recent"])
def test_cache_extensions_vs_oracle(tmp_path, policy):
    """batch 2, GQA 4:2, top-4 sparse residual; token-by-token decode appends through every tier."""
    rng = np.random.default_rng(11)
    kw = dict(hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=16, subspace_dim=4, num_rvq_layers=1,
              rvq_codebook_size=256, rvq_sparsity_threshold=-1.0, hot_capacity=16, warm_capacity=32,
              block_size_seq=16, num_kv_heads=2, sparse_topk=4, hot_policy=policy)
    cfg = RFSNConfig(batch_size=2, disk_cache_dir=str(tmp_path), **kw)
    ocfg = R.OracleConfig(**kw)
    pq = (rng.standard_normal((16, 256, 4)) * 0.7).astype(np.float16)
    rvq = (rng.standard_normal((1, 256, 64)) * 0.3).astype(np.float16)
    qz = HybridQuantizerMLX(cfg)
    qz.pq.codebooks, qz.rvq.codebooks = torch.from_numpy(pq).cuda(), torch.from_numpy(rvq).cuda()
    oc = R.OracleCache(ocfg, R.Quantizer(pq, rvq, -1.0, sparse_topk=4), batch=2)
    cache = RFSNv10KVCacheMLX(cfg, layer_idx=1)
    k = rng.standard_normal((2, 90, 2, 64)).astype(np.float16)
    v = rng.standard_normal((2, 90, 2, 64)).astype(np.float16)
    cache.update(torch.from_numpy(k[:, :70]).cuda(), torch.from_numpy(v[:, :70]).cuda(), qz)
    oc.update(k[:, :70], v[:, :70])
    for t in range(70, 90):
        cache.update(torch.from_numpy(k[:, t:t + 1]).cuda(), torch.from_numpy(v[:, t:t + 1]).cuda(), qz)
        oc.update(k[:, t:t + 1], v[:, t:t + 1])
    assert (cache.num_hot, cache.num_warm, cache.num_cold) == (oc.num_hot, oc.num_warm, oc.num_cold)
    kg, vg, _ = cache.materialize_window()
    ko, vo, _ = oc.materialize_window()
    np.testing.assert_array_equal(u16(kg), u16(ko))
    np.testing.assert_array_equal(u16(vg), u16(vo))
    q = rng.standard_normal((2, 4, 64)).astype(np.float16)
    for pos in (89, 60):
        for win in (None, 40, 17):
            out = cache.attention_forward(torch.from_numpy(q).cuda(), causal=True, query_positions=[pos],
                                          context_window=win)
            ref = oc.attention_forward(q[:, None], causal=True, query_positions=[pos], context_window=win)
            close(out.cpu().numpy(), ref[:, 0], f"position {pos} window {win}")
    cache.close()


@pytest.mark.parametrize("policy", ["recent", "prefix"])
def test_centroid_routed_cold_tier_vs_oracle(tmp_path, policy):
    """Centroid routing (extension): each step attends hot + warm + the top-4 cold chunks by
    mean-key score, prefetched on the router's stream into a 5-slot pool (smaller than the
    12 cold chunks, so steps copy chunks in).  The chosen chunks equal the oracle's choice
    except where two scores tie to fp32 rounding, and the output equals the oracle's
    attention over the same routed window."""
    rng = np.random.default_rng(23)
    kw = dict(hidden_dim=512, num_heads=8, head_dim=64, num_subspaces=16, subspace_dim=4, num_rvq_layers=1,
              rvq_codebook_size=256, rvq_sparsity_threshold=-1.0, hot_capacity=32, warm_capacity=64,
              block_size_seq=32, num_kv_heads=2, sparse_topk=8, hot_policy=policy)
    cfg = RFSNConfig(batch_size=2, disk_cache_dir=str(tmp_path), cold_routing="centroid", cold_route_top_k=4,
                     cold_pool_chunks=5, prefetch_throttle_s=0.0, **kw)
    pq = (rng.standard_normal((16, 256, 4)) * 0.7).astype(np.float16)
    rvq = (rng.standard_normal((1, 256, 64)) * 0.3).astype(np.float16)
    oc = R.OracleCache(R.OracleConfig(**kw), R.Quantizer(pq, rvq, -1.0, sparse_topk=8), batch=2)
    qz = HybridQuantizerMLX(cfg)
    qz.pq.codebooks, qz.rvq.codebooks = torch.from_numpy(pq).cuda(), torch.from_numpy(rvq).cuda()
    cache = RFSNv10KVCacheMLX(cfg, layer_idx=2)
    router = AsyncHierarchicalRouterMLX(cfg, layer_idx=2)
    T = 480
    walk = np.cumsum(rng.standard_normal((T // 32, 1, 64)) * 0.5, axis=0).repeat(32, axis=0)
    k = (rng.standard_normal((2, T, 2, 64)) + walk[None]).astype(np.float16)
    v = rng.standard_normal((2, T, 2, 64)).astype(np.float16)
    for a in range(0, T, 96):
        cache.update(torch.from_numpy(k[:, a:a + 96]).cuda(), torch.from_numpy(v[:, a:a + 96]).cuda(), qz)
        oc.update(k[:, a:a + 96], v[:, a:a + 96])
    assert (cache.num_hot, cache.num_warm, cache.num_cold) == (oc.num_hot, oc.num_warm, oc.num_cold)
    assert len(cache.cold_chunk_metadata) == 12
    ids, cent = oc.chunk_centroids()
    misses = 0
    for step in range(6):
        q = (rng.standard_normal((2, 8, 64)) * (1 + step)).astype(np.float16)
        out = cache.attention_forward(torch.from_numpy(q).cuda(), causal=True, router=router,
                                      current_position=T - 1, context_window=T)
        chosen = cache.last_routed_chunks
        st = cache.get_last_access_stats()
        assert st["cold_chunks_touched"] == 4
        assert st["cold_chunk_cache_hits"] + st["cold_chunk_cache_misses"] == 4
        misses += st["cold_chunk_cache_misses"]
        sel, scores = R.route_topk(q[:, None], cent, 2, 4)
        want = [ids[i] for i in sel]
        if set(chosen) != set(want):  # only fp32 ties may swap: the scores at the boundary agree closely
            got_s = sorted(scores[ids.index(c)] for c in chosen)
            want_s = sorted(scores[i] for i in sel)
            np.testing.assert_allclose(got_s, want_s, rtol=1e-5, atol=1e-5)
        ref = oc.attention_forward(q[:, None], causal=True, context_window=T, current_position=T - 1,
                                   routed_chunks=chosen)
        close(out.cpu().numpy(), ref[:, 0], f"step {step}")
    assert misses >= 4  # the first step finds an empty pool
    cache.close()


def _ref_chunk_cache(tmp_path, spill):
    idx = dict(np.load(GOLDEN / "ref_chunks" / "index.npz"))
    cfg = RFSNConfig(hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=16, subspace_dim=4, num_rvq_layers=1,
                     rvq_codebook_size=256, rvq_sparsity_threshold=0.4, hot_capacity=16, warm_capacity=24,
                     block_size_seq=16, prefetch_throttle_s=0.0, disk_cache_dir=str(tmp_path), cold_host_chunks=spill)
    qz = golden_quantizer(cfg, idx)
    cache = RFSNv10KVCacheMLX(cfg, layer_idx=0)
    s = int(idx["update_split"])
    for a, b in ((0, s), (s, idx["keys"].shape[0])):
        cache.update(torch.from_numpy(idx["keys"][a:b]).cuda(), torch.from_numpy(idx["values"][a:b]).cuda(), qz)
    return idx, cache


def test_cold_tier_spills_to_reference_chunk_files(tmp_path):
    """cold_host_chunks=1 keeps one chunk image in pinned memory and spills the other to its
    layer0_chunk{id}.npz file: the files and load_cold_chunk hold exactly what the reference
    cache wrote for the same tokens (the 20-token merged chunk included), and attention over
    every tier equals the non-spilling cache's and the oracle's."""
    idx, full = _ref_chunk_cache(tmp_path / "full", None)
    _, sp = _ref_chunk_cache(tmp_path / "spill", 1)
    assert [[m["start_token"], m["end_token"]] for m in sp.cold_chunk_metadata] == idx["chunk_bounds"].tolist()
    assert sp._cold.spills >= 1
    files = 0
    for cid in idx["chunk_ids"]:
        ref = np.load(GOLDEN / "ref_chunks" / f"layer0_chunk{int(cid)}.npz")
        written = tmp_path / "spill" / f"layer0_chunk{int(cid)}.npz"
        got = [sp.load_cold_chunk(int(cid)), full.load_cold_chunk(int(cid))]
        if written.exists():
            files += 1
            got.append(dict(np.load(written)))
        for d in got:
            assert sorted(d) == sorted(ref.files)
            for k in ref.files:
                np.testing.assert_array_equal(d[k], ref[k], err_msg=k)
    assert files >= 1
    oc = R.OracleCache(R.OracleConfig(hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=16, subspace_dim=4,
                                      num_rvq_layers=1, rvq_codebook_size=256, rvq_sparsity_threshold=0.4,
                                      hot_capacity=16, warm_capacity=24, block_size_seq=16),
                       R.Quantizer(idx["pq_codebooks"], idx["rvq_codebooks"], 0.4))
    s = int(idx["update_split"])
    oc.update(idx["keys"][None, :s], idx["values"][None, :s])
    oc.update(idx["keys"][None, s:], idx["values"][None, s:])
    q = np.random.default_rng(5).standard_normal((1, 4, 64)).astype(np.float16)
    for pos, win in ((69, None), (55, 30), (45, 10)):
        a = full.attention_forward(torch.from_numpy(q).cuda(), query_positions=[pos], context_window=win)
        b = sp.attention_forward(torch.from_numpy(q).cuda(), query_positions=[pos], context_window=win)
        assert torch.equal(a, b), (pos, win)
        ref = oc.attention_forward(q[None], query_positions=[pos], context_window=win)
        close(b.cpu().numpy(), ref[0], f"position {pos} window {win}")
    assert sp._cold.unspills >= 1  # attention brought a spilled chunk back from its file
    full.close()
    sp.close()


def test_reference_chunk_file_into_device_store():
    """A chunk file written by the reference, read into a device code store, decodes on the GPU
    bit-exactly as the oracle decodes the file's codes."""
    from apple_b200.chunk_io import load_compressed_chunk, npz_to_store
    from apple_b200 import kernels as K
    idx = dict(np.load(GOLDEN / "ref_chunks" / "index.npz"))
    qz = K.QuantizerBuffers(torch.from_numpy(idx["pq_codebooks"]).cuda(), torch.from_numpy(idx["rvq_codebooks"]).cuda(),
                            0.4, 0)
    oq = R.Quantizer(idx["pq_codebooks"], idx["rvq_codebooks"], 0.4)
    path = GOLDEN / "ref_chunks" / f"layer0_chunk{int(idx['chunk_ids'][0])}.npz"
    st = K.CodeStoreBuffers(qz, rows=4, cap=32)
    n = npz_to_store(path, st)
    f = load_compressed_chunk(path)
    for kv, prefix in ((0, "key"), (1, "value")):
        mask = f[f"{prefix}_rvq_mask"]
        rvq = np.zeros((n * 4, 1), np.uint16)
        rvq[f[f"{prefix}_rvq_offsets"]] = f[f"{prefix}_rvq_codes"]
        codes = R.Codes(f[f"{prefix}_pq_codes"], rvq.reshape(n, 4, 1), mask, np.zeros((n, 4, 0), np.uint8),
                        np.zeros((n, 4, 0), np.float16))
        out = torch.empty((1, n, 4, 64), dtype=torch.float16, device="cuda")
        K.decode_codes(qz, st, 0, 0, n, out, kv=kv)
        np.testing.assert_array_equal(u16(out[0]), u16(oq.decode(codes)))


@pytest.mark.parametrize("layer_linear", [False, True])
def test_llama_layer_golden(tmp_path, monkeypatch, layer_linear):
    """Llama32DecoderLayerMLX (llama32_adapter.py:417-662) against the reference run through the
    shim: prefill, 20 cache-backed decode steps through hot, warm and cold, and the dense path;
    projections on cuBLAS and on rfsn_linear_f16.  fp16 outputs up to ~5 in magnitude: within
    one fp16 step (atol 4e-3) plus 2e-3 relative."""
    from apple_b200 import kernels as Kmod
    from apple_b200.llama import Llama32DecoderLayerMLX
    monkeypatch.setattr(Kmod, "LAYER_LINEAR", layer_linear)
    g = dict(np.load(GOLDEN / "llama_layer.npz"))
    D = 64
    hidden = g["x"].shape[-1]
    heads = g["w_q_proj"].shape[0] // D
    cfg = tiers_config(tmp_path, hidden_dim=hidden, num_heads=heads, head_dim=D, num_subspaces=16, subspace_dim=4,
                       num_rvq_layers=1, rvq_sparsity_threshold=0.2)
    w = {k[2:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("w_")}
    layer = Llama32DecoderLayerMLX(cfg, 0, int(g["kv_heads"]), float(g["eps"]), w["input_layernorm"],
                                   w["post_attention_layernorm"], w["q_proj"], w["k_proj"], w["v_proj"], w["o_proj"],
                                   w["gate_proj"], w["up_proj"], w["down_proj"])
    layer.quantizer.pq.codebooks = torch.from_numpy(g["pq_codebooks"]).cuda()
    layer.quantizer.rvq.codebooks = torch.from_numpy(g["rvq_codebooks"]).cuda()
    n = int(g["n_prefill"])
    x = torch.from_numpy(g["x"]).cuda()
    layer.prefill_cache(x[:, :n], position_embeddings=(g["cos"][:, :n], g["sin"][:, :n]))
    outs = [layer(x[:, t:t + 1], position_embeddings=(g["cos"][:, t:t + 1], g["sin"][:, t:t + 1]), use_cache=True)
            for t in range(n, x.shape[1])]
    assert [layer.cache.num_hot, layer.cache.num_warm, layer.cache.num_cold] == list(g["tiers"])
    assert [layer.cache.last_access_stats[k] for k in STAT_KEYS] == list(g["last_stats"])
    got = torch.cat(outs, 1).float().cpu().numpy()
    np.testing.assert_allclose(got, g["decode_out"].astype(np.float32), atol=4e-3, rtol=2e-3)
    dense = layer(torch.from_numpy(g["x_dense"]).cuda(), position_embeddings=(g["cos_dense"], g["sin_dense"]))
    np.testing.assert_allclose(dense.float().cpu().numpy(), g["dense_out"].astype(np.float32), atol=4e-3, rtol=2e-3)
    with pytest.raises(RuntimeError):
        layer(x[:, :1], use_cache=True)  # no position tables and no rotary module
    layer.cache.close()


def test_llama_ops_vs_oracle():
    """The Llama adapter's RMSNorm (+ residual add), RoPE and SwiGLU kernels against the numpy
    restatement: fp16 results within one fp16 step (the last fp32 bit of sqrt, exp or the mean
    can cross an fp16 rounding boundary), and equal in most elements."""
    from apple_b200 import kernels as K
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((5, 3, 256)) * 2).astype(np.float16)
    r = rng.standard_normal((5, 3, 256)).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(256)).astype(np.float16)
    y, s = K.llama_rms_norm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), 1e-5,
                            residual=torch.from_numpy(r).cuda())
    s_ref = (x.astype(np.float32) + r.astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(u16(s), u16(s_ref))
    ref = R.llama_rms_norm(s_ref, w, 1e-5).astype(np.float32)
    got = y.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-3)
    assert (got == ref).mean() > 0.99
    q = rng.standard_normal((2, 7, 4, 64)).astype(np.float16)
    k = rng.standard_normal((2, 7, 2, 64)).astype(np.float16)
    ang = np.arange(7)[:, None] * (1.0 / (10000 ** (np.arange(0, 64, 2) / 64)))[None]
    cos = np.cos(np.concatenate([ang, ang], -1)).astype(np.float16)[None]
    sin = np.sin(np.concatenate([ang, ang], -1)).astype(np.float16)[None]
    qr, kr = R.apply_rope(q, k, cos, sin)
    np.testing.assert_array_equal(u16(K.rope(torch.from_numpy(q).cuda(), torch.from_numpy(cos), torch.from_numpy(sin))),
                                  u16(qr))
    np.testing.assert_array_equal(u16(K.rope(torch.from_numpy(k).cuda(), torch.from_numpy(cos), torch.from_numpy(sin))),
                                  u16(kr))
    gt = (rng.standard_normal(4096) * 3).astype(np.float16)
    up = rng.standard_normal(4096).astype(np.float16)
    got = K.silu_mul(torch.from_numpy(gt).cuda(), torch.from_numpy(up).cuda()).float().cpu().numpy()
    ref = (R.silu(gt).astype(np.float32) * up.astype(np.float32)).astype(np.float16).astype(np.float32)
    np.testing.assert_allclose(got, ref, rtol=2e-3, atol=1e-4)
    assert (got == ref).mean() > 0.99


def test_affine_codebooks_for_ane():
    """quantize_codebooks_for_ane (quantization.py:159-175, 277-293, 321-327): the kernel's codes,
    scales, biases and dequantized values equal the oracle's affine restatement; the quantizer then
    reads the dequantized codebooks (the reference's quantized fast path test, rfsn_v10_mlx_ane_
    complete.py:404-416: every codebook quantized, finite round-trip error)."""
    from apple_b200 import kernels as K
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((64, 256)) * 0.5).astype(np.float16).astype(np.float32)
    q, sc, bi, deq = K.affine_quantize(torch.from_numpy(w).cuda(), 6, 128)
    rq, rsc, rbi, rdeq = R.affine_quantize(w, 6, 128)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(sc.cpu().numpy(), rsc)
    np.testing.assert_array_equal(bi.cpu().numpy(), rbi)
    np.testing.assert_array_equal(deq.cpu().numpy(), rdeq)
    cfg = RFSNConfig(hidden_dim=512, num_heads=8, head_dim=64, num_subspaces=16, subspace_dim=4, num_rvq_layers=2,
                     rvq_codebook_size=256, rvq_sparsity_threshold=0.3)
    hq = HybridQuantizerMLX(cfg)
    x = torch.randn((512, 64), generator=torch.Generator().manual_seed(3)).half().cuda()
    mse0 = float(((x.float() - hq.decode(*hq.encode(x)).float()) ** 2).mean())
    pq_before = hq.pq.codebooks.clone()
    report = hq.quantize_codebooks_for_ane()
    assert report == {"pq_quantized": 16, "rvq_quantized": 2}
    # PQ codebooks [256, 4] quantize transposed in groups of 128 along the centroids; RVQ [256, 64]
    # in groups of 64 along each row
    m0 = hq.pq._ane_codebooks[0]
    assert m0.transposed and m0.group_size == 128 and hq.rvq._ane_codebooks[0].group_size == 64
    _, _, _, d0 = R.affine_quantize(pq_before[0].float().cpu().numpy().T.copy(), 6, 128)
    np.testing.assert_array_equal(u16(hq.pq.effective_codebooks()[0]), u16(d0.T.astype(np.float16)))
    mse1 = float(((x.float() - hq.decode(*hq.encode(x)).float()) ** 2).mean())
    assert np.isfinite(mse1) and mse1 < 1.5 * mse0 + 1e-3


def test_quantizer_api_golden():
    """HybridQuantizerMLX encode/decode and the compressed-tensor helpers vs reference vectors."""
    g = dict(np.load(GOLDEN / "quant_d128_m8x16_rvq3.npz"))
    cfg = RFSNConfig(hidden_dim=512, num_heads=4, head_dim=128, num_subspaces=8, subspace_dim=16,
                     num_rvq_layers=3, rvq_codebook_size=256, rvq_sparsity_threshold=float(g["threshold"]))
    qz = golden_quantizer(cfg, g)
    x = torch.from_numpy(g["x"]).cuda()
    pq, rvq, mask, offs = qz.encode(x)
    np.testing.assert_array_equal(pq.cpu().numpy(), g["pq_codes"])
    np.testing.assert_array_equal(mask.cpu().numpy(), g["rvq_mask"])
    np.testing.assert_array_equal(offs.cpu().numpy(), g["rvq_offsets"])
    np.testing.assert_array_equal(rvq.cpu().numpy(), g["rvq_codes"].astype(np.int32))
    np.testing.assert_array_equal(u16(qz.decode(pq, rvq, mask, offs)), u16(g["decoded"]))
    np.testing.assert_array_equal(u16(qz.pq.decode(pq)), u16(g["pq_decoded"]))
    codes, residual = qz.pq.quantize(x)
    np.testing.assert_array_equal(u16(residual), u16(g["residual"]))
    ct = _compress_tensor_sequence(x.view(24, 4, 128), qz)
    np.testing.assert_array_equal(u16(_decode_compressed_tensor(ct, qz)), u16(g["decoded"].reshape(24, 4, 128)))
    part = _slice_compressed_tensor(ct, 5, 17)
    np.testing.assert_array_equal(u16(_decode_compressed_tensor(part, qz)),
                                  u16(g["decoded"].reshape(24, 4, 128)[5:17]))


def test_hybrid_attention_api_golden():
    """RFSNHybridAttentionMLX and _blockwise_exact_attention vs the reference outputs."""
    g = dict(np.load(GOLDEN / "attention_hybrid.npz"))
    cfg = RFSNConfig(hidden_dim=512, num_heads=4, head_dim=128, num_subspaces=8, subspace_dim=16,
                     num_rvq_layers=3, rvq_codebook_size=256, rvq_sparsity_threshold=float(g["threshold"]),
                     block_size_seq=16)
    qz = golden_quantizer(cfg, g)
    ks = _compress_tensor_sequence(torch.from_numpy(g["keys"]).cuda(), qz)
    vs = _compress_tensor_sequence(torch.from_numpy(g["values"]).cuda(), qz)
    attn = RFSNHybridAttentionMLX(cfg)
    q = torch.from_numpy(g["q"]).cuda()
    close(attn(q, ks, vs, qz, causal=True, query_positions=g["positions"]).cpu().numpy(), g["out_causal"], "causal")
    close(attn(q, ks, vs, qz, causal=False).cpu().numpy(), g["out_plain"], "plain")
    close(attn(q, ks, vs, qz, causal=True, query_positions=g["positions_bh"]).cpu().numpy(), g["out_bh"], "bh")
    dk = torch.from_numpy(g["decoded_keys"]).cuda()
    dv = torch.from_numpy(g["decoded_values"]).cuda()
    out = _blockwise_exact_attention(q, dk, dv, 128 ** -0.5, 16, True, g["positions"])
    close(out.cpu().numpy(), g["out_causal"], "blockwise")


def test_decoder_layer_cached_decode_matches_dense(tmp_path):
    """RFSNDecoderLayerMLX: with every token in the exact hot tier, cache-backed decode
    equals the dense causal layer on the full sequence (last position)."""
    cfg = RFSNConfig(hidden_dim=512, num_heads=8, head_dim=64, num_subspaces=8, subspace_dim=8, num_rvq_layers=0,
                     rvq_codebook_size=256, hot_capacity=4096, warm_capacity=64, block_size_seq=16,
                     num_kv_heads=4, disk_cache_dir=str(tmp_path))
    layer = RFSNDecoderLayerMLX(cfg, layer_idx=0, init="normal", seed=3)
    g = torch.Generator().manual_seed(5)
    x = torch.randn((1, 40, 512), generator=g).cuda()
    layer.prefill_cache(x[:, :32])
    for t in range(32, 40):
        y = layer(x[:, t:t + 1], use_cache=True)
    dense = layer(x, use_cache=False)
    close(y[0, 0].float().cpu().numpy(), dense[0, -1].float().cpu().numpy(), "decoder layer")
    assert layer.cache_tokens == 40


@pytest.mark.parametrize("layer_linear", [False, True])
def test_decoder_layer_golden(tmp_path, monkeypatch, layer_linear):
    """RFSNDecoderLayerMLX vs the reference layer (rfsn_v10_mlx_ane_complete.py:55-172): prefill 40
    tokens, 24 cache-backed decode steps through hot, warm and cold tiers, and the dense path;
    projections on cuBLAS, and on rfsn_linear_f16 with the GELU and residual add fused."""
    from apple_b200 import kernels as Kmod
    monkeypatch.setattr(Kmod, "LAYER_LINEAR", layer_linear)
    g = dict(np.load(GOLDEN / "decoder_layer.npz"))
    cfg = RFSNConfig(hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=8, subspace_dim=8, num_rvq_layers=1,
                     rvq_codebook_size=64, rvq_sparsity_threshold=0.3, hot_capacity=16, warm_capacity=24,
                     block_size_seq=16, disk_cache_dir=str(tmp_path))
    layer = RFSNDecoderLayerMLX(cfg, layer_idx=0)
    for nm in ("q_proj", "k_proj", "v_proj", "o_proj", "ffn_up", "ffn_down"):
        getattr(layer, nm).weight = torch.from_numpy(g[f"w_{nm}"].astype(np.float32)).cuda()
    layer.quantizer.pq.codebooks = torch.from_numpy(g["pq_codebooks"]).cuda()
    layer.quantizer.rvq.codebooks = torch.from_numpy(g["rvq_codebooks"]).cuda()
    x = torch.from_numpy(g["x"]).cuda()
    P = int(g["n_prefill"])
    layer.prefill_cache(x[:, :P])
    outs = [layer(x[:, t:t + 1], use_cache=True) for t in range(P, x.shape[1])]
    got = torch.cat(outs, 1).float().cpu().numpy()
    close(got, g["decode_out"], "cache-backed decode")
    assert [layer.cache.last_access_stats[k] for k in STAT_KEYS] == list(g["last_stats"])
    assert [layer.cache.num_hot, layer.cache.num_warm, layer.cache.num_cold] == list(g["tiers"])
    dense = layer(torch.from_numpy(g["x_dense"]).cuda(), use_cache=False).float().cpu().numpy()
    close(dense, g["dense_out"], "dense path")
    layer.cache.close()


def test_calibration_golden():
    """calibrate_quantizer on the GPU (PQ encoder kernel + mean updates) from the reference's samples."""
    from apple_b200.layer import calibrate_quantizer
    g = dict(np.load(GOLDEN / "calibration_kmeans.npz"))
    cfg = RFSNConfig(hidden_dim=512, num_heads=8, head_dim=64, num_subspaces=8, subspace_dim=8, num_rvq_layers=0,
                     rvq_sparsity_threshold=float(g["threshold"]))
    hq = HybridQuantizerMLX(cfg)
    metrics = calibrate_quantizer(hq, torch.from_numpy(g["vectors"]).cuda(), num_iterations=int(g["iters"]),
                                  sample_idx=torch.from_numpy(g["sample_idx"]))
    cb = hq.pq.codebooks.cpu().numpy()
    assert (cb.view(np.uint16) == g["codebooks"].view(np.uint16)).mean() > 0.995
    np.testing.assert_allclose(cb.astype(np.float32), g["codebooks"].astype(np.float32), atol=4e-3, rtol=0)
    np.testing.assert_allclose(metrics["avg_distortion"], g["avg_distortion"], rtol=1e-3)
    np.testing.assert_allclose(metrics["sparsity_fraction"], g["sparsity_fraction"], atol=1e-3)


def _stack(tmp_path, n_layers, batch, prefill):
    cfg = RFSNConfig(hidden_dim=256, num_heads=8, num_kv_heads=2, head_dim=64, num_subspaces=8, subspace_dim=8,
                     num_rvq_layers=0, hot_capacity=32, warm_capacity=1024, block_size_seq=16, batch_size=batch,
                     disk_cache_dir=str(tmp_path))
    g = torch.Generator(device="cuda").manual_seed(7)
    layers = []
    for i in range(n_layers):
        layer = RFSNDecoderLayerMLX(cfg, layer_idx=i, weight_dtype=torch.float16, init="normal", seed=2)
        k = torch.randn((batch, prefill, 2, 64), generator=g, device="cuda").half()
        v = torch.randn((batch, prefill, 2, 64), generator=g, device="cuda").half()
        idx = torch.randint(0, batch * prefill * 2, (8, 256), generator=g, device="cuda")
        flat = k.reshape(-1, 64)
        layer.quantizer.pq.codebooks = torch.stack([flat[idx[m], 8 * m:8 * m + 8] for m in range(8)]).contiguous()
        layer.cache.update(k, v, layer.quantizer)
        layers.append(layer)
    return layers


def test_decoder_stack_graph_replay_matches_eager(tmp_path):
    """A multi-layer cache-backed decode step through the public layer API captures into one
    CUDA graph (no host syncs or pageable uploads on the path).  Each replay re-encodes the
    step's token into the same slot and reruns every layer's attention: replays with new
    inputs written into the captured input buffer (output first filled with NaN) equal the
    eager step at the same position on those inputs."""
    xs = torch.randn((5, 2, 1, 256), generator=torch.Generator().manual_seed(11)).half().cuda()

    def step(layers, x):
        for layer in layers:
            x = layer(x, use_cache=True)
        return x

    refs = {}
    for last in (3, 4):  # eager stacks stepped with xs[0..2], then xs[last] as the fourth token
        eager = _stack(tmp_path / f"e{last}", 3, 2, 200)
        for t in range(3):
            step(eager, xs[t])
        refs[last] = step(eager, xs[last]).float().cpu().numpy()
        assert eager[0].cache.total_tokens == 204
        for layer in eager:
            layer.cache.close()
    graphed = _stack(tmp_path / "g", 3, 2, 200)
    for t in range(3):
        step(graphed, xs[t])
    torch.cuda.synchronize()
    xin = xs[3].clone()
    out = torch.empty_like(xin)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        out.copy_(step(graphed, xin))
    for last in (3, 4, 3, 4):
        xin.copy_(xs[last])
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        close(got, refs[last], f"graph replay with token {last} vs eager")
    assert graphed[0].cache.total_tokens == 204
    del graph
    for layer in graphed:
        layer.cache.close()
