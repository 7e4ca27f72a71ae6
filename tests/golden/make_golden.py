"""Generate golden fixtures by running the *reference's own* RFSN code.

Run with RFSN_REFERENCE_DIR pointing at a checkout of the reference sources:

    RFSN_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py

The reference is imported unmodified through the torch-CPU ``mlx`` shim
(``oracle/mlx_shim``).  Inputs and codebooks come from numpy generators with
fixed seeds and are injected into the reference objects, exactly as
rfsn_v10_eval_benchmark.py:112-114 injects codebooks.  Each case is written
to ``tests/golden/<case>.npz``; ``tests/test_oracle_golden.py`` checks the
numpy restatement (``oracle/restate.py``) against them and the ``-m gpu``
tests check the CUDA path against the same files.  The files are small and
committed; the GPU machines never need the reference.
"""
from __future__ import annotations

import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.ref_loader import load_reference  # noqa: E402

OUT = Path(__file__).resolve().parent


def seeded_codebooks(rng, m, k, ds, layers, kr, d):
    """PQ ~ N(0, 2/ds) and RVQ ~ N(0, 2/D) fp16 with RVQ row 0 zeroed, as the
    reference initialises them (quantization.py:108-115, 188-197)."""
    pq = (rng.standard_normal((m, k, ds)).astype(np.float32) * np.float32((2.0 / ds) ** 0.5)).astype(np.float16)
    rvq = (rng.standard_normal((layers, kr, d)).astype(np.float32) * np.float32((2.0 / d) ** 0.5)).astype(np.float16)
    if layers:
        rvq[:, 0] = 0
    return pq, rvq


def make_config(ref, **kw):
    base = dict(hidden_dim=512, num_heads=4, head_dim=128, num_layers=2, num_subspaces=8, subspace_dim=16,
                num_rvq_layers=3, rvq_codebook_size=256, rvq_sparsity_threshold=0.25, hot_capacity=16,
                warm_capacity=24, cold_capacity=128, block_size_seq=16, prefetch_throttle_s=0.0)
    base.update(kw)
    return ref["storage"].RFSNConfig(**base)


def make_quantizer(ref, config, pq_cb, rvq_cb):
    mx = sys.modules["mlx.core"]
    hq = ref["quantization"].HybridQuantizerMLX(config)
    hq.pq.codebooks = mx.array(pq_cb, dtype=mx.float16)
    hq.rvq.codebooks = mx.array(rvq_cb, dtype=mx.float16)
    return hq


def case_quantizer(ref, name, seed, cfg_kw, n, scale_half=None, outliers=0):
    """PQ quantize / RVQ encode / hybrid decode on [n, D] fp16 vectors."""
    mx = sys.modules["mlx.core"]
    rng = np.random.default_rng(seed)
    config = make_config(ref, **cfg_kw)
    d, m, ds = config.head_dim, config.num_subspaces, config.subspace_dim
    pq_cb, rvq_cb = seeded_codebooks(rng, m, 1 << config.pq_bits, ds, config.num_rvq_layers,
                                     config.rvq_codebook_size, d)
    x = rng.standard_normal((n, d)).astype(np.float32)
    if scale_half is not None:
        x[: n // 2] *= scale_half
    if outliers:
        ch = rng.choice(d, size=outliers, replace=False)
        x[:, ch] *= 10.0
    x = x.astype(np.float16)
    hq = make_quantizer(ref, config, pq_cb, rvq_cb)
    xa = mx.array(x, dtype=mx.float16)
    pq_codes, residual = hq.pq.quantize(xa)
    rvq_codes, mask, offsets = hq.rvq.encode(residual)
    decoded = hq.decode(pq_codes, rvq_codes, mask, offsets)
    pq_only = hq.pq.decode(pq_codes)
    np.savez_compressed(
        OUT / f"{name}.npz", x=x, pq_codebooks=pq_cb, rvq_codebooks=rvq_cb,
        threshold=np.float32(config.rvq_sparsity_threshold),
        pq_codes=np.asarray(pq_codes), residual=np.asarray(residual), rvq_codes=np.asarray(rvq_codes),
        rvq_mask=np.asarray(mask), rvq_offsets=np.asarray(offsets), decoded=np.asarray(decoded),
        pq_decoded=np.asarray(pq_only))


def case_attention(ref, name, seed):
    """RFSNHybridAttentionMLX on compressed stores vs blockwise over decoded K/V
    (rfsn_v10_mlx_ane_complete.py:418-446), plus a non-causal and a default-position call."""
    mx = sys.modules["mlx.core"]
    q_mod, a_mod = ref["quantization"], ref["attention"]
    rng = np.random.default_rng(seed)
    config = make_config(ref)
    pq_cb, rvq_cb = seeded_codebooks(rng, 8, 256, 16, 3, 256, 128)
    hq = make_quantizer(ref, config, pq_cb, rvq_cb)
    q = rng.standard_normal((2, 4, 128)).astype(np.float16)
    keys = rng.standard_normal((24, 4, 128)).astype(np.float16)
    values = rng.standard_normal((24, 4, 128)).astype(np.float16)
    ks = q_mod._compress_tensor_sequence(mx.array(keys), hq)
    vs = q_mod._compress_tensor_sequence(mx.array(values), hq)
    dk = q_mod._decode_compressed_tensor(ks, hq)
    dv = q_mod._decode_compressed_tensor(vs, hq)
    attn = a_mod.RFSNHybridAttentionMLX(config)
    qa = mx.array(q)
    pos = mx.array([12, 18], dtype=mx.int32)
    out_causal = attn(q=qa, key_store=ks, value_store=vs, quantizer=hq, causal=True, query_positions=pos)
    out_plain = attn(q=qa, key_store=ks, value_store=vs, quantizer=hq, causal=False)
    pos_bh = np.array([[3, 9, 15, 23], [0, 1, 2, 23]], dtype=np.int32)
    out_bh = a_mod._blockwise_exact_attention(q=qa, keys=dk, values=dv, scale=128 ** -0.5, block_size=16,
                                              causal=True, query_positions=mx.array(pos_bh))
    np.savez_compressed(
        OUT / f"{name}.npz", q=q, keys=keys, values=values, pq_codebooks=pq_cb, rvq_codebooks=rvq_cb,
        threshold=np.float32(0.25), positions=np.array([12, 18], np.int32), positions_bh=pos_bh,
        key_pq=np.asarray(ks.pq_codes), key_rvq=np.asarray(ks.rvq_codes), key_mask=np.asarray(ks.rvq_mask),
        key_offsets=np.asarray(ks.rvq_offsets), val_pq=np.asarray(vs.pq_codes),
        decoded_keys=np.asarray(dk), decoded_values=np.asarray(dv),
        out_causal=np.asarray(out_causal), out_plain=np.asarray(out_plain), out_bh=np.asarray(out_bh))


STAT_KEYS = ("window_start", "window_end", "window_tokens", "context_window", "query_tokens", "used_router",
             "hot_tokens_materialized", "warm_tokens_materialized", "cold_tokens_materialized",
             "reconstructed_tokens", "warm_chunk_decodes", "cold_chunk_decodes", "cold_chunks_touched",
             "cold_chunk_cache_hits", "cold_chunk_cache_misses")


def case_cache(ref, name, seed, n_tokens, queries, windows):
    """RFSNv10KVCacheMLX tiering + materialize + attention (cache.py:89-428) with
    the reference test config (hot 16, warm 24, 16-token cold chunks)."""
    mx = sys.modules["mlx.core"]
    rng = np.random.default_rng(seed)
    tmp = Path(tempfile.mkdtemp(prefix="rfsn_golden_"))
    try:
        config = make_config(ref, disk_cache_dir=str(tmp))
        pq_cb, rvq_cb = seeded_codebooks(rng, 8, 256, 16, 3, 256, 128)
        hq = make_quantizer(ref, config, pq_cb, rvq_cb)
        keys = rng.standard_normal((n_tokens, 4, 128)).astype(np.float16)
        values = rng.standard_normal((n_tokens, 4, 128)).astype(np.float16)
        q = rng.standard_normal((1, 4, 128)).astype(np.float16)
        cache = ref["cache"].RFSNv10KVCacheMLX(config, layer_idx=0)
        # two updates so the cold path exercises the partial-chunk merge (cache.py:157-176)
        split = n_tokens - 3
        cache.update(mx.array(keys[:split]), mx.array(values[:split]), hq, disk_dir=tmp)
        cache.update(mx.array(keys[split:]), mx.array(values[split:]), hq, disk_dir=tmp)
        rec = dict(keys=keys, values=values, q=q, pq_codebooks=pq_cb, rvq_codebooks=rvq_cb,
                   threshold=np.float32(0.25), update_split=np.int32(split),
                   tiers=np.array([cache.num_hot, cache.num_warm, cache.num_cold], np.int32),
                   cold_chunk_ids=np.array([m["chunk_id"] for m in cache.cold_chunk_metadata], np.int32),
                   cold_chunk_bounds=np.array([[m["start_token"], m["end_token"]] for m in cache.cold_chunk_metadata],
                                              np.int32).reshape(-1, 2))
        cases = []
        for qi, qpos in enumerate(queries):
            for wi, win in enumerate(windows):
                tag = f"q{qi}_w{wi}"
                kw = dict(query_positions=mx.array([qpos], dtype=mx.int32), context_window=win)
                out = cache.attention_forward(mx.array(q), causal=True, **kw)
                stats_attn = cache.get_last_access_stats()
                k_w, v_w, adj = cache.materialize_window(**kw)
                rec[f"{tag}_out"] = np.asarray(out)
                rec[f"{tag}_keys"] = np.asarray(k_w)
                rec[f"{tag}_values"] = np.asarray(v_w)
                rec[f"{tag}_adjusted"] = np.asarray(adj) if adj is not None else np.array([], np.int32)
                rec[f"{tag}_stats"] = np.array([stats_attn[k] for k in STAT_KEYS], np.int64)
                cases.append((qpos, -1 if win is None else win))
        rec["cases"] = np.array(cases, np.int32)
        mem = cache.memory_usage_bytes()
        rec["memory"] = np.array([mem["hot_bytes"], mem["warm_pq_bytes"], mem["warm_rvq_bytes"],
                                  mem["cold_chunks"], mem["cold_tokens"]], np.int64)
        np.savez_compressed(OUT / f"{name}.npz", **rec)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def case_router(ref, name):
    """AsyncHierarchicalRouterMLX candidate ordering (storage.py:166-182) over chunk files."""
    tmp = Path(tempfile.mkdtemp(prefix="rfsn_router_"))
    try:
        config = make_config(ref, disk_cache_dir=str(tmp), block_size_seq=16)
        ids = [0, 1, 2, 3, 5, 8, 9]
        for cid in ids:
            p = ref["storage"].chunk_file_path(tmp, 0, cid)
            p.write_bytes(b"")
        router = ref["storage"].AsyncHierarchicalRouterMLX(config, layer_idx=0)
        router._load_chunk_sync = lambda cid: {"id": cid}  # no real NPZ needed for ordering
        queries = [(0, 1024, 1), (47, 16, 3), (100, 40, 4), (130, 100, 8), (60, 0, 2)]
        results = []
        for pos, win, k in queries:
            router._cache.clear()
            results.append(router.prefetch_sync(current_position=pos, context_window=win, top_k=k))
        width = max(len(r) for r in results)
        res = np.full((len(results), width), -1, np.int32)
        for i, r in enumerate(results):
            res[i, :len(r)] = r
        np.savez_compressed(OUT / f"{name}.npz", chunk_ids=np.array(ids, np.int32),
                            queries=np.array(queries, np.int32), loaded=res, chunk_size=np.int32(16))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def case_decoder_layer(ref, name, seed):
    """RFSNDecoderLayerMLX (rfsn_v10_mlx_ane_complete.py:55-172): prefill, then cache-backed
    decode steps through hot, warm and cold tiers, plus the dense (no-cache) path.
    Weights are seeded N(0, 1/in) and injected; they are stored as fp16 because the
    reference's Linear casts its weights to the fp16 activations (mlx.nn.Linear)."""
    mx = sys.modules["mlx.core"]
    rng = np.random.default_rng(seed)
    tmp = Path(tempfile.mkdtemp(prefix="rfsn_layer_"))
    try:
        hidden, heads, hd = 256, 4, 64
        config = make_config(ref, hidden_dim=hidden, num_heads=heads, head_dim=hd, num_subspaces=8, subspace_dim=8,
                             num_rvq_layers=1, rvq_codebook_size=64, rvq_sparsity_threshold=0.3, hot_capacity=16,
                             warm_capacity=24, block_size_seq=16, disk_cache_dir=str(tmp))
        layer = ref["rfsn_v10_mlx_ane_complete"].RFSNDecoderLayerMLX(config, layer_idx=0)
        rec = {}
        for nm, (o, i) in dict(q_proj=(hidden, hidden), k_proj=(hidden, hidden), v_proj=(hidden, hidden),
                               o_proj=(hidden, hidden), ffn_up=(2 * hidden, hidden),
                               ffn_down=(hidden, 2 * hidden)).items():
            w = (rng.standard_normal((o, i)) / np.sqrt(i)).astype(np.float16)
            getattr(layer, nm).weight = mx.array(w.astype(np.float32), dtype=mx.float32)
            rec[f"w_{nm}"] = w
        pq_cb, rvq_cb = seeded_codebooks(rng, 8, 256, 8, 1, 64, hd)
        layer.quantizer.pq.codebooks = mx.array(pq_cb, dtype=mx.float16)
        layer.quantizer.rvq.codebooks = mx.array(rvq_cb, dtype=mx.float16)
        rec.update(pq_codebooks=pq_cb, rvq_codebooks=rvq_cb)
        n_prefill, n_decode = 40, 24
        x = rng.standard_normal((1, n_prefill + n_decode, hidden)).astype(np.float16)
        layer.prefill_cache(mx.array(x[:, :n_prefill]))
        outs = []
        for t in range(n_prefill, n_prefill + n_decode):
            outs.append(np.asarray(layer(mx.array(x[:, t:t + 1]), use_cache=True)))
        stats = layer.cache.get_last_access_stats()
        x2 = rng.standard_normal((2, 6, hidden)).astype(np.float16)
        dense = np.asarray(layer(mx.array(x2), use_cache=False))
        rec.update(x=x, n_prefill=np.int32(n_prefill), decode_out=np.concatenate(outs, 1), x_dense=x2,
                   dense_out=dense, last_stats=np.array([stats[k] for k in STAT_KEYS], np.int64),
                   tiers=np.array([layer.cache.num_hot, layer.cache.num_warm, layer.cache.num_cold], np.int32))
        np.savez_compressed(OUT / f"{name}.npz", **rec)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def case_calibration(ref, name, seed, n=2048, iters=10):
    """calibrate_quantizer (rfsn_v10_mlx_ane_complete.py:175-225): k-means PQ codebooks from
    sampled initial centroids.  The sample indices the reference draws are recorded so the
    B200 build can start from the same centroids."""
    mx = sys.modules["mlx.core"]
    rng = np.random.default_rng(seed)
    config = make_config(ref, hidden_dim=512, num_heads=8, head_dim=64, num_subspaces=8, subspace_dim=8,
                         num_rvq_layers=0, rvq_sparsity_threshold=0.5)
    hq = ref["quantization"].HybridQuantizerMLX(config)
    vectors = rng.standard_normal((n, 64)).astype(np.float16)
    drawn = []
    orig = mx.random.randint

    def recording_randint(*a, **kw):
        out = orig(*a, **kw)
        drawn.append(np.asarray(out).astype(np.int64))
        return out

    mx.random.randint = recording_randint
    try:
        metrics = ref["rfsn_v10_mlx_ane_complete"].calibrate_quantizer(hq, mx.array(vectors), num_iterations=iters)
    finally:
        mx.random.randint = orig
    np.savez_compressed(OUT / f"{name}.npz", vectors=vectors, sample_idx=np.stack(drawn),
                        codebooks=np.asarray(hq.pq.codebooks), iters=np.int32(iters),
                        avg_distortion=np.array(metrics["avg_distortion"], np.float64),
                        sparsity_fraction=np.array(metrics["sparsity_fraction"], np.float64), threshold=np.float32(0.5))


def case_gqa_batch(ref, name, seed, batch=3, kv_heads=2, group=4, n_tokens=60, queries=(59, 44, 20),
                   windows=(None, 8, 30)):
    """GQA and batch > 1 pinned to the reference.  GQA: the reference's own Llama adapter
    repeats each KV head over its query group with _repeat_kv (llama32_adapter.py:380-386,
    580-581) before the cache sees it, so the reference result is a cache over the repeated
    heads.  Batch: the reference cache holds one sequence, so a batch is a loop of reference
    caches, one per sequence, each asked at the same query position and window.  Codebooks:
    PQ 16x4 and one dense RVQ stage (threshold -1), the headline configuration's layout."""
    mx = sys.modules["mlx.core"]
    import importlib
    repeat_kv = importlib.import_module("llama32_adapter")._repeat_kv
    rng = np.random.default_rng(seed)
    hq, d = kv_heads * group, 64
    tmp = Path(tempfile.mkdtemp(prefix="rfsn_gqa_"))
    try:
        pq_cb, rvq_cb = seeded_codebooks(rng, 16, 256, 4, 1, 256, d)
        keys = rng.standard_normal((batch, n_tokens, kv_heads, d)).astype(np.float32)
        keys[..., rng.choice(d, size=4, replace=False)] *= 10.0
        keys = keys.astype(np.float16)
        values = rng.standard_normal((batch, n_tokens, kv_heads, d)).astype(np.float16)
        q = rng.standard_normal((batch, hq, d)).astype(np.float16)
        split = n_tokens - 3
        outs = np.zeros((len(queries) * len(windows), batch, hq, d), np.float16)
        stats = np.zeros((len(queries) * len(windows), batch, len(STAT_KEYS)), np.int64)
        cases = []
        for b in range(batch):
            config = make_config(ref, hidden_dim=hq * d, num_heads=hq, head_dim=d, num_subspaces=16, subspace_dim=4,
                                 num_rvq_layers=1, rvq_sparsity_threshold=-1.0, disk_cache_dir=str(tmp / f"s{b}"))
            hqz = make_quantizer(ref, config, pq_cb, rvq_cb)
            cache = ref["cache"].RFSNv10KVCacheMLX(config, layer_idx=0)
            rk = repeat_kv(mx.array(keys[b:b + 1]), group)[0]
            rv = repeat_kv(mx.array(values[b:b + 1]), group)[0]
            cache.update(rk[:split], rv[:split], hqz, disk_dir=tmp / f"s{b}")
            cache.update(rk[split:], rv[split:], hqz, disk_dir=tmp / f"s{b}")
            i = 0
            for qpos in queries:
                for win in windows:
                    out = cache.attention_forward(mx.array(q[b:b + 1]), causal=True,
                                                  query_positions=mx.array([qpos], dtype=mx.int32), context_window=win)
                    outs[i, b] = np.asarray(out)[0]
                    st = cache.get_last_access_stats()
                    stats[i, b] = [st[k] for k in STAT_KEYS]
                    if b == 0:
                        cases.append((qpos, -1 if win is None else win))
                    i += 1
        np.savez_compressed(OUT / f"{name}.npz", keys=keys, values=values, q=q, pq_codebooks=pq_cb,
                            rvq_codebooks=rvq_cb, threshold=np.float32(-1.0), update_split=np.int32(split),
                            group=np.int32(group), cases=np.array(cases, np.int32), out=outs, stats=stats)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def case_chunk_files(ref, name, seed, n_tokens=70, split=44):
    """Cold chunk files written by the reference cache itself (cache.py:134-191 through
    save_compressed_chunk, storage.py:117-135), copied to tests/golden/<name>/ beside an index
    of the inputs that made them.  The first update leaves a 4-token partial chunk; the second
    update's first 16-token piece merges onto it (a 20-token chunk), its rest opens the next."""
    mx = sys.modules["mlx.core"]
    rng = np.random.default_rng(seed)
    tmp = Path(tempfile.mkdtemp(prefix="rfsn_chunks_"))
    try:
        config = make_config(ref, hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=16, subspace_dim=4,
                             num_rvq_layers=1, rvq_sparsity_threshold=0.4, disk_cache_dir=str(tmp))
        pq_cb, rvq_cb = seeded_codebooks(rng, 16, 256, 4, 1, 256, 64)
        hq = make_quantizer(ref, config, pq_cb, rvq_cb)
        keys = rng.standard_normal((n_tokens, 4, 64)).astype(np.float16)
        values = rng.standard_normal((n_tokens, 4, 64)).astype(np.float16)
        cache = ref["cache"].RFSNv10KVCacheMLX(config, layer_idx=0)
        cache.update(mx.array(keys[:split]), mx.array(values[:split]), hq, disk_dir=tmp)
        cache.update(mx.array(keys[split:]), mx.array(values[split:]), hq, disk_dir=tmp)
        outdir = OUT / name
        if outdir.exists():
            shutil.rmtree(outdir)
        outdir.mkdir()
        meta = cache.cold_chunk_metadata
        for m in meta:
            shutil.copy(m["path"], outdir / Path(m["path"]).name)
        np.savez_compressed(outdir / "index.npz", keys=keys, values=values, pq_codebooks=pq_cb, rvq_codebooks=rvq_cb,
                            threshold=np.float32(0.4), update_split=np.int32(split),
                            chunk_ids=np.array([m["chunk_id"] for m in meta], np.int32),
                            chunk_bounds=np.array([[m["start_token"], m["end_token"]] for m in meta], np.int32))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def rope_tables(positions, head_dim, theta=500000.0):
    """Standard rotary tables cos/sin [1, len, head_dim] (the half-split layout of the Llama
    rotary module), as float32."""
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    ang = np.asarray(positions, np.float64)[:, None] * inv[None]
    emb = np.concatenate([ang, ang], axis=-1)
    return np.cos(emb)[None].astype(np.float32), np.sin(emb)[None].astype(np.float32)


def case_llama_layer(ref, name, seed):
    """Llama32DecoderLayerMLX (llama32_adapter.py:417-662): RMSNorm with weights, q/k/v
    projections, RoPE from given position tables, GQA by _repeat_kv, the RFSN cache (prefill,
    then cache-backed decode steps through hot, warm and cold), o_proj, SwiGLU MLP, residuals;
    plus the dense path.  Weights are seeded and injected as fp16."""
    import importlib
    mx = sys.modules["mlx.core"]
    adapter = importlib.import_module("llama32_adapter")
    rng = np.random.default_rng(seed)
    tmp = Path(tempfile.mkdtemp(prefix="rfsn_llama_"))
    try:
        hidden, heads, kv_heads, hd, inter = 128, 2, 1, 64, 256
        config = make_config(ref, hidden_dim=hidden, num_heads=heads, head_dim=hd, num_subspaces=16, subspace_dim=4,
                             num_rvq_layers=1, rvq_codebook_size=256, rvq_sparsity_threshold=0.2, hot_capacity=16,
                             warm_capacity=24, block_size_seq=16, disk_cache_dir=str(tmp))
        w = {}
        for nm, (o, i) in dict(q_proj=(heads * hd, hidden), k_proj=(kv_heads * hd, hidden),
                               v_proj=(kv_heads * hd, hidden), o_proj=(hidden, heads * hd), gate_proj=(inter, hidden),
                               up_proj=(inter, hidden), down_proj=(hidden, inter)).items():
            w[nm] = (rng.standard_normal((o, i)) / np.sqrt(i)).astype(np.float16)
        w["input_layernorm"] = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float16)
        w["post_attention_layernorm"] = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float16)
        layer = adapter.Llama32DecoderLayerMLX(
            config, 0, kv_heads, 1e-5, mx.array(w["input_layernorm"]), mx.array(w["post_attention_layernorm"]),
            *(mx.array(w[k]) for k in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")))
        pq_cb, rvq_cb = seeded_codebooks(rng, 16, 256, 4, 1, 256, hd)
        layer.quantizer.pq.codebooks = mx.array(pq_cb, dtype=mx.float16)
        layer.quantizer.rvq.codebooks = mx.array(rvq_cb, dtype=mx.float16)
        n_prefill, n_decode = 40, 20
        x = rng.standard_normal((1, n_prefill + n_decode, hidden)).astype(np.float16)
        cos, sin = rope_tables(np.arange(n_prefill + n_decode), hd)
        layer.prefill_cache(mx.array(x[:, :n_prefill]), position_embeddings=(cos[:, :n_prefill], sin[:, :n_prefill]))
        outs = []
        for t in range(n_prefill, n_prefill + n_decode):
            outs.append(np.asarray(layer(mx.array(x[:, t:t + 1]), position_embeddings=(cos[:, t:t + 1], sin[:, t:t + 1]),
                                         use_cache=True)))
        stats = layer.cache.get_last_access_stats()
        x2 = rng.standard_normal((1, 6, hidden)).astype(np.float16)
        c2, s2 = rope_tables(np.arange(6), hd)
        dense = np.asarray(layer(mx.array(x2), position_embeddings=(c2, s2), use_cache=False))
        np.savez_compressed(OUT / f"{name}.npz", **{f"w_{k}": v for k, v in w.items()}, pq_codebooks=pq_cb,
                            rvq_codebooks=rvq_cb, x=x, n_prefill=np.int32(n_prefill), cos=cos, sin=sin,
                            decode_out=np.concatenate(outs, 1), x_dense=x2, cos_dense=c2, sin_dense=s2,
                            dense_out=dense, last_stats=np.array([stats[k] for k in STAT_KEYS], np.int64),
                            tiers=np.array([layer.cache.num_hot, layer.cache.num_warm, layer.cache.num_cold],
                                           np.int32), kv_heads=np.int32(kv_heads), eps=np.float32(1e-5))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


CASES = {
    "quant": lambda ref: (
        case_quantizer(ref, "quant_d128_m8x16_rvq3", seed=11, cfg_kw={}, n=96, scale_half=0.01),
        case_quantizer(ref, "quant_d64_m16x4_rvq1_dense", seed=12,
                       cfg_kw=dict(head_dim=64, num_subspaces=16, subspace_dim=4, num_rvq_layers=1,
                                   rvq_sparsity_threshold=-1.0), n=512, outliers=4),
        case_quantizer(ref, "quant_d64_m8x8_rvq1", seed=13,
                       cfg_kw=dict(head_dim=64, num_subspaces=8, subspace_dim=8, num_rvq_layers=1,
                                   rvq_sparsity_threshold=0.5), n=512),
        case_quantizer(ref, "quant_d64_m8x8_pqonly", seed=14,
                       cfg_kw=dict(head_dim=64, num_subspaces=8, subspace_dim=8, num_rvq_layers=1,
                                   rvq_sparsity_threshold=float("inf")), n=256)),
    "attention": lambda ref: case_attention(ref, "attention_hybrid", seed=21),
    "cache": lambda ref: case_cache(ref, "cache_tiers", seed=31, n_tokens=60, queries=[59, 50, 20],
                                    windows=[None, 8, 30]),
    "router": lambda ref: case_router(ref, "router_order"),
    "layer": lambda ref: case_decoder_layer(ref, "decoder_layer", seed=41),
    "calibration": lambda ref: case_calibration(ref, "calibration_kmeans", seed=51),
    "gqa_batch": lambda ref: case_gqa_batch(ref, "gqa_batch_cache", seed=61),
    "chunk_files": lambda ref: case_chunk_files(ref, "ref_chunks", seed=71),
    "llama": lambda ref: case_llama_layer(ref, "llama_layer", seed=81),
}


def main() -> None:
    """python tests/golden/make_golden.py [case ...]  (default: every case)."""
    ref = load_reference()
    for name in (sys.argv[1:] or list(CASES)):
        CASES[name](ref)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
