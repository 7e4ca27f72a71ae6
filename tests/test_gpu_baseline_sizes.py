"""Parity at the BASELINE configurations' own sizes (configs 2, 3, 4 and 5).

The smaller parity cases elsewhere cover the edge cases; these run the product
kernels on the full workloads the benchmark times and check them against the
numpy oracle (oracle/restate.py) on sampled rows:

* config 2: batch 8, 8 KV heads, GQA 4, 32768-token window (1024 hot fp16 +
  31744 warm PQ 16x4 + dense RVQ + top-8 sparse); 4 rows through the oracle.
* config 3: batch 32, 4 KV heads, GQA 8, 16384-token window (512 hot + PQ 8x8);
  4 rows.
* config 4: batch 4, 131072-token window: 188 cold chunks of 512 tokens in a
  device chunk pool + 32768 warm + 2048 hot, 190 segments; 2 rows.
* config 5: 1,048,576 vectors through the spill encoder; every PQ and RVQ code
  compared with the oracle encoder.

Codes: equal to the oracle's except where the two candidates' squared
distances tie to fp32 rounding, proven per mismatch in float64 against the
rounding bound of the reference's formula (tie_bound).  RVQ codes are compared
on vectors whose PQ codes agree (a PQ tie changes the residual the RVQ stage
sees).  Attention: the elementwise bound |out - ref| <= 2e-3 |ref| + 2e-3 rms
and, per query head, ||out - ref||_2 <= 2e-3 ||ref||_2; the observed maximum
relative errors are printed beside the bounds (pytest -s).
"""
import numpy as np
import pytest
import torch

from oracle import restate as R
from tests.parity import check_codes

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from apple_b200 import kernels as K


def attn_stats(out, ref, what):
    """Assert both attention bounds; return the observed maxima."""
    out = np.asarray(out, np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    err = np.abs(out - ref)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    bad = err > 2e-3 * np.abs(ref) + 2e-3 * rms
    assert not bad.any(), f"{what}: {int(bad.sum())} elements off (max err {err.max():.3e}, rms {rms:.3e})"
    vec_rel = np.linalg.norm(out - ref, axis=1) / np.maximum(np.linalg.norm(ref, axis=1), 1e-30)
    assert (vec_rel <= 2e-3).all(), f"{what}: per-head relative error {vec_rel.max():.3e} > 2e-3"
    big = np.abs(ref) >= 0.05 * rms
    s = {"max_abs": float(err.max()), "max_rel_vs_rms": float(err.max() / rms),
         "max_rel_elem": float((err[big] / np.abs(ref[big])).max()), "max_rel_head_l2": float(vec_rel.max())}
    print(f"{what}: max |d| {s['max_abs']:.2e} = {s['max_rel_vs_rms']:.2e} rms; max elementwise relative "
          f"{s['max_rel_elem']:.2e} (|ref| >= 0.05 rms); max per-head l2 relative {s['max_rel_head_l2']:.2e} "
          f"(bound 2e-3)")
    return s


def row_codes(store, kv, slot, row, first, count, qz):
    """Oracle Codes [count, 1, ...] of one row's tokens read back from a device code store."""
    pq = store.read(kv, "pq", slot, row, first, count).cpu().numpy()
    if qz.L:
        rvq = store.read(kv, "rvq", slot, row, first, count).cpu().numpy().astype(np.uint16)
        mask = store.read(kv, "active", slot, row, first, count)[:, 0].cpu().numpy().astype(bool)
    else:
        rvq = np.zeros((count, 0), np.uint16)
        mask = np.zeros((count,), bool)
    if qz.sparse_topk:
        spi = store.read(kv, "sp_idx", slot, row, first, count).cpu().numpy()
        spv = store.read(kv, "sp_val", slot, row, first, count).cpu().numpy()
    else:
        spi, spv = np.zeros((count, 0), np.uint8), np.zeros((count, 0), np.float16)
    return R.Codes(pq[:, None], rvq[:, None], mask[:, None], spi[:, None], spv[:, None])


def as_dict(c, L):
    d = {"pq": c.pq[:, 0], "mask": c.mask[:, 0], "rvq": c.rvq[:, 0, 0] if L else None}
    if c.sp_idx.shape[-1]:
        d["sp_idx"], d["sp_val"] = c.sp_idx[:, 0], c.sp_val[:, 0]
    return d


def sampled_codebooks(flat, M, ds, Kr, L, g, gc):
    """PQ centroids sampled from the data (a k-means initialisation step); RVQ rows from PQ residuals."""
    D = flat.shape[1]
    idx = torch.randint(0, flat.shape[0], (M, 256), generator=g, device=flat.device)
    pq_cb = torch.stack([flat[idx[m], m * ds:(m + 1) * ds] for m in range(M)]).contiguous()
    if not L:
        return pq_cb, None
    qz_pq = K.QuantizerBuffers(pq_cb, None, float("inf"), 0)
    samp = flat[torch.randint(0, flat.shape[0], (4096,), generator=g, device=flat.device)].contiguous()
    st = K.CodeStoreBuffers(qz_pq, rows=1, cap=4096)
    res = torch.empty_like(samp)
    K.encode(qz_pq, samp.view(1, 4096, 1, D), st, 0, 0, residual_out=res.view(1, 4096, 1, D))
    rvq_cb = res[torch.randperm(4096, generator=gc)[:Kr].to(flat.device)].reshape(1, Kr, D).clone()
    rvq_cb[:, 0] = 0
    return pq_cb, rvq_cb


def check_rows(out, q, rows, Hkv, G, window, what):
    """Oracle attention (attention.py:39-105 restated) of sampled rows over their windows.

    window(b, h) -> list of (tier name, K [n, 1, D] fp16, V [n, 1, D] fp16) in window order:
    the oracle's decode of the device codes for coded tiers, the exact tokens for the hot tier."""
    D = q.shape[-1]
    stats = []
    for row in rows:
        b, h = divmod(row, Hkv)
        parts_k, parts_v = [], []
        for _, a, bb in window(b, h):
            parts_k.append(a)
            parts_v.append(bb)
        kw = np.concatenate(parts_k, 0)
        vw = np.concatenate(parts_v, 0)
        T = kw.shape[0]
        qh = q[b, :, h * G:(h + 1) * G].astype(np.float16)
        ref = R.blockwise_exact_attention(qh, kw, vw, D ** -0.5, 128, True, np.full((1, G), T - 1, np.int32))
        stats.append(attn_stats(out[b, :, h * G:(h + 1) * G], ref, f"{what} row {row}"))
    return stats


def _decode_check(qz, store, kv, slot, row, first, count, codes, oq):
    """The device decoder on these tokens is bit-exact with the oracle decode; returns the window part."""
    dev = torch.empty((1, count, 1, qz.D), dtype=torch.float16, device="cuda")
    one = K.CodeStoreBuffers(qz, rows=1, cap=count)
    # copy the row's blocks into a one-row store so the public decoder can read them
    nb = (count + 15) // 16
    b0 = first // 16
    one.data[0, 0, :nb].copy_(store.data[slot, row, b0:b0 + nb])
    K.decode_codes(qz, one, 0, first - b0 * 16, count, dev, kv=kv)
    ref = oq.decode(codes)
    np.testing.assert_array_equal(dev.cpu().numpy()[0, :, 0].view(np.uint16), ref[:, 0].view(np.uint16))
    return ref[:, 0]


def test_config2_full_size():
    """BASELINE configs[1] at its own size: B8, Hq32/Hkv8, D64, 32768 tokens, the headline workload."""
    B, Hq, Hkv, D, T, hot, M, ds, S = 8, 32, 8, 64, 32768, 1024, 16, 4, 8
    G, warm = Hq // Hkv, T - hot
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(1)
    gc = torch.Generator().manual_seed(1)
    k = torch.randn((B, T, Hkv, D), generator=g, device=dev)
    k[..., torch.randperm(D, generator=gc)[:4].to(dev)] *= 10.0
    k = k.half()
    v = torch.randn((B, T, Hkv, D), generator=g, device=dev).half()
    pq_cb, rvq_cb = sampled_codebooks(torch.cat([k.reshape(-1, D), v.reshape(-1, D)]), M, ds, 256, 1, g, gc)
    qz = K.QuantizerBuffers(pq_cb, rvq_cb, -1.0, S)
    ws = K.CodeStoreBuffers(qz, rows=B * Hkv, cap=warm)
    K.encode_kv(qz, k[:, :warm], v[:, :warm], ws, 0, 0)
    hot_k = k[:, warm:].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    hot_v = v[:, warm:].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    q = torch.randn((B, 1, Hq, D), generator=g, device=dev).half()
    qpos = torch.full((B, 1, Hq), T - 1, dtype=torch.int32, device=dev)
    out = torch.full_like(q, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    segs = [(K.STORE_WARM, 0, 0, warm, 0), (K.STORE_HOT, 0, 0, hot, warm)]
    K.decode_attention(qz, q, out, segs, kv_heads=Hkv, qpos=qpos, hot=(hot_k, hot_v), warm=ws, device_status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    outh, qh = out.cpu().numpy(), q.cpu().numpy()
    assert np.isfinite(outh).all()
    pq_h, rvq_h = pq_cb.cpu().numpy(), rvq_cb.cpu().numpy()
    oq = R.Quantizer(pq_h, rvq_h, -1.0, sparse_topk=S)
    kh, vh = k[:, :, :, :].cpu().numpy(), v.cpu().numpy()
    ties = [0, 0]
    for row in (0, 21, 42, 63):
        b, h = divmod(row, Hkv)
        for kv, x in ((0, kh), (1, vh)):
            got = row_codes(ws, kv, 0, row, 0, warm, qz)
            want = oq.compress(x[b, :warm, h:h + 1])
            t = check_codes(x[b, :warm, h], pq_h, rvq_h, -1.0, as_dict(got, 1), as_dict(want, 1), f"cfg2 row {row}")
            ties[0] += t[0]
            ties[1] += t[1]
    print(f"cfg2 codes of 4 rows x K,V x {warm} tokens: {ties[0]} PQ and {ties[1]} RVQ mismatches, all fp32 ties")

    def window(b, h):
        row = b * Hkv + h
        kc, vc = row_codes(ws, 0, 0, row, 0, warm, qz), row_codes(ws, 1, 0, row, 0, warm, qz)
        wk = _decode_check(qz, ws, 0, 0, row, 0, warm, kc, oq)
        wv = _decode_check(qz, ws, 1, 0, row, 0, warm, vc, oq)
        return [("warm", wk, wv), ("hot", kh[b, warm:, h], vh[b, warm:, h])]

    check_rows(outh, qh, (0, 21, 42, 63), Hkv, G, lambda b, h: [(n, a[:, None], c[:, None]) for n, a, c in window(b, h)],
               "cfg2")


def test_config3_full_size():
    """BASELINE configs[2]'s attention at its own size: B32, Hq32/Hkv4 (GQA 8), 16384 tokens,
    512 hot (the first tokens) + PQ 8x8 warm."""
    B, Hq, Hkv, D, T, hot, M, ds = 32, 32, 4, 64, 16384, 512, 8, 8
    G, warm = Hq // Hkv, T - hot
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(2)
    gc = torch.Generator().manual_seed(2)
    k = torch.randn((B, T, Hkv, D), generator=g, device=dev).half()
    v = torch.randn((B, T, Hkv, D), generator=g, device=dev).half()
    pq_cb, _ = sampled_codebooks(torch.cat([k.reshape(-1, D), v.reshape(-1, D)]), M, ds, 0, 0, g, gc)
    qz = K.QuantizerBuffers(pq_cb, None, 0.0, 0)
    ws = K.CodeStoreBuffers(qz, rows=B * Hkv, cap=warm)
    K.encode_kv(qz, k[:, hot:], v[:, hot:], ws, 0, 0)
    hot_k = k[:, :hot].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    hot_v = v[:, :hot].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    q = torch.randn((B, 1, Hq, D), generator=g, device=dev).half()
    qpos = torch.full((B, 1, Hq), T - 1, dtype=torch.int32, device=dev)
    out = torch.full_like(q, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    segs = [(K.STORE_HOT, 0, 0, hot, 0), (K.STORE_WARM, 0, 0, warm, hot)]
    K.decode_attention(qz, q, out, segs, kv_heads=Hkv, qpos=qpos, hot=(hot_k, hot_v), warm=ws, device_status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    outh, qh = out.cpu().numpy(), q.cpu().numpy()
    pq_h = pq_cb.cpu().numpy()
    oq = R.Quantizer(pq_h, np.zeros((0, 256, D), np.float16), 0.0)
    kh, vh = k.cpu().numpy(), v.cpu().numpy()
    rows = (0, 37, 90, 127)
    n_pq = 0
    for row in rows:
        b, h = divmod(row, Hkv)
        for kv, x in ((0, kh), (1, vh)):
            got = row_codes(ws, kv, 0, row, 0, warm, qz)
            want = oq.compress(x[b, hot:, h:h + 1])
            n_pq += check_codes(x[b, hot:, h], pq_h, None, 0.0, as_dict(got, 0), as_dict(want, 0), f"cfg3 row {row}")[0]
    print(f"cfg3 codes of 4 rows x K,V x {warm} tokens: {n_pq} PQ mismatches, all fp32 ties")

    def window(b, h):
        row = b * Hkv + h
        wk = _decode_check(qz, ws, 0, 0, row, 0, warm, row_codes(ws, 0, 0, row, 0, warm, qz), oq)
        wv = _decode_check(qz, ws, 1, 0, row, 0, warm, row_codes(ws, 1, 0, row, 0, warm, qz), oq)
        return [("hot", kh[b, :hot, h][:, None], vh[b, :hot, h][:, None]), ("warm", wk[:, None], wv[:, None])]

    check_rows(outh, qh, rows, Hkv, G, window, "cfg3")


def test_config4_full_size():
    """BASELINE configs[3] at its own size: B4, Hq32/Hkv8, 131072 tokens = 188 cold chunks of 512
    (device chunk pool, one segment each) + 32768 warm + 2048 hot; keys drift per chunk
    (random walk of the chunk mean, step 0.05) plus N(0, 1) noise."""
    B, Hq, Hkv, D, T, hot, warm, chunk, M, ds, S = 4, 32, 8, 64, 131072, 2048, 32768, 512, 16, 4, 8
    G = Hq // Hkv
    n_cold = T - hot - warm
    n_chunks = n_cold // chunk
    assert n_chunks == 188
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(3)
    gc = torch.Generator().manual_seed(3)
    steps = torch.randn((B, T // chunk, 1, D), generator=g, device=dev) * 0.05
    mean = torch.cumsum(steps, dim=1).repeat_interleave(chunk, dim=1)
    k = (torch.randn((B, T, Hkv, D), generator=g, device=dev) + mean).half()
    v = torch.randn((B, T, Hkv, D), generator=g, device=dev).half()
    pq_cb, rvq_cb = sampled_codebooks(torch.cat([k.reshape(-1, D), v.reshape(-1, D)]), M, ds, 256, 1, g, gc)
    qz = K.QuantizerBuffers(pq_cb, rvq_cb, -1.0, S)
    pool = K.CodeStoreBuffers(qz, rows=B * Hkv, cap=chunk, slots=n_chunks)
    for c in range(n_chunks):
        K.encode_kv(qz, k[:, c * chunk:(c + 1) * chunk], v[:, c * chunk:(c + 1) * chunk], pool, c, 0)
    ws = K.CodeStoreBuffers(qz, rows=B * Hkv, cap=warm)
    K.encode_kv(qz, k[:, n_cold:n_cold + warm], v[:, n_cold:n_cold + warm], ws, 0, 0)
    hot_k = k[:, T - hot:].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    hot_v = v[:, T - hot:].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    segs = [(K.STORE_COLD, c, 0, chunk, c * chunk) for c in range(n_chunks)]
    segs += [(K.STORE_WARM, 0, 0, warm, n_cold), (K.STORE_HOT, 0, 0, hot, n_cold + warm)]
    q = torch.randn((B, 1, Hq, D), generator=g, device=dev).half()
    qpos = torch.full((B, 1, Hq), T - 1, dtype=torch.int32, device=dev)
    out = torch.full_like(q, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    K.decode_attention(qz, q, out, segs, kv_heads=Hkv, qpos=qpos, hot=(hot_k, hot_v), warm=ws, cold=pool,
                       device_status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    outh, qh = out.cpu().numpy(), q.cpu().numpy()
    oq = R.Quantizer(pq_cb.cpu().numpy(), rvq_cb.cpu().numpy(), -1.0, sparse_topk=S)
    rows = (5, 30)
    kh = {r: k[r // Hkv, :, r % Hkv].cpu().numpy() for r in rows}
    vh = {r: v[r // Hkv, :, r % Hkv].cpu().numpy() for r in rows}
    # codes of one cold chunk and of the warm run of each sampled row vs the oracle encoder
    for row in rows:
        for kv, x in ((0, kh[row]), (1, vh[row])):
            c = 101
            check_codes(x[c * chunk:(c + 1) * chunk], oq.pq_codebooks, oq.rvq_codebooks, -1.0,
                        as_dict(row_codes(pool, kv, c, row, 0, chunk, qz), 1),
                        as_dict(oq.compress(x[c * chunk:(c + 1) * chunk, None]), 1), f"cfg4 row {row} chunk {c}")

    def window(b, h):
        row = b * Hkv + h
        parts = []
        for c in range(n_chunks):
            kc, vc = row_codes(pool, 0, c, row, 0, chunk, qz), row_codes(pool, 1, c, row, 0, chunk, qz)
            parts.append(("cold", oq.decode(kc), oq.decode(vc)))
        kc, vc = row_codes(ws, 0, 0, row, 0, warm, qz), row_codes(ws, 1, 0, row, 0, warm, qz)
        parts.append(("warm", _decode_check(qz, ws, 0, 0, row, 0, warm, kc, oq)[:, None],
                      _decode_check(qz, ws, 1, 0, row, 0, warm, vc, oq)[:, None]))
        parts.append(("hot", kh[row][T - hot:, None], vh[row][T - hot:, None]))
        return parts

    check_rows(outh, qh, rows, Hkv, G, window, "cfg4")


def config5_inputs(seed=4, N=1 << 20, D=64):
    """BASELINE configs[4]'s vectors and codebooks: half N(0,1), half a 256-component Gaussian
    mixture (centres N(0,1), sigma 0.1); PQ 8x8 and RVQ Kr256 codebooks seeded alike."""
    rng = np.random.default_rng(seed)
    half = N // 2
    centres = rng.standard_normal((256, D)).astype(np.float32)
    x = np.concatenate([rng.standard_normal((half, D)).astype(np.float32),
                        centres[rng.integers(0, 256, N - half)] + 0.1 * rng.standard_normal((N - half, D))])
    pq_cb = (rng.standard_normal((8, 256, 8)) * 0.8).astype(np.float16)
    rvq_cb = (rng.standard_normal((1, 256, D)) * 0.3).astype(np.float16)
    rvq_cb[:, 0] = 0
    return x.astype(np.float16), pq_cb, rvq_cb


def test_config5_every_code_of_1m_vectors():
    """Spill encoder on all 1,048,576 vectors: every PQ and RVQ code vs the oracle encoder."""
    x, pq_cb, rvq_cb = config5_inputs()
    N, D = x.shape
    thr = 0.005
    qz = K.QuantizerBuffers(torch.from_numpy(pq_cb).cuda(), torch.from_numpy(rvq_cb).cuda(), thr, 0)
    st = K.CodeStoreBuffers(qz, rows=1, cap=N)
    K.encode(qz, torch.from_numpy(x).cuda().view(1, N, 1, D), st, 0, 0)
    torch.cuda.synchronize()
    got = {"pq": st.read_rows(0, "pq", 0, 0, N)[0].cpu().numpy(),
           "mask": st.read_rows(0, "active", 0, 0, N)[0, :, 0].cpu().numpy().astype(bool),
           "rvq": st.read_rows(0, "rvq", 0, 0, N)[0, :, 0].cpu().numpy().astype(np.int64)}
    oq = R.Quantizer(pq_cb, rvq_cb, thr)
    n_pq = n_rvq = 0
    step = 1 << 17
    for a in range(0, N, step):
        pqc, rvc, mask, offs, _, _ = oq.encode_flat(x[a:a + step])
        dense = np.zeros(mask.shape[0], np.int64)
        dense[offs] = rvc[:, 0]
        want = {"pq": pqc, "mask": mask, "rvq": dense}
        part = {kk: vv[a:a + step] for kk, vv in got.items()}
        t = check_codes(x[a:a + step], pq_cb, rvq_cb, thr, part, want, f"cfg5 vectors {a}..")
        n_pq += t[0]
        n_rvq += t[1]
    print(f"cfg5: {N} vectors, {N * 8} PQ codes ({n_pq} fp32-tie mismatches), RVQ codes of the active vectors "
          f"({n_rvq} fp32-tie mismatches)")
