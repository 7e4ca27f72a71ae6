"""Decode-attention benchmark for the B200 RFSN compressed-KV path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (Llama-3.2-1B-shaped layer): batch 8, 32 query
heads, 8 KV heads (GQA 4), head_dim 64, 32768-token context = 1024 hot fp16
tokens + 31744 warm tokens coded as PQ M=16x4 (K=256) + one dense RVQ stage
(Kr=256) + top-8 fp16 sparse residual; K has 4 outlier channels x10; seed 1.
A step is one fused decode-attention pass (new query vs the whole window) for
the batch.  Inputs are larger than L2 (183 MB of codes + hot KV per step), so
no L2 flush is needed between steps.

value     steps/s with inputs resident in HBM (CUDA events on the launch stream).
e2e       the same metric through the public API (RFSNv10KVCacheMLX.attention_forward),
          with the query copied from pinned host memory and the output copied back
          to host every step.
roofline  algorithmic bytes of one step / its duration vs MEASURED_PEAKS.json hbm_gbs.
cpu_baseline  the numpy oracle (oracle/restate.py) on a bounded sample, host cores.

Multi-GPU (torchrun): every rank runs the full per-GPU workload (weak scaling);
after each step the ranks all-gather their outputs over NCCL; time is the max
over ranks.  --impl reference times the CPU oracle port (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode attn steps/s per layer at 32K ctx"
UNIT = "steps/s"
CFG = dict(batch=8, q_heads=32, kv_heads=8, head_dim=64, context=32768, hot=1024, M=16, ds=4, K=256, L=1, Kr=256,
           sparse=8, outliers=4, seed=1)


def workload_desc(n_gpus: int) -> dict:
    return {"workload": "BASELINE configs[1]: Llama-3.2-1B-shaped layer decode, random init",
            "global_batch": CFG["batch"] * n_gpus, "batch_per_gpu": CFG["batch"], "seq_len": CFG["context"],
            "q_heads": CFG["q_heads"], "kv_heads": CFG["kv_heads"], "head_dim": CFG["head_dim"],
            "hot_tokens": CFG["hot"], "warm_tokens": CFG["context"] - CFG["hot"],
            "warm_codes": "PQ M16x4 K256 u8 + RVQ L1 Kr256 u8 (dense) + top-8 sparse fp16/u8",
            "parallelism": f"batch-shard dp{n_gpus}", "l2": "inputs > L2 (183 MB/step), no flush"}


def algorithmic_bytes() -> int:
    c = CFG
    rows = c["batch"] * c["kv_heads"]
    warm = c["context"] - c["hot"]
    per_row = c["hot"] * 2 * c["head_dim"] * 2 + warm * 2 * (c["M"] + c["L"] + 3 * c["sparse"])
    qo = 2 * c["batch"] * c["q_heads"] * c["head_dim"] * 2
    return rows * per_row + qo


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# synthetic workload (GPU)
# ---------------------------------------------------------------------------

def build_workload(device, seed):
    import torch
    from apple_b200 import kernels as K
    c = CFG
    g = torch.Generator(device=device).manual_seed(seed)
    B, Hkv, D, T, hot = c["batch"], c["kv_heads"], c["head_dim"], c["context"], c["hot"]
    warm = T - hot
    k = torch.randn((B, T, Hkv, D), generator=g, device=device, dtype=torch.float32)
    gc = torch.Generator().manual_seed(seed)
    ch = torch.randperm(D, generator=gc)[: c["outliers"]]
    k[..., ch.to(device)] *= 10.0
    k = k.half()
    v = torch.randn((B, T, Hkv, D), generator=g, device=device, dtype=torch.float32).half()
    # codebooks: PQ centroids sampled from the data (k-means init step), RVQ rows from PQ residuals
    M, ds, Kc = c["M"], c["ds"], c["K"]
    flat = torch.cat([k.reshape(-1, D), v.reshape(-1, D)], 0)
    idx = torch.randint(0, flat.shape[0], (M, Kc), generator=g, device=device)
    pq_cb = torch.stack([flat[idx[m], m * ds:(m + 1) * ds] for m in range(M)]).contiguous()
    qz_pq = K.QuantizerBuffers(pq_cb, None, float("inf"), 0)
    samp = flat[torch.randint(0, flat.shape[0], (4096,), generator=g, device=device)].contiguous()
    st = K.CodeStoreBuffers(qz_pq, rows=1, cap=4096)
    res = torch.empty_like(samp)
    K.encode(qz_pq, samp.view(1, 4096, 1, D), st, 0, 0, residual_out=res.view(1, 4096, 1, D))
    rvq_cb = res[torch.randperm(4096, generator=gc)[: c["Kr"]].to(device)].reshape(1, c["Kr"], D).clone()
    rvq_cb[:, 0] = 0
    qz = K.QuantizerBuffers(pq_cb, rvq_cb, -1.0, c["sparse"])
    ws = K.CodeStoreBuffers(qz, rows=B * Hkv, cap=warm)
    K.encode(qz, k[:, :warm], ws, 0, 0, kv=0)
    K.encode(qz, v[:, :warm], ws, 0, 0, kv=1)
    hot_k = k[:, warm:].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    hot_v = v[:, warm:].permute(0, 2, 1, 3).reshape(B * Hkv, hot, D).contiguous()
    q = torch.randn((B, 1, c["q_heads"], D), generator=g, device=device).half()
    qpos = torch.full((B, 1, c["q_heads"]), T - 1, dtype=torch.int32, device=device)
    segs = [(K.STORE_WARM, 0, 0, warm, 0), (K.STORE_HOT, 0, 0, hot, warm)]
    torch.cuda.synchronize()
    return dict(qz=qz, warm=ws, hot=(hot_k, hot_v), q=q, qpos=qpos, segs=segs, k=k, v=v)


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    def __init__(self, device_index: int):
        self.proc = None
        self.idx = device_index
        self.path = ROOT / "gpurun_out" / f"clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}",
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        try:
            rows = [l.split(",") for l in self.path.read_text().strip().splitlines() if l.strip()]
            sm = [float(r[0]) for r in rows]
            mx = [float(r[1]) for r in rows]
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[3 + i] and "Not" not in r[3 + i]})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                    "reasons": reasons, "samples": len(rows)}
        except Exception as e:  # pragma: no cover - best effort
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": str(e)}


# ---------------------------------------------------------------------------
# CPU baseline: the numpy oracle on a sample of (sequence, KV-head) rows
# ---------------------------------------------------------------------------

def build_cpu_sample(kv_heads_sample: int, seed: int = 1):
    """Seeded synthetic rows of the same workload, encoded by the oracle (setup, untimed)."""
    from oracle import restate as R
    c = CFG
    D, T, hot, M, ds = c["head_dim"], c["context"], c["hot"], c["M"], c["ds"]
    warm = T - hot
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((T, kv_heads_sample, D)).astype(np.float32)
    k[..., rng.choice(D, c["outliers"], replace=False)] *= 10.0
    k = k.astype(np.float16)
    v = rng.standard_normal((T, kv_heads_sample, D)).astype(np.float16)
    flat = np.concatenate([k.reshape(-1, D), v.reshape(-1, D)], 0)
    pq_cb = np.stack([flat[rng.integers(0, flat.shape[0], c["K"]), m * ds:(m + 1) * ds] for m in range(M)])
    _, res = R.pq_quantize(flat[rng.integers(0, flat.shape[0], 4096)], pq_cb)
    rvq_cb = res[rng.permutation(4096)[: c["Kr"]]].reshape(1, c["Kr"], D).copy()
    rvq_cb[:, 0] = 0
    oq = R.Quantizer(pq_cb, rvq_cb, -1.0, c["sparse"])
    kc, vc = oq.compress(k[:warm]), oq.compress(v[:warm])
    G = c["q_heads"] // c["kv_heads"]
    q = rng.standard_normal((1, kv_heads_sample * G, D)).astype(np.float16)
    return dict(oq=oq, kc=kc, vc=vc, hot_k=k[warm:], hot_v=v[warm:], q=q, rows=kv_heads_sample)


def time_cpu_step(s) -> float:
    """Seconds per full-batch decode step: materialise the window (decode) + fp32 blockwise
    attention, as the reference does (cache.py:344-428, attention.py:39-105), scaled from
    the sampled rows to batch x kv_heads rows."""
    from oracle import restate as R
    c = CFG
    D, T = c["head_dim"], c["context"]
    t0 = time.perf_counter()
    kw = np.concatenate([s["oq"].decode(s["kc"]), s["hot_k"]], 0)
    vw = np.concatenate([s["oq"].decode(s["vc"]), s["hot_v"]], 0)
    R.blockwise_exact_attention(s["q"], kw, vw, D ** -0.5, 128, True, np.full((1, s["q"].shape[1]), T - 1))
    dt = time.perf_counter() - t0
    return dt * (c["batch"] * c["kv_heads"]) / s["rows"]


def run_reference(args) -> None:
    """CPU oracle port of the reference algorithm on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    try:
        import torch
        torch.set_num_threads(os.cpu_count() or 1)
    except ImportError:
        pass
    heads = 1
    s = build_cpu_sample(heads, CFG["seed"])
    for _ in range(max(0, args.warmup)):
        time_cpu_step(s)
    times = [time_cpu_step(s) for _ in range(args.steps)]
    sec = statistics.mean(times)
    val = 1.0 / sec
    sample = f"1 sequence x {heads} of 8 KV heads (4 query heads each), full 32K window; scaled x{64 // heads}"
    line = {"metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": workload_desc(args.gpus),
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

def run_b200(args) -> None:
    import torch
    import torch.distributed as dist
    from apple_b200 import kernels as K

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    w = build_workload(dev, CFG["seed"] + rank)
    out = torch.empty_like(w["q"])
    gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=dev) if world > 1 else None
    launches_per_step = 2  # fused decode-attention + LSE merge

    def step():
        K.decode_attention(w["qz"], w["q"], out, w["segs"], kv_heads=CFG["kv_heads"], qpos=w["qpos"], causal=True,
                           hot=w["hot"], warm=w["warm"])
        if gathered is not None:
            dist.all_gather_into_tensor(gathered, out)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_per_step = ms / args.steps
    value = world * 1e3 / ms_per_step

    # kernel-only timing for the roofline (no collective in between)
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        K.decode_attention(w["qz"], w["q"], out, w["segs"], kv_heads=CFG["kv_heads"], qpos=w["qpos"], causal=True,
                           hot=w["hot"], warm=w["warm"])
    e3.record(stream)
    torch.cuda.synchronize()
    kern_ms = e2.elapsed_time(e3) / args.steps

    # end-to-end through the public API with host buffers
    e2e = e2e_public_api(w, args, dev)

    if world > 1:
        dist.barrier()
    if rank == 0:
        peak, peak_kind = measured_peak()
        nbytes = algorithmic_bytes()
        achieved = nbytes / (kern_ms * 1e-3) / 1e9
        cs = build_cpu_sample(2, CFG["seed"])
        time_cpu_step(cs)
        cpu_sec = statistics.mean([time_cpu_step(cs) for _ in range(3)])
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": workload_desc(world),
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                             "algorithmic_bytes_per_step": nbytes, "kernel_ms": kern_ms},
                "cpu_baseline": {"value": 1.0 / cpu_sec, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                                 "sample": "numpy oracle: 1 sequence x 2 of 8 KV heads, full 32K window, "
                                           "mean of 3 steps, scaled x32"},
                "e2e": e2e, "gpu_launches": launches_per_step * args.steps, "clocks": clocks.summary()}
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def e2e_public_api(w, args, dev) -> dict:
    """Same decode step through the public cache API with pinned-host q in and output out."""
    import torch
    try:
        from apple_b200.cache import RFSNv10KVCacheMLX  # noqa: F401
        from apple_b200.bench_support import public_api_step
    except ImportError:
        public_api_step = None
    c = CFG
    h_q = w["q"].cpu().pin_memory()
    h_out = torch.empty_like(h_q).pin_memory()
    if public_api_step is None:
        from apple_b200 import kernels as K
        d_q = torch.empty_like(w["q"])
        d_out = torch.empty_like(w["q"])

        def step():
            d_q.copy_(h_q, non_blocking=True)
            K.decode_attention(w["qz"], d_q, d_out, w["segs"], kv_heads=c["kv_heads"], qpos=w["qpos"], causal=True,
                               hot=w["hot"], warm=w["warm"])
            h_out.copy_(d_out, non_blocking=True)
        api = "kernels.decode_attention (C ABI)"
    else:
        step, api = public_api_step(w, h_q, h_out)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        step()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    nb = h_q.numel() * h_q.element_size()
    return {"value": 1e3 / ms, "unit": UNIT, "h2d_bytes_per_step": nb, "d2h_bytes_per_step": nb, "api": api}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
