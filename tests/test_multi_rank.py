"""Multi-rank host logic on CPU: shard plans and the output all-gather over gloo (world size 2).

Each rank computes the oracle's decode attention for its own (sequence,
KV-head) units only; the gathered output must equal the single-process result
bit for bit (the units are independent, so sharding changes no arithmetic).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from apple_b200.sharding import Shard, plan_shards


def test_plan_shards_batch_split():
    assert plan_shards(8, 8, 2) == [Shard(0, 4, 0, 8), Shard(4, 8, 0, 8)]
    assert [s.batch for s in plan_shards(5, 8, 2)] == [3, 2]
    assert plan_shards(8, 8, 1) == [Shard(0, 8, 0, 8)]


def test_plan_shards_head_split():
    assert plan_shards(1, 8, 2) == [Shard(0, 1, 0, 4), Shard(0, 1, 4, 8)]
    assert plan_shards(2, 8, 8)[5] == Shard(1, 2, 2, 4)  # sequence 1, heads [2, 4)
    with pytest.raises(ValueError):
        plan_shards(3, 8, 4)   # world not a multiple of batch
    with pytest.raises(ValueError):
        plan_shards(1, 6, 4)   # heads do not split into 4 groups


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, Hkv, G, T, D, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, 1, Hkv * G, D)).astype(np.float16)
    k = rng.standard_normal((B, T, Hkv, D)).astype(np.float16)
    v = rng.standard_normal((B, T, Hkv, D)).astype(np.float16)
    return q, k, v


def _attend(q, k, v, b0, b1, h0, h1, G):
    from oracle import restate as R
    D = q.shape[-1]
    outs = []
    for b in range(b0, b1):
        qs = q[b][:, h0 * G:h1 * G]
        outs.append(R.blockwise_exact_attention(qs, k[b][:, h0:h1], v[b][:, h0:h1], D ** -0.5, 16, False))
    return np.stack(outs)


def _worker(rank, world, port, case, result_q):
    import torch.distributed as dist
    from apple_b200.sharding import gather_outputs, plan_shards
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, Hkv, G, T, D = case
        q, k, v = _inputs(B, Hkv, G, T, D)
        shards = plan_shards(B, Hkv, world)
        s = shards[rank]
        local = torch.from_numpy(_attend(q, k, v, s.batch0, s.batch1, s.head0, s.head1, G))
        full = gather_outputs(local, shards, rank, world, G)
        if rank == 0:
            result_q.put(full.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(4, 2, 2, 40, 16), (3, 2, 2, 24, 16), (1, 4, 2, 32, 16)])
def test_gather_outputs_two_ranks(case):
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = result_q.get(timeout=90)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    B, Hkv, G, T, D = case
    q, k, v = _inputs(B, Hkv, G, T, D)
    want = _attend(q, k, v, 0, B, 0, Hkv, G)
    np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))
