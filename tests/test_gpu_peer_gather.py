"""The output all-gather fused into decode attention over NVLink peer memory (rfsn_peer_gather).

Needs two GPUs (one rank per GPU; the kernel's last CTA waits on the other GPU's
launch): skipped on a one-GPU machine.  Each rank holds its own batch shard;
after every gathered launch -- eager calls and CUDA-graph replays with new
queries -- every rank's gathered output must equal the concatenation of all
ranks' local outputs, exchanged for the check over NCCL.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int) -> None:
    import datetime

    import torch.distributed as dist

    from apple_b200 import kernels as K
    from apple_b200.sharding import PeerGather
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        B, Hkv, G, D, T = 3, 4, 4, 64, 700
        Hq = Hkv * G
        pq = torch.randn((8, 256, 8), generator=g, device=dev).half()
        qz = K.QuantizerBuffers(pq, None, 0.0, 0)
        warm = K.CodeStoreBuffers(qz, rows=B * Hkv, cap=T)
        k = torch.randn((B, T, Hkv, D), generator=g, device=dev).half()
        v = torch.randn((B, T, Hkv, D), generator=g, device=dev).half()
        K.encode_kv(qz, k, v, warm, 0, 0)
        segs = [(K.STORE_WARM, 0, 0, T, 0)]
        qpos = torch.full((B, 1, Hq), T - 1, dtype=torch.int32, device=dev)
        q = torch.randn((B, 1, Hq, D), generator=g, device=dev).half()
        out = torch.empty_like(q)
        peer = PeerGather(B, 1, Hq, D, rank, world, dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        entry = K.attention_call(qz, q, out, segs, kv_heads=Hkv, qpos=qpos, warm=warm, memo=False, gather=peer)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            K.run_attention(entry, q, out, qpos, status)
        full_ref = torch.empty((B * world, 1, Hq, D), dtype=torch.float16, device=dev)
        for it in range(6):
            q.copy_(torch.randn(q.shape, generator=g, device=dev).half())
            peer.full.fill_(float("nan"))
            if it % 2:
                graph.replay()
            else:
                K.run_attention(entry, q, out, qpos, status)
            torch.cuda.synchronize()
            dist.all_gather_into_tensor(full_ref, out)
            torch.cuda.synchronize()
            assert int(status.item()) == 0, status.item()
            assert torch.equal(peer.full, full_ref), f"rank {rank} iteration {it}"
        del graph
        torch.cuda.synchronize()
        dist.barrier()
        peer.close()
    finally:
        dist.destroy_process_group()


def test_peer_gather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs (one rank per GPU)")
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")
