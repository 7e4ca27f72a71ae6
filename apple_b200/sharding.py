"""Batch x KV-head sharding of decode attention over the GPUs of one node.

Every (sequence, KV head) row of the cache is independent: its hot tokens,
codes and attention never touch another row, and the codebooks (a few tens of
KB) are replicated.  So the units are split across ranks with no exchange in
the kernel:

* batch >= world: contiguous sequence ranges (sizes differ by at most one);
* batch < world: each sequence is split over world // batch ranks by
  contiguous KV-head groups (with their query heads), which needs
  world % batch == 0 and kv_heads % (world // batch) == 0.

The one exchange is the all-gather of the attention outputs (fp16
[b, Q, Hq_local, D] per rank), since the output projection needs every head
of every sequence.  Two forms:

* ``PeerGather``: fused into the attention kernel over NVLink peer memory
  (rfsn_peer_gather): the CTA that merges a row stores its output into every
  rank's gathered-output buffer, and the launch's last CTA waits for every
  rank before copying the complete output out (batch shards of equal size).
* ``gather_outputs``: a separate collective over the process group's backend
  (NCCL on GPUs, gloo for the CPU tests); shards of unequal size are padded
  to the largest.
"""
from __future__ import annotations

from dataclasses import dataclass
import ctypes as C
from typing import List, Optional

import torch


@dataclass(frozen=True)
class Shard:
    batch0: int  # sequences [batch0, batch1)
    batch1: int
    head0: int   # KV heads [head0, head1)
    head1: int

    @property
    def batch(self) -> int:
        return self.batch1 - self.batch0

    @property
    def kv_heads(self) -> int:
        return self.head1 - self.head0


def plan_shards(batch: int, kv_heads: int, world: int) -> List[Shard]:
    """The shard of every rank (index = rank)."""
    if batch <= 0 or kv_heads <= 0 or world <= 0:
        raise ValueError("batch, kv_heads and world must be positive")
    if batch >= world:
        base, extra = divmod(batch, world)
        out, b = [], 0
        for r in range(world):
            n = base + (1 if r < extra else 0)
            out.append(Shard(b, b + n, 0, kv_heads))
            b += n
        return out
    if world % batch:
        raise ValueError(f"with batch {batch} < world {world}, world must be a multiple of batch")
    groups = world // batch
    if kv_heads % groups:
        raise ValueError(f"kv_heads {kv_heads} must split into {groups} groups per sequence")
    per = kv_heads // groups
    return [Shard(r // groups, r // groups + 1, (r % groups) * per, (r % groups + 1) * per) for r in range(world)]


def gather_outputs(local: torch.Tensor, shards: List[Shard], rank: int, group_size: int, q_per_kv: int,
                   group=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather each rank's attention output [b_r, Q, Hq_r, D] into the full [B, Q, Hq, D].

    Hq_r = shard.kv_heads * q_per_kv (query head h reads KV head h // q_per_kv).  ``out``
    (contiguous, [B, Q, Hq, D]) receives the result when given; a decode loop passes the
    same buffer every step."""
    import torch.distributed as dist
    if len(shards) != group_size:
        raise ValueError("one shard per rank")
    me = shards[rank]
    Q, D = local.shape[1], local.shape[3]
    if tuple(local.shape) != (me.batch, Q, me.kv_heads * q_per_kv, D):
        raise ValueError(f"rank {rank}: local output {tuple(local.shape)} does not match its shard {me}")
    B = max(s.batch1 for s in shards)
    Hq = max(s.head1 for s in shards) * q_per_kv
    if all(s.batch == me.batch and s.head0 == 0 and s.head1 * q_per_kv == Hq and s.batch0 == r * me.batch
           for r, s in enumerate(shards)):
        # equal batch shards in rank order: gather straight into the full output
        full = out if out is not None else torch.empty((B, Q, Hq, D), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(full, local.contiguous(), group=group)
        return full
    max_b = max(s.batch for s in shards)
    max_h = max(s.kv_heads for s in shards) * q_per_kv
    buf = torch.zeros((max_b, Q, max_h, D), dtype=local.dtype, device=local.device)
    buf[: me.batch, :, : local.shape[2]] = local
    flat = torch.empty((group_size * max_b,) + tuple(buf.shape[1:]), dtype=buf.dtype, device=buf.device)
    dist.all_gather_into_tensor(flat, buf, group=group)  # rank r's shard at rows [r*max_b, (r+1)*max_b)
    allbuf = flat.view((group_size,) + tuple(buf.shape))
    full = out if out is not None else torch.empty((B, Q, Hq, D), dtype=local.dtype, device=local.device)
    for r, s in enumerate(shards):
        full[s.batch0:s.batch1, :, s.head0 * q_per_kv:s.head1 * q_per_kv] = \
            allbuf[r, : s.batch, :, : s.kv_heads * q_per_kv]
    return full


class PeerGather:
    """Fused output all-gather over peer memory for one decode-attention shape (rfsn_peer_gather).

    Each rank holds ``local_seqs`` consecutive sequences (rank r: [r * local_seqs, (r + 1) *
    local_seqs)) of the ``world * local_seqs`` in the gathered output ``full`` [total, Q, Hq, D]
    fp16.  The constructor is collective: every rank allocates its peer-visible buffers
    (rfsn_peer_alloc), the CUDA IPC handles are exchanged over the process group, and every rank
    maps the others' (rfsn_peer_open).  Pass the instance as ``gather`` to a decode-attention call:
    that launch then also leaves the whole batch's output in ``full`` on every rank.  Every rank
    must make the same sequence of gathered launches, each rank on its own GPU."""

    def __init__(self, local_seqs: int, queries: int, q_heads: int, head_dim: int, rank: int, world: int,
                 device: torch.device, group=None):
        import torch.distributed as dist
        from . import _lib
        if not 2 <= world <= _lib.RFSN_MAX_PEERS:
            raise ValueError(f"peer gather needs 2..{_lib.RFSN_MAX_PEERS} ranks, got {world}")
        self.rank, self.world = rank, world
        self.total = local_seqs * world
        self.full = torch.empty((self.total, queries, q_heads, head_dim), dtype=torch.float16, device=device)
        buf_bytes = 2 * self.full.numel() * 2
        self._flag_off = (buf_bytes + 255) // 256 * 256
        self._step_off = self._flag_off + 8 * world
        lib = _lib.lib()
        with torch.cuda.device(device):
            own = C.c_void_p()
            handle = (C.c_char * 64)()
            _lib.check("rfsn_peer_alloc", lib.rfsn_peer_alloc(self._step_off + 8, C.byref(own), handle))
            self._own = own.value
            handles: List[bytes] = [b""] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self._opened: List[int] = []
            bases = []
            for r in range(world):
                if r == rank:
                    bases.append(self._own)
                    continue
                ptr = C.c_void_p()
                _lib.check("rfsn_peer_open", lib.rfsn_peer_open((C.c_char * 64).from_buffer_copy(handles[r]),
                                                                C.byref(ptr)))
                self._opened.append(ptr.value)
                bases.append(ptr.value)
        st = _lib.PeerGather()
        st.num_ranks, st.rank = world, rank
        st.seq_offset, st.total_seqs = rank * local_seqs, self.total
        for r, base in enumerate(bases):
            st.buffers[r] = base
            st.flags[r] = base + self._flag_off
        st.step = self._own + self._step_off
        st.out_full = self.full.data_ptr()
        self.struct = st
        self.pointer = C.pointer(st)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank's last gathered launch)."""
        from . import _lib
        lib = _lib.lib()
        for ptr in self._opened:
            lib.rfsn_peer_close(C.c_void_p(ptr))
        self._opened = []
        if self._own:
            lib.rfsn_peer_free(C.c_void_p(self._own))
            self._own = None
