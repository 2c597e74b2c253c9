"""Context-parallel ring attention (causal, zig-zag), one process per GPU.

The reference is single-GPU (every run is on cuda:0, avo/benchmark.py:212); this is
new.  The sequence of S positions is cut into 2N chunks of L = S / 2N; rank r holds
the query, key and value rows of chunks r and 2N-1-r ("zig-zag", which gives every
rank the same amount of causal work).  Over N steps each rank's K/V pair travels
around the ring (rank r sends to r+1 and receives from r-1, NCCL point-to-point over
NVLink/NVSwitch, issued before the step's compute so the transfer overlaps it).  At
step s a rank holds the K/V of rank src = (r - s) mod N and computes:

* s == 0 (own K/V): early Q x early K/V (causal diagonal), late Q x early K/V (full),
  late Q x late K/V (causal diagonal);
* src < r: both Q chunks x the early K/V chunk of src (full: every key precedes);
* src > r: the late Q chunk x both K/V chunks of src (full); the early Q chunk sees
  none of them.

Each block yields a normalised partial (O_i bf16, LSE_i fp32); partials are folded
into an fp32 accumulator by log-sum-exp: LSE = log sum_i exp(LSE_i),
O = sum_i exp(LSE_i - LSE) O_i.  The received blocks land in local HBM through NCCL
before any kernel reads them: no kernel reads peer memory.

The compute is injected through ``RingBackend`` so the schedule can be checked on CPU
(gloo) with the oracle in tests; ``CudaRingBackend`` is the product path and calls
only the C-ABI kernels.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Protocol


def zigzag_chunks(rank: int, world: int) -> tuple[int, int]:
    """Chunk indices (early, late) of ``rank`` among 2*world chunks."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return rank, 2 * world - 1 - rank


def zigzag_shard(x, rank: int, world: int, dim: int = -2):
    """Rows of chunks (early, late) of ``rank`` along ``dim``, concatenated."""
    import torch

    seq = x.shape[dim]
    if seq % (2 * world) != 0:
        raise ValueError(f"sequence {seq} not divisible by 2*world={2 * world}")
    chunk = seq // (2 * world)
    early, late = zigzag_chunks(rank, world)
    return torch.cat([x.narrow(dim, early * chunk, chunk), x.narrow(dim, late * chunk, chunk)], dim=dim)


def zigzag_unshard(shards, world: int, dim: int = -2):
    """Inverse of ``zigzag_shard`` given every rank's shard in rank order."""
    import torch

    chunk = shards[0].shape[dim] // 2
    pieces = [None] * (2 * world)
    for rank, shard in enumerate(shards):
        early, late = zigzag_chunks(rank, world)
        pieces[early] = shard.narrow(dim, 0, chunk)
        pieces[late] = shard.narrow(dim, chunk, chunk)
    return torch.cat(pieces, dim=dim)


@dataclass(frozen=True)
class Block:
    """One partial attention: local query rows [q_start, q_start+q_len) of this rank's
    shard against rows [kv_start, kv_start+kv_len) of the K/V shard held at this step."""

    q_start: int
    q_len: int
    kv_start: int
    kv_len: int
    causal: bool
    q_pos0: int
    kv_pos0: int


def step_blocks(rank: int, world: int, step: int, chunk: int) -> list[Block]:
    """The blocks rank ``rank`` computes at ``step`` (chunk = rows per chunk)."""
    src = (rank - step) % world
    my_early, my_late = zigzag_chunks(rank, world)
    src_early, src_late = zigzag_chunks(src, world)
    if step == 0:
        return [
            Block(0, chunk, 0, chunk, True, my_early * chunk, my_early * chunk),
            Block(chunk, chunk, 0, chunk, False, my_late * chunk, my_early * chunk),
            Block(chunk, chunk, chunk, chunk, True, my_late * chunk, my_late * chunk),
        ]
    if src < rank:
        return [Block(0, 2 * chunk, 0, chunk, False, my_early * chunk, src_early * chunk)]
    return [Block(chunk, chunk, 0, 2 * chunk, False, my_late * chunk, src_early * chunk)]


class RingBackend(Protocol):
    def block(self, q, k, v, out, lse, *, causal: bool, q_pos0: int, kv_pos0: int) -> None: ...

    def merge(self, acc_o, acc_lse, part_o, part_lse) -> None: ...

    def finalize(self, acc_o, out) -> None: ...


class CudaRingBackend:
    """The sm_100a kernels through the C ABI (attention block, LSE merge, fp32->bf16)."""

    def __init__(self, binding: Any):
        self.binding = binding

    def block(self, q, k, v, out, lse, *, causal, q_pos0, kv_pos0):
        self.binding.attention_block(q, k, v, out, lse, causal=causal, q_pos0=q_pos0, kv_pos0=kv_pos0)

    def merge(self, acc_o, acc_lse, part_o, part_lse):
        self.binding.lse_merge(acc_o, acc_lse, part_o, part_lse)

    def finalize(self, acc_o, out):
        self.binding.acc_to_bf16(acc_o, out)


class RingAttention:
    """Reusable buffers + schedule for one rank.  ``q``, ``k``, ``v`` are this rank's
    zig-zag shards, [BH, 2L, 128] bf16 contiguous."""

    def __init__(self, q, k, v, *, rank: int, world: int, backend: RingBackend, group=None,
                 comm_stream=None):
        import torch

        if q.dim() != 3 or q.shape != k.shape or q.shape != v.shape:
            raise ValueError("q, k, v must be [BH, 2L, D] shards of equal shape")
        if q.shape[1] % 2:
            raise ValueError("shard length must be even (two chunks)")
        self.q, self.k, self.v = q, k, v
        self.rank, self.world, self.backend, self.group = rank, world, backend, group
        self.chunk = q.shape[1] // 2
        bh, rows, dim = q.shape
        self.acc_o = torch.empty((bh, rows, dim), dtype=torch.float32, device=q.device)
        self.acc_lse = torch.empty((bh, rows), dtype=torch.float32, device=q.device)
        self.part_o = torch.empty((bh, rows, dim), dtype=q.dtype, device=q.device)
        self.part_lse = torch.empty((bh, rows), dtype=torch.float32, device=q.device)
        self.out = torch.empty_like(q)
        self.kv_bufs = [torch.empty((2, bh, rows, dim), dtype=q.dtype, device=q.device) for _ in range(2)]
        self.comm_stream = comm_stream

    def _exchange(self, send_buf, recv_buf):
        import torch.distributed as dist

        nxt = (self.rank + 1) % self.world
        prv = (self.rank - 1) % self.world
        ops = [dist.P2POp(dist.isend, send_buf, nxt, group=self.group),
               dist.P2POp(dist.irecv, recv_buf, prv, group=self.group)]
        return dist.batch_isend_irecv(ops)

    def forward(self):
        """Run the N steps; returns (O bf16 [BH, 2L, D], LSE fp32 [BH, 2L])."""
        self.acc_lse.fill_(float("-inf"))
        self.acc_o.zero_()
        cur = self.kv_bufs[0]
        cur[0].copy_(self.k)
        cur[1].copy_(self.v)
        for step in range(self.world):
            reqs = None
            nxt = self.kv_bufs[(step + 1) % 2]
            if step + 1 < self.world:
                reqs = self._exchange(cur, nxt)
            for blk in step_blocks(self.rank, self.world, step, self.chunk):
                q = self.q[:, blk.q_start:blk.q_start + blk.q_len]
                k = cur[0][:, blk.kv_start:blk.kv_start + blk.kv_len]
                v = cur[1][:, blk.kv_start:blk.kv_start + blk.kv_len]
                po = self.part_o[:, blk.q_start:blk.q_start + blk.q_len]
                pl = self.part_lse[:, blk.q_start:blk.q_start + blk.q_len]
                self.backend.block(q, k, v, po, pl, causal=blk.causal, q_pos0=blk.q_pos0,
                                   kv_pos0=blk.kv_pos0)
                self.backend.merge(self.acc_o[:, blk.q_start:blk.q_start + blk.q_len],
                                   self.acc_lse[:, blk.q_start:blk.q_start + blk.q_len], po, pl)
            if reqs is not None:
                for req in reqs:
                    req.wait()
            cur = nxt
        self.backend.finalize(self.acc_o, self.out)
        return self.out, self.acc_lse
