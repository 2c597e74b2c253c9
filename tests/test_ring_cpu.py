"""Context-parallel ring schedule on CPU gloo ranks (world 2 and 3).

The ring's host logic (zig-zag sharding, per-step block selection, K/V rotation with
send/recv, log-sum-exp merging) runs unchanged; the block compute is the CPU oracle,
injected through the RingBackend interface.  A rank that dies mid-ring must make the
others fail fast instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket
import tempfile
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import attention_oracle as oracle


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleBackend:
    """Test-only compute for the ring: fp64 oracle blocks, fp64 LSE merge."""

    def block(self, q, k, v, out, lse, *, causal, q_pos0, kv_pos0):
        o, l = oracle.attention_fp64(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal,
                                     q_pos0=q_pos0, kv_pos0=kv_pos0)
        out.copy_(torch.from_numpy(o))
        lse.copy_(torch.from_numpy(l))

    def merge(self, acc_o, acc_lse, part_o, part_lse):
        o, l = oracle.lse_merge([(acc_o.double().numpy(), acc_lse.double().numpy()),
                                 (part_o.double().numpy(), part_lse.double().numpy())])
        acc_o.copy_(torch.from_numpy(o))
        acc_lse.copy_(torch.from_numpy(l))

    def finalize(self, acc_o, out):
        out.copy_(acc_o)


def _full_inputs(bh=2, seq=96, dim=128):
    g = torch.Generator().manual_seed(1)
    return tuple(torch.randn((bh, seq, dim), generator=g, dtype=torch.float32) for _ in range(3))


def _ring_rank(rank, world, port, outdir, die_at_step):
    import torch.distributed as dist

    from avo import ring

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        q, k, v = (ring.zigzag_shard(t, rank, world, dim=1).contiguous() for t in _full_inputs())
        runner = ring.RingAttention(q, k, v, rank=rank, world=world, backend=OracleBackend())
        if die_at_step is not None and rank == world - 1:
            # Leave between steps, with nothing in flight: the peers must notice.
            os._exit(3)
        out, lse = runner.forward()
        torch.save({"out": out, "lse": lse}, os.path.join(outdir, f"rank{rank}.pt"))
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"rank{rank}.err"), "w") as fh:
            fh.write(traceback.format_exc())
        os._exit(1)


@pytest.mark.parametrize("world", [1, 2, 3])
def test_ring_matches_full_causal_attention(world):
    from avo import ring

    port = _port()
    with tempfile.TemporaryDirectory() as outdir:
        mp.start_processes(_ring_rank, args=(world, port, outdir, None), nprocs=world, join=True,
                           start_method="spawn")
        shards = [torch.load(os.path.join(outdir, f"rank{r}.pt")) for r in range(world)]
    out = ring.zigzag_unshard([s["out"] for s in shards], world, dim=1)
    lse = ring.zigzag_unshard([s["lse"].unsqueeze(-1) for s in shards], world, dim=1).squeeze(-1)
    q, k, v = _full_inputs()
    ref_o, ref_lse = oracle.attention_fp64(q.numpy(), k.numpy(), v.numpy(), True)
    assert np.abs(out.numpy() - ref_o).max() < 1e-5
    assert np.abs(lse.numpy() - ref_lse).max() < 1e-5


def test_dead_rank_fails_peers_fast():
    """Rank 1 exits between steps; rank 0, left alone, must end with an error of its own
    (connection closed or process-group timeout) well inside the bound, not hang."""
    port = _port()
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as outdir:
        procs = [ctx.Process(target=_ring_rank, args=(r, 2, port, outdir, 0)) for r in range(2)]
        for p in procs:
            p.start()
        procs[0].join(timeout=60)
        alive = procs[0].is_alive()
        for p in procs:
            if p.is_alive():
                p.kill()
            p.join()
        assert not alive, "surviving rank hung after its peer died"
        assert procs[1].exitcode == 3
        assert procs[0].exitcode != 0
        assert os.path.exists(os.path.join(outdir, "rank0.err"))


def test_step_blocks_cover_causal_triangle_exactly():
    from avo import ring

    for world in (1, 2, 3, 4, 8):
        chunk = 4
        seq = 2 * world * chunk
        covered = np.zeros((seq, seq), dtype=int)
        for rank in range(world):
            early, late = ring.zigzag_chunks(rank, world)
            q_positions = list(range(early * chunk, (early + 1) * chunk)) + list(
                range(late * chunk, (late + 1) * chunk))
            for step in range(world):
                src = (rank - step) % world
                s_early, s_late = ring.zigzag_chunks(src, world)
                kv_positions = list(range(s_early * chunk, (s_early + 1) * chunk)) + list(
                    range(s_late * chunk, (s_late + 1) * chunk))
                for b in ring.step_blocks(rank, world, step, chunk):
                    for i in range(b.q_len):
                        qp = q_positions[b.q_start + i]
                        assert qp == b.q_pos0 + i or b.q_len > chunk
                        for j in range(b.kv_len):
                            kp = kv_positions[b.kv_start + j]
                            if not b.causal or kp <= qp:
                                covered[qp, kp] += 1
        assert np.array_equal(covered, np.tril(np.ones((seq, seq), dtype=int))), world


def test_step_blocks_balance_work():
    from avo import ring

    world, chunk = 8, 16
    for rank in range(world):
        for step in range(world):
            work = 0
            for b in ring.step_blocks(rank, world, step, chunk):
                work += b.q_len * b.kv_len // (2 if b.causal else 1)
            assert work == 2 * chunk * chunk


def test_zigzag_round_trip():
    from avo import ring

    x = torch.arange(2 * 3 * 24 * 2).reshape(2, 3, 24, 2)
    shards = [ring.zigzag_shard(x, r, 3, dim=2) for r in range(3)]
    assert torch.equal(ring.zigzag_unshard(shards, 3, dim=2), x)
    with pytest.raises(ValueError):
        ring.zigzag_shard(x, 0, 5, dim=2)
