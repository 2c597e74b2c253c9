"""GPU parity of the block kernel (strided views, position offsets), the LSE merge and
fp32->bf16 kernels, and the ring schedule on one GPU, all through the C ABI."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu


def _rand_bf16(shape, seed):
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(torch.bfloat16)


@pytest.mark.parametrize(
    "seq_q,seq_kv,causal,q_pos0,kv_pos0",
    [
        (256, 256, True, 0, 0),        # plain diagonal
        (256, 384, False, 0, 0),       # rectangular, full
        (300, 200, True, 1000, 900),   # offsets, ragged, partially masked
        (128, 128, True, 96, 100),     # first rows see no key at all
        (512, 128, True, 0, 10000),    # every row sees nothing: O = 0, LSE = -inf
        (640, 1000, True, 400, 0),     # long rectangular causal
    ],
)
def test_block_kernel_with_offsets_and_strides(b200, seq_q, seq_kv, causal, q_pos0, kv_pos0):
    import torch

    bh = 3
    # Views with head strides larger than the rows they cover.
    q_buf = _rand_bf16((bh, seq_q + 64, 128), 1).cuda()
    kv_buf = _rand_bf16((2, bh, seq_kv + 128, 128), 2).cuda()
    q = q_buf[:, 32:32 + seq_q]
    k = kv_buf[0, :, 128:128 + seq_kv]
    v = kv_buf[1, :, 128:128 + seq_kv]
    out_buf = torch.full((bh, seq_q + 16, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    out = out_buf[:, 8:8 + seq_q]
    lse_buf = torch.full((bh, seq_q + 8), 7.0, dtype=torch.float32, device="cuda")
    lse = lse_buf[:, 4:4 + seq_q]
    b200.attention_block(q, k, v, out, lse, causal=causal, q_pos0=q_pos0, kv_pos0=kv_pos0)
    torch.cuda.synchronize()
    b200.check_status("cuda:0")
    ref_o, ref_lse = oracle.attention_fp64(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                           v.float().cpu().numpy(), causal, q_pos0=q_pos0, kv_pos0=kv_pos0)
    got_o = out.float().cpu().numpy()
    got_lse = lse.cpu().numpy()
    metrics = oracle.error_metrics(got_o, ref_o, got_lse, ref_lse)
    assert metrics["max_abs"] <= oracle.MAX_ABS_TOL and metrics["mean_abs"] <= oracle.MEAN_ABS_TOL, metrics
    assert metrics["lse_max_abs"] <= oracle.LSE_TOL, metrics
    assert np.array_equal(np.isneginf(got_lse), np.isneginf(ref_lse))
    # Nothing outside the views was written.
    assert torch.all(out_buf[:, :8] == 7.0) and torch.all(out_buf[:, 8 + seq_q:] == 7.0)
    assert torch.all(lse_buf[:, :4] == 7.0) and torch.all(lse_buf[:, 4 + seq_q:] == 7.0)


def test_lse_merge_and_finalize(b200):
    import torch

    bh, rows = 4, 300
    g = torch.Generator().manual_seed(5)
    acc_o = torch.randn((bh, rows, 128), generator=g)
    acc_lse = torch.randn((bh, rows), generator=g) * 4
    acc_lse[0, :10] = float("-inf")                    # empty accumulator rows
    part_o = torch.randn((bh, rows, 128), generator=g).to(torch.bfloat16)
    part_lse = torch.randn((bh, rows), generator=g) * 4
    part_lse[1, :7] = float("-inf")                    # empty partial rows
    part_lse[0, :3] = float("-inf")                    # both empty
    want_o, want_lse = oracle.lse_merge([(acc_o.numpy(), acc_lse.numpy()),
                                         (part_o.float().numpy(), part_lse.numpy())])
    d_acc_o, d_acc_lse = acc_o.cuda(), acc_lse.cuda()
    # Merge into a row-slice view of a larger accumulator (head stride != rows*128).
    big_o = torch.zeros((bh, rows + 20, 128), device="cuda")
    big_lse = torch.zeros((bh, rows + 20), device="cuda")
    big_o[:, 20:] = d_acc_o
    big_lse[:, 20:] = d_acc_lse
    b200.lse_merge(big_o[:, 20:], big_lse[:, 20:], part_o.cuda(), part_lse.cuda())
    out = torch.empty((bh, rows, 128), dtype=torch.bfloat16, device="cuda")
    b200.acc_to_bf16(big_o[:, 20:], out)
    torch.cuda.synchronize()
    got_o = big_o[:, 20:].cpu().numpy()
    got_lse = big_lse[:, 20:].cpu().numpy()
    assert np.array_equal(np.isneginf(got_lse), np.isneginf(want_lse))
    fin = np.isfinite(want_lse)
    assert np.abs(got_lse[fin] - want_lse[fin]).max() < 1e-5
    assert np.abs(got_o - want_o).max() < 1e-4
    assert np.abs(out.float().cpu().numpy() - got_o).max() <= np.abs(got_o).max() * 2 ** -8
    assert torch.all(big_o[:, :20] == 0)


def test_ring_single_gpu_equals_causal_attention(b200):
    import torch

    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "avo-ampere_b200"))
    from avo import ring

    q, k, v = oracle.make_inputs((1, 4, 1024, 128), seed=21)
    dq, dk, dv = (t.reshape(4, 1024, 128).cuda() for t in (q, k, v))
    runner = ring.RingAttention(dq, dk, dv, rank=0, world=1, backend=ring.CudaRingBackend(b200))
    out, lse = runner.forward()
    torch.cuda.synchronize()
    b200.check_status("cuda:0")
    ref_o, ref_lse = oracle.attention_fp64(*(t.reshape(4, 1024, 128).float().numpy() for t in (q, k, v)), True)
    metrics = oracle.error_metrics(out.float().cpu().numpy(), ref_o, lse.cpu().numpy(), ref_lse)
    assert oracle.within_tolerance(metrics), metrics
    # Same again with reused buffers.
    out2, _ = runner.forward()
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
