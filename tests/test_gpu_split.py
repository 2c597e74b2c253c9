"""Split work plans on the B200 (avo_b200_attn_fwd_ws): items cut between CTAs and merged
by log-sum-exp inside the launch.

Each case first asserts, through the host-side plan enumeration, that the sizes really
select the plan under test (1 = whole-item waves plus a split tail, 2 = causal head
groups), then compares the split launch with the whole-item launch (avo_b200_attn_fwd)
and with an fp32 reference of the same bf16 inputs: O max-abs <= 2e-2, mean-abs <= 2e-3,
LSE max-abs <= 1e-3.  Three launches in a row check that the workspace flags come back
to zero after each launch.
"""

from __future__ import annotations

import pytest

from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu

CASES = [
    # (batch, heads, seq, causal, plan mode)
    ((1, 2, 4096, 128), False, 1),     # 32 items on 148 SMs: every item in 4 pieces
    ((1, 8, 8192, 128), False, 1),     # the target point's head shard on one of 8 GPUs
    ((1, 2, 16384, 128), False, 1),    # B1 H16 S16384's shard on one of 8 GPUs
    ((1, 1, 1000, 128), False, 1),     # 4 items of 8 tiles: each in 2 pieces
    ((1, 4, 512, 128), False, 0),      # 8 items of 4 tiles: splitting would not pay
    ((1, 20, 4096, 128), True, 2),     # causal: per-CTA lists over groups of heads
    ((1, 160, 1000, 128), True, 2),    # the same with a clipped last block
    ((1, 3, 1000, 128), True, 0),      # causal, few items: longest first in waves
]


def _fp32_ref(q, k, v, causal):
    from avo.benchmark import fp32_reference

    return fp32_reference(q, k, v, causal)


@pytest.mark.parametrize("shape,causal,mode", CASES)
def test_split_plan_matches_whole_items_and_reference(b200, shape, causal, mode):
    import torch

    batch, heads, seq, _ = shape
    got_mode = b200.schedule_units(batch * heads, seq, seq, causal, split=True,
                                   sm_count=torch.cuda.get_device_properties(0).multi_processor_count)[0]
    assert got_mode == mode
    q, k, v = oracle.make_inputs(shape, seed=5)
    dq, dk, dv = (t.cuda() for t in (q, k, v))
    whole_o, whole_lse = b200.attention_forward(dq, dk, dv, causal, split=False)
    ref_o, ref_lse = _fp32_ref(dq, dk, dv, causal)
    for _ in range(3):
        out, lse = b200.attention_forward(dq, dk, dv, causal, split=True)
        torch.cuda.synchronize()
        b200.check_status(dq.device)
        assert torch.isfinite(out.float()).all()
        diff = (out.float() - ref_o).abs()
        assert diff.max().item() <= oracle.MAX_ABS_TOL, diff.max().item()
        assert diff.mean().item() <= oracle.MEAN_ABS_TOL, diff.mean().item()
        assert (lse - ref_lse).abs().max().item() <= oracle.LSE_TOL
        # against the whole-item launch: only the accumulation order differs
        assert (out.float() - whole_o.float()).abs().max().item() <= 1.6e-2
        assert (lse - whole_lse).abs().max().item() <= 1e-4
    ws = b200.workspace(dq.device)
    assert int(ws[:4096].view(torch.int32).abs().sum().item()) == 0  # flags back to zero


def test_split_plan_small_case_against_fp64_oracle(b200):
    import numpy as np
    import torch

    shape = (1, 2, 2048, 128)
    assert b200.schedule_units(2, 2048, 2048, False, split=True,
                               sm_count=torch.cuda.get_device_properties(0).multi_processor_count)[0] == 1
    q, k, v = oracle.make_inputs(shape, seed=11)
    out, lse = b200.attention_forward(*(t.cuda() for t in (q, k, v)), False, split=True)
    torch.cuda.synchronize()
    b200.check_status(out.device)
    ref_o, ref_lse = oracle.attention_fp64(*(t.float().numpy() for t in (q, k, v)), False)
    metrics = oracle.error_metrics(out.float().cpu().numpy(), ref_o, lse.cpu().numpy(), ref_lse)
    assert np.isfinite(out.float().cpu().numpy()).all()
    assert oracle.within_tolerance(metrics), metrics
