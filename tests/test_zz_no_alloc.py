"""avo_b200_attn_fwd_split_noalloc: the no-allocation entry point against the existing one.

The entry point computes the same forward as avo_b200_attn_fwd as consecutive key/value
blocks merged by log-sum-exp in scratch the library holds statically.  Each case runs it
twice in a row (the scratch is re-initialised by every call) and compares both results
with avo_b200_attn_fwd on the same inputs, and once with the fp64 oracle.  The file name
puts it last in collection, so it also runs after every other GPU test in one process;
it passes on its own too.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu

# (shape, causal, n_splits); batch*heads*seq <= 16384 rows (the static scratch).
CASES = [
    ((1, 4, 2048, 128), False, 3),
    ((2, 2, 4096, 128), True, 4),    # exactly the row capacity
    ((1, 3, 1000, 128), True, 2),    # ragged sequence, partial last tile in each block
]


@pytest.mark.parametrize("shape,causal,n_splits", CASES)
def test_noalloc_matches_existing_entry_point(b200, shape, causal, n_splits):
    import torch

    q, k, v = oracle.make_inputs(shape, seed=3)
    dq, dk, dv = (t.cuda() for t in (q, k, v))
    ref_o, ref_lse = b200.attention_forward(dq, dk, dv, causal)
    torch.cuda.synchronize()
    b200.check_status(dq.device)
    for _ in range(2):
        out, lse = b200.attention_forward_noalloc(dq, dk, dv, causal, n_splits=n_splits)
        torch.cuda.synchronize()
        b200.check_status(dq.device)
        diff = (out.float() - ref_o.float()).abs()
        # partials pass through bf16 once more than the single-launch path
        assert diff.max().item() <= 2e-2, diff.max().item()
        assert diff.mean().item() <= 2e-3, diff.mean().item()
        assert (lse - ref_lse).abs().max().item() <= 1e-3
    ref64_o, ref64_lse = oracle.attention_fp64(*(t.float().numpy() for t in (q, k, v)), causal)
    metrics = oracle.error_metrics(out.float().cpu().numpy(), ref64_o, lse.cpu().numpy(), ref64_lse)
    assert np.isfinite(out.float().cpu().numpy()).all()
    assert metrics["max_abs"] <= oracle.MAX_ABS_TOL, metrics
    assert metrics["mean_abs"] <= oracle.MEAN_ABS_TOL, metrics
    assert metrics["lse_max_abs"] <= oracle.LSE_TOL, metrics


def test_noalloc_rejects_problems_beyond_its_scratch(b200):
    import torch

    shape = (1, 1, b200.NOALLOC_MAX_ROWS + 128, 128)
    q = torch.zeros(shape, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(b200.B200AttentionError, match="too large"):
        b200.attention_forward_noalloc(q, q, q, False)
