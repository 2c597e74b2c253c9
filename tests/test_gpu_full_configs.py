"""Full-size workloads on one B200 against a plain PyTorch fp32 reference of the same
bf16 inputs (computed on the GPU, TF32 off), plus sampled rows against the fp64 CPU
oracle.  Tolerance: O max-abs <= 2e-2, mean-abs <= 2e-3, LSE max-abs <= 1e-3, and the
reference scorer's torch.allclose(atol=3e-2, rtol=3e-2) against bf16 SDPA."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu

CONFIGS = {
    "b4_h16_s4096_noncausal": ((4, 16, 4096, 128), False, 1.0),
    "b2_h16_s8192_causal": ((2, 16, 8192, 128), True, 1.0),
    "b1_h16_s16384_noncausal_k3": ((1, 16, 16384, 128), False, 3.0),
    "b1_h16_s32768_causal": ((1, 16, 32768, 128), True, 1.0),
    "b4_h16_s8192_noncausal": ((4, 16, 8192, 128), False, 1.0),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_config_against_fp32_reference(b200, name):
    import torch
    import torch.nn.functional as F

    from avo.benchmark import error_metrics, fp32_reference

    shape, causal, k_scale = CONFIGS[name]
    q, k, v = oracle.make_inputs(shape, seed=0, k_scale=k_scale)
    dq, dk, dv = (t.cuda() for t in (q, k, v))
    out, lse = b200.attention_forward(dq, dk, dv, causal)
    torch.cuda.synchronize()
    b200.check_status("cuda:0")
    assert out.isfinite().all()
    ref_o, ref_lse = fp32_reference(dq, dk, dv, causal)
    metrics = error_metrics(out, ref_o, lse, ref_lse)
    assert metrics["max_abs"] <= oracle.MAX_ABS_TOL, metrics
    assert metrics["mean_abs"] <= oracle.MEAN_ABS_TOL, metrics
    assert metrics["lse_max_abs"] <= oracle.LSE_TOL, metrics
    del ref_o, ref_lse
    sdpa = F.scaled_dot_product_attention(dq, dk, dv, is_causal=causal)
    assert torch.allclose(out.float(), sdpa.float(), atol=oracle.ALLCLOSE_ATOL, rtol=oracle.ALLCLOSE_RTOL)
    del sdpa
    # Sampled rows of a few heads against the fp64 CPU oracle.
    rng = np.random.default_rng(0)
    seq = shape[2]
    rows = np.sort(rng.choice(seq, size=48, replace=False))
    for b, h in ((0, 0), (shape[0] - 1, shape[1] - 1)):
        qr = q[b, h, rows].float().numpy()
        limit = int(rows.max()) + 1 if causal else seq
        kf = k[b, h, :limit].float().numpy()
        vf = v[b, h, :limit].float().numpy()
        s = (qr.astype(np.float64) @ kf.T.astype(np.float64)) / np.sqrt(128.0)
        if causal:
            s = np.where(np.arange(limit)[None, :] > rows[:, None], -np.inf, s)
        m = s.max(axis=1, keepdims=True)
        p = np.exp(s - m)
        ref = (p @ vf) / p.sum(axis=1, keepdims=True)
        ref_l = (m + np.log(p.sum(axis=1, keepdims=True)))[:, 0]
        got = out[b, h, torch.from_numpy(rows).cuda()].float().cpu().numpy()
        got_l = lse[b, h, torch.from_numpy(rows).cuda()].cpu().numpy()
        assert np.abs(got - ref).max() <= oracle.MAX_ABS_TOL
        assert np.abs(got_l - ref_l).max() <= oracle.LSE_TOL


def test_scorer_end_to_end_on_candidate(b200):
    from pathlib import Path

    from avo.benchmark import score_backend
    from avo.config import cases_from_cli

    seed = Path(__file__).resolve().parents[1] / "avo-ampere_b200" / "candidates" / "cuda_b200_attention_seed.py"
    cases = cases_from_cli("4096", "both", total_tokens=8192)
    summary = score_backend("candidate", cases, warmup=2, repeats=3, candidate=seed)
    assert summary["all_correct"], summary
    assert summary["benchmark"]["target"]["sm"] == "sm_100a"
    for case in summary["cases"]:
        assert case["tflops"] > 100.0
        assert case["lse_max_abs_error"] <= oracle.LSE_TOL


def test_run_to_run_determinism(b200):
    import torch

    q, k, v = oracle.make_inputs((2, 8, 2048, 128), seed=9)
    dq, dk, dv = (t.cuda() for t in (q, k, v))
    first, lse1 = b200.attention_forward(dq, dk, dv, True)
    second, lse2 = b200.attention_forward(dq, dk, dv, True)
    torch.cuda.synchronize()
    assert torch.equal(first, second) and torch.equal(lse1, lse2)
