"""Scorer arithmetic, mirroring the reference's tests/test_benchmark_math.py with the
B200 target."""

from __future__ import annotations

import pytest

from avo.benchmark import (
    CaseScore,
    attention_forward_flops,
    benchmark_metadata,
    geometric_mean,
    score_summary,
    tflops_from_ms,
    timing_summary,
)
from avo.config import NAMED_CASES, AttentionCase


def test_attention_flops_dense_and_causal() -> None:
    dense = AttentionCase(seq_len=4096, causal=False)
    causal = AttentionCase(seq_len=4096, causal=True)
    assert attention_forward_flops(dense) == 4 * 8 * 16 * 4096 * 4096 * 128
    assert attention_forward_flops(causal) == attention_forward_flops(dense) // 2


def test_named_workload_flops() -> None:
    assert attention_forward_flops(NAMED_CASES["b1_h4_s512_noncausal"]) == 536870912
    assert attention_forward_flops(NAMED_CASES["b4_h16_s4096_noncausal"]) == 549755813888
    assert attention_forward_flops(NAMED_CASES["b2_h16_s8192_causal"]) == 549755813888
    assert attention_forward_flops(NAMED_CASES["b1_h16_s16384_noncausal_k3"]) == 2199023255552
    assert attention_forward_flops(NAMED_CASES["b1_h16_s32768_causal"]) == 4398046511104
    assert attention_forward_flops(NAMED_CASES["b4_h16_s8192_noncausal"]) == 2199023255552


def test_tflops_from_ms() -> None:
    case = AttentionCase(seq_len=4096, causal=False)
    assert tflops_from_ms(case, 1.0) == attention_forward_flops(case) / 1e-3 / 1e12


def test_geometric_mean_ignores_zero_failed_scores() -> None:
    assert geometric_mean([2.0, 8.0, 0.0]) == 4.0
    assert geometric_mean([0.0]) == 0.0


def test_score_summary_treats_empty_case_set_as_not_correct() -> None:
    summary = score_summary("candidate", [])
    assert summary["all_correct"] is False
    assert summary["geomean_tflops"] == 0.0
    assert summary["cases"] == []


def test_timing_summary_reports_replicate_statistics() -> None:
    summary = timing_summary([3.0, 1.0, 2.0])
    assert summary["samples_ms"] == [3.0, 1.0, 2.0]
    assert summary["trials"] == 3
    assert summary["min_ms"] == 1.0
    assert summary["median_ms"] == 2.0
    assert summary["mean_ms"] == 2.0
    assert summary["cv"] == pytest.approx(0.40824829046)


def test_case_score_serializes_empty_timing_and_new_fields() -> None:
    payload = CaseScore(backend="mock", case=AttentionCase(seq_len=16, causal=False), correct=False,
                        milliseconds=None, tflops=0.0, max_abs_error=None, error="failed").as_dict()
    assert payload["timing"] == {"samples_ms": [], "trials": 0, "min_ms": None, "median_ms": None,
                                 "mean_ms": None, "cv": None}
    assert "mean_abs_error" not in payload and "per_gpu_ms" not in payload
    multi = CaseScore(backend="candidate", case=AttentionCase(seq_len=16, causal=False, gpus=2),
                      correct=True, milliseconds=1.0, tflops=10.0, max_abs_error=0.01,
                      mean_abs_error=0.001, lse_max_abs_error=1e-4, per_gpu_ms=(1.0, 0.9)).as_dict()
    assert multi["tflops_per_gpu"] == 5.0 and multi["per_gpu_ms"] == [1.0, 0.9]
    assert multi["case"]["gpus"] == 2


def test_benchmark_metadata_records_settings_and_b200_target() -> None:
    metadata = benchmark_metadata(cases=[AttentionCase(seq_len=16, causal=False)], warmup=1, repeats=2,
                                  trials=3, seed=4)
    assert metadata["settings"] == {"warmup": 1, "repeats": 2, "trials": 3, "seed": 4, "case_count": 1}
    assert metadata["target"]["sm"] == "sm_100a"
    assert metadata["target"]["compute_capability"] == [10, 0]
    assert metadata["target"]["nvcc_gencode"] == "-gencode=arch=compute_100a,code=sm_100a"
    assert metadata["flop_accounting"] == {
        "name": "flash_attention_forward_compatible",
        "formula": "4 * batch_size * num_heads * seq_len**2 * head_dim // (2 if causal else 1)",
        "scope": "forward QK and PV matmul FLOPs only; excludes softmax, masking, and projections",
        "causal_convention": "half_dense",
    }
    assert "measured_at" in metadata and "environment" in metadata


def test_host_inputs_match_oracle_generator() -> None:
    import torch

    from avo.benchmark import host_inputs
    from oracle.attention_oracle import make_inputs

    case = AttentionCase(seq_len=64, causal=False, num_heads=2, total_tokens=128, k_scale=3.0)
    ours = host_inputs(case, seed=9)
    theirs = make_inputs(case.shape, seed=9, k_scale=3.0)
    for a, b in zip(ours, theirs):
        assert torch.equal(a, b)


def test_scorer_refuses_without_b200() -> None:
    from avo.benchmark import _require_torch

    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="CUDA is not available"):
        _require_torch()
