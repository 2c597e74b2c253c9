"""Cases and targets (mirrors the reference's tests/test_config.py for B200)."""

from __future__ import annotations

import pytest

from avo.config import ACTIVE_TARGET, AMPERE_A6000, B200, DEFAULT_CASES, AttentionCase, cases_from_cli


def test_b200_target_gencode() -> None:
    assert ACTIVE_TARGET is B200
    assert B200.compute == "compute_100a"
    assert B200.sm == "sm_100a"
    assert B200.nvcc_gencode == "-gencode=arch=compute_100a,code=sm_100a"
    assert B200.torch_arch_list == "10.0a"
    assert AMPERE_A6000.nvcc_gencode == "-gencode=arch=compute_86,code=sm_86"


def test_default_cases_cover_the_eight_case_suite() -> None:
    assert [(c.seq_len, c.causal) for c in DEFAULT_CASES] == [
        (4096, False), (4096, True), (8192, False), (8192, True),
        (16384, False), (16384, True), (32768, False), (32768, True),
    ]
    assert all(c.batch_size * c.seq_len == 32768 for c in DEFAULT_CASES)


def test_case_signature_unchanged_for_defaults() -> None:
    payload = AttentionCase(seq_len=4096, causal=True).as_dict()
    assert set(payload) == {"seq_len", "causal", "mask_mode", "head_dim", "num_heads", "total_tokens",
                            "batch_size", "dtype"}
    extended = AttentionCase(seq_len=4096, causal=True, k_scale=3.0, gpus=8).as_dict()
    assert extended["k_scale"] == 3.0 and extended["gpus"] == 8


def test_cases_from_cli() -> None:
    cases = cases_from_cli("4096,8192", "both", total_tokens=16384, k_scale=3.0, gpus=2)
    assert [(c.seq_len, c.causal, c.batch_size, c.k_scale, c.gpus) for c in cases] == [
        (4096, False, 4, 3.0, 2), (4096, True, 4, 3.0, 2), (8192, False, 2, 3.0, 2), (8192, True, 2, 3.0, 2)]
    with pytest.raises(ValueError, match="causal must be one of"):
        cases_from_cli("4096", "maybe")
    with pytest.raises(ValueError, match="at least one sequence length"):
        cases_from_cli("", "true")
    with pytest.raises(ValueError, match="must be divisible"):
        AttentionCase(seq_len=3000, causal=False).batch_size
