"""The reference's comparison lanes on the B200 (avo/benchmark.py:314-403 there):
``score_backend("torch-sdpa", ...)`` and ``score_backend("flash-attn", ...)`` through this
repo's scorer, on the bench workload shapes.  The flash-attn lane is skipped only when
the ``flash_attn`` wheel is not importable on the machine."""

from __future__ import annotations

import importlib.util

import pytest

from avo.benchmark import score_backend
from avo.config import AttentionCase

pytestmark = pytest.mark.gpu

CASES = [AttentionCase(seq_len=4096, causal=False, total_tokens=16384),
         AttentionCase(seq_len=4096, causal=True, total_tokens=16384)]


def _check(payload, backend):
    assert payload["backend"] == backend
    assert payload["all_correct"], payload["cases"]
    assert payload["geomean_tflops"] > 50.0, payload["geomean_tflops"]
    assert payload["benchmark"]["target"]["sm"] == "sm_100a"
    for case in payload["cases"]:
        assert case["milliseconds"] > 0 and case["error"] is None


def test_torch_sdpa_lane():
    _check(score_backend("torch-sdpa", CASES, warmup=2, repeats=5), "torch-sdpa")


def test_flash_attn_lane():
    if importlib.util.find_spec("flash_attn") is None:
        pytest.skip("flash_attn is not installed on this machine")
    _check(score_backend("flash-attn", CASES, warmup=2, repeats=5), "flash-attn")
