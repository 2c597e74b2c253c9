"""The candidate module obeys the AVO contract (CPU checks; the GPU path is in the
-m gpu tests)."""

from __future__ import annotations

import importlib.util
import re
from pathlib import Path

import pytest

PKG = Path(__file__).resolve().parents[1] / "avo-ampere_b200"
SEED = PKG / "candidates" / "cuda_b200_attention_seed.py"
COMPANION = PKG / "candidates" / "cuda_b200_attention"


def _load():
    spec = importlib.util.spec_from_file_location("avo_candidate_contract_check", SEED)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_scorer_loads_candidate_and_finds_attention():
    from avo.benchmark import _load_candidate

    module = _load_candidate(SEED)
    assert callable(module.attention) and callable(module.attention_with_lse)


def test_declared_sources_exist_and_are_captured():
    from avo.benchmark import _candidate_source_files

    module = _load()
    files = _candidate_source_files(module, SEED)
    for rel in module.AVO_SOURCE_FILES:
        assert (SEED.parent / rel).is_file(), rel
    assert any(f.endswith("attn_fwd.cuh") for f in files)
    assert not any("__pycache__" in f or f.endswith(".so") for f in files)


def test_cpu_tensors_are_rejected_like_the_reference_binding():
    import torch

    module = _load()
    q = torch.zeros((1, 1, 128, 128), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        module.attention(q, q, q, False)


def test_wrapper_and_kernel_agree_on_head_dim():
    binding = (COMPANION / "b200_attention.py").read_text()
    kernel = (COMPANION / "attn_fwd.cuh").read_text()
    wrapper_dim = int(re.search(r"^HEAD_DIM = (\d+)", binding, re.M).group(1))
    kernel_dim = int(re.search(r"constexpr int kHeadDim = (\d+);", kernel).group(1))
    assert wrapper_dim == kernel_dim == 128


def test_failed_candidate_scores_zero(tmp_path):
    from avo.benchmark import score_backend

    bad = tmp_path / "bad_seed.py"
    bad.write_text("x = 1\n")
    from avo.config import AttentionCase

    summary = score_backend("candidate", [AttentionCase(seq_len=128, causal=False)], warmup=0, repeats=1,
                            candidate=bad)
    assert summary["all_correct"] is False
    assert summary["cases"][0]["tflops"] == 0.0
    assert "attention" in summary["cases"][0]["error"]


def test_no_cpu_fallback_in_product_sources():
    for path in [SEED, *COMPANION.glob("*.py")]:
        text = path.read_text()
        assert "oracle" not in text, path
        assert "scaled_dot_product_attention" not in text, path
