"""AVO candidate: B200-native (sm_100a) BF16 attention forward, head_dim 128.

Obeys the candidate contract of the AVO scorer: a module-level callable
``attention(q, k, v, causal) -> Tensor[B, H, S, D]`` (reference: loader
avo/benchmark.py:406-418; the SDPA seed candidates/torch_sdpa_seed.py:6-7).  Inputs are
contiguous CUDA bf16 ``[B, H, S, 128]``; the output is a new tensor of the same shape
and dtype, as ``torch::empty_like`` gives in the reference seeds
(candidates/cuda_mma_attention/attention_kernel.cu:188).

Additive export ``attention_with_lse(q, k, v, causal) -> (O, LSE)`` returns the fp32
natural-log LSE ``[B, H, S]`` as well.

The kernel lives in the companion directory ``cuda_b200_attention/`` (TMA +
tcgen05/TMEM, warp-specialised, built ahead of time by nvcc for sm_100a and called
through a C ABI).  There is no CPU or eager fallback.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

_DIR = Path(__file__).resolve().parent / "cuda_b200_attention"
_BINDING = "avo_b200_attention_binding"

AVO_SOURCE_FILES = (
    "cuda_b200_attention/sm100_ptx.cuh",
    "cuda_b200_attention/schedule.cuh",
    "cuda_b200_attention/attn_fwd.cuh",
    "cuda_b200_attention/attn_abi.cu",
    "cuda_b200_attention/fast_call.c",
    "cuda_b200_attention/b200_attention.py",
    "cuda_b200_attention/build.py",
)


def _binding():
    module = sys.modules.get(_BINDING)
    if module is None:
        spec = importlib.util.spec_from_file_location(_BINDING, _DIR / "b200_attention.py")
        module = importlib.util.module_from_spec(spec)
        sys.modules[_BINDING] = module
        spec.loader.exec_module(module)
    return module


def attention(q, k, v, causal: bool):
    out, _ = _binding().attention_forward(q, k, v, causal, need_lse=False)
    return out


def attention_with_lse(q, k, v, causal: bool):
    return _binding().attention_forward(q, k, v, causal, need_lse=True)
