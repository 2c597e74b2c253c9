"""Scorer for attention candidates on the B200.

Host-side mirror of the reference scorer ``avo/benchmark.py`` with the same public
names and payload keys (``CaseScore`` :30-50, ``attention_forward_flops`` /
``tflops_from_ms`` :54-62, ``timing_summary`` :65-84, ``geometric_mean`` :87-91,
``score_summary`` :94-100, ``score_backend`` :103-175, ``benchmark_metadata`` :178-204,
``_time_cuda_samples`` :285-311, ``_score_candidate`` :616-666), so the lineage gate and
CLI consume its JSON unchanged.  Differences, all B200-first:

* ``_require_torch`` accepts compute capability 10.0 (the reference demands 8.6).
* Inputs are drawn on the host from a seeded ``torch.Generator`` and copied to the
  GPU, so the CPU oracle, the GPU and every rank of a multi-GPU run see identical bits
  (the reference draws on the GPU, :256-272).  ``k_scale`` multiplies k before the
  bf16 cast.
* Correctness keeps the reference's gate (finite output, same shape,
  ``torch.allclose(atol=3e-2, rtol=3e-2)`` against bf16 SDPA, :630-639) and adds the
  stricter fp32 check: max-abs <= 2e-2 and mean-abs <= 2e-3 against an fp32 reference
  of the same bf16 inputs, and LSE max-abs <= 1e-3 when the candidate exports
  ``attention_with_lse``.
* Multi-GPU (``case.gpus > 1``) is delegated to ``avo.multigpu`` (head-sharded
  processes, device-event timing, max over ranks).
"""

from __future__ import annotations

import importlib.util
import math
import os
import platform
import statistics
import time
from collections.abc import Callable, Iterable
from dataclasses import dataclass, field
from datetime import UTC, datetime
from pathlib import Path, PurePosixPath
from typing import Any, Literal

from .config import ACTIVE_TARGET, AttentionCase

BackendName = Literal["torch-sdpa", "flash-attn", "candidate"]
CANDIDATE_SOURCE_FILE_ATTRIBUTES = ("AVO_SOURCE_FILES", "__avo_source_files__")
CANDIDATE_RUNTIME_SOURCE_SUFFIXES = frozenset({".py", ".cpp", ".cu", ".cuh", ".h", ".hpp"})
FLOP_ACCOUNTING = {
    "name": "flash_attention_forward_compatible",
    "formula": "4 * batch_size * num_heads * seq_len**2 * head_dim // (2 if causal else 1)",
    "scope": "forward QK and PV matmul FLOPs only; excludes softmax, masking, and projections",
    "causal_convention": "half_dense",
}

# Tolerances against the fp32 reference of the same bf16 inputs.
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3
LSE_TOL = 1e-3
# The reference scorer's own gate against bf16 SDPA (avo/benchmark.py:638-639).
ALLCLOSE_ATOL = 3e-2
ALLCLOSE_RTOL = 3e-2


@dataclass(frozen=True)
class CaseScore:
    backend: str
    case: AttentionCase
    correct: bool
    milliseconds: float | None
    tflops: float
    max_abs_error: float | None
    error: str | None = None
    timing_samples_ms: tuple[float, ...] = ()
    mean_abs_error: float | None = None
    lse_max_abs_error: float | None = None
    per_gpu_ms: tuple[float, ...] = field(default=())

    def as_dict(self) -> dict[str, Any]:
        payload = {
            "backend": self.backend,
            "case": self.case.as_dict(),
            "correct": self.correct,
            "milliseconds": self.milliseconds,
            "tflops": self.tflops,
            "max_abs_error": self.max_abs_error,
            "error": self.error,
            "timing": timing_summary(self.timing_samples_ms),
        }
        if self.mean_abs_error is not None:
            payload["mean_abs_error"] = self.mean_abs_error
        if self.lse_max_abs_error is not None:
            payload["lse_max_abs_error"] = self.lse_max_abs_error
        if self.per_gpu_ms:
            payload["per_gpu_ms"] = list(self.per_gpu_ms)
            payload["tflops_per_gpu"] = self.tflops / max(1, self.case.gpus)
        return payload


def attention_forward_flops(case: AttentionCase) -> int:
    dense = 4 * case.batch_size * case.num_heads * case.seq_len * case.seq_len * case.head_dim
    return dense // 2 if case.causal else dense


def tflops_from_ms(case: AttentionCase, milliseconds: float) -> float:
    if milliseconds <= 0:
        return math.inf
    return attention_forward_flops(case) / (milliseconds / 1000.0) / 1e12


def timing_summary(samples_ms: Iterable[float]) -> dict[str, Any]:
    samples = tuple(float(sample) for sample in samples_ms)
    if not samples:
        return {"samples_ms": [], "trials": 0, "min_ms": None, "median_ms": None,
                "mean_ms": None, "cv": None}
    mean = statistics.fmean(samples)
    return {
        "samples_ms": list(samples),
        "trials": len(samples),
        "min_ms": min(samples),
        "median_ms": statistics.median(samples),
        "mean_ms": mean,
        "cv": statistics.pstdev(samples) / mean if mean > 0 and len(samples) > 1 else 0.0,
    }


def geometric_mean(values: Iterable[float]) -> float:
    positive = [value for value in values if value > 0 and math.isfinite(value)]
    if not positive:
        return 0.0
    return math.exp(sum(math.log(value) for value in positive) / len(positive))


def score_summary(backend: str, scores: list[CaseScore]) -> dict[str, Any]:
    return {
        "backend": backend,
        "all_correct": bool(scores) and all(score.correct for score in scores),
        "geomean_tflops": geometric_mean(score.tflops for score in scores if score.correct),
        "cases": [score.as_dict() for score in scores],
    }


def score_backend(
    backend: BackendName,
    cases: list[AttentionCase],
    warmup: int,
    repeats: int,
    trials: int = 1,
    seed: int = 0,
    candidate: Path | None = None,
) -> dict[str, Any]:
    source_files: tuple[str, ...] = ()
    if backend == "torch-sdpa":
        scores = [_score_torch_sdpa(case, warmup, repeats, trials, seed) for case in cases]
    elif backend == "flash-attn":
        scores = [_score_flash_attn(case, warmup, repeats, trials, seed) for case in cases]
    elif backend == "candidate":
        if candidate is None:
            raise ValueError("candidate backend requires --candidate")
        try:
            module = _load_candidate(candidate)
            source_files = _candidate_source_files(module, candidate)
            scores = [
                _score_candidate(module, candidate, case, warmup, repeats, trials, seed)
                for case in cases
            ]
        except Exception as exc:
            source_files = _candidate_companion_source_files(candidate)
            scores = [_failed_score("candidate", case, f"{type(exc).__name__}: {exc}") for case in cases]
    else:
        raise ValueError(f"unsupported backend: {backend}")
    summary = score_summary(backend, scores)
    summary["benchmark"] = benchmark_metadata(
        cases=cases, warmup=warmup, repeats=repeats, trials=trials, seed=seed
    )
    if backend == "candidate" and candidate is not None:
        summary["candidate_path"] = str(candidate)
        if source_files:
            summary["candidate_source_files"] = list(source_files)
    return summary


def benchmark_metadata(*, cases: list[AttentionCase], warmup: int, repeats: int, trials: int,
                       seed: int) -> dict[str, Any]:
    return {
        "measured_at": datetime.now(UTC).isoformat(),
        "settings": {
            "warmup": warmup,
            "repeats": repeats,
            "trials": trials,
            "seed": seed,
            "case_count": len(cases),
        },
        "target": {
            "name": ACTIVE_TARGET.name,
            "compute_capability": list(ACTIVE_TARGET.compute_capability),
            "compute": ACTIVE_TARGET.compute,
            "sm": ACTIVE_TARGET.sm,
            "nvcc_gencode": ACTIVE_TARGET.nvcc_gencode,
        },
        "flop_accounting": dict(FLOP_ACCOUNTING),
        "environment": _benchmark_environment(),
    }


def _require_torch(device: int = 0):
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available")
    capability = torch.cuda.get_device_capability(device)
    if capability != ACTIVE_TARGET.compute_capability:
        raise RuntimeError(f"expected {ACTIVE_TARGET.sm}/B200-like GPU, got compute capability {capability}")
    return torch


def _benchmark_environment() -> dict[str, Any]:
    payload: dict[str, Any] = {"python": platform.python_version(), "platform": platform.platform()}
    try:
        import torch
    except ModuleNotFoundError as exc:
        payload["torch"] = {"installed": False, "error": f"{type(exc).__name__}: {exc}"}
        return payload
    payload["torch"] = {
        "installed": True,
        "version": torch.__version__,
        "cuda": torch.version.cuda,
        "cuda_available": torch.cuda.is_available(),
    }
    payload["host"] = {"cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads()}
    if not torch.cuda.is_available():
        return payload
    index = torch.cuda.current_device()
    props = torch.cuda.get_device_properties(index)
    payload["gpu"] = {
        "index": index,
        "name": torch.cuda.get_device_name(index),
        "compute_capability": list(torch.cuda.get_device_capability(index)),
        "total_memory_bytes": props.total_memory,
        "multi_processor_count": props.multi_processor_count,
        "device_count": torch.cuda.device_count(),
    }
    return payload


def host_inputs(case: AttentionCase, seed: int):
    """Seeded host q, k, v in the case's dtype: N(0,1) fp32 from a CPU generator,
    k *= case.k_scale, then cast."""
    import torch

    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}.get(case.dtype)
    if dtype is None:
        raise ValueError("dtype must be one of: bf16, fp16, fp32")
    generator = torch.Generator().manual_seed(seed)
    shape = case.shape
    q = torch.randn(shape, generator=generator, dtype=torch.float32)
    k = torch.randn(shape, generator=generator, dtype=torch.float32)
    v = torch.randn(shape, generator=generator, dtype=torch.float32)
    if case.k_scale != 1.0:
        k = k * case.k_scale
    return q.to(dtype), k.to(dtype), v.to(dtype)


def _make_inputs(case: AttentionCase, seed: int, device: str = "cuda"):
    _require_torch()
    return tuple(t.to(device) for t in host_inputs(case, seed))


def _reference_sdpa(q, k, v, causal: bool):
    import torch.nn.functional as F

    return F.scaled_dot_product_attention(q, k, v, dropout_p=0.0, is_causal=causal)


def fp32_reference(q, k, v, causal: bool, *, chunk_rows: int = 4096):
    """fp32 O and natural-log LSE of the same inputs, computed row-chunk by row-chunk
    (plain matmul + softmax, TF32 off) so S=32768 fits in memory."""
    import torch

    batch, heads, seq, dim = q.shape
    scale = 1.0 / math.sqrt(dim)
    out = torch.empty((batch, heads, seq, dim), dtype=torch.float32, device=q.device)
    lse = torch.empty((batch, heads, seq), dtype=torch.float32, device=q.device)
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for b in range(batch):
            for h in range(heads):
                kf = k[b, h].float()
                vf = v[b, h].float()
                for start in range(0, seq, chunk_rows):
                    stop = min(seq, start + chunk_rows)
                    limit = stop if causal else seq
                    s = (q[b, h, start:stop].float() @ kf[:limit].T) * scale
                    if causal:
                        rows = torch.arange(start, stop, device=q.device)[:, None]
                        cols = torch.arange(limit, device=q.device)[None, :]
                        s.masked_fill_(cols > rows, float("-inf"))
                    lse[b, h, start:stop] = torch.logsumexp(s, dim=-1)
                    out[b, h, start:stop] = torch.softmax(s, dim=-1) @ vf[:limit]
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    return out, lse


def error_metrics(candidate, reference_o, lse=None, reference_lse=None) -> dict[str, float]:
    diff = (candidate.float() - reference_o.float()).abs()
    metrics = {"max_abs": float(diff.max().item()), "mean_abs": float(diff.mean().item())}
    if lse is not None and reference_lse is not None:
        metrics["lse_max_abs"] = float((lse.float() - reference_lse.float()).abs().max().item())
    return metrics


def _time_cuda(fn: Callable[[], object], warmup: int, repeats: int) -> float:
    return _time_cuda_samples(fn, warmup=warmup, repeats=repeats, trials=1)[0]


def _time_cuda_samples(fn: Callable[[], object], warmup: int, repeats: int,
                       trials: int) -> tuple[float, ...]:
    if warmup < 0:
        raise ValueError("warmup must be non-negative")
    if repeats <= 0:
        raise ValueError("repeats must be positive")
    if trials <= 0:
        raise ValueError("trials must be positive")
    torch = _require_torch()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    samples = []
    stream = torch.cuda.current_stream()
    for _ in range(trials):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(repeats):
            fn()
        end.record(stream)
        torch.cuda.synchronize()
        samples.append(float(start.elapsed_time(end)) / repeats)
    return tuple(samples)


def _score_torch_sdpa(case: AttentionCase, warmup: int, repeats: int, trials: int,
                      seed: int) -> CaseScore:
    try:
        q, k, v = _make_inputs(case, seed)
        output = _reference_sdpa(q, k, v, case.causal)
        if not output.isfinite().all().item():
            raise RuntimeError("reference output contains non-finite values")
        samples = _time_cuda_samples(lambda: _reference_sdpa(q, k, v, case.causal),
                                     warmup=warmup, repeats=repeats, trials=trials)
        ms = statistics.median(samples)
        return CaseScore(backend="torch-sdpa", case=case, correct=True, milliseconds=ms,
                         tflops=tflops_from_ms(case, ms), max_abs_error=0.0,
                         timing_samples_ms=samples)
    except Exception as exc:
        return _failed_score("torch-sdpa", case, f"{type(exc).__name__}: {exc}")


def _score_flash_attn(case: AttentionCase, warmup: int, repeats: int, trials: int,
                      seed: int) -> CaseScore:
    try:
        torch = _require_torch()
        from flash_attn import flash_attn_func

        q_bhsd, k_bhsd, v_bhsd = _make_inputs(case, seed)
        q, k, v = (t.transpose(1, 2).contiguous() for t in (q_bhsd, k_bhsd, v_bhsd))
        reference = _reference_sdpa(q_bhsd, k_bhsd, v_bhsd, case.causal).transpose(1, 2)
        candidate = flash_attn_func(q, k, v, dropout_p=0.0, causal=case.causal)
        max_abs = float((candidate.float() - reference.float()).abs().max().item())
        correct = bool(torch.allclose(candidate.float(), reference.float(),
                                      atol=ALLCLOSE_ATOL, rtol=ALLCLOSE_RTOL))
        samples = _time_cuda_samples(
            lambda: flash_attn_func(q, k, v, dropout_p=0.0, causal=case.causal),
            warmup=warmup, repeats=repeats, trials=trials)
        ms = statistics.median(samples)
        return CaseScore(backend="flash-attn", case=case, correct=correct, milliseconds=ms,
                         tflops=tflops_from_ms(case, ms) if correct else 0.0,
                         max_abs_error=max_abs, timing_samples_ms=samples,
                         error=None if correct else "flash-attn output failed tolerance check")
    except Exception as exc:
        return _failed_score("flash-attn", case, f"{type(exc).__name__}: {exc}")


def _load_candidate(path: Path):
    if not path.exists():
        raise FileNotFoundError(path)
    module_name = f"avo_candidate_{abs(hash(path.resolve()))}"
    spec = importlib.util.spec_from_file_location(module_name, path)
    if spec is None or spec.loader is None:
        raise RuntimeError(f"could not load candidate module from {path}")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    attention = getattr(module, "attention", None)
    if not callable(attention):
        raise ValueError("candidate module must define callable attention(q, k, v, causal)")
    return module


def _candidate_source_files(module: Any, candidate: Path) -> tuple[str, ...]:
    """Declared AVO_SOURCE_FILES / __avo_source_files__ plus the companion directory
    (``<stem>/`` or ``<stem minus _seed>/`` next to the candidate)."""
    paths: list[str] = []
    for attribute in CANDIDATE_SOURCE_FILE_ATTRIBUTES:
        raw = getattr(module, attribute, None)
        if raw is None:
            continue
        values = (raw,) if isinstance(raw, (str, os.PathLike)) else tuple(raw)
        for value in values:
            path = Path(os.fspath(value))
            if not path.is_absolute() and not path.as_posix().startswith("candidates/"):
                path = candidate.parent / path
            paths.append(path.as_posix())
    paths.extend(_candidate_companion_source_files(candidate))
    return tuple(dict.fromkeys(paths))


def _candidate_companion_source_files(candidate: Path) -> tuple[str, ...]:
    stems = [candidate.stem]
    if candidate.stem.endswith("_seed"):
        stems.insert(0, candidate.stem.removesuffix("_seed"))
    paths: list[str] = []
    for stem in dict.fromkeys(stems):
        root = candidate.parent / stem
        if not root.is_dir() or root.is_symlink():
            continue
        for file_path in sorted(root.rglob("*")):
            if (file_path.is_file() and file_path.suffix in CANDIDATE_RUNTIME_SOURCE_SUFFIXES
                    and "__pycache__" not in file_path.parts):
                paths.append(PurePosixPath(file_path).as_posix())
    return tuple(paths)


def _score_candidate(module: Any, candidate_path: Path, case: AttentionCase, warmup: int,
                     repeats: int, trials: int, seed: int) -> CaseScore:
    if case.gpus > 1:
        from .multigpu import score_head_sharded

        return score_head_sharded(candidate_path, case, warmup=warmup, repeats=repeats,
                                  trials=trials, seed=seed)
    try:
        torch = _require_torch()
        q, k, v = _make_inputs(case, seed)
        with_lse = getattr(module, "attention_with_lse", None)
        lse = None
        if callable(with_lse):
            candidate, lse = with_lse(q, k, v, case.causal)
        else:
            candidate = module.attention(q, k, v, case.causal)
        torch.cuda.synchronize()
        if tuple(candidate.shape) != tuple(q.shape):
            raise RuntimeError(f"candidate output shape {tuple(candidate.shape)} != reference {tuple(q.shape)}")
        if not candidate.isfinite().all().item():
            raise RuntimeError("candidate output contains non-finite values")
        reference = _reference_sdpa(q, k, v, case.causal)
        max_abs_bf16 = float((candidate.float() - reference.float()).abs().max().item())
        gate = bool(torch.allclose(candidate.float(), reference.float(),
                                   atol=ALLCLOSE_ATOL, rtol=ALLCLOSE_RTOL))
        del reference
        ref_o, ref_lse = fp32_reference(q, k, v, case.causal)
        metrics = error_metrics(candidate, ref_o, lse, ref_lse if lse is not None else None)
        del ref_o, ref_lse
        correct = (gate and metrics["max_abs"] <= MAX_ABS_TOL
                   and metrics["mean_abs"] <= MEAN_ABS_TOL
                   and metrics.get("lse_max_abs", 0.0) <= LSE_TOL)
        samples = _time_cuda_samples(lambda: module.attention(q, k, v, case.causal),
                                     warmup=warmup, repeats=repeats, trials=trials)
        ms = statistics.median(samples)
        return CaseScore(
            backend="candidate", case=case, correct=correct, milliseconds=ms,
            tflops=tflops_from_ms(case, ms) if correct else 0.0,
            max_abs_error=max(metrics["max_abs"], max_abs_bf16) if not correct else metrics["max_abs"],
            mean_abs_error=metrics["mean_abs"], lse_max_abs_error=metrics.get("lse_max_abs"),
            timing_samples_ms=samples,
            error=None if correct else f"{candidate_path} failed tolerance check {metrics}",
        )
    except Exception as exc:
        return _failed_score("candidate", case, f"{type(exc).__name__}: {exc}")


def _failed_score(backend: str, case: AttentionCase, error: str) -> CaseScore:
    return CaseScore(backend=backend, case=case, correct=False, milliseconds=None, tflops=0.0,
                     max_abs_error=None, error=error)


def sleep_score(seconds: float) -> dict[str, Any]:
    time.sleep(seconds)
    return {"slept": seconds}
