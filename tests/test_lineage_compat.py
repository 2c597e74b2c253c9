"""A B200 score payload passes through the reference's lineage gate as intended (CPU).

The reference's evolve loop commits a candidate only through ``decide_gate``
(avo/lineage.py:81-135): reject if not ``all_correct``, if ``cases`` is empty, if the
geomean is not a positive finite number, if the case signature (sorted JSON of every
``cases[].case`` dict, :425-436) differs from the current best's, if the geomean
regressed (1e-9 slack), or if a best exists and the score is one-shot (settings repeats
<= 1 and warmup <= 1, :413-422; confirmation wants repeats >= 3 / warmup >= 2).
``gate`` below restates those rules in that order; the payloads come from this repo's
scorer (``score_summary`` + ``benchmark_metadata``), including the keys the B200 scorer
adds (``mean_abs_error``, ``lse_max_abs_error``, ``per_gpu_ms``, ``tflops_per_gpu``) and
the case fields ``k_scale`` / ``gpus``, which appear only away from their defaults.
"""

from __future__ import annotations

import json
import math

from avo.benchmark import CaseScore, benchmark_metadata, score_summary
from avo.config import DEFAULT_CASES, AttentionCase


def signature(payload: dict) -> tuple[str, ...]:
    cases = payload.get("cases")
    if not isinstance(cases, list):
        return ()
    return tuple(sorted(json.dumps(c["case"], sort_keys=True, separators=(",", ":"))
                        for c in cases if isinstance(c, dict) and isinstance(c.get("case"), dict)))


def one_shot(payload: dict) -> bool:
    settings = payload.get("benchmark", {}).get("settings")
    if not isinstance(settings, dict):
        return False
    try:
        return int(settings.get("repeats", 0)) <= 1 and int(settings.get("warmup", 0)) <= 1
    except (TypeError, ValueError):
        return False


def gate(candidate: dict, best_geomean: float, best_payload: dict | None = None) -> tuple[bool, str]:
    geo = float(candidate.get("geomean_tflops") or 0.0)
    if not candidate.get("all_correct"):
        return False, "failed correctness"
    if not isinstance(candidate.get("cases"), list) or not candidate["cases"]:
        return False, "no scored cases"
    if not math.isfinite(geo) or geo <= 0.0:
        return False, "non-positive geomean"
    if best_payload is not None and signature(candidate) != signature(best_payload):
        return False, "cases differ"
    if geo + 1e-9 < best_geomean:
        return False, "regressed"
    if best_payload is not None and best_geomean > 0.0 and one_shot(candidate):
        return False, "one-shot"
    return True, "established" if best_payload is None and best_geomean <= 0.0 else "passed"


def b200_payload(cases, tflops: float, *, warmup: int = 5, repeats: int = 20, correct: bool = True) -> dict:
    scores = []
    for case in cases:
        ms = 4 * case.batch_size * case.num_heads * case.seq_len**2 * case.head_dim / (2 if case.causal else 1)
        ms = ms / (tflops * 1e12) * 1e3
        scores.append(CaseScore(
            backend="candidate", case=case, correct=correct, milliseconds=ms,
            tflops=tflops if correct else 0.0, max_abs_error=7.8e-3, timing_samples_ms=(ms,),
            mean_abs_error=2.1e-4, lse_max_abs_error=3.0e-6,
            per_gpu_ms=tuple(ms for _ in range(case.gpus)) if case.gpus > 1 else ()))
    payload = score_summary("candidate", scores)
    payload["benchmark"] = benchmark_metadata(cases=list(cases), warmup=warmup, repeats=repeats, trials=1,
                                              seed=0)
    return json.loads(json.dumps(payload))  # the gate reads what was written as JSON


def test_default_suite_keeps_the_reference_signature():
    payload = b200_payload(DEFAULT_CASES, 1300.0)
    keys = {"seq_len", "causal", "mask_mode", "head_dim", "num_heads", "total_tokens", "batch_size", "dtype"}
    assert all(set(c["case"]) == keys for c in payload["cases"])
    assert all("mean_abs_error" in c and "lse_max_abs_error" in c for c in payload["cases"])
    assert gate(payload, 0.0) == (True, "established")


def test_improvement_accepted_regression_rejected():
    best = b200_payload(DEFAULT_CASES, 1200.0)
    better = b200_payload(DEFAULT_CASES, 1300.0)
    worse = b200_payload(DEFAULT_CASES, 1100.0)
    assert gate(better, best["geomean_tflops"], best) == (True, "passed")
    assert gate(worse, best["geomean_tflops"], best) == (False, "regressed")
    # equal within the 1e-9 slack is not a regression
    assert gate(b200_payload(DEFAULT_CASES, 1200.0), best["geomean_tflops"], best)[0]


def test_one_shot_score_needs_confirmation():
    best = b200_payload(DEFAULT_CASES, 1200.0)
    quick = b200_payload(DEFAULT_CASES, 1300.0, warmup=1, repeats=1)
    assert gate(quick, best["geomean_tflops"], best) == (False, "one-shot")
    confirmed = b200_payload(DEFAULT_CASES, 1300.0, warmup=2, repeats=3)
    assert gate(confirmed, best["geomean_tflops"], best) == (True, "passed")
    # with no best yet, a one-shot score may establish the case set
    assert gate(quick, 0.0) == (True, "established")


def test_incorrect_or_empty_payloads_rejected():
    assert gate(b200_payload(DEFAULT_CASES, 1300.0, correct=False), 0.0) == (False, "failed correctness")
    empty = b200_payload(DEFAULT_CASES, 1300.0)
    empty["cases"] = []
    assert gate(empty, 0.0) == (False, "no scored cases")


def test_new_case_fields_form_their_own_lane():
    """k_scale and gpus change the signature by design, so a multi-GPU or k x 3 score is
    gated against its own lane, never against the single-GPU default suite."""
    default = b200_payload(DEFAULT_CASES, 1200.0)
    sharded_cases = [AttentionCase(seq_len=c.seq_len, causal=c.causal, gpus=8) for c in DEFAULT_CASES]
    sharded = b200_payload(sharded_cases, 9000.0)
    assert all(c["case"]["gpus"] == 8 and "per_gpu_ms" in c and "tflops_per_gpu" in c for c in sharded["cases"])
    assert gate(sharded, default["geomean_tflops"], default) == (False, "cases differ")
    assert gate(sharded, 0.0) == (True, "established")
    stress = b200_payload([AttentionCase(seq_len=16384, causal=False, total_tokens=16384, k_scale=3.0)], 1300.0)
    assert signature(stress) != signature(b200_payload(
        [AttentionCase(seq_len=16384, causal=False, total_tokens=16384)], 1300.0))
