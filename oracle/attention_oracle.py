"""CPU oracle for the attention-forward hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this module,
and only as the checker or the timed CPU baseline - never as the product path.

What it restates (reference = coder-2011/avo-ampere):

* ``sdpa_reference`` - the reference's oracle seed
  ``candidates/torch_sdpa_seed.py:6-7``: ``F.scaled_dot_product_attention(q, k, v,
  dropout_p=0.0, is_causal=causal)``.  That call lives in the third-party dependency
  torch (pinned 2.11.0 in the reference's ``uv.lock:911-912``); its published
  algorithm is softmax(q k^T / sqrt(D) + M) v with M = -inf above the diagonal when
  ``is_causal``.  The same function is what the reference scorer compares every
  candidate against (``avo/benchmark.py:275-278``).
* ``attention_fp64`` - that algorithm written out in numpy float64, with the natural
  log-sum-exp (``LSE``) the candidate also returns.  Causal masking follows
  ``candidates/cuda_naive_attention/attention_kernel.cu:28`` (query i sees keys <= i),
  generalised to sequence positions (``q_pos0``/``kv_pos0``) for context-parallel
  blocks.
* ``attention_online`` - the tiled online-softmax recurrence of
  ``candidates/cuda_tiled_attention/attention_kernel.cu:84-99`` (running max, rescale
  of the partial sum and output on every tile), plus the conditional-rescale variant
  the B200 kernel uses (the max is only raised past a 2^threshold growth).
* ``lse_merge`` - combination of partial (O, LSE) pairs by log-sum-exp, the merge
  step of ring context parallelism.
* ``make_inputs`` - seeded host generator: i.i.d. N(0,1) fp32 drawn on the CPU with
  ``torch.Generator().manual_seed(seed)``, optionally k *= k_scale, then cast to bf16.
  (The reference draws on the GPU, ``avo/benchmark.py:256-272``; drawing on the host
  gives the CPU oracle and the GPU the identical bits.)

Parity pin: ``tests/golden/`` holds outputs of the reference seed itself, generated
by ``tests/golden/make_golden.py`` importing ``candidates/torch_sdpa_seed.py`` from the
reference checkout; ``tests/test_oracle_golden.py`` checks this module against them.
"""

from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634
LN2 = 0.6931471805599453


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16_bits(x))


def causal_mask(seq_q: int, seq_kv: int, q_pos0: int = 0, kv_pos0: int = 0) -> np.ndarray:
    """Boolean [seq_q, seq_kv]: True where key position > query position (masked)."""
    qpos = q_pos0 + np.arange(seq_q)[:, None]
    kpos = kv_pos0 + np.arange(seq_kv)[None, :]
    return kpos > qpos


def attention_fp64(q, k, v, causal: bool, scale: float | None = None,
                   q_pos0: int = 0, kv_pos0: int = 0):
    """O and natural-log LSE of softmax(scale q k^T [+ mask]) v in float64.

    ``q`` is [..., Sq, D], ``k``/``v`` [..., Skv, D] (any float dtype, upcast).
    Rows that see no key get O = 0 and LSE = -inf.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    if causal:
        s = np.where(causal_mask(q.shape[-2], k.shape[-2], q_pos0, kv_pos0), -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    finite = np.isfinite(m)
    m_safe = np.where(finite, m, 0.0)
    p = np.exp(s - m_safe)
    l = p.sum(axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        o = np.where(l > 0, np.matmul(p, v) / np.where(l > 0, l, 1.0), 0.0)
        lse = np.where(l[..., 0] > 0, m_safe[..., 0] + np.log(np.where(l > 0, l, 1.0))[..., 0],
                       -np.inf)
    return o, lse


def attention_online(q, k, v, causal: bool, scale: float | None = None, block: int = 128,
                     rescale_threshold: float | None = None, q_pos0: int = 0, kv_pos0: int = 0):
    """Tiled online-softmax forward over key blocks of ``block`` keys (float64).

    ``rescale_threshold=None`` rescales on every max increase, as the reference's
    tiled kernel does; a number t (log2 units) keeps a stale max until the tile max
    exceeds it by more than t, as the B200 kernel does.  Returns (O, LSE).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    c = scale * LOG2E
    seq_q, seq_kv = q.shape[-2], k.shape[-2]
    batch_shape = q.shape[:-2]
    m = np.full(batch_shape + (seq_q, 1), -np.inf)
    l = np.zeros(batch_shape + (seq_q, 1))
    acc = np.zeros(batch_shape + (seq_q, v.shape[-1]))
    for start in range(0, seq_kv, block):
        stop = min(start + block, seq_kv)
        s = np.matmul(q, np.swapaxes(k[..., start:stop, :], -1, -2)) * c
        if causal:
            s = np.where(causal_mask(seq_q, stop - start, q_pos0, kv_pos0 + start), -np.inf, s)
        m_tile = s.max(axis=-1, keepdims=True)
        m_new = np.maximum(m, m_tile)
        if rescale_threshold is None:
            grow = m_new > m
        else:
            grow = m_new > m + rescale_threshold
        with np.errstate(invalid="ignore"):
            factor = np.where(grow, np.exp2(np.where(np.isfinite(m), m, -np.inf) - m_new), 1.0)
        factor = np.where(np.isnan(factor), 0.0, factor)
        m = np.where(grow, m_new, m)
        acc = acc * factor
        l = l * factor
        m_sub = np.where(np.isfinite(m), m, 0.0)
        p = np.exp2(s - m_sub)
        l = l + p.sum(axis=-1, keepdims=True)
        acc = acc + np.matmul(p, v[..., start:stop, :])
    with np.errstate(divide="ignore", invalid="ignore"):
        o = np.where(l > 0, acc / np.where(l > 0, l, 1.0), 0.0)
        lse = np.where(l[..., 0] > 0,
                       (np.where(np.isfinite(m), m, 0.0) + np.log2(np.where(l > 0, l, 1.0)))[..., 0]
                       * LN2, -np.inf)
    return o, lse


def lse_merge(parts):
    """Merge [(O_i, LSE_i), ...] computed over disjoint key sets into (O, LSE)."""
    lses = np.stack([np.asarray(lse, dtype=np.float64) for _, lse in parts])
    outs = np.stack([np.asarray(o, dtype=np.float64) for o, _ in parts])
    m = lses.max(axis=0)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(lses - m_safe)
    total = w.sum(axis=0)
    with np.errstate(divide="ignore", invalid="ignore"):
        o = np.where(total[..., None] > 0,
                     (w[..., None] * outs).sum(axis=0) / np.where(total > 0, total, 1.0)[..., None],
                     0.0)
        lse = np.where(total > 0, m_safe + np.log(np.where(total > 0, total, 1.0)), -np.inf)
    return o, lse


def sdpa_reference(q, k, v, causal: bool):
    """The reference seed's call, verbatim in meaning (candidates/torch_sdpa_seed.py:6-7)."""
    import torch.nn.functional as F

    return F.scaled_dot_product_attention(q, k, v, dropout_p=0.0, is_causal=causal)


def make_inputs(shape, seed: int = 0, k_scale: float = 1.0):
    """Seeded host q, k, v: N(0,1) fp32 on the CPU generator, k *= k_scale, cast to bf16."""
    import torch

    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape, generator=g, dtype=torch.float32)
    k = torch.randn(shape, generator=g, dtype=torch.float32)
    v = torch.randn(shape, generator=g, dtype=torch.float32)
    if k_scale != 1.0:
        k = k * k_scale
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


def error_metrics(out, ref_o, lse=None, ref_lse=None) -> dict:
    """max-abs / mean-abs error of O and max-abs error of LSE (finite rows only)."""
    out = np.asarray(out, dtype=np.float64)
    ref_o = np.asarray(ref_o, dtype=np.float64)
    diff = np.abs(out - ref_o)
    metrics = {"max_abs": float(diff.max()) if diff.size else 0.0,
               "mean_abs": float(diff.mean()) if diff.size else 0.0}
    if lse is not None and ref_lse is not None:
        lse = np.asarray(lse, dtype=np.float64)
        ref_lse = np.asarray(ref_lse, dtype=np.float64)
        both_inf = np.isneginf(lse) & np.isneginf(ref_lse)
        with np.errstate(invalid="ignore"):
            d = np.where(both_inf, 0.0, np.abs(lse - ref_lse))
        metrics["lse_max_abs"] = float(d.max()) if d.size else 0.0
    return metrics


# Tolerances of the hot path (max-abs and mean-abs of O against the fp32/fp64 oracle
# of the same bf16 inputs, max-abs of LSE), plus the reference scorer's own gate
# torch.allclose(atol=3e-2, rtol=3e-2) (avo/benchmark.py:638-639).
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3
LSE_TOL = 1e-3
ALLCLOSE_ATOL = 3e-2
ALLCLOSE_RTOL = 3e-2


def within_tolerance(metrics: dict) -> bool:
    ok = metrics["max_abs"] <= MAX_ABS_TOL and metrics["mean_abs"] <= MEAN_ABS_TOL
    if "lse_max_abs" in metrics:
        ok = ok and metrics["lse_max_abs"] <= LSE_TOL
    return ok
