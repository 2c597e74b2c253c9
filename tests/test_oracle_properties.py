"""Size-independent properties of the oracle restatements (CPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention_oracle as oracle


def _rand(shape, seed=0, scale=1.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape) * scale).astype(np.float64)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("threshold", [None, 0.0, 8.0, 30.0])
def test_online_equals_direct(causal, threshold):
    q, k, v = _rand((2, 200, 128), 1), _rand((2, 200, 128), 2, 3.0), _rand((2, 200, 128), 3)
    o, lse = oracle.attention_fp64(q, k, v, causal)
    o2, lse2 = oracle.attention_online(q, k, v, causal, block=64, rescale_threshold=threshold)
    assert np.abs(o - o2).max() < 1e-12
    assert np.abs(lse - lse2).max() < 1e-12


@pytest.mark.parametrize("splits", [[0, 64, 200], [0, 1, 2, 150, 200], [0, 128, 129, 200]])
def test_lse_merge_of_key_partitions(splits):
    q, k, v = _rand((3, 90, 128), 4), _rand((3, 200, 128), 5), _rand((3, 200, 128), 6)
    o, lse = oracle.attention_fp64(q, k, v, False)
    parts = [oracle.attention_fp64(q, k[:, a:b], v[:, a:b], False) for a, b in zip(splits, splits[1:])]
    o2, lse2 = oracle.lse_merge(parts)
    assert np.abs(o - o2).max() < 1e-12 and np.abs(lse - lse2).max() < 1e-12


def test_causal_positions_and_empty_rows():
    q, k, v = _rand((1, 8, 128), 7), _rand((1, 8, 128), 8), _rand((1, 8, 128), 9)
    # Keys at positions 100..107, queries at 96..103: rows 96..99 see nothing.
    o, lse = oracle.attention_fp64(q, k, v, True, q_pos0=96, kv_pos0=100)
    assert np.all(o[0, :4] == 0) and np.all(np.isneginf(lse[0, :4]))
    assert np.isfinite(lse[0, 4:]).all()
    o2, lse2 = oracle.attention_online(q, k, v, True, block=3, q_pos0=96, kv_pos0=100)
    assert np.abs(o - o2).max() < 1e-12
    assert np.array_equal(np.isneginf(lse), np.isneginf(lse2))


def test_merge_with_empty_partial_is_identity():
    q, k, v = _rand((1, 16, 128), 10), _rand((1, 32, 128), 11), _rand((1, 32, 128), 12)
    full = oracle.attention_fp64(q, k, v, False)
    empty = (np.zeros_like(full[0]), np.full_like(full[1], -np.inf))
    o, lse = oracle.lse_merge([full, empty])
    assert np.abs(o - full[0]).max() < 1e-12 and np.abs(lse - full[1]).max() < 1e-12


def test_bf16_rounding_matches_torch():
    x = np.concatenate([_rand(10000, 13, 100.0), [0.0, -0.0, 1e-40, 3.0e38, np.inf, -np.inf]]).astype(np.float32)
    ours = oracle.f32_to_bf16_bits(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


def test_sdpa_reference_is_the_seed_call():
    q, k, v = oracle.make_inputs((1, 2, 64, 128), seed=3)
    got = oracle.sdpa_reference(q.float(), k.float(), v.float(), True).numpy()
    want, _ = oracle.attention_fp64(q.float().numpy(), k.float().numpy(), v.float().numpy(), True)
    assert np.abs(got - want).max() < 2e-5


def test_tolerance_helper():
    assert oracle.within_tolerance({"max_abs": 0.01, "mean_abs": 0.001, "lse_max_abs": 1e-4})
    assert not oracle.within_tolerance({"max_abs": 0.03, "mean_abs": 0.001})
    assert not oracle.within_tolerance({"max_abs": 0.01, "mean_abs": 0.001, "lse_max_abs": 2e-3})
