"""Head-sharding arithmetic and the rank launcher (CPU)."""

from __future__ import annotations

import json

import pytest

from avo.benchmark import CaseScore
from avo.config import AttentionCase
from avo.multigpu import case_from_dict, launch_command, score_from_dict, shard_range, worker_env


@pytest.mark.parametrize("total,world", [(64, 1), (64, 8), (16, 8), (16, 3), (5, 8), (32, 4)])
def test_shard_range_partitions_exactly(total, world):
    ranges = [shard_range(total, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def test_launch_command_is_torchrun_on_loopback():
    case = AttentionCase(seq_len=4096, causal=False, total_tokens=16384, gpus=4)
    cmd = launch_command("cand.py", case, warmup=3, repeats=5, trials=1, seed=0, mode="head", port=29555)
    assert cmd[1:4] == ["-m", "torch.distributed.run", "--nnodes=1"]
    assert "--nproc-per-node=4" in cmd and "--master-addr=127.0.0.1" in cmd and "--master-port=29555" in cmd
    payload = json.loads(cmd[cmd.index("--case-json") + 1])
    assert case_from_dict(payload) == case
    assert worker_env({"PYTHONPATH": "x"})["PYTHONPATH"].endswith("x")
    assert worker_env({})["NCCL_NVLS_ENABLE"] == "0"


def test_score_round_trip():
    case = AttentionCase(seq_len=32768, causal=True, gpus=8)
    score = CaseScore(backend="candidate", case=case, correct=True, milliseconds=1.5, tflops=100.0,
                      max_abs_error=0.01, timing_samples_ms=(1.5,), mean_abs_error=0.001,
                      lse_max_abs_error=1e-4, per_gpu_ms=tuple([1.5] * 8))
    again = score_from_dict(score.as_dict())
    assert again == score
