"""CLI surface (CPU): parsing, worker argv, the ncu wrapper's command and CSV parsing."""

from __future__ import annotations

import pytest

from avo.cli import build_parser, parse_ncu_raw_csv, profile_command, worker_argv


def test_score_args_forward_to_worker():
    args = build_parser().parse_args([
        "score", "--backend", "candidate", "--candidate", "c.py", "--seq-lens", "8192", "--causal", "false",
        "--trials", "3", "--gpus", "2", "--mode", "head", "--k-scale", "3", "--seed", "7"])
    argv = worker_argv(args)
    assert argv[1:4] == ["-m", "avo", "worker-score"]
    for flag, value in (("--trials", "3"), ("--gpus", "2"), ("--k-scale", "3.0"), ("--seed", "7"),
                        ("--candidate", "c.py"), ("--mode", "head")):
        assert argv[argv.index(flag) + 1] == value


def test_profile_never_locks_clocks():
    args = build_parser().parse_args(["profile", "--backend", "candidate", "--candidate", "c.py",
                                      "--seq-lens", "4096", "--causal", "false"])
    cmd = profile_command("/usr/bin/ncu", args)
    assert cmd[cmd.index("--clock-control") + 1] == "none"
    assert cmd[cmd.index("--kernel-name") + 1] == "regex:attn_fwd"
    assert "worker-score" in cmd
    assert "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed" in cmd[cmd.index("--metrics") + 1]


def test_profile_refuses_multi_gpu(capsys):
    from avo.cli import main

    with pytest.raises(ValueError, match="one GPU"):
        main(["profile", "--backend", "candidate", "--candidate", "c.py", "--gpus", "2"])


def test_parse_ncu_raw_csv():
    text = ('==PROF== Connected\n"ID","Kernel Name","gpu__time_duration.sum"\n"","","nsecond"\n'
            '"0","attn_fwd_kernel","500000"\nAVO_RESULT_JSON={}\n')
    rows = parse_ncu_raw_csv(text)
    assert rows == [{"ID": "0", "Kernel Name": "attn_fwd_kernel", "gpu__time_duration.sum": "500000"}]
    assert parse_ncu_raw_csv("nothing") == []


def test_cases_and_env_commands(capsys):
    from avo.cli import main

    assert main(["cases"]) == 0
    assert "b4_h16_s8192_noncausal" in capsys.readouterr().out
    assert main(["env"]) == 0
    assert "sm_100a" in capsys.readouterr().out
