"""``python -m avo`` - the hot-path commands of the reference CLI, retargeted to B200.

Mirrors the reference's ``avo/cli.py`` subcommands that touch the attention path:
``env`` (:97-98), ``compile`` (:113-116), ``score`` (:118-120, :420-453),
``profile`` (:122-131, :456-590) and the child ``worker-score`` (:725-743), with the
same flags (``add_score_args`` :258-273) plus ``--gpus``, ``--mode head|ring``,
``--k-scale`` and ``--seed``.  The LLM agent, evolve, knowledge and lineage commands
are not part of the hot path and are not provided.

``score`` runs ``worker-score`` in an isolated child (``avo.isolation``); with
``--gpus N > 1`` the worker launches N ranks (``avo.multigpu``).  ``profile`` wraps
the same worker in Nsight Compute, always with ``--clock-control none`` so the GPU's
clocks are never locked, and reports counters only.
"""

from __future__ import annotations

import argparse
import json
import shutil
import subprocess
import sys
from pathlib import Path

from .config import NAMED_CASES, cases_from_cli
from .isolation import extract_payload, module_worker_args, print_result, run_json_worker

PROFILE_TIMEOUT_CAP_S = 300
PROFILE_METRICS = (
    "gpu__time_duration.sum",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "launch__registers_per_thread",
)


def add_score_args(parser: argparse.ArgumentParser) -> None:
    parser.add_argument("--backend", choices=["torch-sdpa", "flash-attn", "candidate"], required=True)
    parser.add_argument("--candidate", type=Path, default=None)
    parser.add_argument("--seq-lens", default="4096,8192,16384,32768")
    parser.add_argument("--causal", choices=["true", "false", "both"], default="both")
    parser.add_argument("--head-dim", type=int, default=128)
    parser.add_argument("--num-heads", type=int, default=16)
    parser.add_argument("--total-tokens", type=int, default=32768)
    parser.add_argument("--dtype", choices=["bf16", "fp16", "fp32"], default="bf16")
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--repeats", type=int, default=20)
    parser.add_argument("--trials", type=int, default=1)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--k-scale", type=float, default=1.0)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--mode", choices=["head", "ring"], default="head")


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="avo")
    sub = parser.add_subparsers(dest="command", required=True)
    sub.add_parser("env")
    sub.add_parser("cases")

    compile_parser = sub.add_parser("compile")
    compile_parser.add_argument("--source", type=Path, required=True)
    compile_parser.add_argument("--out-dir", type=Path, required=True)
    compile_parser.add_argument("--timeout-s", type=int, default=120)

    score_parser = sub.add_parser("score")
    add_score_args(score_parser)
    score_parser.add_argument("--timeout-s", type=int, default=900)

    profile_parser = sub.add_parser("profile")
    add_score_args(profile_parser)
    profile_parser.add_argument("--timeout-s", type=int, default=300)
    profile_parser.add_argument("--kernel-name", default="regex:attn_fwd")
    profile_parser.add_argument("--launch-count", type=int, default=1)
    profile_parser.add_argument("--launch-skip", type=int, default=0)
    profile_parser.add_argument("--metric", action="append", default=[])

    worker = sub.add_parser("worker-score")
    add_score_args(worker)

    rank = sub.add_parser("worker-rank")
    rank.add_argument("--candidate", type=Path, required=True)
    rank.add_argument("--case-json", required=True)
    rank.add_argument("--warmup", type=int, default=5)
    rank.add_argument("--repeats", type=int, default=20)
    rank.add_argument("--trials", type=int, default=1)
    rank.add_argument("--seed", type=int, default=0)
    rank.add_argument("--mode", choices=["head", "ring"], default="head")
    return parser


def main(argv: list[str] | None = None) -> int:
    args = build_parser().parse_args(argv)
    if args.command == "env":
        from .cuda_env import environment_report

        print(json.dumps(environment_report(), indent=2, sort_keys=True, default=str))
        return 0
    if args.command == "cases":
        print(json.dumps({name: case.as_dict() for name, case in NAMED_CASES.items()}, indent=2))
        return 0
    if args.command == "compile":
        from .compile import compile_cuda_source

        result = compile_cuda_source(args.source, args.out_dir, timeout_s=args.timeout_s)
        print(json.dumps(result.as_dict(), indent=2, sort_keys=True))
        return 0 if result.ok else 2
    if args.command == "score":
        return _score(args)
    if args.command == "profile":
        return _profile(args)
    if args.command == "worker-score":
        return _worker_score(args)
    if args.command == "worker-rank":
        from .multigpu import case_from_dict, rank_main

        return rank_main(args.candidate, case_from_dict(json.loads(args.case_json)), warmup=args.warmup,
                         repeats=args.repeats, trials=args.trials, seed=args.seed, mode=args.mode)
    raise AssertionError(args.command)


def worker_argv(args: argparse.Namespace) -> list[str]:
    argv = module_worker_args(
        "worker-score", "--backend", args.backend, "--seq-lens", args.seq_lens, "--causal", args.causal,
        "--head-dim", str(args.head_dim), "--num-heads", str(args.num_heads),
        "--total-tokens", str(args.total_tokens), "--dtype", args.dtype, "--warmup", str(args.warmup),
        "--repeats", str(args.repeats), "--trials", str(args.trials), "--seed", str(args.seed),
        "--k-scale", str(args.k_scale), "--gpus", str(args.gpus), "--mode", args.mode,
    )
    if args.candidate:
        argv.extend(["--candidate", str(args.candidate)])
    return argv


def _worker_env() -> dict[str, str]:
    from .cuda_env import prepare_torch_extension_env
    from .multigpu import worker_env

    env = worker_env()
    prepare_torch_extension_env(env)
    return env


def _score(args: argparse.Namespace) -> int:
    result = run_json_worker(worker_argv(args), timeout_s=args.timeout_s, cwd=Path.cwd(), env=_worker_env())
    print(json.dumps(result.as_dict(), indent=2, sort_keys=True))
    return 0 if result.ok else 2


def _worker_score(args: argparse.Namespace) -> int:
    from .benchmark import score_backend

    cases = cases_from_cli(args.seq_lens, args.causal, head_dim=args.head_dim, num_heads=args.num_heads,
                           total_tokens=args.total_tokens, dtype=args.dtype, k_scale=args.k_scale,
                           gpus=args.gpus)
    if args.gpus > 1:
        if args.backend != "candidate" or args.candidate is None:
            raise SystemExit("--gpus > 1 needs --backend candidate --candidate PATH")
        from .benchmark import benchmark_metadata, score_summary
        from .multigpu import score_head_sharded

        scores = [score_head_sharded(args.candidate, case, warmup=args.warmup, repeats=args.repeats,
                                     trials=args.trials, seed=args.seed, mode=args.mode) for case in cases]
        payload = score_summary("candidate", scores)
        payload["benchmark"] = benchmark_metadata(cases=cases, warmup=args.warmup, repeats=args.repeats,
                                                  trials=args.trials, seed=args.seed)
        payload["candidate_path"] = str(args.candidate)
        payload["mode"] = args.mode
    else:
        payload = score_backend(args.backend, cases, warmup=args.warmup, repeats=args.repeats,
                                trials=args.trials, seed=args.seed, candidate=args.candidate)
    print_result(payload)
    return 0


def profile_command(ncu: str, args: argparse.Namespace) -> list[str]:
    metrics = list(args.metric) or list(PROFILE_METRICS)
    return [
        ncu, "--target-processes", "all", "--clock-control", "none",
        "--metrics", ",".join(metrics), "--kernel-name", args.kernel_name,
        "--launch-count", str(args.launch_count), "--launch-skip", str(args.launch_skip),
        "--csv", "--page", "raw", *worker_argv(args),
    ]


def parse_ncu_raw_csv(text: str) -> list[dict[str, str]]:
    """Launch rows of ``ncu --csv --page raw`` output: a header row of metric names,
    a row of units, then one row per profiled launch."""
    import csv

    rows = list(csv.reader(line for line in text.splitlines() if line.startswith('"')))
    if len(rows) < 3:
        return []
    header = rows[0]
    return [dict(zip(header, row)) for row in rows[2:]]


def _profile(args: argparse.Namespace) -> int:
    if args.backend != "candidate" or args.candidate is None:
        raise ValueError("profile requires --backend candidate --candidate PATH")
    if args.gpus != 1:
        raise ValueError("profile runs on one GPU only (never a multi-rank command under ncu)")
    if args.launch_count <= 0 or args.launch_skip < 0:
        raise ValueError("profile requires --launch-count > 0 and --launch-skip >= 0")
    ncu = shutil.which("ncu")
    settings = {"kernel_name": args.kernel_name, "launch_count": args.launch_count,
                "launch_skip": args.launch_skip, "clock_control": "none"}
    if ncu is None:
        print(json.dumps({"ok": False, "profiler_error": "ncu_not_found", "settings": settings}, indent=2))
        return 2
    command = profile_command(ncu, args)
    timeout_s = min(args.timeout_s, PROFILE_TIMEOUT_CAP_S)
    try:
        completed = subprocess.run(command, env=_worker_env(), stdin=subprocess.DEVNULL, text=True,
                                   capture_output=True, timeout=timeout_s, check=False)
    except subprocess.TimeoutExpired:
        print(json.dumps({"ok": False, "profiler_error": "timeout", "command": command,
                          "settings": settings}, indent=2))
        return 2
    launches = parse_ncu_raw_csv(completed.stdout)
    payload = {
        "ok": completed.returncode == 0 and bool(launches),
        "returncode": completed.returncode,
        "command": command,
        "settings": settings,
        "launches": launches,
        "score": extract_payload(completed.stdout),
        "stderr_tail": completed.stderr[-2000:],
    }
    print(json.dumps(payload, indent=2, sort_keys=True))
    return 0 if payload["ok"] else 2


if __name__ == "__main__":
    sys.exit(main())
