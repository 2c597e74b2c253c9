"""Multi-GPU scoring: head-sharded launches and the context-parallel ring.

The reference runs every case on cuda:0 (avo/benchmark.py:212, 242); this module is
new.  Both modes run one process per GPU under ``torch.distributed.run`` inside the
isolation wrapper (a crash or hang of any rank becomes a failed record,
avo/isolation.py), with NCCL used only for the host barrier, the max-over-ranks
reduction of timings and errors, and - in ring mode - the K/V rotation.

* ``head``: the B*H independent (batch, head) pairs are split into contiguous,
  balanced ranges, one per rank; every rank calls the candidate's
  ``attention(q, k, v, causal)`` on its [1, n, S, D] slice.  No data-path collective.
* ``ring``: causal context parallelism (``avo.ring``); each rank holds two zig-zag
  sequence chunks of every head.

Timing: ranks pass a barrier, synchronize, then time ``repeats`` calls with CUDA
events on their launching stream; the aggregate TFLOPS is total FLOPs divided by the
slowest rank's time (max over ranks).  Correctness: every rank compares its rows with
an fp32 reference of the same rows; the worst error over ranks is reported.
"""

from __future__ import annotations

import json
import os
import socket
import statistics
import sys
from pathlib import Path
from typing import Any

from .benchmark import (
    ALLCLOSE_ATOL,
    ALLCLOSE_RTOL,
    LSE_TOL,
    MAX_ABS_TOL,
    MEAN_ABS_TOL,
    CaseScore,
    _failed_score,
    _load_candidate,
    attention_forward_flops,
    host_inputs,
    tflops_from_ms,
)
from .config import AttentionCase
from .isolation import print_result, run_json_worker

PKG_ROOT = Path(__file__).resolve().parents[1]


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced [start, stop) of ``total`` items for ``rank`` of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def case_from_dict(payload: dict[str, Any]) -> AttentionCase:
    return AttentionCase(
        seq_len=int(payload["seq_len"]), causal=bool(payload["causal"]),
        head_dim=int(payload.get("head_dim", 128)), num_heads=int(payload.get("num_heads", 16)),
        total_tokens=int(payload.get("total_tokens", 32768)), dtype=str(payload.get("dtype", "bf16")),
        k_scale=float(payload.get("k_scale", 1.0)), gpus=int(payload.get("gpus", 1)),
    )


def score_from_dict(payload: dict[str, Any]) -> CaseScore:
    timing = payload.get("timing") or {}
    return CaseScore(
        backend=payload["backend"], case=case_from_dict(payload["case"]), correct=bool(payload["correct"]),
        milliseconds=payload.get("milliseconds"), tflops=float(payload.get("tflops", 0.0)),
        max_abs_error=payload.get("max_abs_error"), error=payload.get("error"),
        timing_samples_ms=tuple(timing.get("samples_ms") or ()),
        mean_abs_error=payload.get("mean_abs_error"), lse_max_abs_error=payload.get("lse_max_abs_error"),
        per_gpu_ms=tuple(payload.get("per_gpu_ms") or ()),
    )


def launch_command(candidate: Path, case: AttentionCase, *, warmup: int, repeats: int, trials: int,
                   seed: int, mode: str, port: int | None = None) -> list[str]:
    return [
        sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
        f"--nproc-per-node={case.gpus}", "--master-addr=127.0.0.1",
        f"--master-port={port or free_port()}",
        "-m", "avo", "worker-rank",
        "--candidate", str(candidate), "--case-json", json.dumps(case.as_dict()),
        "--warmup", str(warmup), "--repeats", str(repeats), "--trials", str(trials),
        "--seed", str(seed), "--mode", mode,
    ]


def worker_env(base: dict[str, str] | None = None) -> dict[str, str]:
    env = dict(os.environ if base is None else base)
    env["PYTHONPATH"] = os.pathsep.join([str(PKG_ROOT), *filter(None, [env.get("PYTHONPATH")])])
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    return env


def score_head_sharded(candidate: Path, case: AttentionCase, *, warmup: int, repeats: int, trials: int,
                       seed: int, mode: str = "head", timeout_s: float = 900) -> CaseScore:
    """Score ``case`` over ``case.gpus`` GPUs in isolated ranks; rank 0's payload."""
    command = launch_command(Path(candidate).resolve(), case, warmup=warmup, repeats=repeats,
                             trials=trials, seed=seed, mode=mode)
    result = run_json_worker(command, timeout_s=timeout_s, env=worker_env())
    if not result.ok:
        reason = "timed out" if result.timed_out else f"exit {result.returncode}"
        return _failed_score("candidate", case, f"multi-GPU ranks failed ({reason}): {result.stderr_tail[-800:]}")
    return score_from_dict(result.payload)


# ---------------------------------------------------------------- inside a rank
def _fp32_rows_reference(q, k, v, causal: bool, rows: list[tuple[int, int]]):
    """fp32 O and LSE of query rows ``rows`` (list of [start, stop) of the full
    sequence) for every head of [BH, S, D] tensors on the GPU."""
    import math

    import torch

    bh, seq, dim = q.shape
    scale = 1.0 / math.sqrt(dim)
    outs, lses = [], []
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for start, stop in rows:
            o_part = torch.empty((bh, stop - start, dim), dtype=torch.float32, device=q.device)
            l_part = torch.empty((bh, stop - start), dtype=torch.float32, device=q.device)
            for h in range(bh):
                for s0 in range(start, stop, 4096):
                    s1 = min(stop, s0 + 4096)
                    limit = s1 if causal else seq
                    s = (q[h, s0:s1].float() @ k[h, :limit].float().T) * scale
                    if causal:
                        r = torch.arange(s0, s1, device=q.device)[:, None]
                        c = torch.arange(limit, device=q.device)[None, :]
                        s.masked_fill_(c > r, float("-inf"))
                    l_part[h, s0 - start:s1 - start] = torch.logsumexp(s, dim=-1)
                    o_part[h, s0 - start:s1 - start] = torch.softmax(s, dim=-1) @ v[h, :limit].float()
            outs.append(o_part)
            lses.append(l_part)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return torch.cat(outs, dim=1), torch.cat(lses, dim=1)


def _time_rank(fn, *, warmup: int, repeats: int, trials: int, dist, device) -> list[float]:
    import torch

    for _ in range(warmup):
        fn()
    samples = []
    stream = torch.cuda.current_stream(device)
    for _ in range(trials):
        dist.barrier(device_ids=[device.index])
        torch.cuda.synchronize(device)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(repeats):
            fn()
        end.record(stream)
        torch.cuda.synchronize(device)
        samples.append(start.elapsed_time(end) / repeats)
    return samples


def rank_main(candidate: Path, case: AttentionCase, *, warmup: int, repeats: int, trials: int, seed: int,
              mode: str) -> int:
    """Body of one rank (``python -m avo worker-rank``)."""
    import datetime

    import torch
    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    error = None
    metrics = torch.zeros(3, dtype=torch.float64, device=device)
    local_ms: list[float] = []
    try:
        module = _load_candidate(candidate)
        q_h, k_h, v_h = host_inputs(case, seed)
        bh = case.batch_size * case.num_heads
        seq, dim = case.seq_len, case.head_dim
        q_all, k_all, v_all = (t.reshape(bh, seq, dim) for t in (q_h, k_h, v_h))
        if mode == "head":
            start, stop = shard_range(bh, world, rank)
            q, k, v = (t[start:stop].unsqueeze(0).contiguous().to(device) for t in (q_all, k_all, v_all))
            with_lse = getattr(module, "attention_with_lse", None)
            if callable(with_lse):
                out, lse = with_lse(q, k, v, case.causal)
            else:
                out, lse = module.attention(q, k, v, case.causal), None
            torch.cuda.synchronize(device)
            ref_o, ref_lse = _fp32_rows_reference(q[0], k[0], v[0], case.causal, [(0, seq)])
            diff = (out[0].float() - ref_o).abs()
            gate = bool(torch.allclose(out[0].float(), ref_o, atol=ALLCLOSE_ATOL, rtol=ALLCLOSE_RTOL))
            metrics[0] = diff.max() if diff.numel() else 0.0
            metrics[1] = diff.mean() if diff.numel() else 0.0
            if lse is not None:
                metrics[2] = (lse[0] - ref_lse).abs().max() if lse.numel() else 0.0
            if not gate:
                metrics[0] = max(float(metrics[0]), 1e9)
            del ref_o, ref_lse
            local_ms = _time_rank(lambda: module.attention(q, k, v, case.causal), warmup=warmup,
                                  repeats=repeats, trials=trials, dist=dist, device=device)
        elif mode == "ring":
            from . import ring

            if not case.causal:
                raise ValueError("ring mode is the causal context-parallel schedule")
            binding = _binding_for(candidate)
            q, k, v = (ring.zigzag_shard(t, rank, world, dim=1).contiguous().to(device)
                       for t in (q_all, k_all, v_all))
            runner = ring.RingAttention(q, k, v, rank=rank, world=world,
                                        backend=ring.CudaRingBackend(binding))
            out, lse = runner.forward()
            torch.cuda.synchronize(device)
            binding.check_status(device)
            chunk = seq // (2 * world)
            early, late = ring.zigzag_chunks(rank, world)
            rows = [(early * chunk, (early + 1) * chunk), (late * chunk, (late + 1) * chunk)]
            ref_o, ref_lse = _fp32_rows_reference(q_all.to(device), k_all.to(device), v_all.to(device),
                                                  True, rows)
            diff = (out.float() - ref_o).abs()
            metrics[0] = diff.max()
            metrics[1] = diff.mean()
            metrics[2] = (lse - ref_lse).abs().max()
            del ref_o, ref_lse
            local_ms = _time_rank(runner.forward, warmup=warmup, repeats=repeats, trials=trials,
                                  dist=dist, device=device)
        else:
            raise ValueError(f"unknown mode {mode!r}")
    except Exception as exc:  # report through rank 0; every rank still joins the collectives
        error = f"rank {rank}: {type(exc).__name__}: {exc}"
        metrics.fill_(float("inf"))
        local_ms = [float("inf")] * trials
    dist.all_reduce(metrics, op=dist.ReduceOp.MAX)
    per_rank = [None] * world
    dist.all_gather_object(per_rank, {"ms": local_ms, "error": error})
    dist.barrier(device_ids=[device.index])
    if rank == 0:
        errors = [p["error"] for p in per_rank if p["error"]]
        samples = tuple(max(p["ms"][t] for p in per_rank) for t in range(trials))
        max_abs, mean_abs, lse_err = (float(x) for x in metrics.tolist())
        correct = (not errors and max_abs <= MAX_ABS_TOL and mean_abs <= MEAN_ABS_TOL
                   and lse_err <= LSE_TOL)
        ms = statistics.median(samples) if not errors else None
        score = CaseScore(
            backend="candidate", case=case, correct=correct, milliseconds=ms,
            tflops=tflops_from_ms(case, ms) if (correct and ms) else 0.0,
            max_abs_error=None if errors else max_abs,
            mean_abs_error=None if errors else mean_abs,
            lse_max_abs_error=None if errors else lse_err,
            timing_samples_ms=samples if not errors else (),
            per_gpu_ms=tuple(statistics.median(p["ms"]) for p in per_rank) if not errors else (),
            error="; ".join(errors) if errors else (None if correct else f"{mode} mode failed tolerance check"),
        )
        payload = score.as_dict()
        payload["mode"] = mode
        payload["flops"] = attention_forward_flops(case)
        print_result(payload)
    dist.destroy_process_group()
    return 0


def _binding_for(candidate: Path):
    """The candidate's C-ABI binding (companion directory of the seed)."""
    import importlib.util

    name = "avo_b200_attention_binding"
    module = sys.modules.get(name)
    if module is None:
        stem = candidate.stem.removesuffix("_seed")
        path = candidate.resolve().parent / stem / "b200_attention.py"
        spec = importlib.util.spec_from_file_location(name, path)
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
    return module
