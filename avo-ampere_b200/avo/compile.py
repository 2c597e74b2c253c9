"""Compile-only nvcc diagnostics for a CUDA source, targeting sm_100a.

Mirror of the reference's ``avo/compile.py`` (``compile_cuda_source`` :40-84): same
flags (``-std=c++17 -O3 -lineinfo --expt-relaxed-constexpr``, the torch-extension
``-D__CUDA_NO_*`` defines, ``--ptxas-options=-v``, ``-c``) with the gencode switched
from ``compute_86/sm_86`` to the B200's arch-specific ``compute_100a/sm_100a``, so
ptxas reports registers, spills and shared memory for the target that runs it.
"""

from __future__ import annotations

import os
import subprocess
from collections.abc import Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from .config import ACTIVE_TARGET

TORCH_EXTENSION_CUDA_DEFINES = (
    "__CUDA_NO_HALF_OPERATORS__",
    "__CUDA_NO_HALF_CONVERSIONS__",
    "__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "__CUDA_NO_HALF2_OPERATORS__",
)


@dataclass(frozen=True)
class CompileResult:
    ok: bool
    command: list[str]
    returncode: int
    object_path: Path
    stdout_tail: str
    stderr_tail: str

    def as_dict(self) -> dict[str, Any]:
        return {
            "ok": self.ok,
            "command": self.command,
            "returncode": self.returncode,
            "object_path": str(self.object_path),
            "stdout_tail": self.stdout_tail,
            "stderr_tail": self.stderr_tail,
        }


def compile_command(source: Path, object_path: Path, compiler: str,
                    include_dirs: Sequence[str | Path] = ()) -> list[str]:
    return [
        compiler,
        ACTIVE_TARGET.nvcc_gencode,
        "-std=c++17",
        "-O3",
        "-lineinfo",
        "--expt-relaxed-constexpr",
        *[f"-D{define}" for define in TORCH_EXTENSION_CUDA_DEFINES],
        "--ptxas-options=-v",
        *[flag for include_dir in include_dirs for flag in ("-I", str(include_dir))],
        "-c",
        str(source),
        "-o",
        str(object_path),
    ]


def compile_cuda_source(source: Path, out_dir: Path, *, timeout_s: int = 120, nvcc: str | None = None,
                        env: dict[str, str] | None = None,
                        include_dirs: Sequence[str | Path] = ()) -> CompileResult:
    if not source.exists():
        raise FileNotFoundError(source)
    out_dir.mkdir(parents=True, exist_ok=True)
    object_path = out_dir / f"{source.stem}.o"
    compiler = nvcc or _default_nvcc(env or dict(os.environ))
    command = compile_command(source, object_path, compiler, include_dirs)
    completed = subprocess.run(command, text=True, capture_output=True, timeout=timeout_s,
                               check=False, env=env)
    return CompileResult(
        ok=completed.returncode == 0 and object_path.exists(),
        command=command,
        returncode=completed.returncode,
        object_path=object_path,
        stdout_tail=_tail(completed.stdout),
        stderr_tail=_tail(completed.stderr),
    )


def _default_nvcc(env: dict[str, str]) -> str:
    cuda_home = env.get("CUDA_HOME")
    if cuda_home:
        candidate = Path(cuda_home) / "bin" / "nvcc"
        if candidate.exists():
            return str(candidate)
    return "nvcc"


def _tail(text: str, limit: int = 4000) -> str:
    return text[-limit:]
