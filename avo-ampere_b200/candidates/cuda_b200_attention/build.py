"""Builds libavo_b200_attn.so in place with nvcc for sm_100a.

The reference JIT-builds each CUDA seed through ``torch.utils.cpp_extension.load``
(candidates/cuda_mma_attention_seed.py:16-30) with the arch list pinned to sm_86
(avo/cuda_env.py:37).  This candidate ships a plain C-ABI shared library instead, so
it is built once, ahead of time, by nvcc with ``-gencode arch=compute_100a,code=sm_100a``
and loaded with ctypes; the built ``.so`` sits next to its sources.

Usage: ``python build.py [--force] [--ptxas-verbose]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_NAME = "libavo_b200_attn.so"
LIB_PATH = HERE / LIB_NAME
SOURCES = ("attn_abi.cu",)
HEADERS = ("attn_fwd.cuh", "sm100_ptx.cuh", "schedule.cuh")
GENCODE = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = (
    *GENCODE,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
)


FAST_SOURCE = HERE / "fast_call.c"
FAST_PATH = HERE / ("_avo_b200_fast" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


class BuildError(RuntimeError):
    """nvcc failed or could not be found."""


def build_fast(*, force: bool = False) -> Path | None:
    """Compile the CPython binding of the per-call entry (fast_call.c) with the host C
    compiler, if it is missing or older than its source.  Returns its path, or None when
    no compiler or no Python headers are available (the ctypes binding is then used)."""
    if not force and FAST_PATH.is_file() and FAST_PATH.stat().st_mtime >= FAST_SOURCE.stat().st_mtime:
        return FAST_PATH
    compiler = shutil.which(os.environ.get("CC", "") or "gcc") or shutil.which("cc")
    include = sysconfig.get_paths().get("include")
    if compiler is None or not include or not (Path(include) / "Python.h").is_file():
        return None
    fd, tmp_name = tempfile.mkstemp(prefix="._avo_b200_fast.", suffix=".so", dir=HERE)
    os.close(fd)
    tmp = Path(tmp_name)
    try:
        command = [compiler, "-O2", "-shared", "-fPIC", "-I", include, str(FAST_SOURCE), "-o", str(tmp)]
        completed = subprocess.run(command, text=True, capture_output=True, check=False)
        if completed.returncode != 0:
            raise BuildError(f"{' '.join(command)} failed:\n{completed.stderr[-2000:]}")
        os.replace(tmp, FAST_PATH)
    finally:
        if tmp.exists():
            tmp.unlink()
    return FAST_PATH


def include_dir() -> Path:
    """Directory holding avo_b200_attn.h (the repository's ``include/``)."""
    env = os.environ.get("AVO_B200_INCLUDE")
    candidates = [Path(env)] if env else []
    candidates += [HERE / "include", HERE.parents[2] / "include"]
    for candidate in candidates:
        if (candidate / "avo_b200_attn.h").is_file():
            return candidate
    raise BuildError("avo_b200_attn.h not found; set AVO_B200_INCLUDE to its directory")


def nvcc_path() -> str:
    for key in ("CUDA_HOME", "CUDA_PATH"):
        root = os.environ.get(key)
        if root and (Path(root) / "bin" / "nvcc").is_file():
            return str(Path(root) / "bin" / "nvcc")
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    if default.is_file():
        return str(default)
    raise BuildError("nvcc not found (set CUDA_HOME)")


def source_files() -> list[Path]:
    files = [HERE / name for name in (*SOURCES, *HEADERS)]
    try:
        files.append(include_dir() / "avo_b200_attn.h")
    except BuildError:
        pass
    return files


def needs_build() -> bool:
    if not LIB_PATH.is_file():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(path.is_file() and path.stat().st_mtime > built for path in source_files())


def build_command(output: Path, *, ptxas_verbose: bool = False) -> list[str]:
    command = [nvcc_path(), *NVCC_FLAGS, "-I", str(include_dir())]
    if ptxas_verbose:
        command.append("-Xptxas=-v")
    command += [str(HERE / name) for name in SOURCES]
    command += ["-o", str(output)]
    return command


def build(*, force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the library (and the CPython binding of its per-call entry) if missing or
    older than their sources; return the library's path."""
    build_fast(force=force)
    if not force and not needs_build():
        return LIB_PATH
    fd, tmp_name = tempfile.mkstemp(prefix=".libavo_b200_attn.", suffix=".so", dir=HERE)
    os.close(fd)
    tmp = Path(tmp_name)
    try:
        command = build_command(tmp, ptxas_verbose=ptxas_verbose)
        completed = subprocess.run(command, text=True, capture_output=True, check=False)
        if verbose or ptxas_verbose:
            sys.stderr.write(completed.stdout + completed.stderr)
        if completed.returncode != 0:
            raise BuildError(
                f"nvcc failed ({completed.returncode}): {' '.join(command)}\n"
                f"{completed.stderr[-4000:]}"
            )
        os.replace(tmp, LIB_PATH)
    finally:
        if tmp.exists():
            tmp.unlink()
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=True, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
