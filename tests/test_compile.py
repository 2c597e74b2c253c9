"""Compile helper flags with a fake nvcc (mirrors the reference's tests/test_compile.py)."""

from __future__ import annotations

import os
import stat
from pathlib import Path

from avo.compile import compile_cuda_source


def _fake_nvcc(tmp_path: Path) -> Path:
    log = tmp_path / "argv.log"
    script = tmp_path / "nvcc"
    script.write_text(
        "#!/bin/bash\n"
        f"printf '%s\\n' \"$@\" > {log}\n"
        "while [ $# -gt 0 ]; do if [ \"$1\" = -o ]; then touch \"$2\"; fi; shift; done\n"
    )
    script.chmod(script.stat().st_mode | stat.S_IEXEC)
    return script


def test_compile_uses_sm100a_gencode(tmp_path):
    source = tmp_path / "k.cu"
    source.write_text("__global__ void k() {}\n")
    nvcc = _fake_nvcc(tmp_path)
    result = compile_cuda_source(source, tmp_path / "out", nvcc=str(nvcc), include_dirs=[tmp_path])
    argv = (tmp_path / "argv.log").read_text().split("\n")
    assert result.ok
    assert "-gencode=arch=compute_100a,code=sm_100a" in argv
    assert "--ptxas-options=-v" in argv and "-lineinfo" in argv and "-c" in argv
    assert "-D__CUDA_NO_BFLOAT16_CONVERSIONS__" in argv
    assert argv[argv.index("-I") + 1] == str(tmp_path)


def test_compile_real_nvcc_for_sm100a(tmp_path):
    if not Path("/usr/local/cuda/bin/nvcc").exists():
        return
    source = tmp_path / "smoke.cu"
    source.write_text('extern "C" __global__ void avo_smoke_kernel(int* out) { out[0] = 1; }\n')
    result = compile_cuda_source(source, tmp_path / "out", nvcc="/usr/local/cuda/bin/nvcc",
                                 env=dict(os.environ))
    assert result.ok, result.stderr_tail
    assert "sm_100a" in result.stderr_tail or "sm_100a" in result.stdout_tail
