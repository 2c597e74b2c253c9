"""The C-ABI library builds for sm_100a, loads without a GPU, and exports exactly what
include/avo_b200_attn.h declares; host-side argument checks answer without a device."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "avo_b200_attn.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(avo_b200_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    assert "avo_b200_attn_fwd" in names and "avo_b200_attn_fwd_block" in names
    assert "avo_b200_lse_merge" in names and "avo_b200_watchdog_selftest" in names


def test_library_exports_every_declared_symbol(b200):
    path = b200.library_path()
    lib = ctypes.CDLL(str(path))
    for name in declared_functions():
        assert hasattr(lib, name), name
    exported = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True,
                              check=True).stdout
    public = sorted(set(re.findall(r"\bT (avo_b200_\w+)", exported)))
    assert public == declared_functions()
    assert set(b200.SIGNATURES) == set(declared_functions())


def test_abi_version_and_strerror(b200):
    lib = b200.load_library()
    assert lib.avo_b200_abi_version() == b200.ABI_VERSION
    assert b200.strerror(0) == "ok"
    assert "invalid" in b200.strerror(1)
    assert "B200" in b200.strerror(2)
    assert b200.strerror(99) == "unknown error"
    assert "register count" in b200.strerror(7) and "168" in b200.strerror(7)


def test_library_links_no_driver_library(b200):
    needed = subprocess.run(["readelf", "-d", str(b200.library_path())], capture_output=True, text=True,
                            check=True).stdout
    assert "libcuda.so" not in needed  # the tensor-map encoder is fetched at run time


def test_host_side_argument_checks(b200):
    lib = b200.load_library()
    # Null tensors, a wrong head_dim or a non-positive scale are rejected before any
    # CUDA call, so these run without a GPU.
    assert lib.avo_b200_attn_fwd(None, None, None, None, None, 1, 1, 128, 128, 0, 0.088, None, None) == 1
    fake = ctypes.c_void_p(0x10000)
    assert lib.avo_b200_attn_fwd(fake, fake, fake, fake, None, 1, 1, 128, 64, 0, 0.088, None, None) == 1
    assert lib.avo_b200_attn_fwd(fake, fake, fake, fake, None, 1, 1, 128, 128, 0, 0.0, None, None) == 1
    assert lib.avo_b200_attn_fwd(fake, fake, fake, fake, None, -1, 1, 128, 128, 0, 0.088, None, None) == 1
    misaligned = ctypes.c_void_p(0x10008)
    assert lib.avo_b200_attn_fwd(misaligned, fake, fake, fake, None, 1, 1, 128, 128, 0, 0.088, None, None) == 1
    # Empty problems are a no-op success.
    assert lib.avo_b200_attn_fwd(fake, fake, fake, fake, None, 0, 16, 128, 128, 0, 0.088, None, None) == 0
    assert lib.avo_b200_attn_fwd_block(fake, fake, fake, fake, None, 2, 64, 64, 128, 100, 64 * 128,
                                       64 * 128, 64, 0, 0.088, 0, 0, None, None) == 1  # stride % 8
    assert lib.avo_b200_lse_merge(None, None, None, None, 1, 1, 128, 128, 1, 128, 1, None) == 1
    assert lib.avo_b200_acc_to_bf16(fake, fake, 1, 4, 128, 100, 512, None) == 1
    assert lib.avo_b200_watchdog_selftest(0, fake, None) == 1
    # The no-allocation entry point: argument errors, then a problem beyond its static
    # scratch (16384 rows) is refused with its own code before any device work.
    noalloc = lib.avo_b200_attn_fwd_split_noalloc
    assert noalloc(None, fake, fake, fake, None, 1, 1, 128, 128, 0, 0.088, 2, None, None) == 1
    assert noalloc(fake, fake, fake, fake, None, 1, 1, 128, 128, 0, 0.088, 0, None, None) == 1
    assert noalloc(fake, fake, fake, fake, None, 1, 1, 128, 128, 0, 0.088, 65, None, None) == 1
    assert noalloc(fake, fake, fake, fake, None, 1, 1, 16384 + 128, 128, 0, 0.088, 2, None, None) == 6
    assert noalloc(fake, fake, fake, fake, None, 2, 16, 1024, 128, 0, 0.088, 2, None, None) == 6
    assert noalloc(fake, fake, fake, fake, None, 0, 16, 1024, 128, 0, 0.088, 2, None, None) == 0
    # Dimensions whose row product overflows 64 bits are refused as too large, not wrapped.
    int_max = 2**31 - 1
    assert noalloc(fake, fake, fake, fake, None, int_max, int_max, 4, 128, 0, 0.088, 2, None, None) == 6
    assert noalloc(fake, fake, fake, fake, None, int_max, int_max, int_max, 128, 0, 0.088, 2, None, None) == 6
    assert noalloc(fake, fake, fake, fake, None, 1, int_max, 2, 128, 0, 0.088, 2, None, None) == 6
    assert "too large" in b200.strerror(6)


def test_no_gpu_means_enodev(b200):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = b200.load_library()
    fake = ctypes.c_void_p(0x10000)
    assert lib.avo_b200_attn_fwd(fake, fake, fake, fake, None, 1, 1, 128, 128, 0, 0.088, None, None) == 2


def test_build_flags_target_sm100a():
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "avo_b200_build_check", ROOT / "avo-ampere_b200" / "candidates" / "cuda_b200_attention" / "build.py")
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    command = build.build_command(Path("/tmp/x.so"))
    assert "arch=compute_100a,code=sm_100a" in command
    assert "-shared" in command and "-lineinfo" in command


def test_cpython_binding_builds_and_checks_arguments():
    # The per-call entry's CPython binding (fast_call.c) compiles with the host compiler and
    # refuses a wrong argument count before it touches the library (no GPU needed).
    import importlib.util
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parents[1] / "avo-ampere_b200" / "candidates" / "cuda_b200_attention"
    spec = importlib.util.spec_from_file_location("avo_b200_build_for_test", here / "build.py")
    builder = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(builder)
    path = builder.build_fast()
    if path is None:
        pytest.skip("no C compiler or Python headers")
    spec = importlib.util.spec_from_file_location("_avo_b200_fast", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    with pytest.raises(TypeError):
        module.fwd_ws(1, 2, 3)
    assert sys.modules.get("avo_b200_build_for_test") is None
