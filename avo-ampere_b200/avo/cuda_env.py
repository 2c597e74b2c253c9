"""CUDA toolchain environment and the B200 hardware check.

Mirror of the reference's ``avo/cuda_env.py`` (``prepare_torch_extension_env`` :31-46,
``nvcc_cuda_version`` / ``parse_nvcc_release`` :111-146, ``cuda_build_compatibility``
:149-175) retargeted to the B200:

* the torch-extension arch list becomes ``10.0a`` (the reference pins ``8.6``, :37);
* ``check_b200`` / ``require_b200`` replace the scorer's sm_86 assertion with a check
  for compute capability 10.0;
* ``library_build_compatibility`` states the rule for the candidate's C-ABI library:
  it links the CUDA runtime statically, so it needs only a driver at least as new as
  the nvcc that built it (not a torch-matching toolkit).
"""

from __future__ import annotations

import os
import re
import shutil
import subprocess
from collections.abc import MutableMapping
from pathlib import Path
from typing import Any

from .config import ACTIVE_TARGET

DEFAULT_CUDA_HOME = "/usr/local/cuda"


def prepare_torch_extension_env(env: MutableMapping[str, str] | None = None, *,
                                max_jobs: str = "2") -> MutableMapping[str, str]:
    target = os.environ if env is None else env
    target.setdefault("TORCH_CUDA_ARCH_LIST", ACTIVE_TARGET.torch_arch_list)
    target.setdefault("MAX_JOBS", max_jobs)
    if "CUDA_HOME" not in target and (Path(DEFAULT_CUDA_HOME) / "bin" / "nvcc").exists():
        target["CUDA_HOME"] = DEFAULT_CUDA_HOME
    return target


def nvcc_path_from_env(env: dict[str, str]) -> str | None:
    cuda_home = env.get("CUDA_HOME") or env.get("CUDA_PATH")
    if cuda_home:
        return str(Path(cuda_home) / "bin" / "nvcc")
    return shutil.which("nvcc", path=env.get("PATH"))


def torch_cuda_version() -> str | None:
    try:
        import torch
    except Exception:
        return None
    return torch.version.cuda


def nvcc_cuda_version(nvcc_path: str | None, env: dict[str, str]) -> tuple[str | None, str | None]:
    if nvcc_path is None:
        return None, "nvcc was not found in CUDA_HOME, CUDA_PATH, or PATH"
    try:
        completed = subprocess.run([nvcc_path, "--version"], check=True, capture_output=True,
                                   env=env, text=True, timeout=10)
    except FileNotFoundError:
        return None, f"nvcc was not found at {nvcc_path}"
    except subprocess.TimeoutExpired:
        return None, f"{nvcc_path} --version timed out"
    except subprocess.CalledProcessError as exc:
        output = (exc.stdout or exc.stderr or "").strip()
        return None, f"{nvcc_path} --version failed" + (f": {output}" if output else "")
    version = parse_nvcc_release(f"{completed.stdout}\n{completed.stderr}")
    if version is None:
        return None, f"could not parse CUDA release from {nvcc_path} --version"
    return version, None


def parse_nvcc_release(output: str) -> str | None:
    match = re.search(r"release\s+(\d+\.\d+)", output)
    return match.group(1) if match else None


def _major_minor(version: str | None) -> tuple[int, int] | None:
    if version is None:
        return None
    match = re.match(r"^\s*(\d+)\.(\d+)", version)
    return (int(match.group(1)), int(match.group(2))) if match else None


def cuda_build_compatibility(torch_cuda: str | None, nvcc_cuda: str | None) -> tuple[str, str | None]:
    """Torch-extension rule (same classes as the reference): exact, minor_mismatch, major_mismatch."""
    if torch_cuda is None:
        return "missing_torch_cuda", "torch.version.cuda is unavailable"
    if nvcc_cuda is None:
        return "missing_nvcc", "nvcc CUDA version is unavailable"
    tv, nv = _major_minor(torch_cuda), _major_minor(nvcc_cuda)
    if tv is None:
        return "unparseable_torch_cuda", f"could not parse torch CUDA version {torch_cuda!r}"
    if nv is None:
        return "unparseable_nvcc_cuda", f"could not parse nvcc CUDA version {nvcc_cuda!r}"
    if tv == nv:
        return "exact", None
    if tv[0] == nv[0]:
        return ("minor_mismatch", "PyTorch extension builds may warn: "
                f"nvcc reports CUDA {nvcc_cuda} but torch was compiled with CUDA {torch_cuda}")
    return ("major_mismatch", "PyTorch extension builds will fail: "
            f"nvcc reports CUDA {nvcc_cuda} but torch was compiled with CUDA {torch_cuda}")


def library_build_compatibility(driver_cuda: str | None, nvcc_cuda: str | None) -> tuple[str, str | None]:
    """The C-ABI library links cudart statically: the driver must support nvcc's CUDA."""
    dv, nv = _major_minor(driver_cuda), _major_minor(nvcc_cuda)
    if dv is None or nv is None:
        return "unknown", f"driver CUDA {driver_cuda!r}, nvcc CUDA {nvcc_cuda!r}"
    if dv >= nv:
        return "ok", None
    return "driver_too_old", f"driver supports CUDA {driver_cuda} < nvcc CUDA {nvcc_cuda}"


def driver_cuda_version() -> str | None:
    try:
        import torch

        if not torch.cuda.is_available():
            return None
        from ctypes import CDLL, byref, c_int

        version = c_int(0)
        CDLL("libcuda.so.1").cuDriverGetVersion(byref(version))
        return f"{version.value // 1000}.{(version.value % 1000) // 10}"
    except Exception:
        return None


def check_b200(device_index: int = 0) -> dict[str, Any]:
    """Facts about ``cuda:device_index`` and whether it is a B200 (capability 10.0)."""
    report: dict[str, Any] = {"ok": False, "device": device_index}
    try:
        import torch
    except Exception as exc:
        report["reason"] = f"torch unavailable: {exc}"
        return report
    if not torch.cuda.is_available():
        report["reason"] = "CUDA is not available"
        return report
    if device_index >= torch.cuda.device_count():
        report["reason"] = f"no CUDA device {device_index} (count {torch.cuda.device_count()})"
        return report
    props = torch.cuda.get_device_properties(device_index)
    capability = (props.major, props.minor)
    report.update(name=props.name, compute_capability=list(capability),
                  multi_processor_count=props.multi_processor_count, total_memory_bytes=props.total_memory)
    if capability != ACTIVE_TARGET.compute_capability:
        report["reason"] = f"expected compute capability {ACTIVE_TARGET.compute_capability}, got {capability}"
        return report
    report["ok"] = True
    return report


def require_b200(device_index: int = 0) -> dict[str, Any]:
    report = check_b200(device_index)
    if not report["ok"]:
        raise RuntimeError(f"B200 required: {report.get('reason')}")
    return report


def environment_report(env: dict[str, str] | None = None) -> dict[str, Any]:
    env = dict(os.environ if env is None else env)
    prepare_torch_extension_env(env)
    nvcc = nvcc_path_from_env(env)
    nvcc_cuda, nvcc_error = nvcc_cuda_version(nvcc, env)
    torch_cuda = torch_cuda_version()
    driver = driver_cuda_version()
    ext_status, ext_note = cuda_build_compatibility(torch_cuda, nvcc_cuda)
    lib_status, lib_note = library_build_compatibility(driver, nvcc_cuda)
    return {
        "target": {"name": ACTIVE_TARGET.name, "sm": ACTIVE_TARGET.sm, "gencode": ACTIVE_TARGET.nvcc_gencode},
        "torch_cuda_arch_list": env.get("TORCH_CUDA_ARCH_LIST"),
        "nvcc": nvcc, "nvcc_cuda": nvcc_cuda, "nvcc_error": nvcc_error,
        "torch_cuda": torch_cuda, "driver_cuda": driver,
        "torch_extension_compatibility": {"status": ext_status, "note": ext_note},
        "library_compatibility": {"status": lib_status, "note": lib_note},
        "device": check_b200(0),
    }
