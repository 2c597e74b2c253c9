"""CUDA toolchain environment and the B200 hardware check.

Serves the same callers as the reference's ``avo/cuda_env.py`` (the CLI's ``env`` report
and the environment handed to build workers), retargeted to the B200:

* the torch-extension arch list is ``10.0a`` (the reference pins ``8.6``);
* ``check_b200`` / ``require_b200`` replace the scorer's sm_86 assertion with a check
  for compute capability 10.0;
* the toolkit probe reports nvcc's path and release in one record, and two rules say
  whether a build can work: a torch extension wants nvcc's major version to match
  torch's CUDA, while the candidate's C-ABI library links the CUDA runtime statically
  and only needs a driver at least as new as the nvcc that built it.
"""

from __future__ import annotations

import os
import re
import shutil
import subprocess
from collections.abc import MutableMapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from .config import ACTIVE_TARGET

DEFAULT_CUDA_HOME = "/usr/local/cuda"
_VERSION_RE = re.compile(r"(\d+)\.(\d+)")


def prepare_torch_extension_env(env: MutableMapping[str, str] | None = None, *,
                                max_jobs: str = "2") -> MutableMapping[str, str]:
    """Fill in the build variables a worker needs, keeping any the caller set."""
    target = os.environ if env is None else env
    defaults = {"TORCH_CUDA_ARCH_LIST": ACTIVE_TARGET.torch_arch_list, "MAX_JOBS": max_jobs}
    if Path(DEFAULT_CUDA_HOME, "bin", "nvcc").exists():
        defaults["CUDA_HOME"] = DEFAULT_CUDA_HOME
    for key, value in defaults.items():
        if key not in target:
            target[key] = value
    return target


def version_tuple(text: str | None) -> tuple[int, int] | None:
    """(major, minor) of the first ``X.Y`` in ``text``."""
    if not text:
        return None
    found = _VERSION_RE.search(text)
    return (int(found.group(1)), int(found.group(2))) if found else None


@dataclass(frozen=True)
class NvccProbe:
    path: str | None
    release: str | None  # "12.9"
    error: str | None


def find_nvcc(env: MutableMapping[str, str]) -> str | None:
    """nvcc under CUDA_HOME (or CUDA_PATH) if either is set, else the first on PATH."""
    for key in ("CUDA_HOME", "CUDA_PATH"):
        if env.get(key):
            return os.path.join(env[key], "bin", "nvcc")
    return shutil.which("nvcc", path=env.get("PATH"))


def probe_nvcc(env: MutableMapping[str, str]) -> NvccProbe:
    """Run ``nvcc --version`` and read its ``release X.Y``."""
    path = find_nvcc(env)
    if path is None:
        return NvccProbe(None, None, "no nvcc under CUDA_HOME/CUDA_PATH or on PATH")
    try:
        proc = subprocess.run([path, "--version"], capture_output=True, text=True, env=dict(env),
                              timeout=10)
    except (OSError, subprocess.TimeoutExpired) as exc:
        return NvccProbe(path, None, f"{path} --version: {type(exc).__name__}: {exc}")
    text = proc.stdout + "\n" + proc.stderr
    if proc.returncode != 0:
        return NvccProbe(path, None, f"{path} --version exited {proc.returncode}: {text.strip()[:200]}")
    release = re.search(r"release\s+(\d+\.\d+)", text)
    if release is None:
        return NvccProbe(path, None, f"no 'release X.Y' in the output of {path} --version")
    return NvccProbe(path, release.group(1), None)


def torch_cuda_version() -> str | None:
    try:
        import torch
    except ImportError:
        return None
    return torch.version.cuda


def torch_extension_compatibility(torch_cuda: str | None, nvcc_cuda: str | None) -> tuple[str, str | None]:
    """Whether a torch C++/CUDA extension builds with this nvcc: "exact", "minor_mismatch"
    (builds, may warn), "major_mismatch" (fails), or "unknown" with the reason."""
    tv, nv = version_tuple(torch_cuda), version_tuple(nvcc_cuda)
    if tv is None or nv is None:
        return "unknown", f"torch CUDA {torch_cuda!r}, nvcc CUDA {nvcc_cuda!r}"
    if tv == nv:
        return "exact", None
    note = f"nvcc CUDA {nvcc_cuda} vs torch CUDA {torch_cuda}"
    return ("minor_mismatch", note) if tv[0] == nv[0] else ("major_mismatch", note)


def library_build_compatibility(driver_cuda: str | None, nvcc_cuda: str | None) -> tuple[str, str | None]:
    """The C-ABI library links cudart statically: the driver must support nvcc's CUDA."""
    dv, nv = version_tuple(driver_cuda), version_tuple(nvcc_cuda)
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
    probe = probe_nvcc(env)
    nvcc, nvcc_cuda, nvcc_error = probe.path, probe.release, probe.error
    torch_cuda = torch_cuda_version()
    driver = driver_cuda_version()
    ext_status, ext_note = torch_extension_compatibility(torch_cuda, nvcc_cuda)
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
