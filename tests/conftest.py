"""Shared pytest configuration.

``-m gpu`` tests need a B200 and call the CUDA path through the C ABI; everything
else runs on the CPU.  The package directory ``avo-ampere_b200`` (not importable by
name because of the hyphen) is put on ``sys.path`` so tests import ``avo`` and the
candidate modules the way the reference's own tests do (``pythonpath=["."]``).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "avo-ampere_b200"
for path in (str(ROOT), str(PKG)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (run with -m gpu)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def b200():
    """The ctypes binding, loaded once; skips nothing - a GPU test without a B200 fails."""
    import importlib.util

    name = "avo_b200_attention_binding"
    module = sys.modules.get(name)
    if module is None:
        spec = importlib.util.spec_from_file_location(
            name, PKG / "candidates" / "cuda_b200_attention" / "b200_attention.py"
        )
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
    module.load_library()
    return module
