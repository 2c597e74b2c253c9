"""The kernel's FMA-pipe exp2 (``exp2_poly_x2`` in sm100_ptx.cuh).

CPU: the four coefficients compiled into the header are the fp32 rounding of the
degree-3 relative-minimax fit that ``exp2_poly.py`` derives (Remez exchange), and an
fp32 restatement of the evaluation scheme (Cody-Waite split, Horner, 2^j added to the
exponent bits) stays within the stated relative error bound over the whole input range
the kernel uses.  GPU: the device function itself, through the C ABI, against CUDA's
exp2f (torch.exp2) and against exact 2^x.
"""

from __future__ import annotations

import importlib.util
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
CAND = ROOT / "avo-ampere_b200" / "candidates" / "cuda_b200_attention"
REL_BOUND = 7.5e-5
LO, HI = -125.0, 127.0


def _fit_module():
    spec = importlib.util.spec_from_file_location("avo_b200_exp2_fit", CAND / "exp2_poly.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def header_coefficients() -> list[float]:
    text = (CAND / "sm100_ptx.cuh").read_text()
    body = text[text.index("exp2_poly_x2"):]
    found = {int(m.group(1)): float(m.group(2))
             for m in re.finditer(r"c(\d) = f2_pack\(([-0-9.e]+)f,", body)}
    return [found[i] for i in range(4)]


def test_header_constants_are_the_fitted_polynomial():
    coeffs, bound = _fit_module().float32_coefficients(3)
    header = header_coefficients()
    assert np.array_equal(np.float32(header), np.float32(coeffs)), (header, coeffs)
    assert bound < REL_BOUND


def emulate_fp32(x: np.ndarray) -> np.ndarray:
    """The device evaluation restated in fp32 numpy (FMAs as separate multiply + add,
    which can differ from the fused form by an ulp, far inside the bound)."""
    f32 = np.float32
    x = x.astype(f32)
    t = (x + f32(12582912.0)).astype(f32)           # 1.5 * 2^23 + round(x)
    j = (t - f32(12582912.0)).astype(f32)
    f = (x - j).astype(f32)
    c3, c2, c1, c0 = (f32(c) for c in reversed(header_coefficients()))
    p = (c3 * f + c2).astype(f32)
    p = (p * f + c1).astype(f32)
    p = (p * f + c0).astype(f32)
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def test_fp32_restatement_meets_the_bound():
    x = np.concatenate([np.linspace(LO, HI, 2_000_001, dtype=np.float64),
                        np.arange(-125, 128, dtype=np.float64),          # integers: f = 0
                        np.arange(-125, 127, dtype=np.float64) + 0.5])   # rounding ties
    x = x.astype(np.float32)
    y = emulate_fp32(x).astype(np.float64)
    exact = np.exp2(x.astype(np.float64))
    rel = np.abs(y / exact - 1.0)
    assert rel.max() < REL_BOUND, rel.max()
    # 2^j scaling is exact: shifting x by an integer scales the result by exactly 2^n
    # (base values on a 1/64 grid, so that base + n is exact in fp32 as well).
    base = (np.arange(-192, 193) / 64.0).astype(np.float32)
    for n in (-100, -7, 0, 5, 90):
        shifted = emulate_fp32(base + np.float32(n))
        assert np.array_equal(shifted, emulate_fp32(base) * np.float32(2.0) ** n)


@pytest.mark.gpu
def test_device_exp2_poly_against_cuda_exp2f(b200):
    import torch

    x = torch.linspace(LO, HI, 4_000_001, dtype=torch.float64)
    x = torch.cat([x, torch.arange(-125, 128, dtype=torch.float64),
                   torch.arange(-125, 127, dtype=torch.float64) + 0.5]).float().cuda()
    y = b200.exp2_poly_eval(x)
    ref = torch.exp2(x)  # CUDA exp2f
    torch.cuda.synchronize()
    rel_cuda = ((y.double() / ref.double()) - 1.0).abs().max().item()
    rel_exact = ((y.double() / torch.exp2(x.double())) - 1.0).abs().max().item()
    assert rel_cuda < REL_BOUND, rel_cuda
    assert rel_exact < REL_BOUND, rel_exact
    # exact 2^n scaling on the device too (1/64 grid: base + n exact in fp32)
    base = (torch.arange(-192, 193, dtype=torch.float32) / 64.0).cuda()
    for n in (-100, -7, 5, 90):
        assert torch.equal(b200.exp2_poly_eval(base + n), b200.exp2_poly_eval(base) * (2.0 ** n))
    # and the device agrees with the fp32 restatement to an ulp or so
    host = emulate_fp32(x.cpu().numpy())
    rel_host = np.abs(y.cpu().numpy().astype(np.float64) / host.astype(np.float64) - 1.0).max()
    assert rel_host < 1e-6, rel_host
