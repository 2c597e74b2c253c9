"""attention() captured in a CUDA graph and replayed (B200).

A server replays a captured forward with new inputs copied into the captured tensors.
Each case first asserts, through the host-side plan enumeration, which launch plan the
sizes select: the whole-item wave plan (launched with programmatic dependent launch
allowed), the causal table plan (its item lists in the kernel's parameter block) and the
split plan (a cooperative launch).  Two replays with fresh inputs must equal direct calls
on the same inputs bit for bit: the graph holds the same kernel and parameters.
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # (shape, causal, plan mode: 0 waves, 1 split tail, 2 causal table)
    ((1, 4, 512, 128), False, 0),
    ((1, 20, 4096, 128), True, 2),
    ((1, 2, 4096, 128), False, 1),
]


def _seed():
    path = Path(__file__).resolve().parents[1] / "avo-ampere_b200" / "candidates" / "cuda_b200_attention_seed.py"
    spec = importlib.util.spec_from_file_location("avo_candidate_b200_seed_graph", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


@pytest.mark.parametrize("shape,causal,mode", CASES)
def test_captured_forward_replays_like_direct_calls(b200, shape, causal, mode):
    import torch

    seed = _seed()
    assert b200.schedule_units(shape[0] * shape[1], shape[2], shape[2], causal, split=True,
                               sm_count=torch.cuda.get_device_properties(0).multi_processor_count)[0] == mode
    gen = torch.Generator(device="cuda").manual_seed(17)
    sq, sk, sv = (torch.randn(shape, device="cuda", generator=gen).bfloat16() for _ in range(3))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up off the capture: the workspace and status word exist
        for _ in range(3):
            seed.attention(sq, sk, sv, causal)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured_out = seed.attention(sq, sk, sv, causal)
    try:
        for _ in range(2):
            nq, nk, nv = (torch.randn(shape, device="cuda", generator=gen).bfloat16() for _ in range(3))
            sq.copy_(nq)
            sk.copy_(nk)
            sv.copy_(nv)
            graph.replay()
            direct = seed.attention(nq, nk, nv, causal)
            torch.cuda.synchronize()
            b200.check_status(sq.device)
            assert torch.equal(captured_out, direct)
    finally:
        del graph
