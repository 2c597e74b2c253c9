"""The attention kernel's own watchdog path: a wait that runs out ends in a reported abort.

A child process sets AVO_B200_TEST_SKIP_LOAD=5, so every CTA's producer never issues its
sixth K/V copy (V_2 of its first work item), and a 20 ms watchdog (both read once per
process).  A second child skips copy 11 (V_1 of the second item) of a problem with about
four items per CTA, so the abort comes in the middle of a CTA's item sequence and the
remaining items run the dry schedule.  The wait for
that copy runs out, the CTA aborts, and every role must leave its pipeline cleanly:
softmax warps keep their place in the MMA warp's named-barrier schedule, the producer
drains the copies it did issue, the MMA warp drains its MMAs.  The launch must return,
set the watchdog bit (never the drain bit), and leave the CUDA context usable.  Nothing
faults, traps or hangs: a copy that is never issued only makes a bounded wait give up.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
BINDING = ROOT / "avo-ampere_b200" / "candidates" / "cuda_b200_attention" / "b200_attention.py"

CHILD = r"""
import importlib.util, sys, torch
spec = importlib.util.spec_from_file_location("avo_b200_attention_binding", sys.argv[1])
b = importlib.util.module_from_spec(spec)
sys.modules[spec.name] = b
spec.loader.exec_module(b)
b.load_library()
g = torch.Generator().manual_seed(0)
shape = tuple(int(x) for x in sys.argv[2].split(","))
q, k, v = (torch.randn(shape, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
for causal in (False, True, False):
    out, lse = b.attention_forward(q, k, v, causal)
    torch.cuda.synchronize()
    word = b.status_word(q.device)
    print("STATUS", int(word.item()), flush=True)
    word.zero_()
# the context is still usable after the aborted launches
print("SUM", float((q.float() * 2).sum().item()), flush=True)
print("DONE", flush=True)
"""


@pytest.mark.parametrize(
    "shape,skip",
    [
        ("1,2,4096,128", 5),   # 32 items, at most one per CTA: abort in the first item
        ("1,300,512,128", 11),  # 600 items of 4 tiles: abort in each CTA's second item
    ],
)
def test_watchdog_abort_returns_and_reports(shape, skip):
    env = dict(os.environ)
    env["AVO_B200_TEST_SKIP_LOAD"] = str(skip)
    env["AVO_B200_WATCHDOG_MS"] = "20"
    proc = subprocess.run([sys.executable, "-c", CHILD, str(BINDING), shape], env=env, capture_output=True,
                          text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-2000:]
    lines = proc.stdout.splitlines()
    assert "DONE" in lines, proc.stdout
    statuses = [int(line.split()[1]) for line in lines if line.startswith("STATUS")]
    assert len(statuses) == 3
    watchdog_bit, drain_bit = 1, 2
    assert all(s & watchdog_bit for s in statuses), statuses
    assert not any(s & drain_bit for s in statuses), statuses
