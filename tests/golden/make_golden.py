"""Generate golden attention vectors from the reference's own oracle seed.

Imports ``candidates/torch_sdpa_seed.py`` from the reference checkout (path given by
the required ``--reference`` flag) and runs its ``attention(q, k, v, causal)``
on the CPU for small seeded cases:

* ``o_bf16``  - the seed on the bf16 inputs (what the reference scorer compares with);
* ``o_fp32``  - the seed on the same inputs upcast to fp32 (the parity oracle).

Inputs are stored as bf16 bit patterns (uint16), outputs as bf16 bits / float32, in
``attention_golden.npz`` next to this script, with a JSON manifest of the cases.  The
reference cannot travel to the GPU machine, so tests use only the stored file.

Usage: ``python tests/golden/make_golden.py --reference PATH``
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name: (shape [B, H, S, D], causal, seed, k_scale).  For the B1 H4 S512 cases the
# inputs are stored only as a SHA-256 of their bf16 bytes (tests regenerate them from
# the seed and check the hash) and o_fp32 keeps heads 0-1, to keep the file small.
HASHED_INPUTS = {"b1_h4_s512_noncausal", "b1_h4_s512_causal"}
FP32_HEADS = {"b1_h4_s512_noncausal": 2, "b1_h4_s512_causal": 2}
CASES = {
    "b1_h4_s512_noncausal": ((1, 4, 512, 128), False, 0, 1.0),
    "b1_h4_s512_causal": ((1, 4, 512, 128), True, 0, 1.0),
    "b1_h1_s128_causal": ((1, 1, 128, 128), True, 1, 1.0),
    "b1_h2_s100_causal_ragged": ((1, 2, 100, 128), True, 2, 1.0),
    "b1_h1_s1_causal": ((1, 1, 1, 128), True, 3, 1.0),
    "b1_h1_s256_noncausal_k3": ((1, 1, 256, 128), False, 4, 3.0),
    "b2_h1_s300_noncausal": ((2, 1, 300, 128), False, 5, 1.0),
}


def seeded_inputs(shape, seed, k_scale):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape, generator=g, dtype=torch.float32)
    k = torch.randn(shape, generator=g, dtype=torch.float32)
    v = torch.randn(shape, generator=g, dtype=torch.float32)
    if k_scale != 1.0:
        k = k * k_scale
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", required=True, help="root of the reference checkout")
    args = parser.parse_args()
    seed_path = Path(args.reference) / "candidates" / "torch_sdpa_seed.py"
    spec = importlib.util.spec_from_file_location("reference_torch_sdpa_seed", seed_path)
    seed_module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(seed_module)

    arrays: dict[str, np.ndarray] = {}
    manifest = {"generator": "tests/golden/make_golden.py", "reference_seed": "candidates/torch_sdpa_seed.py",
                "torch": torch.__version__, "cases": {}}
    for name, (shape, causal, seed, k_scale) in CASES.items():
        q, k, v = seeded_inputs(shape, seed, k_scale)
        o_bf16 = seed_module.attention(q, k, v, causal)
        o_fp32 = seed_module.attention(q.float(), k.float(), v.float(), causal)
        entry = {"shape": list(shape), "causal": causal, "seed": seed, "k_scale": k_scale}
        if name in HASHED_INPUTS:
            entry["input_sha256"] = {
                key: hashlib.sha256(bf16_bits(t).tobytes()).hexdigest()
                for key, t in (("q", q), ("k", k), ("v", v))
            }
        else:
            arrays[f"{name}/q"] = bf16_bits(q)
            arrays[f"{name}/k"] = bf16_bits(k)
            arrays[f"{name}/v"] = bf16_bits(v)
        heads = FP32_HEADS.get(name, shape[1])
        entry["o_fp32_heads"] = heads
        arrays[f"{name}/o_bf16"] = bf16_bits(o_bf16)
        arrays[f"{name}/o_fp32"] = o_fp32[:, :heads].contiguous().numpy().astype(np.float32)
        manifest["cases"][name] = entry
    np.savez_compressed(HERE / "attention_golden.npz", **arrays)
    (HERE / "attention_golden.json").write_text(json.dumps(manifest, indent=2) + "\n")
    print(f"wrote {len(CASES)} cases to {HERE / 'attention_golden.npz'}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
