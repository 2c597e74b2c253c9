"""Attention cases and GPU targets.

Mirrors the reference's ``avo/config.py`` (``AttentionCase`` :9-39, ``DEFAULT_CASES``
:42-47, ``AmpereTarget`` :50-68, ``cases_from_cli`` :71-101) with the same field names,
defaults and error messages, retargeted to the B200:

* ``GpuTarget`` generalises ``AmpereTarget``; ``B200`` (compute capability 10.0,
  arch-specific ``sm_100a``) is the active target, ``AMPERE_A6000`` is kept for
  comparison only.
* ``AttentionCase`` gains two optional fields, ``k_scale`` (k *= k_scale before the
  bf16 cast, the softmax max-rescale stress case) and ``gpus`` (head-sharded launch
  width).  They appear in ``as_dict()`` only when not at their defaults, so default
  cases keep the reference's lineage signature.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

MaskMode = Literal["causal", "noncausal"]


@dataclass(frozen=True)
class AttentionCase:
    seq_len: int
    causal: bool
    head_dim: int = 128
    num_heads: int = 16
    total_tokens: int = 32768
    dtype: str = "bf16"
    k_scale: float = 1.0
    gpus: int = 1

    @property
    def batch_size(self) -> int:
        if self.total_tokens % self.seq_len != 0:
            msg = f"total_tokens={self.total_tokens} must be divisible by seq_len={self.seq_len}"
            raise ValueError(msg)
        return self.total_tokens // self.seq_len

    @property
    def mask_mode(self) -> MaskMode:
        return "causal" if self.causal else "noncausal"

    @property
    def shape(self) -> tuple[int, int, int, int]:
        return (self.batch_size, self.num_heads, self.seq_len, self.head_dim)

    def as_dict(self) -> dict[str, int | bool | str | float]:
        payload: dict[str, int | bool | str | float] = {
            "seq_len": self.seq_len,
            "causal": self.causal,
            "mask_mode": self.mask_mode,
            "head_dim": self.head_dim,
            "num_heads": self.num_heads,
            "total_tokens": self.total_tokens,
            "batch_size": self.batch_size,
            "dtype": self.dtype,
        }
        if self.k_scale != 1.0:
            payload["k_scale"] = self.k_scale
        if self.gpus != 1:
            payload["gpus"] = self.gpus
        return payload


DEFAULT_SEQUENCE_LENGTHS = (4096, 8192, 16384, 32768)
DEFAULT_CASES = tuple(
    AttentionCase(seq_len=seq_len, causal=causal)
    for seq_len in DEFAULT_SEQUENCE_LENGTHS
    for causal in (False, True)
)


@dataclass(frozen=True)
class GpuTarget:
    name: str
    compute_capability: tuple[int, int]
    arch_suffix: str = ""

    @property
    def compute(self) -> str:
        major, minor = self.compute_capability
        return f"compute_{major}{minor}{self.arch_suffix}"

    @property
    def sm(self) -> str:
        major, minor = self.compute_capability
        return f"sm_{major}{minor}{self.arch_suffix}"

    @property
    def nvcc_gencode(self) -> str:
        return f"-gencode=arch={self.compute},code={self.sm}"

    @property
    def torch_arch_list(self) -> str:
        major, minor = self.compute_capability
        return f"{major}.{minor}{self.arch_suffix}"


B200 = GpuTarget(name="NVIDIA B200", compute_capability=(10, 0), arch_suffix="a")
AMPERE_A6000 = GpuTarget(name="NVIDIA RTX A6000", compute_capability=(8, 6))
ACTIVE_TARGET = B200

# The measured workloads of this hot path (all D=128, bf16, scale 1/sqrt(128)).
NAMED_CASES: dict[str, AttentionCase] = {
    # CPU-runnable correctness case: B1 H4 S512 non-causal.
    "b1_h4_s512_noncausal": AttentionCase(seq_len=512, causal=False, num_heads=4, total_tokens=512),
    # B4 H16 S4096 non-causal.
    "b4_h16_s4096_noncausal": AttentionCase(seq_len=4096, causal=False, total_tokens=16384),
    # B2 H16 S8192 causal (O and LSE).
    "b2_h16_s8192_causal": AttentionCase(seq_len=8192, causal=True, total_tokens=16384),
    # B1 H16 S16384 non-causal with k*3.
    "b1_h16_s16384_noncausal_k3": AttentionCase(
        seq_len=16384, causal=False, total_tokens=16384, k_scale=3.0
    ),
    # B1 H16 S32768 causal (head-sharded or context-parallel ring).
    "b1_h16_s32768_causal": AttentionCase(seq_len=32768, causal=True, total_tokens=32768),
    # Throughput target point: B4 H16 S8192 non-causal.
    "b4_h16_s8192_noncausal": AttentionCase(seq_len=8192, causal=False, total_tokens=32768),
    # One GPU's head shard of the target point at 8 GPUs (8 of its 64 pairs).
    "b1_h8_s8192_noncausal": AttentionCase(seq_len=8192, causal=False, num_heads=8, total_tokens=8192),
}


def cases_from_cli(
    seq_lens: str,
    causal: str,
    *,
    head_dim: int = 128,
    num_heads: int = 16,
    total_tokens: int = 32768,
    dtype: str = "bf16",
    k_scale: float = 1.0,
    gpus: int = 1,
) -> list[AttentionCase]:
    lengths = [int(part) for part in seq_lens.split(",") if part.strip()]
    if not lengths:
        raise ValueError("at least one sequence length is required")
    causal_values = {
        "true": [True],
        "false": [False],
        "both": [False, True],
    }.get(causal)
    if causal_values is None:
        raise ValueError("causal must be one of: true, false, both")
    if gpus < 1:
        raise ValueError("gpus must be >= 1")
    return [
        AttentionCase(
            seq_len=seq_len,
            causal=is_causal,
            head_dim=head_dim,
            num_heads=num_heads,
            total_tokens=total_tokens,
            dtype=dtype,
            k_scale=k_scale,
            gpus=gpus,
        )
        for seq_len in lengths
        for is_causal in causal_values
    ]
