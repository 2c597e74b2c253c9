"""Host-side mirror of the reference package ``avo`` (coder-2011/avo-ampere) for the
attention-forward hot path: cases and targets, toolchain environment, compile helper,
process isolation, the scorer, and the multi-GPU harness, retargeted to B200."""

__all__ = ["__version__"]
__version__ = "0.1.0"
