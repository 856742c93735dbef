"""Runtime feature flags (the reference's src/starling/flags.py:51-121 surface).

``multistep_graph`` selects the K-step graphed decoder (default, as in the
reference); ``weight_format`` picks the packed weight format of the native
decoder.  ``batched_encoder`` / ``tolerance_mode`` are kept for API parity: the
encoder is outside this package, so they only carry the reference's
validation rule.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass, replace

from .config import WEIGHT_FORMATS


@dataclass
class OptFlags:
    multistep_graph: bool = True
    batched_encoder: bool = False
    tolerance_mode: bool = False
    weight_format: str = "bf16"
    use_pdl: bool = True

    def __post_init__(self) -> None:
        if self.batched_encoder and not self.tolerance_mode:
            raise ValueError(
                "batched_encoder=True requires tolerance_mode=True (it breaks byte-exactness). "
                "Set tolerance_mode=True or batched_encoder=False."
            )
        if self.weight_format not in WEIGHT_FORMATS:
            raise ValueError(f"weight_format must be one of {WEIGHT_FORMATS}, got {self.weight_format!r}")


_DEFAULT_FLAGS = OptFlags()


def get_default_flags() -> OptFlags:
    return _DEFAULT_FLAGS


def set_default_flags(fl: OptFlags) -> None:
    global _DEFAULT_FLAGS
    _DEFAULT_FLAGS = fl


@contextmanager
def flags(**overrides):
    """Scoped override of the process-global default flags (restored on exit)."""
    global _DEFAULT_FLAGS
    saved = _DEFAULT_FLAGS
    _DEFAULT_FLAGS = replace(saved, **overrides)
    try:
        yield _DEFAULT_FLAGS
    finally:
        _DEFAULT_FLAGS = saved
