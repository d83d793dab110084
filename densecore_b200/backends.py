"""Precision switch of the SDPA kernels.

DenseCore exposes ``densecore.backends.cuda.matmul.allow_tf32`` as a stub that stays False
(python/densecore/_compat.py:220-222). Here it is honoured: False (the default) runs the
tensor-core kernels in the 3xTF32 split, which keeps fp32-class accuracy; True opts into
single-pass TF32. ``set_sdpa_precision("fp32")`` forces the CUDA-core fp32 kernels.
"""
from __future__ import annotations

from types import SimpleNamespace

cuda = SimpleNamespace(matmul=SimpleNamespace(allow_tf32=False))

_FORCED = None
_NAMES = {"3xtf32": 0, "tf32": 1, "fp32": 2}


def set_sdpa_precision(mode: str | None) -> None:
    """Force "3xtf32", "tf32" or "fp32"; None returns to following ``allow_tf32``."""
    global _FORCED
    if mode is not None and mode not in _NAMES:
        raise ValueError(f"precision must be one of {sorted(_NAMES)} or None")
    _FORCED = mode


def precision_code() -> int:
    if _FORCED is not None:
        return _NAMES[_FORCED]
    return 1 if cuda.matmul.allow_tf32 else 0


def precision_name() -> str:
    return {v: k for k, v in _NAMES.items()}[precision_code()]
