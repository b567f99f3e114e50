"""Helpers shared by the functional modules: output allocation, pointer and
stride marshalling, the global matmul precision mode and the host RNG."""

import ctypes
import os

import numpy as np

from .. import validation
from ..Tensor import Tensor
from ..backend.lib import F, check

i64 = ctypes.c_int64


def arr64(values):
    values = list(values)
    return (i64 * max(1, len(values)))(*values)


def empty(shape, dtype="f32", requires_grad=False):
    return Tensor._empty(list(shape), dtype, requires_grad)


def dense(t):
    """``t`` itself when its layout is compact row-major (any offset), else a
    dense copy.  Kernels take the view's base address, so dense views with an
    offset need no copy."""
    if t.is_dense():
        return t
    from .utils import contiguous

    return contiguous(t)


def ptr_or_none(t):
    return None if t is None else t.ptr


# ---------------------------------------------------------------- matmul mode

_MODES = {"tf32": 0, "3xtf32": 1, "fp32": 2}
_matmul_mode = _MODES.get(os.environ.get("WXX_MATMUL_MODE", "tf32").lower(), 0)


def set_matmul_mode(mode):
    """Selects the contraction arithmetic for matmul and conv2d:
    ``"tf32"`` (default, TF32 tensor cores), ``"3xtf32"`` (split-operand TF32,
    fp32-faithful) or ``"fp32"`` (fp32 FMA; conv2d maps it to 3xtf32)."""
    global _matmul_mode
    key = str(mode).lower()
    if key not in _MODES:
        raise ValueError(f"matmul mode must be one of {sorted(_MODES)}, got {mode!r}")
    _matmul_mode = _MODES[key]


def get_matmul_mode():
    return {v: k for k, v in _MODES.items()}[_matmul_mode]


def matmul_mode_code():
    return _matmul_mode


# ---------------------------------------------------------------- host RNG

_rng = None


def manual_seed(seed):
    """Seeds the host generator used by ``normal`` / ``uniform`` and module
    initialisation.  The reference draws from an unseeded
    ``np.random.default_rng()`` on every call (functional/utils.py:644-666);
    without ``manual_seed`` the same happens here."""
    global _rng
    _rng = None if seed is None else np.random.default_rng(seed)


def rng():
    return _rng if _rng is not None else np.random.default_rng()


__all__ = [
    "arr64",
    "check",
    "dense",
    "empty",
    "F",
    "get_matmul_mode",
    "manual_seed",
    "matmul_mode_code",
    "ptr_or_none",
    "rng",
    "set_matmul_mode",
    "Tensor",
    "validation",
]
