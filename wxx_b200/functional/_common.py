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


# ---------------------------------------------------------------- kernel timing

class KernelTimer:
    """Brackets every tensor-core GEMM launch with CUDA events on the library
    stream while active (``with KernelTimer() as t: ...``); ``summary()``
    returns total FLOPs, total device milliseconds and the launch count."""

    def __init__(self):
        self.records = []

    def __enter__(self):
        global _timer
        self._prev = _timer
        _timer = self
        return self

    def __exit__(self, *exc):
        global _timer
        _timer = self._prev

    def start(self):
        from ..backend.device import Event

        return Event().record()

    def stop(self, ev0, flops, label):
        from ..backend.device import Event

        self.records.append((label, flops, ev0, Event().record()))

    def summary(self):
        total_ms = 0.0
        total_flops = 0.0
        per = {}
        for label, flops, e0, e1 in self.records:
            ms = e0.elapsed_ms(e1)
            total_ms += ms
            total_flops += flops
            d = per.setdefault(label, [0, 0.0, 0.0])
            d[0] += 1
            d[1] += ms
            d[2] += flops
        return {"launches": len(self.records), "ms": total_ms, "flops": total_flops,
                "per_shape": per}


_timer = None


def active_timer():
    return _timer
