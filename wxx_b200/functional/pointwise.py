"""Elementwise binary / scalar / unary ops (reference: src/wxx/functional/pointwise.py)."""

import numpy as np

from .. import validation
from ..Tensor import Tensor
from ..backend.dispatch import broadcast_shapes, supports_strided, view_broadcast_strides
from ._common import F, arr64, check, dense, empty

_UNARY = {
    "relu": 0, "gelu": 1, "sigmoid": 2, "sin": 3, "cos": 4, "exp": 5, "log": 6, "sqrt": 7,
    "rsqrt": 8, "abs": 9, "sign": 10, "negate": 11, "square": 12, "silu": 13, "selu": 14,
}


def unary(tensor1, name):
    """Runs the unary kernel ``name`` over a dense copy of ``tensor1``
    (backend/dispatch.py:59-89 _unary_op)."""
    validation.check_rank(tensor1.shape, max_rank=8, name="unary op input")
    x = dense(tensor1)
    out = empty(x.shape, "f32", tensor1.requires_grad)
    check(F.wxx_unary(out.buffer.ptr, x.ptr, validation.numel(x.shape), _UNARY[name]), name)
    return out


def pointwise(tensor1, tensor2, op):
    """Broadcasting ``A op B`` (0 add, 1 sub, 2 mul, 3 div) over strided views
    (functional/pointwise.py:29-98); a scalar ``tensor2`` uses scalarpointwise."""
    if not isinstance(tensor2, Tensor):
        return scalarpointwise(tensor1, tensor2, op)
    if not supports_strided(tensor1):
        tensor1 = tensor1.contiguous()
    if not supports_strided(tensor2):
        tensor2 = tensor2.contiguous()
    if tensor1.type != "f32" or tensor2.type != "f32":
        raise TypeError(
            f"pointwise expects f32 tensors, got {tensor1.type!r} and {tensor2.type!r}"
        )
    out_shape, _, _ = broadcast_shapes(tensor1.shape, tensor2.shape)
    rank = validation.check_rank(out_shape, name="pointwise output")
    sa = view_broadcast_strides(tensor1, out_shape)
    sb = view_broadcast_strides(tensor2, out_shape)
    out = empty(out_shape, "f32", tensor1.requires_grad or tensor2.requires_grad)
    if validation.numel(out_shape):
        check(F.wxx_binary(out.buffer.ptr, tensor1.buffer.ptr, tensor1.offset, arr64(sa),
                           tensor2.buffer.ptr, tensor2.offset, arr64(sb), rank, arr64(out_shape),
                           int(op)), "pointwise")
    return out


def _pointwise(tensor1, tensor2, op):
    """In-place ``A op= B`` with B broadcast to A (functional/pointwise.py:232-291)."""
    a = tensor1 if tensor1.is_dense() else None
    if a is None:
        raise ValueError("_pointwise accumulates into a dense tensor")
    if tensor1.type != "f32" or tensor2.type != "f32":
        raise TypeError(
            f"_pointwise expects f32 tensors, got {tensor1.type!r} and {tensor2.type!r}"
        )
    out_shape, _, _ = broadcast_shapes(tensor1.shape, tensor2.shape)
    if tuple(out_shape) != tuple(tensor1.shape):
        raise ValueError(f"_pointwise cannot broadcast {tensor2.shape} into {tensor1.shape}")
    rank = len(out_shape)
    sa = validation.contiguous_strides(out_shape)
    sb = view_broadcast_strides(tensor2, out_shape)
    if validation.numel(out_shape):
        check(F.wxx_binary(tensor1.ptr, tensor1.ptr, 0, arr64(sa), tensor2.buffer.ptr,
                           tensor2.offset, arr64(sb), rank, arr64(out_shape), int(op)),
              "_pointwise")
    buf = tensor1.buffer
    if hasattr(buf, "version"):
        buf.version += 1      # in-place write: cached weight copies are rebuilt
    return tensor1


def scalarpointwise(tensor1, value, op, reverse=0):
    """``X op value`` (or ``value op X``): op 0 add, 1 sub, 2 mul, 3 pow, 4 div."""
    if tensor1.type != "f32":
        raise TypeError(f"scalarpointwise expects f32 input, got {tensor1.type!r}")
    x = dense(tensor1)
    out = empty(x.shape, "f32", tensor1.requires_grad)
    check(F.wxx_scalar(out.buffer.ptr, x.ptr, validation.numel(x.shape), int(op), float(value),
                       int(bool(reverse))), "scalarpointwise")
    return out


def clamp(tensor1, min, max):
    x = dense(tensor1)
    out = empty(x.shape, "f32", tensor1.requires_grad)
    check(F.wxx_clamp(out.buffer.ptr, x.ptr, validation.numel(x.shape), float(min), float(max)),
          "clamp")
    return out


def negate(tensor1):
    return unary(tensor1, "negate")


def abs(tensor1):
    return unary(tensor1, "abs")


def sign(tensor1):
    return unary(tensor1, "sign")


def square(tensor1):
    return unary(tensor1, "square")


def exp(tensor1):
    return unary(tensor1, "exp")


def sqrt(tensor1):
    return unary(tensor1, "sqrt")


def rsqrt(tensor1):
    return unary(tensor1, "rsqrt")


def log(tensor1):
    return unary(tensor1, "log")


def decay_window(decay, stage, length):
    """``exp(-|decay[stage, d]| * t)`` as a ``(channels, length)`` tensor
    (functional/pointwise.py:357-404)."""
    if decay.type != "f32":
        raise TypeError(f"decay_window expects f32 decay, got {decay.type!r}")
    if len(decay.shape) != 2:
        raise ValueError(f"decay_window expects a 2-D decay, got {decay.shape}")
    rows, channels = decay.shape
    if not isinstance(length, int) or length < 1:
        raise ValueError(f"decay_window length must be a positive int, got {length!r}")
    if not (0 <= stage < rows):
        raise IndexError(f"decay_window stage {stage} out of range for {rows} rows")
    d = dense(decay)
    out = empty((channels, length), "f32", decay.requires_grad)
    check(F.wxx_decay_window(out.buffer.ptr, d.ptr, rows, channels, length, stage),
          "decay_window")
    return out


def hyena_filters(pe, linears1, linears2, omega, decay):
    """All ``n`` implicit filters of a Hyena operator (nn/hyena.py:127-130 and
    :236-239) in one exact-fp32 kernel: filter i is ``(sin(omega * (pe @ W1_i
    + b1_i)) @ W2_i + b2_i)^T * decay_window(decay, i, L)``, returned as an
    (n, D, L) tensor.  ``linears1[i]`` / ``linears2[i]`` are ``(weight,
    bias)`` pairs with weights (F, H) and (H, D).  None when the shapes are
    outside the kernel's limits (n <= 8, F <= 32, H <= 64 and a multiple of 4);
    the caller then composes the separate ops."""
    import ctypes

    L, Fdim = pe.shape
    n = len(linears1)
    if n == 0 or len(linears2) != n or tuple(decay.shape)[0] < n:
        return None
    H = linears1[0][0].shape[1]
    D = linears2[0][0].shape[1]
    if n > 8 or Fdim > 32 or H > 64 or H % 4:
        return None
    for (w1, b1), (w2, b2) in zip(linears1, linears2):
        if (tuple(w1.shape) != (Fdim, H) or b1 is None or tuple(b1.shape) != (H,)
                or tuple(w2.shape) != (H, D) or b2 is None or tuple(b2.shape) != (D,)):
            return None
    if tuple(decay.shape)[1] != D:
        return None
    keep = [dense(t) for pair in list(linears1) + list(linears2) for t in pair]
    ptrs = [t.ptr for t in keep]
    arr = ctypes.c_void_p * n
    w1p = arr(*ptrs[0:2 * n:2])
    b1p = arr(*ptrs[1:2 * n:2])
    w2p = arr(*ptrs[2 * n::2])
    b2p = arr(*ptrs[2 * n + 1::2])
    pd = dense(pe)
    dd = dense(decay)
    out = empty((n, D, L), "f32", False)
    st = F.wxx_hyena_filters(out.buffer.ptr, pd.ptr, L, Fdim, H, D, n, w1p, b1p, w2p, b2p,
                             float(omega), dd.ptr)
    if st != 0:
        check(st, "hyena_filters")
    return out


def _training_only(name):
    def fn(*args, **kwargs):
        raise NotImplementedError(f"{name} is a training kernel; not part of this backend")

    fn.__name__ = name
    return fn


clampbackwards = _training_only("clampbackwards")
decay_window_backward = _training_only("decay_window_backward")
mul_backward = _training_only("mul_backward")

_np = np
