"""Reductions (reference: src/wxx/functional/reductions.py)."""

from ..backend.dispatch import _get_reduce_dims, keepdims_shape
from ._common import F, check, dense, empty
from .pointwise import _training_only


def _reduce(tensor1, axis, keepdims, mode):
    x = dense(tensor1)
    outer, red, inner, out_shape = _get_reduce_dims(x.shape, axis)
    if keepdims:
        out_shape = keepdims_shape(x.shape, axis)
    out = empty(out_shape, "f32")
    check(F.wxx_reduce(out.buffer.ptr, x.ptr, outer, red, inner, mode), "reduce")
    return out


def sum(tensor1, axis=None, keepdims=False, *, keepdim=None):
    """Sum over one run of adjacent axes (or everything for ``axis=None``)."""
    return _reduce(tensor1, axis, keepdims if keepdim is None else keepdim, 0)


def mean(tensor1, axis=None, keepdims=False, *, keepdim=None):
    return _reduce(tensor1, axis, keepdims if keepdim is None else keepdim, 1)


def sumsq(tensor1, axis=None, keepdims=False, *, keepdim=None):
    return _reduce(tensor1, axis, keepdims if keepdim is None else keepdim, 2)


def _minmax(tensor1, axis, keepdims, op):
    """Values and u32 indices with the reference's tie rule (reduce_minmax.wgsl)."""
    x = dense(tensor1)
    outer, red, inner, out_shape = _get_reduce_dims(x.shape, axis)
    if keepdims:
        out_shape = keepdims_shape(x.shape, axis)
    vals = empty(out_shape, "f32")
    idx = empty(out_shape, "u32")
    check(F.wxx_argminmax(vals.buffer.ptr, idx.buffer.ptr, x.ptr, outer, red, inner, op),
          "max/min")
    return vals, idx


def max(tensor1, axis=None, keepdims=False, *, keepdim=None):
    return _minmax(tensor1, axis, keepdims if keepdim is None else keepdim, 0)


def min(tensor1, axis=None, keepdims=False, *, keepdim=None):
    return _minmax(tensor1, axis, keepdims if keepdim is None else keepdim, 1)


def var(tensor1, axis=None, keepdims=False, *, keepdim=None):
    """Population variance (ddof=0), composed as in the reference."""
    from .pointwise import pointwise

    if keepdim is not None:
        keepdims = keepdim
    if tensor1.type != "f32":
        raise TypeError(f"var expects an f32 tensor, got {tensor1.type!r}")
    m = mean(tensor1, axis, keepdims=True)
    diff = pointwise(tensor1, m, 1)
    return mean(pointwise(diff, diff, 2), axis, keepdims)


def std(tensor1, axis=None, keepdims=False, *, keepdim=None):
    from .pointwise import sqrt

    if keepdim is not None:
        keepdims = keepdim
    return sqrt(var(tensor1, axis=axis, keepdims=keepdims))


maxmin_backward = _training_only("maxmin_backward")
