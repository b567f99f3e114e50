"""Shape bookkeeping shared by the functional ops.

Reference: src/wxx/backend/dispatch.py.  The reference's launch helpers
(_dispatch_1d, _dispatch_tiled_rows, _unary_op) are replaced by the kernel
library's own launch logic; the broadcast and reduction shape rules are kept
with the same results and errors.
"""

from .. import validation


def broadcast_shapes(shape_a, shape_b):
    """NumPy broadcasting; returns (out_shape, padded_a, padded_b)."""
    a = validation.normalize_shape(shape_a, name="shape_a")
    b = validation.normalize_shape(shape_b, name="shape_b")
    validation.check_rank(a, name="shape_a")
    validation.check_rank(b, name="shape_b")
    r = max(len(a), len(b))
    pa = (1,) * (r - len(a)) + a
    pb = (1,) * (r - len(b)) + b
    out = []
    for x, y in zip(pa, pb):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise ValueError(f"cannot broadcast shapes {tuple(a)} and {tuple(b)}")
    return tuple(out), pa, pb


def compute_broadcast_strides(padded_shape, out_shape):
    if len(padded_shape) != len(out_shape):
        raise ValueError(
            f"padded shape {tuple(padded_shape)} and output shape {tuple(out_shape)} "
            "must have the same rank"
        )
    strides = [0] * len(out_shape)
    acc = 1
    for i in range(len(out_shape) - 1, -1, -1):
        strides[i] = 0 if padded_shape[i] == 1 else acc
        acc *= padded_shape[i]
    return tuple(strides)


def view_broadcast_strides(tensor, out_shape):
    """Element strides that map ``out_shape`` onto a (possibly strided) view."""
    validation.check_broadcastable(tensor.shape, out_shape, name="pointwise operand")
    lead = len(out_shape) - len(tensor.shape)
    strides = []
    for i in range(len(out_shape)):
        j = i - lead
        strides.append(0 if j < 0 or tensor.shape[j] == 1 else tensor.stride[j])
    return tuple(strides)


def supports_strided(tensor):
    return len(tensor.shape) <= validation.MAX_RANK and all(s >= 0 for s in tensor.stride)


def _get_reduce_dims(shape, axis=None):
    """(outer, reduce, inner, out_shape) for a reduction over one run of axes."""
    shape = validation.normalize_shape(shape, name="reduction input")
    nd = len(shape)
    if nd == 0:
        raise ValueError("cannot reduce a 0-d tensor")
    if axis is None:
        return 1, validation.numel(shape), 1, (1,)
    axes = tuple(sorted(validation.normalize_dims(axis, nd, name="axis", allow_duplicates=False)))
    if not axes:
        raise ValueError("axis must contain at least one dimension")
    if any(axes[i] != axes[i - 1] + 1 for i in range(1, len(axes))):
        raise ValueError(
            f"non-contiguous multi-axis reduction {axes} on shape {shape} "
            "requires permuting the tensor first"
        )
    lo, hi = axes[0], axes[-1]
    outer = validation.numel(shape[:lo])
    red = validation.numel(shape[lo:hi + 1])
    inner = validation.numel(shape[hi + 1:])
    out_shape = tuple(s for d, s in enumerate(shape) if d not in axes) or (1,)
    return outer, red, inner, out_shape


def keepdims_shape(shape, axis):
    if axis is None:
        return (1,) * len(shape)
    red = set(validation.normalize_dims(axis, len(shape)))
    return tuple(1 if d in red else s for d, s in enumerate(shape))
