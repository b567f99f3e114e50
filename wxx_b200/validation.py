"""Shape, dimension and layout checks shared by the wxx ops.

Same contracts and error types as the reference's validators
(src/wxx/validation.py:14-190): metadata only, no device work.  ``MAX_RANK``
stays 6 (the rank every strided kernel of the reference accepts); the CUDA
kernels here accept up to 8, so the limit is the API's, not the hardware's.
"""

import math

MAX_RANK = 6


def numel(shape):
    return int(math.prod(shape)) if len(shape) else 1


def _is_int(v):
    return isinstance(v, int) and not isinstance(v, bool)


def normalize_shape(shape, *, name="shape", allow_infer=False):
    """Tuple of non-negative ints (one ``-1`` allowed when ``allow_infer``)."""
    if _is_int(shape):
        shape = (shape,)
    try:
        dims = tuple(shape)
    except TypeError:
        raise TypeError(
            f"{name} must be an int or an iterable of ints, got {type(shape).__name__}"
        ) from None
    seen_infer = False
    for i, d in enumerate(dims):
        if not _is_int(d):
            raise TypeError(f"{name}[{i}] must be an int, got {type(d).__name__}")
        if d == -1 and allow_infer:
            if seen_infer:
                raise ValueError(f"{name} may contain at most one -1, got {dims}")
            seen_infer = True
        elif d < 0:
            raise ValueError(f"{name}[{i}] must be non-negative, got {d}")
    return dims


def infer_shape(shape, total, *, name="shape"):
    """Resolves a single ``-1`` and checks that the element count is ``total``."""
    dims = normalize_shape(shape, name=name, allow_infer=True)
    if -1 in dims:
        at = dims.index(-1)
        known = numel(dims[:at] + dims[at + 1:])
        if known == 0 or total % known:
            raise ValueError(f"cannot infer {name} {dims} for {total} elements")
        dims = dims[:at] + (total // known,) + dims[at + 1:]
    if numel(dims) != total:
        raise ValueError(f"{name} {dims} describes {numel(dims)} elements, expected {total}")
    return dims


def normalize_dim(dim, rank, *, name="dim"):
    if not _is_int(dim):
        raise TypeError(f"{name} must be an int, got {type(dim).__name__}")
    if rank == 0:
        raise IndexError(f"{name}={dim} is invalid for a 0-d tensor")
    d = dim + rank if dim < 0 else dim
    if d < 0 or d >= rank:
        raise IndexError(f"{name}={dim} is out of range for a tensor of rank {rank}")
    return d


def normalize_dims(dims, rank, *, name="dims", allow_duplicates=True):
    if _is_int(dims):
        dims = (dims,)
    try:
        items = tuple(dims)
    except TypeError:
        raise TypeError(
            f"{name} must be an int or an iterable of ints, got {type(dims).__name__}"
        ) from None
    out = tuple(normalize_dim(d, rank, name=f"{name}[{i}]") for i, d in enumerate(items))
    if not allow_duplicates and len(set(out)) != len(out):
        raise ValueError(f"{name} contains duplicate dimensions: {out}")
    return out


def check_rank(shape, *, min_rank=0, max_rank=MAX_RANK, name="tensor"):
    rank = len(shape)
    if rank < min_rank or (max_rank is not None and rank > max_rank):
        if max_rank is None:
            want = f"at least {min_rank}"
        elif min_rank == max_rank:
            want = str(min_rank)
        else:
            want = f"{min_rank}..{max_rank}"
        raise ValueError(f"{name} must have rank {want}, got {rank}")
    return rank


def check_same_shape(*shapes, name="tensors"):
    if not shapes:
        raise ValueError(f"{name} must contain at least one shape")
    first = tuple(shapes[0])
    for i, s in enumerate(shapes[1:], 1):
        if tuple(s) != first:
            raise ValueError(
                f"{name} must have the same shape, got {first} and {tuple(s)} (at index {i})"
            )
    return first


def check_broadcastable(shape, out_shape, *, name="tensor"):
    if len(shape) > len(out_shape):
        raise ValueError(f"{name} of shape {tuple(shape)} cannot broadcast to {tuple(out_shape)}")
    lead = len(out_shape) - len(shape)
    for i, d in enumerate(shape):
        if d != 1 and d != out_shape[lead + i]:
            raise ValueError(
                f"{name} of shape {tuple(shape)} cannot broadcast to {tuple(out_shape)}"
            )
    return tuple(out_shape)


def contiguous_strides(shape):
    strides = []
    acc = 1
    for d in reversed(tuple(shape)):
        strides.append(acc)
        acc *= d
    return tuple(reversed(strides))


def is_contiguous_layout(shape, stride):
    """Row-major compact layout; size-1 dims may carry any stride."""
    want = 1
    for d, s in zip(reversed(tuple(shape)), reversed(tuple(stride))):
        if d > 1 and s != want:
            return False
        want *= d
    return True


def check_contiguous(tensor, *, name="tensor"):
    if not tensor.is_contiguous():
        raise ValueError(
            f"{name} must be contiguous, got shape={tuple(tensor.shape)} "
            f"stride={tuple(tensor.stride)} offset={tensor.offset}"
        )
    return tensor


def check_no_negative_stride(tensor, *, name="tensor"):
    if any(s < 0 for s in tensor.stride):
        raise ValueError(
            f"{name} has a negative stride {tuple(tensor.stride)}; call .contiguous() first"
        )
    return tensor


__all__ = [
    "MAX_RANK",
    "numel",
    "normalize_shape",
    "infer_shape",
    "normalize_dim",
    "normalize_dims",
    "check_rank",
    "check_same_shape",
    "check_broadcastable",
    "contiguous_strides",
    "is_contiguous_layout",
    "check_contiguous",
    "check_no_negative_stride",
]
