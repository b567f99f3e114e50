"""Metadata checks for the wxx ops: shapes, axes, ranks, broadcasting, layouts.

Pure host code (no device work).  The public names and the exception types
they raise are the interface of the reference's ``wxx.validation`` module
(src/wxx/validation.py): ``TypeError`` for a value of the wrong kind,
``ValueError`` for a bad shape or layout, ``IndexError`` for an axis outside
the tensor's rank.  ``MAX_RANK`` is 6, the rank every strided kernel of the
reference accepts; the CUDA kernels take up to 8, so the limit is the API's.
"""

import math
from numbers import Integral

MAX_RANK = 6


def _int_like(v):
    return isinstance(v, Integral) and not isinstance(v, bool)


def _as_int_tuple(value, what):
    """``value`` as a tuple of Python ints; a bare int becomes a 1-tuple."""
    if _int_like(value):
        return (int(value),)
    if isinstance(value, (str, bytes)) or not hasattr(value, "__iter__"):
        raise TypeError(f"{what}: expected an int or a sequence of ints, "
                        f"not {type(value).__name__}")
    items = tuple(value)
    for pos, item in enumerate(items):
        if not _int_like(item):
            raise TypeError(f"{what}: entry {pos} is a {type(item).__name__}, not an int")
    return tuple(int(i) for i in items)


def numel(shape):
    """Number of elements of ``shape`` (1 for a scalar's empty shape)."""
    return math.prod(int(d) for d in shape)


def normalize_shape(shape, *, name="shape", allow_infer=False):
    """Validated shape tuple: non-negative sizes, plus at most one ``-1``
    placeholder when ``allow_infer`` is set."""
    dims = _as_int_tuple(shape, name)
    placeholders = [i for i, d in enumerate(dims) if d == -1]
    if placeholders and allow_infer:
        if len(placeholders) > 1:
            raise ValueError(f"{name}: only one size may be -1, got {dims}")
        negative = [d for i, d in enumerate(dims) if d < 0 and i != placeholders[0]]
    else:
        negative = [d for d in dims if d < 0]
    if negative:
        raise ValueError(f"{name}: sizes must be >= 0, got {dims}")
    return dims


def infer_shape(shape, total, *, name="shape"):
    """Shape for ``total`` elements, with a ``-1`` (if any) filled in."""
    dims = list(normalize_shape(shape, name=name, allow_infer=True))
    if -1 in dims:
        slot = dims.index(-1)
        rest = numel(dims[:slot] + dims[slot + 1:])
        if rest == 0 or total % rest != 0:
            raise ValueError(f"{name}: {tuple(dims)} cannot hold {total} elements")
        dims[slot] = total // rest
    if numel(dims) != total:
        raise ValueError(f"{name}: {tuple(dims)} holds {numel(dims)} elements, not {total}")
    return tuple(dims)


def normalize_dim(dim, rank, *, name="dim"):
    """Axis ``dim`` (negative counts from the end) as an index in [0, rank)."""
    if not _int_like(dim):
        raise TypeError(f"{name}: expected an int, not {type(dim).__name__}")
    dim = int(dim)
    if not -rank <= dim < rank or rank == 0:
        raise IndexError(f"{name}={dim} does not name an axis of a rank-{rank} tensor")
    return dim % rank


def normalize_dims(dims, rank, *, name="dims", allow_duplicates=True):
    """Each axis of ``dims`` normalised as by ``normalize_dim``."""
    axes = tuple(normalize_dim(d, rank, name=f"{name}[{k}]")
                 for k, d in enumerate(_as_int_tuple(dims, name)))
    if not allow_duplicates and len(frozenset(axes)) < len(axes):
        raise ValueError(f"{name}: an axis appears twice in {axes}")
    return axes


def check_rank(shape, *, min_rank=0, max_rank=MAX_RANK, name="tensor"):
    """Rank of ``shape``, which must lie in [min_rank, max_rank] (no upper
    bound when ``max_rank`` is None)."""
    rank = len(shape)
    hi = math.inf if max_rank is None else max_rank
    if min_rank <= rank <= hi:
        return rank
    if max_rank is None:
        allowed = f">= {min_rank}"
    elif min_rank == max_rank:
        allowed = f"== {min_rank}"
    else:
        allowed = f"in [{min_rank}, {max_rank}]"
    raise ValueError(f"{name}: rank {rank} not supported (needs rank {allowed})")


def check_same_shape(*shapes, name="tensors"):
    """The common shape of ``shapes``; raises if any differs."""
    if len(shapes) == 0:
        raise ValueError(f"{name}: no shapes given")
    ref = tuple(shapes[0])
    odd = [(k, tuple(s)) for k, s in enumerate(shapes) if tuple(s) != ref]
    if odd:
        k, s = odd[0]
        raise ValueError(f"{name}: shape {s} at position {k} differs from {ref}")
    return ref


def check_broadcastable(shape, out_shape, *, name="tensor"):
    """``out_shape`` if ``shape`` broadcasts to it (numpy rules, trailing
    axes aligned, size 1 stretches)."""
    src, dst = tuple(shape), tuple(out_shape)
    fits = len(src) <= len(dst) and all(
        s in (1, d) for s, d in zip(reversed(src), reversed(dst)))
    if not fits:
        raise ValueError(f"{name}: shape {src} does not broadcast to {dst}")
    return dst


def contiguous_strides(shape):
    """Element strides of a dense row-major tensor of ``shape``."""
    strides = [1] * len(shape)
    for axis in range(len(shape) - 2, -1, -1):
        strides[axis] = strides[axis + 1] * int(shape[axis + 1])
    return tuple(strides)


def is_contiguous_layout(shape, stride):
    """True if (shape, stride) addresses a dense row-major block; axes of
    size 1 are never stepped along, so their stride does not matter."""
    dense = contiguous_strides(shape)
    return all(n == 1 or s == d for n, s, d in zip(shape, stride, dense))


def check_contiguous(tensor, *, name="tensor"):
    if not tensor.is_contiguous():
        raise ValueError(f"{name}: needs a contiguous tensor, got shape "
                         f"{tuple(tensor.shape)}, stride {tuple(tensor.stride)}, "
                         f"offset {tensor.offset}")
    return tensor


def check_no_negative_stride(tensor, *, name="tensor"):
    if min(tensor.stride, default=0) < 0:
        raise ValueError(f"{name}: negative stride in {tuple(tensor.stride)}; "
                         f"make it contiguous first")
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
