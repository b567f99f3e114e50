"""Dense tensors in B200 device memory.

API of the reference's ``Tensor`` (src/wxx/Tensor.py:28-872): a logical
``shape`` (a list), a row-major ``stride`` and an ``offset`` in elements, a
``type`` of ``"f32"``, ``"u32"`` or ``"c64"`` (interleaved float pairs), and a
``buffer`` holding the storage.  Views (indexing, ``narrow``, ``permute``,
``transpose``, ...) share the buffer and carry their own offset/stride;
operations route through ``wxx_b200.autograd`` to ``wxx_b200.functional``.

``buffer`` is a :class:`wxx_b200.backend.device.DeviceBuffer` (a device
allocation freed when the last tensor referencing it goes away) instead of a
wgpu buffer.  Host access (``numpy``, ``item``, ``repr``) synchronises the
stream, as ``read_buffer`` does in the reference.
"""

import ctypes
import numbers

import os

import numpy as np

from . import validation
from .backend import device as _dev
from .backend.lib import F, check

_DTYPES = ("f32", "u32", "c64")
_NP = {"f32": np.float32, "u32": np.uint32, "c64": np.complex64}


# Check mode (WXX_CHECK=1, or wxx_b200.backend.observe.set_check_mode): every
# view is checked to address only its own storage.
_CHECK = {"views": os.environ.get("WXX_CHECK", "") == "1"}


def _check_view_extent(t):
    n = validation.numel(t.shape)
    if n == 0 or t.buffer is None:
        return
    lo = t.offset + sum(min(0, (d - 1) * s) for d, s in zip(t.shape, t.stride))
    hi = t.offset + sum(max(0, (d - 1) * s) for d, s in zip(t.shape, t.stride))
    size = getattr(t.buffer, "size", None)
    if lo < 0 or (size is not None and (hi + 1) * _itemsize(t.type) > size):
        raise IndexError(f"view shape={t.shape} stride={t.stride} offset={t.offset} reaches "
                         f"elements [{lo}, {hi}] outside its {size}-byte storage")


def _itemsize(dtype):
    return 8 if dtype == "c64" else 4


class Tensor:
    """N-dimensional tensor backed by a device buffer."""

    def __init__(self, shape, buffer=None, data=None, value=1.0, offset=0, stride=None,
                 requires_grad=False, dtype=None):
        shape = validation.normalize_shape(shape)
        if not isinstance(offset, int) or isinstance(offset, bool) or offset < 0:
            raise ValueError(f"offset must be a non-negative int, got {offset!r}")
        if dtype is not None and dtype not in _DTYPES:
            raise ValueError(f"unsupported dtype {dtype!r}; expected one of {_DTYPES}")
        self.shape = list(shape)
        self.offset = offset
        self._base = None
        self.type = dtype if dtype is not None else "f32"
        if stride is None:
            self.stride = validation.contiguous_strides(self.shape)
        else:
            stride = tuple(stride)
            if len(stride) != len(self.shape):
                raise ValueError(
                    f"stride {stride} must have one entry per shape dimension "
                    f"{tuple(self.shape)}"
                )
            self.stride = stride
        n = validation.numel(self.shape)
        self.nbytes = n * self.itemsize()
        if buffer is None:
            buffer = _dev.DeviceBuffer(max(self.nbytes, 4), "Tensor")
            if data is not None:
                raw = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
                if raw.nbytes < self.nbytes:
                    raise ValueError(
                        f"data has {raw.nbytes} bytes, shape {tuple(self.shape)} needs {self.nbytes}"
                    )
                raw = np.ascontiguousarray(raw[: self.nbytes])
                check(F.wxx_memcpy_h2d(buffer.ptr, raw.ctypes.data, self.nbytes), "upload")
            elif n:
                # every fill is a library kernel (c64 zeros: 2n zero words)
                words = 2 * n if self.type == "c64" else n
                bits = 0 if self.type == "c64" else _fill_bits(value, self.type)
                shp = (ctypes.c_int64 * 1)(words)
                one = (ctypes.c_int64 * 1)(1)
                check(F.wxx_strided_fill(buffer.ptr, 0, one, 1, shp, bits), "fill")
        self.buffer = buffer
        self.requires_grad = requires_grad
        self.creator = None
        self.grad = None

    # ------------------------------------------------------------------ fast paths
    @classmethod
    def _wrap(cls, shape, buffer, dtype="f32", requires_grad=False, stride=None, offset=0,
              base=None):
        """Builds a tensor around an existing buffer without validation (internal)."""
        t = object.__new__(cls)
        t.shape = list(shape)
        t.offset = offset
        t._base = base
        t.type = dtype
        t.stride = tuple(stride) if stride is not None else validation.contiguous_strides(t.shape)
        t.nbytes = validation.numel(t.shape) * _itemsize(dtype)
        t.buffer = buffer
        t.requires_grad = requires_grad
        t.creator = None
        t.grad = None
        if _CHECK["views"]:
            _check_view_extent(t)
        return t

    @classmethod
    def _empty(cls, shape, dtype="f32", requires_grad=False):
        """Uninitialised dense tensor (internal: every op's output)."""
        n = validation.numel(shape)
        buf = _dev.DeviceBuffer(max(n * _itemsize(dtype), 4), "Tensor")
        return cls._wrap(shape, buf, dtype, requires_grad)

    @property
    def ptr(self):
        """Device address of element 0 of this view."""
        return self.buffer.ptr + self.offset * self.itemsize()

    # ------------------------------------------------------------------ layout
    def itemsize(self):
        return 8 if self.type == "c64" else 4

    def calc_contiguous_strides(self):
        return validation.contiguous_strides(self.shape)

    def is_contiguous(self):
        """Compact row-major layout starting at offset 0 (reference semantics)."""
        if self.offset != 0:
            return False
        return validation.is_contiguous_layout(self.shape, self.stride)

    def is_dense(self):
        """Compact row-major layout at any offset."""
        return validation.is_contiguous_layout(self.shape, self.stride)

    # ------------------------------------------------------------------ indexing
    def __getitem__(self, index):
        if not isinstance(index, tuple):
            index = (index,)
        if any(item is Ellipsis for item in index):
            at = next(i for i, item in enumerate(index) if item is Ellipsis)
            missing = len(self.shape) - (len(index) - 1)
            if missing < 0:
                raise IndexError("too many indices for tensor")
            index = index[:at] + (slice(None),) * missing + index[at + 1:]
        items = []
        advanced = False
        for item in index:
            if isinstance(item, (list, np.ndarray)):
                item = np.asarray(item)
                advanced = True
            elif isinstance(item, Tensor):
                advanced = True
            items.append(item)
        index = tuple(items)
        if advanced:
            return self._advanced_getitem(index)
        if len(index) < len(self.shape):
            index = index + (slice(None),) * (len(self.shape) - len(index))
        if len(index) > len(self.shape):
            raise IndexError("too many indices for tensor")
        return self._basic_getitem(index)

    def _basic_getitem(self, index):
        off = self.offset
        shape, stride = [], []
        for axis, item in enumerate(index):
            if isinstance(item, slice):
                start, stop, step = item.indices(self.shape[axis])
                off += start * self.stride[axis]
                length = max(0, (stop - start + (step - 1 if step > 0 else step + 1)) // step)
                shape.append(length)
                stride.append(self.stride[axis] * step)
            elif isinstance(item, int) and not isinstance(item, bool):
                pos = item if item >= 0 else self.shape[axis] + item
                if not 0 <= pos < self.shape[axis]:
                    raise IndexError(
                        f"index {item} out of bounds for axis {axis} with size {self.shape[axis]}"
                    )
                off += pos * self.stride[axis]
            else:
                raise IndexError(f"unsupported index type {type(item).__name__}")
        return Tensor._wrap(shape, self.buffer, self.type, self.requires_grad, stride, off, self)

    def _advanced_getitem(self, index):
        host = self.numpy()
        np_index = tuple(
            item.numpy().astype(np.int64) if isinstance(item, Tensor) else item for item in index
        )
        first = np_index[0]
        if isinstance(first, np.ndarray) and first.dtype == np.bool_ and len(np_index) == 1:
            result = host.reshape(-1)[np.flatnonzero(first)]
        else:
            result = host[np_index]
        out = _from_host(np.ascontiguousarray(result), self.type)
        out.requires_grad = self.requires_grad
        return out

    def __setitem__(self, index, value):
        from . import functional

        functional.assign(self[index], value)

    # ------------------------------------------------------------------ views
    def narrow(self, dim, start, length):
        rank = len(self.shape)
        dim = validation.normalize_dim(dim, rank)
        if not isinstance(start, int) or isinstance(start, bool):
            raise TypeError(f"start must be an int, got {type(start).__name__}")
        if not isinstance(length, int) or isinstance(length, bool):
            raise TypeError(f"length must be an int, got {type(length).__name__}")
        if start < 0 or length < 0 or start + length > self.shape[dim]:
            raise IndexError(
                f"narrow bounds out of range: start={start}, length={length}, "
                f"dim {dim} has size {self.shape[dim]}"
            )
        shape = list(self.shape)
        shape[dim] = length
        return Tensor._wrap(shape, self.buffer, self.type, self.requires_grad, self.stride,
                            self.offset + start * self.stride[dim], self)

    def slice(self, dim, start, length):
        return self.narrow(dim, start, length)

    def chunk(self, chunks, dim=0):
        rank = len(self.shape)
        dim = validation.normalize_dim(dim, rank, name="dim")
        if not isinstance(chunks, int) or isinstance(chunks, bool) or chunks < 1:
            raise ValueError(f"chunks must be a positive int, got {chunks!r}")
        size = self.shape[dim]
        if size % chunks:
            raise ValueError(
                f"cannot split dimension {dim} of size {size} into {chunks} equal chunks"
            )
        step = size // chunks
        return tuple(self.narrow(dim, i * step, step) for i in range(chunks))

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        from . import autograd

        return autograd.reshape(self).forward(self, tuple(shape))

    def view(self, *shape):
        return self.reshape(*shape)

    def permute(self, *axis):
        from . import autograd

        if len(axis) == 1 and isinstance(axis[0], (tuple, list)):
            axis = tuple(axis[0])
        return autograd.permute(self).forward(self, axis)

    def transpose(self, dim0, dim1):
        rank = len(self.shape)
        d0 = validation.normalize_dim(dim0, rank, name="dim0")
        d1 = validation.normalize_dim(dim1, rank, name="dim1")
        axes = list(range(rank))
        axes[d0], axes[d1] = axes[d1], axes[d0]
        return self.permute(*axes)

    def t(self):
        if len(self.shape) < 2:
            raise IndexError("t() expects a tensor with at least 2 dimensions")
        return self.transpose(-1, -2)

    def contiguous(self):
        from . import autograd

        return autograd.contiguous(self).forward(self)

    def unsqueeze(self, dim):
        rank = len(self.shape)
        dim = validation.normalize_dim(dim, rank + 1, name="dim")
        shape = list(self.shape)
        stride = list(self.stride)
        inner = stride[dim] * shape[dim] if dim < rank else 1
        shape.insert(dim, 1)
        stride.insert(dim, inner)
        return Tensor._wrap(shape, self.buffer, self.type, self.requires_grad, stride,
                            self.offset, self)

    def squeeze(self, dim=None):
        if dim is None:
            keep = [i for i, s in enumerate(self.shape) if s != 1]
        else:
            d = validation.normalize_dim(dim, len(self.shape), name="dim")
            keep = [i for i in range(len(self.shape)) if i != d or self.shape[i] != 1]
        shape = [self.shape[i] for i in keep]
        stride = [self.stride[i] for i in keep]
        return Tensor._wrap(shape, self.buffer, self.type, self.requires_grad, stride,
                            self.offset, self)

    def flatten(self, start_dim=0, end_dim=-1):
        nd = len(self.shape)
        s = validation.normalize_dim(start_dim, nd, name="start_dim")
        e = validation.normalize_dim(end_dim, nd, name="end_dim")
        if s > e:
            raise ValueError(f"start_dim ({s}) must be <= end_dim ({e})")
        merged = validation.numel(self.shape[s:e + 1])
        return self.reshape(tuple(self.shape[:s]) + (merged,) + tuple(self.shape[e + 1:]))

    def detach(self):
        if self.buffer is None:
            raise RuntimeError("cannot detach a tensor whose buffer was released")
        return Tensor._wrap(self.shape, self.buffer, self.type, False, self.stride, self.offset,
                            self)

    def detach_(self):
        self.requires_grad = False
        self.creator = None
        self.grad = None
        return self

    def backward(self, grad=None):
        """Back-propagates from this tensor (the reference's Tensor.backward):
        the recorded ops are visited in reverse topological order, each op's
        ``backward`` turns its output gradient into its inputs' gradients,
        gradients reaching one tensor along several paths are added, and
        leaf tensors (parameters) receive theirs in ``.grad`` (added to an
        existing ``.grad``).  The seed is ``grad`` or ones.  The graph is
        released as it is consumed."""
        from . import functional
        from .backend.context import inferenceMode

        if not self.requires_grad:
            raise RuntimeError("cannot call backward on a tensor that does not require gradients")
        seed = grad if grad is not None else Tensor(self.shape, value=1.0, dtype=self.type)
        # reverse topological order of the tensors that need a gradient
        order, seen = [], set()
        stack = [(self, False)]
        while stack:
            t, done = stack.pop()
            if done:
                order.append(t)
                continue
            if id(t) in seen:
                continue
            seen.add(id(t))
            stack.append((t, True))
            fn = t.creator
            if fn is not None and fn.inputs is not None:
                for parent in fn.inputs:
                    if isinstance(parent, Tensor) and parent.requires_grad and \
                            id(parent) not in seen:
                        stack.append((parent, False))
        grads = {id(self): seed}
        with inferenceMode():
            for t in reversed(order):
                g = grads.pop(id(t), None)
                fn = t.creator
                if fn is None:
                    if g is not None:
                        t.grad = g if t.grad is None else functional.pointwise(t.grad, g, 0)
                    continue
                if g is not None:
                    parts = fn.backward(g)
                    if not isinstance(parts, (tuple, list)):
                        parts = (parts,)
                    if len(parts) != len(fn.inputs):
                        raise RuntimeError(f"{type(fn).__name__}.backward returned {len(parts)} "
                                           f"gradients for {len(fn.inputs)} inputs")
                    for parent, pg in zip(fn.inputs, parts):
                        if pg is None or not isinstance(parent, Tensor) or \
                                not parent.requires_grad:
                            continue
                        prev = grads.get(id(parent))
                        grads[id(parent)] = pg if prev is None else functional.pointwise(prev, pg, 0)
                fn.inputs = None
                t.creator = None

    # ------------------------------------------------------------------ host access
    def numpy(self):
        """Copies this tensor to a NumPy array (synchronises the stream)."""
        if self.type not in _NP:
            raise TypeError(f"unsupported tensor type {self.type!r}")
        src = self if self.is_dense() else self.contiguous()
        out = np.empty(tuple(self.shape), dtype=_NP[self.type])
        if out.nbytes:
            check(F.wxx_memcpy_d2h(out.ctypes.data, src.ptr, out.nbytes), "download")
        return out

    def read_buffer(self):
        _dev.synchronize()

    def __repr__(self):
        arr = np.array2string(self.numpy(), prefix="tensor(", precision=4, suppress_small=True)
        return f"tensor({arr}, shape={self.shape}), require grad={self.requires_grad}"

    def item(self):
        if validation.numel(self.shape) != 1:
            raise RuntimeError("cannot convert a tensor with more than one element to a scalar")
        return self.numpy().item()

    def destroy(self):
        """Drops this tensor's reference to its storage (freed with the last one)."""
        self.buffer = None

    # ------------------------------------------------------------------ arithmetic
    def __add__(self, other):
        from . import autograd

        if not isinstance(other, Tensor):
            return autograd.addscaler(self).forward(self, float(other))
        return autograd.add(self, other).forward(self, other)

    def __radd__(self, other):
        return self.__add__(other)

    def __sub__(self, other):
        from . import autograd

        if not isinstance(other, Tensor):
            return autograd.subscaler(self).forward(self, float(other))
        return autograd.sub(self, other).forward(self, other)

    def __rsub__(self, other):
        from . import functional

        return functional.scalarpointwise(self, float(other), 1, reverse=1)

    def __neg__(self):
        from . import autograd

        return autograd.negate(self).forward(self)

    def __mul__(self, other):
        from . import autograd

        if not isinstance(other, Tensor):
            return autograd.mulscaler(self).forward(self, float(other))
        return autograd.mul(self, other).forward(self, other)

    def __rmul__(self, other):
        return self.__mul__(other)

    def __truediv__(self, other):
        from . import autograd

        if not isinstance(other, Tensor):
            return autograd.mulscaler(self).forward(self, 1.0 / float(other))
        return autograd.div(self, other).forward(self, other)

    def __rtruediv__(self, other):
        from . import autograd

        if not isinstance(other, numbers.Real):
            return NotImplemented
        return autograd.rdivscaler(self).forward(self, float(other))

    def __matmul__(self, other):
        from . import autograd

        return autograd.matmul(self, other).forward(self, other)

    def matmul(self, other):
        return self.__matmul__(other)

    def __pow__(self, other):
        from . import autograd

        if isinstance(other, numbers.Real) and other == 2:
            return autograd.square(self).forward(self)
        if isinstance(other, numbers.Real):
            return autograd.powscaler(self).forward(self, float(other))
        raise TypeError(f"tensor exponents are not supported, got {type(other).__name__}")

    def __rpow__(self, other):
        from . import autograd

        if not isinstance(other, numbers.Real):
            return NotImplemented
        base = float(other)
        if base <= 0.0:
            raise ValueError(f"a tensor exponent requires a positive base, got {base}")
        return autograd.rpowscaler(self).forward(self, base)

    def pow(self, exponent):
        return self.__pow__(exponent)

    def __eq__(self, other):
        from . import functional

        return functional.equal(self, other)

    __hash__ = object.__hash__

    def matmul_add(self, other, bias):
        from . import autograd

        return autograd.matmuladd(self, other, bias).forward(self, other, bias)

    # ------------------------------------------------------------------ unary / reductions
    def relu(self):
        from . import functional

        return functional.relu(self)

    def gelu(self):
        from . import autograd

        return autograd.gelu(self).forward(self)

    def sin(self):
        from . import functional

        return functional.sin(self)

    def cos(self):
        from . import functional

        return functional.cos(self)

    def sigmoid(self):
        from . import functional

        return functional.sigmoid(self)

    def silu(self):
        from . import functional

        return functional.sigmoid(self) * self

    def selu(self):
        from . import functional

        return functional.selu(self)

    def softmax(self, dim=-1):
        from . import autograd

        return autograd.softmax(self).forward(self, dim)

    def square(self):
        from . import functional

        return functional.square(self)

    def exp(self):
        from . import functional

        return functional.exp(self)

    def sqrt(self):
        from . import functional

        return functional.sqrt(self)

    def rsqrt(self):
        from . import functional

        return functional.rsqrt(self)

    def log(self):
        from . import functional

        return functional.log(self)

    def abs(self):
        from . import functional

        return functional.abs(self)

    def sign(self):
        from . import functional

        return functional.sign(self)

    def clamp(self, min=np.finfo(np.float32).min, max=np.finfo(np.float32).max):
        from . import functional

        return functional.clamp(self, min, max)

    def sum(self, axis=None, keepdims=False, *, keepdim=None):
        from . import autograd

        return autograd.sum(self).forward(self, axis, keepdims if keepdim is None else keepdim)

    def mean(self, axis=None, keepdims=False, *, keepdim=None):
        from . import autograd

        return autograd.mean(self).forward(self, axis, keepdims if keepdim is None else keepdim)

    def var(self, axis=None, keepdims=False, *, keepdim=None):
        from . import functional

        return functional.var(self, axis, keepdims if keepdim is None else keepdim)

    def std(self, axis=None, keepdims=False, *, keepdim=None):
        from . import functional

        return functional.std(self, axis, keepdims if keepdim is None else keepdim)

    def max(self, dim=None, keepdims=False, *, keepdim=None):
        from . import functional

        return functional.max(self, dim, keepdims if keepdim is None else keepdim)[0]

    def min(self, dim=None, keepdims=False, *, keepdim=None):
        from . import functional

        return functional.min(self, dim, keepdims if keepdim is None else keepdim)[0]

    def argmax(self, dim=None, keepdims=False, *, keepdim=None):
        from . import functional

        return functional.max(self, dim, keepdims if keepdim is None else keepdim)[1]

    def argmin(self, dim=None, keepdims=False, *, keepdim=None):
        from . import functional

        return functional.min(self, dim, keepdims if keepdim is None else keepdim)[1]

    # ------------------------------------------------------------------ FFT / complex
    def rfft(self, n=None):
        from . import functional

        return functional.rfft(self, n)[0]

    def irfft(self, n=None):
        from . import functional

        return functional.irfft(self, n)

    def complex_mul(self, other):
        from . import functional

        return functional.complex_mul(self, other)

    def conj(self):
        from . import functional

        return functional.complex_conj(self)


class Parameter(Tensor):
    """A tensor registered as a learnable parameter (shares the tensor's storage)."""

    def __init__(self, tensor, requires_grad=True):
        self.shape = list(tensor.shape)
        self.offset = tensor.offset
        self.stride = tuple(tensor.stride)
        self.type = tensor.type
        self.nbytes = tensor.nbytes
        self.buffer = tensor.buffer
        self._base = tensor
        self.Tensor = tensor
        self.requires_grad = requires_grad
        self.creator = None
        self.grad = None


def _fill_bits(value, dtype):
    if dtype == "u32":
        return int(value) & 0xFFFFFFFF
    return int(np.array([value], dtype=np.float32).view(np.uint32)[0])


def _from_host(array, dtype):
    """Uploads a contiguous host array as a new tensor of ``dtype``."""
    if dtype == "c64":
        array = np.ascontiguousarray(array, dtype=np.complex64)
    elif dtype == "u32":
        array = np.ascontiguousarray(array, dtype=np.uint32)
    else:
        array = np.ascontiguousarray(array, dtype=np.float32)
    t = Tensor._empty(list(array.shape), dtype)
    if array.nbytes:
        check(F.wxx_memcpy_h2d(t.buffer.ptr, array.ctypes.data, array.nbytes), "upload")
    return t
