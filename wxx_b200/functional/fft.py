"""FFT and complex primitives (reference: src/wxx/functional/fft.py).

Complex tensors are interleaved (re, im) float pairs with ``type == "c64"``;
their logical shape omits the pair, so a spectrum of K bins has shape
``(..., K)``.  ``rfft``/``irfft`` follow ``numpy.fft.rfft``/``irfft`` with
the transform length ``n`` (zero-pad or truncate); ``n`` must be a power of
two as in the reference.  ``fftconv`` is the fused
``irfft(rfft(x, n) * rfft(h, n), n)[..., :L]`` used by Hyena.
"""

import numpy as np

from .. import validation
from ..Tensor import Tensor, _from_host
from ..backend.dispatch import broadcast_shapes
from ._common import F, arr64, check, dense, empty

MAX_RANK = 6


def _prod(shape):
    return validation.numel(shape)


def _check_pow2(n):
    if n < 1 or (n & (n - 1)) != 0:
        raise ValueError(f"FFT length must be a positive power of two, got {n}")


def from_numpy_complex(array):
    array = np.asarray(array)
    if not np.iscomplexobj(array):
        array = array.astype(np.float32)
    return _from_host(np.ascontiguousarray(array, dtype=np.complex64), "c64")


def complex_weights(weights):
    return from_numpy_complex(np.asarray(weights, dtype=np.float32).astype(np.complex64))


def _broadcast_strides(tensor, out_shape):
    rank = len(out_shape)
    lead = rank - len(tensor.shape)
    if lead < 0:
        raise ValueError(f"cannot broadcast shape {tuple(tensor.shape)} to {tuple(out_shape)}")
    strides = []
    for i in range(rank):
        if i < lead:
            strides.append(0)
            continue
        d = tensor.shape[i - lead]
        if d == out_shape[i]:
            strides.append(tensor.stride[i - lead])
        elif d == 1:
            strides.append(0)
        else:
            raise ValueError(
                f"cannot broadcast shape {tuple(tensor.shape)} to {tuple(out_shape)}"
            )
    return tuple(strides)


def complex_mul(tensor_a, tensor_b, conj_a=False, conj_b=False):
    """Broadcasting complex product of strided c64 views."""
    if tensor_a.type != "c64" or tensor_b.type != "c64":
        raise TypeError("complex_mul expects complex64 tensors")
    out_shape, _, _ = broadcast_shapes(tensor_a.shape, tensor_b.shape)
    rank = len(out_shape)
    if rank > MAX_RANK:
        raise ValueError(f"Maximum rank supported by complex kernels is {MAX_RANK}")
    sa = _broadcast_strides(tensor_a, out_shape)
    sb = _broadcast_strides(tensor_b, out_shape)
    out = empty(out_shape, "c64", tensor_a.requires_grad or tensor_b.requires_grad)
    if _prod(out_shape):
        check(F.wxx_complex_mul(out.buffer.ptr, tensor_a.buffer.ptr, tensor_a.offset, arr64(sa),
                                tensor_b.buffer.ptr, tensor_b.offset, arr64(sb), rank,
                                arr64(out_shape), int(bool(conj_a)), int(bool(conj_b))),
              "complex_mul")
    return out


def complex_contiguous(tensor1):
    if tensor1.type != "c64":
        raise TypeError("complex_contiguous expects a complex64 tensor")
    from .utils import contiguous

    return contiguous(tensor1)


def complex_conj(tensor1):
    x = dense(tensor1)
    out = empty(x.shape, "c64", tensor1.requires_grad)
    check(F.wxx_complex_conj(out.buffer.ptr, x.ptr, _prod(x.shape)), "complex_conj")
    return out


def complex_add_inplace(accumulator, tensor1):
    if tuple(accumulator.shape) != tuple(tensor1.shape):
        raise ValueError("complex_add_inplace expects equal shapes")
    if not accumulator.is_dense():
        raise ValueError("complex_add_inplace accumulates into a dense tensor")
    x = dense(tensor1)
    check(F.wxx_complex_add_inplace(accumulator.ptr, x.ptr, _prod(x.shape)),
          "complex_add_inplace")
    from .utils import mark_written

    mark_written(accumulator)
    return accumulator


def complex_pad(tensor1, out_len):
    """Zero-pads or truncates the last (complex) axis to ``out_len``."""
    x = dense(tensor1)
    shape = list(x.shape)
    out_shape = shape[:-1] + [int(out_len)]
    out = Tensor(out_shape, value=0.0, dtype="c64")
    keep = min(shape[-1], int(out_len))
    if keep:
        from .utils import assign

        assign(out.narrow(len(shape) - 1, 0, keep), x.narrow(len(shape) - 1, 0, keep))
    return out


def rfft(tensor1, n=None):
    """Real FFT of the last axis; returns ``(spectrum, n)`` with ``n//2 + 1`` bins."""
    if tensor1.type == "c64":
        raise TypeError("rfft expects a real-valued tensor")
    validation.check_rank(tensor1.shape, min_rank=1, max_rank=8, name="rfft input")
    x = dense(tensor1)
    shape = list(x.shape)
    in_len = shape[-1]
    n = in_len if n is None else int(n)
    _check_pow2(n)
    rows = _prod(shape[:-1])
    bins = n // 2 + 1
    out = empty(shape[:-1] + [bins], "c64", tensor1.requires_grad)
    check(F.wxx_rfft(out.buffer.ptr, bins, x.ptr, in_len, rows, in_len, n), "rfft")
    return out, n


def irfft(tensor1, n=None):
    """Inverse real FFT of a one-sided spectrum; last axis becomes ``n``
    (default ``2 * (bins - 1)``)."""
    if tensor1.type != "c64":
        raise TypeError("irfft expects a complex64 tensor")
    validation.check_rank(tensor1.shape, min_rank=1, max_rank=8, name="irfft input")
    x = dense(tensor1)
    shape = list(x.shape)
    in_len = shape[-1]
    n = 2 * (in_len - 1) if n is None else int(n)
    _check_pow2(n)
    if n < 2:
        raise ValueError("irfft length must be at least 2")
    rows = _prod(shape[:-1])
    out = empty(shape[:-1] + [n], "f32", tensor1.requires_grad)
    check(F.wxx_irfft(out.buffer.ptr, n, x.ptr, in_len, rows, in_len, n), "irfft")
    return out


def filter_spectrum(h, n):
    """The spectra of the (R, Lh) filters ``h`` for ``fftconv_spectrum`` at
    FFT size ``n``: a (R, n//2 + 2) c64 tensor whose rows hold the n//2 + 1
    bins of ``rfft(h, n)`` (one pad value a row keeps every row 16-byte
    aligned for the fused kernel's bulk copies).  One launch for all rows."""
    if len(h.shape) != 2:
        raise ValueError(f"filter_spectrum expects (R, Lh) filters, got {h.shape}")
    n = int(n)
    _check_pow2(n)
    hd = dense(h)
    R, Lh = hd.shape
    ld = n // 2 + 2
    out = empty((R, ld), "c64")
    check(F.wxx_rfft(out.buffer.ptr, ld, hd.ptr, Lh, R, Lh, n), "filter_spectrum")
    return out


def fftconv_spectrum(x, H, n, out_len=None, gate=None):
    """``fftconv`` with the filter given by its spectrum ``H`` (a (D, >= n//2 +
    1) c64 view with unit column stride, as ``filter_spectrum`` returns), so a
    filter that does not change between calls is transformed once."""
    if len(x.shape) != 3 or len(H.shape) != 2 or H.type != "c64":
        raise ValueError(f"fftconv_spectrum expects x (B, D, L) and a c64 H (D, bins), got "
                         f"{x.shape}, {H.shape}")
    B, D, L = x.shape
    n = int(n)
    _check_pow2(n)
    if H.shape[0] != D or H.shape[1] < n // 2 + 1 or H.stride[1] != 1:
        raise ValueError(f"fftconv_spectrum: spectrum {tuple(H.shape)} does not fit D = {D}, "
                         f"n = {n}")
    out_len = L if out_len is None else int(out_len)
    if not 0 <= out_len <= n:
        raise ValueError(f"fftconv_spectrum: out_len {out_len} outside [0, {n}]")
    if any(s < 0 for s in x.stride):
        x = x.contiguous()
    out = empty((B, D, out_len), "f32")
    if gate is None:
        check(F.wxx_fftconv_spectrum(out.buffer.ptr, x.buffer.ptr, x.offset, x.stride[0],
                                     x.stride[1], x.stride[2], H.ptr, H.stride[0], B, D, L, n,
                                     out_len), "fftconv_spectrum")
        return out
    if tuple(gate.shape) != (B, D, out_len):
        raise ValueError(f"fftconv_spectrum: gate shape {gate.shape} != {(B, D, out_len)}")
    if any(s < 0 for s in gate.stride):
        gate = gate.contiguous()
    check(F.wxx_fftconv_spectrum_gated(out.buffer.ptr, x.buffer.ptr, x.offset, x.stride[0],
                                       x.stride[1], x.stride[2], H.ptr, H.stride[0], B, D, L, n,
                                       out_len, gate.buffer.ptr, gate.offset, gate.stride[0],
                                       gate.stride[1], gate.stride[2]), "fftconv_spectrum")
    return out


def fftconv(x, h, n, out_len=None, gate=None):
    """Causal FFT convolution ``irfft(rfft(x, n) * rfft(h, n), n)[..., :out_len]``
    of a (B, D, L) view ``x`` with a (D, Lh) filter ``h`` broadcast over the
    batch, in one fused pass per row (the spectra stay on chip).  With a
    (B, D, out_len) ``gate`` view the result is ``gate * fftconv(x, h)``
    (Hyena's ``gates[i] * fft_conv1d(z, h)``), multiplied as it is stored."""
    if len(x.shape) != 3 or len(h.shape) != 2:
        raise ValueError(f"fftconv expects x (B, D, L) and h (D, Lh), got {x.shape}, {h.shape}")
    B, D, L = x.shape
    if h.shape[0] != D:
        raise ValueError(f"fftconv: filter has {h.shape[0]} channels, input has {D}")
    n = int(n)
    _check_pow2(n)
    out_len = L if out_len is None else int(out_len)
    if not 0 <= out_len <= n:
        raise ValueError(f"fftconv: out_len {out_len} outside [0, {n}]")
    if any(s < 0 for s in x.stride):
        x = x.contiguous()
    hd = dense(h)
    if gate is None:
        out = empty((B, D, out_len), "f32", x.requires_grad or h.requires_grad)
        check(F.wxx_fftconv(out.buffer.ptr, x.buffer.ptr, x.offset, x.stride[0], x.stride[1],
                            x.stride[2], hd.ptr, h.shape[1], h.shape[1], B, D, L, n, out_len),
              "fftconv")
        return out
    if tuple(gate.shape) != (B, D, out_len):
        raise ValueError(f"fftconv: gate shape {gate.shape} != {(B, D, out_len)}")
    if any(s < 0 for s in gate.stride):
        gate = gate.contiguous()
    out = empty((B, D, out_len), "f32", x.requires_grad or h.requires_grad or gate.requires_grad)
    check(F.wxx_fftconv_gated(out.buffer.ptr, x.buffer.ptr, x.offset, x.stride[0], x.stride[1],
                              x.stride[2], hd.ptr, h.shape[1], h.shape[1], B, D, L, n, out_len,
                              gate.buffer.ptr, gate.offset, gate.stride[0], gate.stride[1],
                              gate.stride[2]),
          "fftconv")
    return out
