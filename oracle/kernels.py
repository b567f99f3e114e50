"""CPU oracle: numpy restatement of the reference's WGSL kernels.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (wxx_b200) imports this
package; tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it as the checker and as the
timed CPU implementation of the path.

Each function restates one reference kernel (paths relative to the reference
project Mo-Ehab/wxx, src/wxx/...) on numpy arrays: fp32 storage, with the
accumulation precision stated per function.  The reference cannot run here
(wgpu needs a graphics adapter that neither machine has), so the oracle is
pinned against the reference's own known-answer tests and golden vectors
generated from its pure-numpy test helpers (tests/golden/), and against
independent float64 implementations (numpy.fft, float64 matmul).
"""

import numpy as np

F32 = np.float32


# ----------------------------------------------------------------- elementwise

def pointwise(a, b, op):
    """shaders/pointwise/pointwise.wgsl:46-57: broadcast a op b (0 add 1 sub 2 mul 3 div)."""
    a = np.asarray(a, F32)
    b = np.asarray(b, F32)
    with np.errstate(all="ignore"):
        return [np.add, np.subtract, np.multiply, np.divide][op](a, b).astype(F32)


def scalarpointwise(x, c, op, reverse=0):
    """shaders/pointwise/scalarpointwise.wgsl:23-76 (op 0 add 1 sub 2 mul 3 pow 4 div)."""
    x = np.asarray(x, F32)
    c = F32(c)
    with np.errstate(all="ignore"):
        if op == 0:
            return (x + c).astype(F32)
        if op == 1:
            return (c - x if reverse else x - c).astype(F32)
        if op == 2:
            return (x * c).astype(F32)
        if op == 4:
            return (c / x if reverse else x / c).astype(F32)
        if op == 3:
            if reverse:
                return np.power(c, x).astype(F32)
            out = np.power(np.abs(x), c).astype(F32)
            neg = x < 0
            if float(c) == np.trunc(float(c)):
                odd = (abs(float(c)) % 2.0) == 1.0
                out = np.where(neg & odd, -out, out)
            else:
                out = np.where(neg, np.float32(np.nan), out)
            return np.where(neg, out, np.power(x, c)).astype(F32)
    raise ValueError(op)


def relu(x):
    """shaders/activations/relu.wgsl: max(0, x)."""
    return np.maximum(np.asarray(x, F32), F32(0))


def gelu(x):
    """shaders/activations/gelu.wgsl:20-27: tanh form, x > 10 -> x, x < -10 -> 0."""
    x = np.asarray(x, F32).astype(np.float64)
    u = 0.7978845608 * (x + 0.044715 * x ** 3)
    y = 0.5 * x * (1.0 + np.tanh(u))
    y = np.where(x > 10.0, x, np.where(x < -10.0, 0.0, y))
    return y.astype(F32)


def sigmoid(x):
    """shaders/activations/sigmoid.wgsl:18-19: input clamped to [-88, 88]."""
    x = np.clip(np.asarray(x, F32).astype(np.float64), -88.0, 88.0)
    return (1.0 / (1.0 + np.exp(-x))).astype(F32)


def silu(x):
    """Tensor.py:724-727: sigmoid(x) * x."""
    return (sigmoid(x) * np.asarray(x, F32)).astype(F32)


def unary(x, name):
    x64 = np.asarray(x, F32).astype(np.float64)
    table = {
        "relu": relu, "gelu": gelu, "sigmoid": sigmoid, "silu": silu,
        "sin": lambda v: np.sin(x64), "cos": lambda v: np.cos(x64), "exp": lambda v: np.exp(x64),
        "log": lambda v: np.log(x64), "sqrt": lambda v: np.sqrt(x64),
        "rsqrt": lambda v: 1.0 / np.sqrt(x64), "abs": lambda v: np.abs(x64),
        "sign": lambda v: np.sign(x64), "negate": lambda v: -x64, "square": lambda v: x64 * x64,
    }
    with np.errstate(all="ignore"):
        return np.asarray(table[name](x), np.float64).astype(F32)


def embed(ids, weight):
    """shaders/layers/embed.wgsl:25-34: out[t, d] = W[ids[t], d] (bit-exact gather)."""
    return np.asarray(weight, F32)[np.asarray(ids, np.int64)]


def causal_conv1d(x, w, b):
    """shaders/helpers/causal_conv1d.wgsl:37-55:
    out[b, d, n] = bias[d] + sum_k w[d, k] * x[b, d, n - k] (float64 accumulation)."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    B, D, L = x.shape
    out = np.broadcast_to(np.asarray(b, np.float64)[None, :, None], (B, D, L)).copy()
    for k in range(w.shape[1]):
        out[:, :, k:] += w[:, k][None, :, None] * x[:, :, : L - k]
    return out.astype(F32)


def decay_window(decay, stage, length):
    """shaders/helpers/decay_window.wgsl:27-34: W[d, t] = exp(-|decay[stage, d]| * t)."""
    rate = np.abs(np.asarray(decay, np.float64)[stage])
    return np.exp(-rate[:, None] * np.arange(length)[None, :]).astype(F32)


def complex_mul(a, b, conj_a=False, conj_b=False):
    """shaders/helpers/complex_mul.wgsl:57-61 (broadcast)."""
    a = np.asarray(a, np.complex128)
    b = np.asarray(b, np.complex128)
    if conj_a:
        a = np.conj(a)
    if conj_b:
        b = np.conj(b)
    return (a * b).astype(np.complex64)


# ----------------------------------------------------------------- reductions

def reduce_dims(shape, axis):
    """backend/dispatch.py:173-214 _get_reduce_dims: (outer, reduce, inner, out_shape)."""
    nd = len(shape)
    if axis is None:
        return 1, int(np.prod(shape)), 1, (1,)
    axes = tuple(sorted(a % nd for a in ((axis,) if np.isscalar(axis) else axis)))
    if any(axes[i] != axes[i - 1] + 1 for i in range(1, len(axes))):
        raise ValueError("non-contiguous multi-axis reduction")
    lo, hi = axes[0], axes[-1]
    outer = int(np.prod(shape[:lo])) if lo else 1
    red = int(np.prod(shape[lo:hi + 1]))
    inner = int(np.prod(shape[hi + 1:])) if hi < nd - 1 else 1
    out_shape = tuple(s for d, s in enumerate(shape) if d not in axes) or (1,)
    return outer, red, inner, out_shape


def reduce(x, axis=None, mode=0, keepdims=False):
    """shaders/helpers/reduce.wgsl:31-66: mode 0 sum, 1 mean, 2 sum of squares
    (float64 accumulation; the reference accumulates fp32 in a 256-wide tree)."""
    x = np.asarray(x, F32)
    o, r, i, out_shape = reduce_dims(x.shape, axis)
    v = x.reshape(o, r, i).astype(np.float64)
    if mode == 2:
        v = v * v
    s = v.sum(axis=1)
    if mode == 1:
        s = s / r
    if keepdims:
        if axis is None:
            out_shape = (1,) * x.ndim
        else:
            axes = {a % x.ndim for a in ((axis,) if np.isscalar(axis) else axis)}
            out_shape = tuple(1 if d in axes else n for d, n in enumerate(x.shape))
    return s.reshape(out_shape).astype(F32)


def argminmax(x, axis=None, op=0):
    """shaders/helpers/reduce_minmax.wgsl:18-77, bit-exact including ties.

    For every output, 256 lanes scan r = lane, lane + 256, ... keeping the
    first strictly better value (start -1e38 for max, 1e38 for min, index 0);
    then a tree with strides 128, 64, ..., 1 where slot i takes slot i + s only
    if strictly better.  Returns (values f32, indices u32)."""
    x = np.asarray(x, F32)
    o, r, i, out_shape = reduce_dims(x.shape, axis)
    v = x.reshape(o, r, i).transpose(0, 2, 1).reshape(o * i, r)
    init = F32(-1e38) if op == 0 else F32(1e38)
    better = (lambda a, b: a > b) if op == 0 else (lambda a, b: a < b)
    rows = v.shape[0]
    pad = (-r) % 256
    vp = np.concatenate([v, np.full((rows, pad), np.nan, F32)], axis=1) if pad else v
    lanes = vp.reshape(rows, -1, 256)               # [rows, steps, lane]
    best = np.full((rows, 256), init, F32)
    arg = np.zeros((rows, 256), np.uint32)
    for step in range(lanes.shape[1]):
        cand = lanes[:, step, :]
        take = better(cand, best)                   # NaN compares false
        best = np.where(take, cand, best)
        arg = np.where(take, np.uint32(step * 256) + np.arange(256, dtype=np.uint32), arg)
    s = 128
    while s >= 1:
        lo_v, hi_v = best[:, :s], best[:, s:2 * s]
        take = better(hi_v, lo_v)
        best[:, :s] = np.where(take, hi_v, lo_v)
        arg[:, :s] = np.where(take, arg[:, s:2 * s], arg[:, :s])
        s //= 2
    return best[:, 0].reshape(out_shape), arg[:, 0].reshape(out_shape).astype(np.uint32)


def softmax(x, dim=-1):
    """shaders/activations/softmax.wgsl:55-74 (max init -1e38; float64 math)."""
    x = np.asarray(x, F32).astype(np.float64)
    m = np.maximum(x.max(axis=dim, keepdims=True), -1e38)
    e = np.exp(x - m)
    return (e / e.sum(axis=dim, keepdims=True)).astype(F32)


def layernorm(x, gamma, beta, axis=-1, eps=1e-5):
    """shaders/layers/meanvarnorm.wgsl:40-102: inv = var > 0 ? rsqrt(var + eps) : 0,
    y = (x - mean) * inv * gamma + beta (float64 statistics).  Returns (y, mean, inv)."""
    x = np.asarray(x, F32)
    o, r, i, out_shape = reduce_dims(x.shape, axis)
    v = x.reshape(o, r, i).astype(np.float64)
    mean = v.mean(axis=1, keepdims=True)
    var = np.maximum(((v - mean) ** 2).mean(axis=1, keepdims=True), 0.0)
    inv = np.where(var > 0, 1.0 / np.sqrt(var + eps), 0.0)
    g = np.asarray(gamma, np.float64).reshape(1, r, 1)
    b = np.asarray(beta, np.float64).reshape(1, r, 1)
    y = (v - mean) * inv * g + b
    return (y.reshape(x.shape).astype(F32), mean.reshape(out_shape).astype(F32),
            inv.reshape(out_shape).astype(F32))


def rmsnorm(x, gamma, axis=-1, eps=1e-6):
    """shaders/layers/rmsnorm.wgsl:30-78: inv = ms > 0 ? rsqrt(ms + eps) : 0,
    y = x * inv * gamma.  Returns (y, inv).  Rows beyond 65535 are normalised
    (the reference's grid leaves them unwritten, rmsnorm.wgsl:23-24)."""
    x = np.asarray(x, F32)
    o, r, i, out_shape = reduce_dims(x.shape, axis)
    v = x.reshape(o, r, i).astype(np.float64)
    ms = (v * v).mean(axis=1, keepdims=True)
    inv = np.where(ms > 0, 1.0 / np.sqrt(ms + eps), 0.0)
    y = v * inv * np.asarray(gamma, np.float64).reshape(1, r, 1)
    return y.reshape(x.shape).astype(F32), inv.reshape(out_shape).astype(F32)


def batchnorm_eval(x, gamma, beta, rmean, rvar, eps=1e-5):
    """shaders/layers/batchnorm.wgsl:112-131: (x - rm) * rsqrt(rv + eps) * g + b;
    the reference's running_std buffer holds a variance (nn/module.py:238)."""
    x = np.asarray(x, np.float64)
    sh = (1, -1) + (1,) * (x.ndim - 2)
    inv = 1.0 / np.sqrt(np.asarray(rvar, np.float64) + eps)
    y = (x - np.asarray(rmean, np.float64).reshape(sh)) * inv.reshape(sh)
    return (y * np.asarray(gamma, np.float64).reshape(sh)
            + np.asarray(beta, np.float64).reshape(sh)).astype(F32)


# ----------------------------------------------------------------- contractions

def matmul_add(a, b, bias=None, transpose_a=False, transpose_b=False):
    """shaders/matmul.wgsl:59-146 + functional/utils.py:378-499: batched
    op(A) @ op(B) (+ bias, modes (N,), (M,N), (batch,M,N)); an unbatched side
    broadcasts.  float64 accumulation."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    if transpose_a:
        a = np.swapaxes(a, -1, -2)
    if transpose_b:
        b = np.swapaxes(b, -1, -2)
    out = np.matmul(a, b)
    if bias is not None:
        out = out + np.asarray(bias, np.float64)
    return out.astype(F32)


def conv2d(x, w, stride=(1, 1), padding=(0, 0), dilation=(1, 1), bias=None):
    """shaders/layers/conv2d.wgsl:32-116: NCHW cross-correlation, zero padding,
    Ho = (H + 2p - d(k-1) - 1) // s + 1 (functional/convolution.py:679-680).
    float64 accumulation via an explicit im2col."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    B, C, H, W = x.shape
    O, _, KH, KW = w.shape
    sh, sw = stride
    ph, pw = padding
    dh, dw = dilation
    Ho = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    Wo = (W + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    xp = np.pad(x, ((0, 0), (0, 0), (ph, ph), (pw, pw)))
    cols = np.empty((B, C, KH, KW, Ho, Wo))
    for i in range(KH):
        for j in range(KW):
            hs, ws = i * dh, j * dw
            cols[:, :, i, j] = xp[:, :, hs:hs + sh * (Ho - 1) + 1:sh, ws:ws + sw * (Wo - 1) + 1:sw]
    out = np.einsum("bckhyx,ockh->boyx", cols.reshape(B, C, KH, KW, Ho, Wo), w, optimize=True)
    if bias is not None:
        out = out + np.asarray(bias, np.float64)[None, :, None, None]
    return out.astype(F32)


def maxpool2d(x, kernel, stride, padding):
    """shaders/layers/maxpool2d.wgsl:35-74: padding excluded, first strictly greater
    value wins (init -1e38, index 0xFFFFFFFF).  Returns (values, flat indices)."""
    x = np.asarray(x, F32)
    B, C, H, W = x.shape
    KH, KW = kernel
    sh, sw = stride
    ph, pw = padding
    Ho = (H + 2 * ph - KH) // sh + 1
    Wo = (W + 2 * pw - KW) // sw + 1
    best = np.full((B, C, Ho, Wo), F32(-1e38))
    arg = np.full((B, C, Ho, Wo), 0xFFFFFFFF, np.uint32)
    plane = (np.arange(B)[:, None] * C + np.arange(C)[None, :]) * (H * W)
    for kh in range(KH):
        for kw in range(KW):
            ih = np.arange(Ho) * sh - ph + kh
            iw = np.arange(Wo) * sw - pw + kw
            vh = (ih >= 0) & (ih < H)
            vw = (iw >= 0) & (iw < W)
            ihc, iwc = np.clip(ih, 0, H - 1), np.clip(iw, 0, W - 1)
            cand = x[:, :, ihc][:, :, :, iwc]
            valid = vh[:, None] & vw[None, :]
            take = valid[None, None] & (cand > best)
            best = np.where(take, cand, best)
            flat = plane[:, :, None, None] + (ihc[:, None] * W + iwc[None, :])[None, None]
            arg = np.where(take, flat.astype(np.uint32), arg)
    return best, arg


def adaptive_avgpool2d(x, out_hw):
    """shaders/layers/adaptive_avgpool2d.wgsl:26-51: windows
    [floor(o*in/out), ceil((o+1)*in/out)) per axis (float64 mean)."""
    x = np.asarray(x, np.float64)
    B, C, H, W = x.shape
    Ho, Wo = out_hw
    out = np.empty((B, C, Ho, Wo))
    for oh in range(Ho):
        hs, he = (oh * H) // Ho, -((-(oh + 1) * H) // Ho)
        for ow in range(Wo):
            ws, we = (ow * W) // Wo, -((-(ow + 1) * W) // Wo)
            out[:, :, oh, ow] = x[:, :, hs:he, ws:we].mean(axis=(2, 3))
    return out.astype(F32)


# ----------------------------------------------------------------- FFT

def rfft(x, n):
    """functional/fft.py:484-563 (fft_bitrev_real + fft_stage + fft_copy_out):
    numpy.fft.rfft semantics, zero-pad / truncate to n (float64)."""
    return np.fft.rfft(np.asarray(x, np.float64), n).astype(np.complex64)


def irfft(X, n):
    """functional/fft.py:566-645 (fft_bitrev_complex + fft_stage + ifft_write_real):
    Hermitian expansion of the first n//2+1 bins (missing bins are zero), inverse
    transform, Re(.)/n -- i.e. numpy.fft.irfft (float64)."""
    return np.fft.irfft(np.asarray(X, np.complex128), n).astype(F32)


def fftconv(x, h, n, out_len=None):
    """nn/hyena.py:208-216 fft_conv1d: irfft(rfft(x, n) * rfft(h, n), n)[..., :L]
    with h (D, Lh) broadcast over the batch (float64)."""
    x = np.asarray(x, np.float64)
    L = x.shape[-1] if out_len is None else out_len
    spec = np.fft.rfft(x, n) * np.fft.rfft(np.asarray(h, np.float64), n)
    return np.fft.irfft(spec, n)[..., :L].astype(F32)
