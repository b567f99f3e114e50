"""Tensor utilities: matmul, copies, views, creation and init helpers.

Reference: src/wxx/functional/utils.py (same names, arguments and errors).
"""

import math

import numpy as np

from .. import validation
from ..Tensor import Tensor, _from_host
from ._common import F, active_timer, arr64, check, dense, empty, matmul_mode_code, rng


def assign(tensor1, val):
    """Copies ``val`` (a tensor of the same shape and dtype, or a scalar) into
    the view ``tensor1`` in place (functional/utils.py:29-101).

    The source view's own offset and strides are honoured (the reference reads
    the source from offset 0)."""
    validation.check_rank(tensor1.shape, name="assign target")
    rank = len(tensor1.shape)
    shape = arr64(tensor1.shape)
    dstride = arr64(tensor1.stride)
    if isinstance(val, (float, int)) and not isinstance(val, bool):
        if tensor1.type == "c64":
            raise TypeError("scalar assign into a c64 tensor is not supported")
        if tensor1.type == "u32":
            bits = int(val) & 0xFFFFFFFF
        else:
            bits = int(np.array([val], dtype=np.float32).view(np.uint32)[0])
        check(F.wxx_strided_fill(tensor1.buffer.ptr, tensor1.offset, dstride, rank, shape, bits),
              "assign")
        mark_written(tensor1)
        return tensor1
    if not isinstance(val, Tensor):
        raise TypeError(f"assign expects a Tensor or a scalar, got {type(val).__name__}")
    if tuple(val.shape) != tuple(tensor1.shape):
        raise ValueError(
            f"assign shape mismatch: target {tuple(tensor1.shape)} vs source {tuple(val.shape)}"
        )
    if val.type != tensor1.type:
        raise TypeError(f"assign dtype mismatch: target {tensor1.type!r} vs source {val.type!r}")
    check(F.wxx_strided_copy(tensor1.buffer.ptr, tensor1.offset, dstride, val.buffer.ptr,
                             val.offset, arr64(val.stride), rank, shape, tensor1.itemsize()),
          "assign")
    mark_written(tensor1)
    return tensor1


def mark_written(tensor):
    """Records an in-place write into ``tensor``'s storage (its buffer's
    version), so copies derived from it (``kmajor_weight``) are rebuilt."""
    buf = tensor.buffer
    if buf is not None and hasattr(buf, "version"):
        buf.version += 1


def permute(tensor1, *axes):
    if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
        axes = tuple(axes[0])
    rank = len(tensor1.shape)
    if len(axes) != rank:
        raise ValueError(
            f"permute expects {rank} axes for shape {tuple(tensor1.shape)}, got {len(axes)}"
        )
    axes = validation.normalize_dims(axes, rank, name="axes", allow_duplicates=False)
    return Tensor._wrap([tensor1.shape[i] for i in axes], tensor1.buffer, tensor1.type,
                        tensor1.requires_grad, [tensor1.stride[i] for i in axes],
                        tensor1.offset, tensor1)


def diagonal(tensor1, offset=0, dim1=0, dim2=1):
    rank = len(tensor1.shape)
    if rank < 2:
        raise ValueError(f"diagonal expects at least 2 dimensions, got shape {tuple(tensor1.shape)}")
    if not isinstance(offset, int) or isinstance(offset, bool):
        raise TypeError(f"offset must be an int, got {type(offset).__name__}")
    d1 = validation.normalize_dim(dim1, rank, name="dim1")
    d2 = validation.normalize_dim(dim2, rank, name="dim2")
    if d1 == d2:
        raise ValueError(f"dim1 and dim2 must differ, got {d1} and {d2}")
    rows, cols = tensor1.shape[d1], tensor1.shape[d2]
    if offset >= 0:
        r0, c0, length = 0, offset, min(rows, cols - offset)
    else:
        r0, c0, length = -offset, 0, min(rows + offset, cols)
    if length <= 0:
        r0 = c0 = length = 0
    shape = [s for a, s in enumerate(tensor1.shape) if a not in (d1, d2)] + [length]
    stride = [s for a, s in enumerate(tensor1.stride) if a not in (d1, d2)]
    stride.append(tensor1.stride[d1] + tensor1.stride[d2])
    off = tensor1.offset + r0 * tensor1.stride[d1] + c0 * tensor1.stride[d2]
    return Tensor._wrap(shape, tensor1.buffer, tensor1.type, tensor1.requires_grad, stride, off,
                        tensor1)


def unfold(tensor1, dimension, size, step=1):
    rank = len(tensor1.shape)
    dim = validation.normalize_dim(dimension, rank, name="dimension")
    if isinstance(size, bool) or not isinstance(size, int):
        raise TypeError(f"size must be an int, got {type(size).__name__}")
    if isinstance(step, bool) or not isinstance(step, int):
        raise TypeError(f"step must be an int, got {type(step).__name__}")
    if size < 1:
        raise ValueError(f"size must be positive, got {size}")
    if step < 1:
        raise ValueError(f"step must be positive, got {step}")
    if rank + 1 > validation.MAX_RANK:
        raise ValueError(
            f"unfold would produce rank {rank + 1}, but the maximum supported rank is "
            f"{validation.MAX_RANK}"
        )
    length = tensor1.shape[dim]
    if size > length:
        raise ValueError(f"size {size} is larger than dimension {dim} of size {length}")
    shape = list(tensor1.shape)
    shape[dim] = (length - size) // step + 1
    shape.append(size)
    stride = list(tensor1.stride)
    stride[dim] *= step
    stride.append(tensor1.stride[dim])
    return Tensor._wrap(shape, tensor1.buffer, tensor1.type, tensor1.requires_grad, stride,
                        tensor1.offset, tensor1)


def reshape(tensor1, new_shape):
    total = validation.numel(tensor1.shape)
    new_shape = validation.infer_shape(new_shape, total, name="new shape")
    src = dense(tensor1)
    return Tensor._wrap(list(new_shape), src.buffer, tensor1.type, tensor1.requires_grad, None,
                        src.offset, src)


def contiguous(tensor1):
    """``tensor1`` when contiguous, else a dense copy (functional/utils.py:316-369)."""
    if tensor1.is_contiguous():
        return tensor1
    rank = validation.check_rank(tensor1.shape, max_rank=8, name="contiguous input")
    out = empty(tensor1.shape, tensor1.type, tensor1.requires_grad)
    check(F.wxx_strided_copy(out.buffer.ptr, 0, arr64(out.stride), tensor1.buffer.ptr,
                             tensor1.offset, arr64(tensor1.stride), rank, arr64(tensor1.shape),
                             tensor1.itemsize()), "contiguous")
    return out


def matmul_add(tensor1, tensor2, tensor3, transpose_A=False, transpose_B=False, *, alpha=1.0):
    """Batched ``op(A) @ op(B) (+ bias)`` (functional/utils.py:378-499).

    Shapes, batch broadcasting (equal batch shapes, or one side unbatched) and
    the four bias modes follow the reference.  The product runs on the tcgen05
    TF32 tensor cores (see ``set_matmul_mode``); ``alpha`` scales the product
    before the bias is added (used to fold attention's 1/sqrt(d) into QK^T).
    """
    validation.check_rank(tensor1.shape, min_rank=2, name="matmul left operand")
    validation.check_rank(tensor2.shape, min_rank=2, name="matmul right operand")
    a = dense(tensor1)
    b = dense(tensor2)
    if transpose_A:
        M, K = a.shape[-1], a.shape[-2]
    else:
        M, K = a.shape[-2], a.shape[-1]
    if transpose_B:
        K_B, N = b.shape[-1], b.shape[-2]
    else:
        K_B, N = b.shape[-2], b.shape[-1]
    if K != K_B:
        raise ValueError(f"Inner dimension mismatch: {K} vs {K_B}")
    batch_a = list(a.shape[:-2])
    batch_b = list(b.shape[:-2])
    if batch_a and batch_b and batch_a != batch_b:
        raise ValueError(
            f"Batch dimensions must match or be unbatched: {batch_a} vs {batch_b}"
        )
    out_batch = batch_a or batch_b
    batch = int(math.prod(out_batch)) if out_batch else 1
    a_bs = M * K if batch_a else 0
    b_bs = K * N if batch_b else 0
    bias_mode = 0
    bias_ptr = None
    if tensor3 is not None and tensor3.shape is not None:
        bias = dense(tensor3)
        bshape = tuple(bias.shape)
        if bshape == (N,):
            bias_mode = 1
        elif bshape == (M, N):
            bias_mode = 2
        elif bshape == tuple(out_batch) + (M, N):
            bias_mode = 3
        else:
            raise ValueError(
                f"Bias shape {bshape} is not broadcastable to {tuple(out_batch) + (M, N)}"
            )
        bias_ptr = bias.ptr
    requires_grad = (
        tensor1.requires_grad or tensor2.requires_grad
        or (tensor3 is not None and tensor3.requires_grad)
    )
    out = empty(out_batch + [M, N], "f32", requires_grad)
    lda = M if transpose_A else K
    ldb = K if transpose_B else N
    timer = active_timer()
    ev0 = timer.start() if timer is not None else None
    check(F.wxx_matmul(out.buffer.ptr, a.ptr, b.ptr, bias_ptr, batch, M, N, K, a_bs, b_bs, lda,
                       ldb, int(bool(transpose_A)), int(bool(transpose_B)), bias_mode,
                       float(alpha), matmul_mode_code()), "matmul_add")
    if timer is not None:
        timer.stop(ev0, 2.0 * batch * M * N * K, f"{batch}x{M}x{N}x{K}")
    return out


_ACTIVATIONS = {None: 0, "gelu": 1, "swiglu": 2}


def _linear_batch_transposed(x, weight, bias, activation, residual, feeds_tf32=False):
    """``linear`` for a (B, M, K) view of a dense (B, K, M) activation (Hyena's
    ``out_proj(z.transpose(1, 2))``, nn/hyena.py:242): the GEMM reads each
    batch's A as a transposed (MN-major) operand instead of copying the view.
    None when the input is not such a view or the fused form does not apply."""
    if len(x.shape) != 3 or activation not in (None, "gelu"):
        return None
    B, M, K = x.shape
    if x.stride[1] != 1 or x.stride[2] != M or M < 2 or K < 2:
        return None
    w = dense(weight)
    N = w.shape[-1]
    mode = matmul_mode_code()
    if (len(w.shape) != 2 or w.shape[0] != K or mode not in (0, 1) or N % 4
            or (mode == 1 and K > 1024)):
        return None
    if bias is not None and tuple(bias.shape) != (N,):
        raise ValueError(f"linear: bias {tuple(bias.shape)} is not ({N},)")
    if residual is not None and tuple(residual.shape) != (B, M, N):
        raise ValueError(f"linear: residual {tuple(residual.shape)} is not {(B, M, N)}")
    requires_grad = (x.requires_grad or weight.requires_grad
                     or (bias is not None and bias.requires_grad)
                     or (residual is not None and residual.requires_grad))
    out = empty([B, M, N], "f32", requires_grad)
    b = dense(bias) if bias is not None else None
    r = dense(residual) if residual is not None else None
    timer = active_timer()
    ev0 = timer.start() if timer is not None else None
    check(F.wxx_linear_batched(out.buffer.ptr, x.ptr, w.ptr, None if b is None else b.ptr,
                               None if r is None else r.ptr, B, M, N, K, x.stride[0], M, 1, N, 0,
                               _ACTIVATIONS[activation], 1.0,
                               3 if (feeds_tf32 and mode == 0) else mode), "linear")
    if timer is not None:
        timer.stop(ev0, 2.0 * B * M * N * K, f"{B}x{M}x{N}x{K}T")
    return out


def linear(x, weight, bias=None, *, activation=None, residual=None, transpose_weight=False,
           feeds_tf32=False):
    """``act(x @ weight + bias) + residual`` with the activation and the
    residual add fused into the GEMM epilogue.

    ``x`` (..., K), ``weight`` (K, N) (nn.Linear layout), ``bias`` (N,) or
    None, ``residual`` shaped like the output or None.  ``activation``:
    None, ``"gelu"`` (tanh form) or ``"swiglu"``: the weight's columns 2j and
    2j+1 hold the gate and the up projection of output column j, and the
    (..., N/2) result is ``silu(gate) * up`` (SwiGLU's ``silu(x W1) * (x W2)``
    from one GEMM; no residual).  The result has the same bits as
    ``matmul_add`` followed by the activation / ``residual + y``, which is the
    path taken when the fused form does not apply (fp32 SIMT mode, N not a
    multiple of 4, 3xTF32 with K > 1024).

    ``transpose_weight``: ``weight`` is given as (N, K) (output, input), i.e.
    the transpose of the nn.Linear layout, and the GEMM reads it as a K-major
    operand -- the faster tensor-core operand form (~15 % on GPT2's K = 1024
    products); the result is ``x @ weight.T``.

    ``feeds_tf32``: the result is read only by TF32 tensor-core products (the
    next GEMM or the attention kernel), so in tf32 mode it is stored rounded
    to the nearest TF32 value, which that product then reads exactly (it would
    otherwise truncate it); no effect in 3xtf32 / fp32 modes."""
    if activation not in _ACTIVATIONS:
        raise ValueError(f"activation must be None, 'gelu' or 'swiglu', got {activation!r}")
    if not transpose_weight:
        y = _linear_batch_transposed(x, weight, bias, activation, residual, feeds_tf32)
        if y is not None:
            return y
    a = dense(x)
    w = dense(weight)
    K = a.shape[-1]
    N = w.shape[0] if transpose_weight else w.shape[-1]
    if len(w.shape) != 2 or w.shape[1 if transpose_weight else 0] != K:
        raise ValueError(f"linear: weight {tuple(w.shape)} does not match input {tuple(a.shape)}")
    glu = activation == "swiglu"
    if glu and (N % 2 or residual is not None):
        raise ValueError("linear: 'swiglu' needs an even output width and no residual")
    out_shape = list(a.shape[:-1]) + [N // 2 if glu else N]
    if bias is not None and tuple(bias.shape) != (N,):
        raise ValueError(f"linear: bias {tuple(bias.shape)} is not ({N},)")
    if residual is not None and list(residual.shape) != out_shape:
        raise ValueError(f"linear: residual {tuple(residual.shape)} is not {tuple(out_shape)}")
    mode = matmul_mode_code()
    M = int(math.prod(a.shape[:-1])) if len(a.shape) > 1 else 1
    # 3xTF32 products with K > 1024 are summed in slices (split-K) to bound
    # the tensor-core accumulation chain; that path has no fused epilogue.
    if (mode not in (0, 1) or N % (8 if glu else 4) or K == 0 or (mode == 1 and K > 1024)):
        y = matmul_add(x, weight, bias, transpose_B=transpose_weight)
        if activation == "gelu":
            y = y.gelu()
        elif glu:
            from .activations import silu
            y = silu(y[..., 0::2]) * y[..., 1::2]
        return y if residual is None else residual + y
    requires_grad = (x.requires_grad or weight.requires_grad
                     or (bias is not None and bias.requires_grad)
                     or (residual is not None and residual.requires_grad))
    out = empty(out_shape, "f32", requires_grad)
    if M == 0:
        return out
    b = dense(bias) if bias is not None else None
    r = dense(residual) if residual is not None else None
    timer = active_timer()
    ev0 = timer.start() if timer is not None else None
    check(F.wxx_linear(out.buffer.ptr, a.ptr, w.ptr, None if b is None else b.ptr,
                       None if r is None else r.ptr, M, N, K, K, K if transpose_weight else N,
                       int(bool(transpose_weight)), _ACTIVATIONS[activation], 1.0,
                       3 if (feeds_tf32 and mode == 0) else mode), "linear")
    if timer is not None:
        timer.stop(ev0, 2.0 * M * N * K, f"{M}x{N}x{K}")
    return out


_E_UNSUPPORTED = -4


def linear_argmax(x, weight, *, transpose_weight=False):
    """``max(x @ weight, -1)[1]`` (or ``x @ weight.T`` with
    ``transpose_weight``) without storing the product: the u32 index of each
    row's maximum, shaped ``x.shape[:-1]``, with the argmax kernel's tie rule.
    For GPT2's forward when its output is the next-token id of every
    position (the LM head's 1.65 GB of logits at the GPT2-scaled shape are
    then neither written nor read back).  None (nothing launched) when the
    product is not one the fused epilogue takes (few output tiles, operands
    the tensor memory accelerator cannot address): compute the product and
    ``max`` it then."""
    a = dense(x)
    w = dense(weight)
    K = a.shape[-1]
    if len(w.shape) != 2 or w.shape[1 if transpose_weight else 0] != K:
        raise ValueError(f"linear_argmax: weight {tuple(w.shape)} does not match input "
                         f"{tuple(a.shape)}")
    N = w.shape[0] if transpose_weight else w.shape[1]
    M = int(math.prod(a.shape[:-1])) if len(a.shape) > 1 else 1
    out = empty(list(a.shape[:-1]), "u32")
    mode = matmul_mode_code()
    if M:
        timer = active_timer()
        ev0 = timer.start() if timer is not None else None
        st = F.wxx_matmul_argmax(out.buffer.ptr, None, a.ptr, w.ptr, 1, M, N, K, 0, 0, K,
                                 K if transpose_weight else N, 0, int(bool(transpose_weight)),
                                 mode if mode in (0, 1, 2) else 0)
        if st == _E_UNSUPPORTED:
            return None
        check(st, "linear_argmax")
        if timer is not None:
            timer.stop(ev0, 2.0 * M * N * K, f"{M}x{N}x{K} argmax")
    return out


def ln_linear(x, gamma, beta, weight, bias=None, *, activation=None, residual=None,
              feeds_tf32=False, eps=1e-5):
    """``linear(LayerNorm(x), weight, bias, ...)`` with ``weight`` given as
    (N, K) (``transpose_weight=True`` layout) and the LayerNorm over x's last
    axis (``gamma``, ``beta``): for a few rows (at most 32, the decode step)
    one launch normalises the rows and streams the weight; otherwise, or for
    shapes that kernel does not take, the LayerNorm kernel and ``linear``."""
    from .normalization import meanvarnorm

    a = dense(x)
    K = a.shape[-1]
    w = dense(weight)
    N = w.shape[0]
    M = int(math.prod(a.shape[:-1])) if len(a.shape) > 1 else 1
    mode = matmul_mode_code()
    if (activation in (None, "gelu") and len(w.shape) == 2 and w.shape[1] == K
            and tuple(gamma.shape) == (K,) and tuple(beta.shape) == (K,) and mode in (0, 1, 2)
            and 1 <= M <= 32):
        out_shape = list(a.shape[:-1]) + [N]
        if residual is not None and list(residual.shape) != out_shape:
            raise ValueError(f"ln_linear: residual {tuple(residual.shape)} is not {out_shape}")
        if bias is not None and tuple(bias.shape) != (N,):
            raise ValueError(f"ln_linear: bias {tuple(bias.shape)} is not ({N},)")
        out = empty(out_shape, "f32")
        g, bt = dense(gamma), dense(beta)
        b = dense(bias) if bias is not None else None
        r = dense(residual) if residual is not None else None
        st = F.wxx_ln_linear(out.buffer.ptr, a.ptr, K, g.ptr, bt.ptr, float(eps), w.ptr, K,
                             None if b is None else b.ptr, None if r is None else r.ptr, M, N, K,
                             _ACTIVATIONS[activation], int(bool(feeds_tf32) and mode == 0))
        if st != _E_UNSUPPORTED:
            check(st, "ln_linear")
            return out
    axis = len(x.shape) - 1
    h = meanvarnorm(x, gamma, beta, axis, feeds_tf32=True)[0]
    return linear(h, weight, bias, activation=activation, residual=residual,
                  transpose_weight=True, feeds_tf32=feeds_tf32)


def transpose_stack(out, weights, *, round_tf32=False):
    """Writes the transposes of ``weights`` (n <= 8 dense-able (K, N) tensors
    of one shape) stacked along rows into the dense (n * N, K) tensor ``out``
    with one kernel launch (values rounded to the nearest TF32 value when
    ``round_tf32``).  False (nothing written) when the shapes do not allow
    it."""
    import ctypes

    n = len(weights)
    if n < 1 or n > 8 or not out.is_dense() or out.type != "f32":
        return False
    K, N = weights[0].shape
    if any(tuple(w.shape) != (K, N) or w.type != "f32" for w in weights):
        return False
    if tuple(out.shape) != (n * N, K):
        return False
    ws = [dense(w) for w in weights]
    srcs = (ctypes.c_void_p * n)(*[w.ptr for w in ws])
    check(F.wxx_transpose_stack(out.ptr, srcs, n, K, N, int(bool(round_tf32))),
          "transpose_stack")
    return True


def linear_short_conv(x, weight, bias, conv_weight, conv_bias):
    """Hyena's projection + transpose + short causal conv (nn/hyena.py:227-234)
    as one tcgen05 GEMM whose epilogue applies the taps and writes channels
    first: ``x`` (B, L, K), ``weight`` (K, N), ``bias`` (N,) or None,
    ``conv_weight`` (C, k), ``conv_bias`` (C,) with column c using conv row
    c % C.  Returns (B, N, L) = ``causal_conv1d(linear(x, weight,
    bias).transpose(1, 2))`` with the conv weights tiled over N.  That
    composition (CUDA kernels too) is taken when the fused kernel does not
    apply: fp32 SIMT mode, more than four taps, or operands the tensor memory
    accelerator cannot address."""
    if len(x.shape) != 3:
        raise ValueError(f"linear_short_conv expects a (B, L, K) input, got {x.shape}")
    Bsz, L, K = x.shape
    w = dense(weight)
    if len(w.shape) != 2 or w.shape[0] != K:
        raise ValueError(f"linear_short_conv: weight {tuple(w.shape)} does not match input {x.shape}")
    N = w.shape[1]
    if len(conv_weight.shape) != 2 or tuple(conv_bias.shape) != (conv_weight.shape[0],):
        raise ValueError("linear_short_conv: conv weight must be (C, k) with a (C,) bias")
    C, taps = conv_weight.shape
    if N % C:
        raise ValueError(f"linear_short_conv: {N} output columns are not a multiple of {C} channels")
    if bias is not None and tuple(bias.shape) != (N,):
        raise ValueError(f"linear_short_conv: bias {tuple(bias.shape)} is not ({N},)")
    mode = matmul_mode_code()
    grad = (x.requires_grad or weight.requires_grad or conv_weight.requires_grad
            or conv_bias.requires_grad or (bias is not None and bias.requires_grad))
    if mode in (0, 1) and 1 <= taps <= 4 and K > 0 and Bsz * L * N > 0:
        a = dense(x)
        cw = dense(conv_weight)
        cb = dense(conv_bias)
        b = dense(bias) if bias is not None else None
        out = empty([Bsz, N, L], "f32", grad)
        timer = active_timer()
        ev0 = timer.start() if timer is not None else None
        st = F.wxx_linear_short_conv(out.buffer.ptr, a.ptr, w.ptr, None if b is None else b.ptr,
                                     Bsz * L, N, K, K, N, 0, L, cw.ptr, cb.ptr, C, taps, mode)
        if st == 0:
            if timer is not None:
                timer.stop(ev0, 2.0 * Bsz * L * N * K, f"{Bsz * L}x{N}x{K}conv")
            return out
        if st != _E_UNSUPPORTED:
            check(st, "linear_short_conv")
    from .convolution import causal_conv1d
    y = linear(x, weight, bias).transpose(1, 2)
    if C == N:
        return causal_conv1d(y, conv_weight, conv_bias)
    parts = [causal_conv1d(y[:, i * C:(i + 1) * C, :], conv_weight, conv_bias)
             for i in range(N // C)]
    return concat(parts, 1)


def _equal_impl(tensor1, tensor2, mode, number=0):
    a = dense(tensor1)
    b = dense(tensor2) if tensor2 is not None else None
    out = empty(a.shape, "f32", tensor1.requires_grad)
    n = validation.numel(a.shape)
    check(F.wxx_equal(out.buffer.ptr, a.ptr, None if b is None else b.ptr, n, mode,
                      int(number) & 0xFFFFFFFF), "equal")
    return out


def equal(tensor1, tensor2):
    if isinstance(tensor2, (int, float)):
        return equal_number(tensor1, tensor2)
    if tensor1.type not in ("f32", "u32") or tensor1.type != tensor2.type:
        raise TypeError(
            f"equal expects matching f32 or u32 tensors, got {tensor1.type!r} and {tensor2.type!r}"
        )
    if tuple(tensor1.shape) != tuple(tensor2.shape):
        raise ValueError(f"equal expects equal shapes, got {tensor1.shape} and {tensor2.shape}")
    return _equal_impl(tensor1, tensor2, 0 if tensor1.type == "f32" else 1)


def equal_number(tensor1, number):
    if tensor1.type == "f32":
        bits = int(np.array([number], dtype=np.float32).view(np.uint32)[0])
        return _equal_impl(tensor1, None, 2, bits)
    if tensor1.type == "u32":
        return _equal_impl(tensor1, None, 3, int(number))
    raise TypeError(f"equal_number expects an f32 or u32 tensor, got {tensor1.type!r}")


def masked_fill(tensor1, number):
    """Keeps nonzero elements and writes ``number`` where the input is zero
    (maskedfill.wgsl: ``select(fill, x, x != 0)``)."""
    x = dense(tensor1)
    out = empty(x.shape, "f32", tensor1.requires_grad)
    check(F.wxx_scalar(out.buffer.ptr, x.ptr, validation.numel(x.shape), 5, float(number), 0),
          "masked_fill")
    return out


def linspace(start, end, steps):
    return from_numpy(np.linspace(start, end, int(steps), dtype=np.float32))


def ones_like(tensor1):
    return Tensor(tensor1.shape, value=1)


def arange(start, shape):
    if isinstance(shape, int):
        shape = (shape,)
    shape = tuple(shape)
    total = int(math.prod(shape))
    values = (np.arange(total) % shape[-1] + start).astype(np.float32)
    return from_numpy(values.reshape(shape))


def normal(mu, sigma, shape):
    if isinstance(shape, int):
        shape = (shape,)
    shape = tuple(shape)
    values = rng().normal(mu, sigma, size=int(math.prod(shape))).astype(np.float32)
    return from_numpy(values.reshape(shape))


def uniform(a, b, shape):
    if isinstance(shape, int):
        shape = (shape,)
    shape = tuple(shape)
    values = rng().uniform(a, b, size=int(math.prod(shape))).astype(np.float32)
    return from_numpy(values.reshape(shape))


def from_numpy(array, dtype=np.float32):
    """Uploads a NumPy array (``np.float32`` default, or ``np.uint32``)."""
    if dtype == np.uint32:
        return _from_host(np.asarray(array), "u32")
    return _from_host(np.asarray(array, dtype=np.float32), "f32")


def from_tensor(array, type=np.float32):
    if hasattr(array, "detach"):
        array = array.detach().cpu().contiguous().numpy()
    array = np.asarray(array, dtype=type, order="C")
    return from_numpy(array, dtype=np.uint32 if type == np.uint32 else np.float32)


def concat(tensors, dim):
    tensors = list(tensors)
    if not tensors:
        raise ValueError("concat expects at least one tensor")
    rank = len(tensors[0].shape)
    dim = validation.normalize_dim(dim, rank, name="dim")
    for t in tensors[1:]:
        if len(t.shape) != rank or any(
            t.shape[i] != tensors[0].shape[i] for i in range(rank) if i != dim
        ):
            raise ValueError("concat: tensors must match except along dim")
    shape = list(tensors[0].shape)
    shape[dim] = sum(t.shape[dim] for t in tensors)
    out = empty(shape, tensors[0].type, any(t.requires_grad for t in tensors))
    start = 0
    for t in tensors:
        assign(out.narrow(dim, start, t.shape[dim]), t)
        start += t.shape[dim]
    return out


def _zero_init(tensor):
    assign(tensor, 0.0)


def _xavier_normal_init(tensor, fan_in, fan_out):
    assign(tensor, normal(0, math.sqrt(2 / (fan_in + fan_out)), tensor.shape))


def _xavier_uniform_init(tensor, fan_in, fan_out):
    a = math.sqrt(6 / (fan_in + fan_out))
    assign(tensor, uniform(-a, a, tensor.shape))


def _kaiming_normal_init(tensor, fan_in):
    assign(tensor, normal(0, math.sqrt(2 / fan_in), tensor.shape))


def _kaiming_uniform_init(tensor, fan_in):
    a = math.sqrt(6 / fan_in)
    assign(tensor, uniform(-a, a, tensor.shape))


def scatter_zeros(grad, out_shape, dim, start):
    """Zero tensor of ``out_shape`` with ``grad`` written at ``start`` along ``dim``."""
    out_shape = list(validation.normalize_shape(out_shape, name="out_shape"))
    rank = validation.check_rank(out_shape, name="scatter_zeros output")
    dim = validation.normalize_dim(dim, rank, name="dim")
    length = grad.shape[dim]
    if not 0 <= start <= out_shape[dim] - length:
        raise IndexError(
            f"scatter_zeros bounds out of range: start={start}, length={length}, "
            f"dim {dim} has size {out_shape[dim]}"
        )
    out = Tensor(out_shape, value=0.0)
    assign(out.narrow(dim, start, length), grad)
    return out


def unfolddx(grad, input_shape, dimension, size, step=1):
    raise NotImplementedError("unfold backward is a training kernel; not part of this backend")
