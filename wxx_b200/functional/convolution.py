"""Convolutions and pooling (reference: src/wxx/functional/convolution.py)."""

from .. import validation
from ._common import F, active_timer, check, dense, empty, matmul_mode_code
from .pointwise import _training_only


def _check_pool_input(tensor1, rank, name):
    if len(tensor1.shape) != rank:
        expected = "(B, C, L)" if rank == 3 else "(B, C, H, W)"
        raise ValueError(f"{name} expects {expected}, got {tensor1.shape}")
    if tensor1.type != "f32":
        raise TypeError(f"{name} expects f32 input, got {tensor1.type!r}")


def maxpool2d(tensor1, kernel, stride, padding, return_indices=False):
    """Window max over (B, C, H, W), padding excluded, first strict maximum wins;
    with ``return_indices`` also the flat input index (u32) of each maximum."""
    _check_pool_input(tensor1, 4, "maxpool2d")
    x = dense(tensor1)
    B, C, H, W = x.shape
    KH, KW = kernel
    sh, sw = stride
    ph, pw = padding
    Ho = (H + 2 * ph - KH) // sh + 1
    Wo = (W + 2 * pw - KW) // sw + 1
    if Ho < 1 or Wo < 1:
        raise ValueError(f"pooling produces an empty output {(Ho, Wo)}")
    out = empty((B, C, Ho, Wo), "f32")
    idx = empty((B, C, Ho, Wo), "u32") if return_indices else None
    check(F.wxx_maxpool2d(out.buffer.ptr, None if idx is None else idx.buffer.ptr, x.ptr, B, C, H,
                          W, KH, KW, sh, sw, ph, pw), "maxpool2d")
    return (out, idx) if return_indices else out


def _normalize_output_size(output_size):
    if isinstance(output_size, int):
        output_size = (output_size, output_size)
    if len(output_size) != 2:
        raise ValueError(f"output_size must be an int or 2-tuple, got {output_size!r}")
    h, w = int(output_size[0]), int(output_size[1])
    if h < 1 or w < 1:
        raise ValueError(f"output_size entries must be positive, got {output_size!r}")
    return h, w


def adaptive_avgpool2d(tensor1, output_size):
    """Adaptive average pooling with windows [floor(o*in/out), ceil((o+1)*in/out))."""
    if tensor1.type != "f32":
        raise TypeError(f"adaptive_avgpool2d expects f32 input, got {tensor1.type!r}")
    if validation.check_rank(tensor1.shape, name="adaptive_avgpool2d input") != 4:
        raise ValueError(f"adaptive_avgpool2d expects (B, C, H, W), got {tensor1.shape}")
    Ho, Wo = _normalize_output_size(output_size)
    x = dense(tensor1)
    B, C, H, W = x.shape
    out = empty((B, C, Ho, Wo), "f32", tensor1.requires_grad)
    check(F.wxx_adaptive_avgpool2d(out.buffer.ptr, x.ptr, B, C, H, W, Ho, Wo),
          "adaptive_avgpool2d")
    return out


def conv2d(tensor1, W, stride, padding, dilation, bias=None):
    """NCHW cross-correlation as an implicit GEMM on the tcgen05 tensor cores
    (functional/convolution.py:658-729): rows = B*Ho*Wo output pixels,
    columns = Cout, K = Cin*KH*KW, the im2col gather done by producer warps."""
    return _conv2d(tensor1, W, stride, padding, dilation, bias, None, None, False)


def conv2d_bn(tensor1, W, stride, padding, dilation, bias=None, *, bn=None, residual=None,
              relu=False):
    """``conv2d`` followed by eval-mode batchnorm, an optional residual add and
    an optional ReLU, all applied in the convolution's epilogue (ResNet's
    conv -> bn (-> + shortcut) -> relu chain, functional/normalization.py:
    148-206 in eval mode).  ``bn`` is ``(running_mean, running_var, gamma,
    beta, eps)`` or None; ``residual`` is shaped like the output.  The values
    equal the separate ``conv2d`` / ``batchnorm`` / ``+`` / ``relu`` ops (the
    same fp32 operations in the same order)."""
    return _conv2d(tensor1, W, stride, padding, dilation, bias, bn, residual, relu)


def conv2d_nhwc_supported(cin, cout, ho, wo):
    """True when ``conv2d_nhwc`` takes these channel counts and output size:
    Cin a multiple of 32, Cout of 4, and 128-pixel output tiles that are
    boxes of the output (Wo a multiple of 128, or Wo dividing 128 and Ho a
    multiple or a divisor of 128 / Wo)."""
    if cin % 32 or cout % 4 or ho < 1 or wo < 1:
        return False
    if wo >= 128:
        return wo % 128 == 0
    if 128 % wo:
        return False
    rows = 128 // wo
    return ho % rows == 0 if ho >= rows else rows % ho == 0


def resnet_stem(tensor1, W, bias=None, *, bn=None, relu=True, packed=None):
    """ResNet's stem in one launch (nn/resnet.py:31-79): ``conv2d`` 7x7 /
    stride 2 / pad 3 to 64 channels, eval batchnorm (``bn`` = (running_mean,
    running_var, gamma, beta, eps) or None), ReLU, ``maxpool2d`` 3x3 / stride 2
    / pad 1, returned channels-last (B, Hp, Wp, 64) -- the same values as those
    ops followed by ``permute(0, 2, 3, 1)``.  None when the shapes are outside
    the kernel's (1..4 input channels, H and W up to 32).  ``packed``: ``W``
    already transposed to a dense (Cin * 49, 64) tensor (the kernel then
    copies it instead of gathering it)."""
    x = dense(tensor1)
    w = dense(W)
    if len(x.shape) != 4 or len(w.shape) != 4:
        return None
    B, Cin, H, Wd = x.shape
    if tuple(w.shape) != (64, Cin, 7, 7) or not (1 <= Cin <= 4 and 1 <= H <= 32 and 1 <= Wd <= 32):
        return None
    if bias is not None and tuple(bias.shape) != (64,):
        return None
    Ho, Wo = (H - 1) // 2 + 1, (Wd - 1) // 2 + 1
    Hp, Wp = (Ho - 1) // 2 + 1, (Wo - 1) // 2 + 1
    out = empty((B, Hp, Wp, 64), "f32")
    if bn is not None:
        rm, rv, g, b, eps = bn
        ptrs = [dense(t).ptr for t in (rm, rv, g, b)]
    else:
        ptrs, eps = [None] * 4, 0.0
    wp = w.ptr
    if packed is not None:
        if tuple(packed.shape) != (Cin * 49, 64) or not packed.is_dense():
            raise ValueError(f"resnet_stem: packed weights {tuple(packed.shape)} are not "
                             f"({Cin * 49}, 64)")
        wp = packed.ptr
    check(F.wxx_resnet_stem(out.buffer.ptr, x.ptr, wp, None if bias is None else dense(bias).ptr,
                            *ptrs, float(eps), int(bool(relu)), B, Cin, H, Wd,
                            int(packed is not None)), "resnet_stem")
    return out


def conv_weight_pack(weights, outs):
    """Reorders each (Cout, Cin, KH, KW) weight in ``weights`` into the dense
    (Cout, KH, KW, Cin) tensor at the same index of ``outs`` -- the K order
    of the channels-last convolution -- in one launch (up to 24 weights).
    False (nothing written) when the arguments do not fit."""
    import ctypes

    n = len(weights)
    if n == 0 or n > 24 or len(outs) != n:
        return False
    ws = [dense(w) for w in weights]
    for w, o in zip(ws, outs):
        co, ci, kh, kw = w.shape
        if tuple(o.shape) != (co, kh, kw, ci) or not o.is_dense() or ci * kh * kw > 51200:
            return False
    ints = ctypes.c_int * n
    ptrs = ctypes.c_void_p * n
    check(F.wxx_conv_weight_pack(ptrs(*[o.ptr for o in outs]), ptrs(*[w.ptr for w in ws]),
                                 ints(*[w.shape[0] for w in ws]), ints(*[w.shape[1] for w in ws]),
                                 ints(*[w.shape[2] * w.shape[3] for w in ws]), n),
          "conv_weight_pack")
    return True


def conv2d_nhwc(tensor1, W, stride, padding, dilation, bias=None, *, bn=None, residual=None,
                relu=False, packed=None):
    """``conv2d_bn`` on channels-last tensors: ``tensor1`` (B, H, W, Cin) NHWC,
    ``W`` (Cout, Cin, KH, KW) as in the reference, ``residual`` and the result
    (B, Ho, Wo, Cout) NHWC.  The implicit GEMM's A operand is fetched by TMA
    boxes (one filter tap x 32 channels x a 128-pixel tile per K-block), so
    the rows of im2col are never gathered by threads; see
    ``conv2d_nhwc_supported`` for the shapes it takes.  ``packed``: ``W``
    already reordered to (Cout, KH, KW, Cin) by ``conv_weight_pack`` (the
    convolution then skips its own reorder launch)."""
    x = dense(tensor1)
    w = dense(W)
    B, H, Wd, Cin = x.shape
    Cout, Cin_w, KH, KW = w.shape
    if Cin_w != Cin:
        raise ValueError(f"conv2d: input has {Cin} channels, weight expects {Cin_w}")
    sh, sw = stride
    ph, pw = padding
    dh, dw = dilation
    Ho = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    Wo = (Wd + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    if not conv2d_nhwc_supported(Cin, Cout, Ho, Wo):
        raise ValueError(f"conv2d_nhwc: unsupported shape Cin={Cin} Cout={Cout} out={(Ho, Wo)}")
    if residual is not None and tuple(residual.shape) != (B, Ho, Wo, Cout):
        raise ValueError(f"conv2d: residual {tuple(residual.shape)} is not {(B, Ho, Wo, Cout)}")
    b = dense(bias) if bias is not None else None
    out = empty((B, Ho, Wo, Cout), "f32", tensor1.requires_grad)
    if bn is not None:
        rm, rv, g, beta, eps = bn
        rm, rv, g, beta = (dense(t) for t in (rm, rv, g, beta))
        bn_args = (rm.ptr, rv.ptr, g.ptr, beta.ptr, float(eps))
    else:
        bn_args = (None, None, None, None, 0.0)
    r = dense(residual) if residual is not None else None
    mode = matmul_mode_code()
    timer = active_timer()
    ev0 = timer.start() if timer is not None else None
    if packed is not None:
        pk = dense(packed)
        if tuple(pk.shape) != (Cout, KH, KW, Cin):
            raise ValueError(f"conv2d_nhwc: packed weight {tuple(pk.shape)} is not "
                             f"{(Cout, KH, KW, Cin)}")
        fn, wptr = F.wxx_conv2d_nhwc_packed, pk.ptr
    else:
        fn, wptr = F.wxx_conv2d_nhwc, w.ptr
    check(fn(out.buffer.ptr, x.ptr, wptr, None if b is None else b.ptr, B, Cin, H,
             Wd, Cout, KH, KW, sh, sw, ph, pw, dh, dw, 0 if mode == 0 else 1,
             *bn_args, None if r is None else r.ptr, int(bool(relu))), "conv2d")
    if timer is not None:
        timer.stop(ev0, 2.0 * B * Ho * Wo * Cout * Cin * KH * KW, f"conv{B}x{H}x{Wd}x{Cin}->{Cout}")
    return out


def _conv2d(tensor1, W, stride, padding, dilation, bias, bn, residual, relu):
    x = dense(tensor1)
    w = dense(W)
    B, Cin, H, Wd = x.shape
    Cout, Cin_w, KH, KW = w.shape
    if Cin_w != Cin:
        raise ValueError(f"conv2d: input has {Cin} channels, weight expects {Cin_w}")
    sh, sw = stride
    ph, pw = padding
    dh, dw = dilation
    Ho = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    Wo = (Wd + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    if Ho < 1 or Wo < 1:
        raise ValueError(f"conv2d produces an empty output {(Ho, Wo)}")
    b = dense(bias) if bias is not None else None
    out = empty((B, Cout, Ho, Wo), "f32", tensor1.requires_grad)
    mode = matmul_mode_code()
    timer = active_timer()
    ev0 = timer.start() if timer is not None else None
    args = (out.buffer.ptr, x.ptr, w.ptr, None if b is None else b.ptr, B, Cin, H, Wd, Cout, KH,
            KW, sh, sw, ph, pw, dh, dw, 0 if mode == 0 else 1)
    if bn is None and residual is None and not relu:
        check(F.wxx_conv2d(*args), "conv2d")
    else:
        if residual is not None and tuple(residual.shape) != (B, Cout, Ho, Wo):
            raise ValueError(f"conv2d: residual {tuple(residual.shape)} is not {(B, Cout, Ho, Wo)}")
        if bn is not None:
            rm, rv, g, beta, eps = bn
            rm, rv, g, beta = (dense(t) for t in (rm, rv, g, beta))
            for t in (rm, rv, g, beta):
                if tuple(t.shape) != (Cout,):
                    raise ValueError(f"conv2d: batchnorm parameter {tuple(t.shape)} is not ({Cout},)")
            bn_args = (rm.ptr, rv.ptr, g.ptr, beta.ptr, float(eps))
        else:
            bn_args = (None, None, None, None, 0.0)
        r = dense(residual) if residual is not None else None
        check(F.wxx_conv2d_bn(*args, *bn_args, None if r is None else r.ptr, int(bool(relu))),
              "conv2d")
    if timer is not None:
        timer.stop(ev0, 2.0 * B * Ho * Wo * Cout * Cin * KH * KW, f"conv{B}x{Cin}x{H}x{Wd}->{Cout}")
    return out


def causal_conv1d(tensor1, weight, bias):
    """Depthwise causal conv ``out[b,d,n] = bias[d] + sum_k w[d,k] x[b,d,n-k]``
    consuming a strided (B, D, L) view directly."""
    if len(tensor1.shape) != 3:
        raise ValueError(f"causal_conv1d expects a 3-D input, got {tensor1.shape}")
    if len(weight.shape) != 2:
        raise ValueError(f"causal_conv1d weight must be (D, K), got {weight.shape}")
    x = tensor1 if all(s >= 0 for s in tensor1.stride) else tensor1.contiguous()
    w = dense(weight)
    b = dense(bias)
    B, D, L = x.shape
    K = w.shape[1]
    out = empty((B, D, L), "f32", tensor1.requires_grad or weight.requires_grad)
    check(F.wxx_causal_conv1d(out.buffer.ptr, x.buffer.ptr, x.offset, x.stride[0], x.stride[1],
                              x.stride[2], w.ptr, b.ptr, B, D, L, K), "causal_conv1d")
    return out


conv2ddx = _training_only("conv2ddx")
conv2ddw = _training_only("conv2ddw")
conv2dtranspose = _training_only("conv2dtranspose")
conv2dtranspose_dx = _training_only("conv2dtranspose_dx")
conv2dtranspose_dw = _training_only("conv2dtranspose_dw")
maxpool2ddx = _training_only("maxpool2ddx")
adaptive_avgpool2ddx = _training_only("adaptive_avgpool2ddx")
avgpool1d = _training_only("avgpool1d")
avgpool1ddx = _training_only("avgpool1ddx")
avgpool2d = _training_only("avgpool2d")
avgpool2ddx = _training_only("avgpool2ddx")
maxpool1d = _training_only("maxpool1d")
maxpool1ddx = _training_only("maxpool1ddx")
causal_conv1d_backward = _training_only("causal_conv1d_backward")
