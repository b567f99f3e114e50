"""Kernel-level operators (reference: src/wxx/functional/__init__.py).

Same names and signatures as the reference; every forward operator runs a
hand-written sm_100a kernel from libwxx_cuda.so.  Names of the reference's
training-only kernels (backward passes, optimiser, loss) and of ops no
forward path uses exist and raise ``NotImplementedError``.
"""

from ._common import get_matmul_mode, manual_seed, set_matmul_mode
from .activations import (
    attention,
    attention_supported,
    cos,
    cosback,
    gelu,
    masked_softmax,
    relu,
    relubackwards,
    selu,
    selubackwards,
    sigmoid,
    sigmoidbackwards,
    silu,
    sin,
    sinback,
    softmax,
)
from .convolution import (
    adaptive_avgpool2d,
    adaptive_avgpool2ddx,
    avgpool1d,
    avgpool1ddx,
    avgpool2d,
    avgpool2ddx,
    causal_conv1d,
    causal_conv1d_backward,
    conv2d,
    conv2d_bn,
    conv2d_nhwc,
    conv_weight_pack,
    resnet_stem,
    conv2d_nhwc_supported,
    conv2ddw,
    conv2ddx,
    conv2dtranspose,
    conv2dtranspose_dw,
    conv2dtranspose_dx,
    maxpool1d,
    maxpool1ddx,
    maxpool2d,
    maxpool2ddx,
)
from .fft import (
    complex_add_inplace,
    complex_conj,
    complex_contiguous,
    complex_mul,
    complex_pad,
    complex_weights,
    fftconv,
    fftconv_spectrum,
    filter_spectrum,
    from_numpy_complex,
    irfft,
    rfft,
)
from .layers import dropout, dropoutdx, embed
from .normalization import (
    batchnorm,
    batchnormdg,
    batchnormdx,
    meanvarnorm,
    rmsnorm,
    rmsnormdg,
    rmsnormdx,
)
from .pointwise import (
    _pointwise,
    abs,
    clamp,
    clampbackwards,
    decay_window,
    decay_window_backward,
    hyena_filters,
    exp,
    log,
    mul_backward,
    negate,
    pointwise,
    rsqrt,
    scalarpointwise,
    sign,
    sqrt,
    square,
)
from .reductions import max, maxmin_backward, mean, min, std, sum, sumsq, var
from .utils import (
    _kaiming_normal_init,
    _kaiming_uniform_init,
    _xavier_normal_init,
    _xavier_uniform_init,
    _zero_init,
    arange,
    assign,
    concat,
    contiguous,
    diagonal,
    equal,
    equal_number,
    from_numpy,
    from_tensor,
    linear,
    ln_linear,
    linear_argmax,
    linear_short_conv,
    transpose_stack,
    linspace,
    masked_fill,
    matmul_add,
    normal,
    ones_like,
    permute,
    reshape,
    scatter_zeros,
    unfold,
    unfolddx,
    uniform,
)


from .training import (  # noqa: E402
    adamw,
    cceloss,
    embeddx,
    gelu_backward,
    gelubackwards,
    layernorm_backward,
    meanvarnormdx,
    meanvarnormdg,
    softmax_backward,
)


__all__ = [name for name in dir() if not name.startswith("__")]

from ..backend import observe as _observe  # noqa: E402

if _observe.nvtx_requested():
    _observe.wrap_namespace(globals(), "wxx")
