"""Normalisations (reference: src/wxx/functional/normalization.py).

The epsilons are the reference's hard-coded values: RMSNorm 1e-6,
LayerNorm 1e-5, BatchNorm 1e-5 with momentum 0.1 (normalization.py:36,94,157).
Unlike the reference kernels (rmsnorm.wgsl:23-24, meanvarnorm.wgsl:28-29),
rows beyond 65535 are normalised too.
"""

from ..backend.dispatch import _get_reduce_dims
from ._common import F, check, dense, empty, get_matmul_mode
from .pointwise import _training_only


def _round_flag(feeds_tf32):
    return int(bool(feeds_tf32) and get_matmul_mode() == "tf32")


def rmsnorm(tensor1, gamma, axis=None, *, feeds_tf32=False):
    """``y = x * rsqrt(mean(x^2) + 1e-6) * gamma`` (inv = 0 for all-zero rows);
    returns ``(y, inv_rms)``.  ``feeds_tf32``: y is read only by TF32 tensor-core
    products, so in tf32 matmul mode it is stored rounded to the nearest TF32
    value (the product then reads it exactly instead of truncating it)."""
    x = dense(tensor1)
    g = dense(gamma)
    outer, red, inner, out_shape = _get_reduce_dims(x.shape, axis)
    out = empty(x.shape, "f32")
    irms = empty(out_shape, "f32")
    check(F.wxx_rmsnorm(out.buffer.ptr, irms.buffer.ptr, x.ptr, g.ptr, outer, red, inner, 1e-6,
                        _round_flag(feeds_tf32)), "rmsnorm")
    return out, irms


def meanvarnorm(tensor1, gamma, beta, axis=None, *, feeds_tf32=False):
    """LayerNorm ``(x - mean) * inv * gamma + beta``, ``inv = rsqrt(var + 1e-5)``
    (0 when the variance is 0); returns ``(y, mean, inv_std)``.  ``feeds_tf32``
    as for ``rmsnorm``."""
    x = dense(tensor1)
    g = dense(gamma)
    b = dense(beta)
    outer, red, inner, out_shape = _get_reduce_dims(x.shape, axis)
    out = empty(x.shape, "f32")
    mean = empty(out_shape, "f32")
    inv = empty(out_shape, "f32")
    check(F.wxx_layernorm(out.buffer.ptr, mean.buffer.ptr, inv.buffer.ptr, x.ptr, g.ptr, b.ptr,
                          outer, red, inner, 1e-5, _round_flag(feeds_tf32)), "meanvarnorm")
    return out, mean, inv


def batchnorm(tensor1, gamma, beta, running_mean, running_std, training=False):
    """BatchNorm over NCHW.  Eval: ``(x - rm) * rsqrt(rv + 1e-5) * g + b`` where
    the reference's ``running_std`` buffer holds a variance; training: batch
    statistics, running statistics updated with momentum 0.1.
    Returns ``(y, saved_mean, saved_inv_std)``."""
    x = dense(tensor1)
    B, C, H, W = x.shape
    g = dense(gamma)
    b = dense(beta)
    out = empty(x.shape, "f32")
    saved_mean = empty((C,), "f32")
    saved_inv = empty((C,), "f32")
    check(F.wxx_batchnorm(out.buffer.ptr, saved_mean.buffer.ptr, saved_inv.buffer.ptr, x.ptr,
                          g.ptr, b.ptr, running_mean.ptr, running_std.ptr, B, C, H * W, 1e-5,
                          0.1, int(bool(training))), "batchnorm")
    return out, saved_mean, saved_inv


rmsnormdx = _training_only("rmsnormdx")
rmsnormdg = _training_only("rmsnormdg")
batchnormdx = _training_only("batchnormdx")
batchnormdg = _training_only("batchnormdg")
