"""Training kernels behind the reference's functional names
(src/wxx/functional/{activations,normalization,layers,loss}.py): GELU, softmax and
LayerNorm backward, the embedding gradient, the softmax cross-entropy loss and
the AdamW step, each one launch of ``csrc/train.cu`` (plus column sums on the
reduction kernels for the LayerNorm affine gradients)."""

import numpy as np

from .. import validation
from ..backend.dispatch import _get_reduce_dims
from ._common import F, check, dense, empty
from .utils import mark_written


def gelu_backward(grad, tensor1):
    """``grad * gelu'(x)`` in one pass (the autograd GELU's backward)."""
    g = dense(grad)
    x = dense(tensor1)
    if tuple(g.shape) != tuple(x.shape):
        raise ValueError(f"gelu_backward: grad {tuple(g.shape)} vs input {tuple(x.shape)}")
    out = empty(x.shape, "f32")
    check(F.wxx_gelu_backward(out.buffer.ptr, g.ptr, x.ptr, validation.numel(x.shape)),
          "gelu_backward")
    return out


def gelubackwards(tensor1):
    """gelu'(x) (functional/activations.py:96, gelubackwards.wgsl)."""
    from .utils import ones_like

    return gelu_backward(ones_like(tensor1), tensor1)


def softmax_backward(grad, out, dim=-1):
    """Gradient of ``softmax(x, dim)`` from its output ``out``:
    ``out * (grad - sum(grad * out, dim))``; ``dim`` is the last axis."""
    y = dense(out)
    g = dense(grad)
    rank = len(y.shape)
    if validation.normalize_dim(dim, rank) != rank - 1:
        raise ValueError("softmax_backward: only the last axis is supported")
    n = y.shape[-1]
    rows = validation.numel(y.shape) // max(n, 1)
    dx = empty(y.shape, "f32")
    check(F.wxx_softmax_backward(dx.buffer.ptr, g.ptr, y.ptr, rows, n), "softmax_backward")
    return dx


def layernorm_backward(grad, tensor1, gamma, mean, inv_std, axis=None):
    """(dx, dgamma, dbeta) of LayerNorm over the trailing run of axes, from
    the forward's saved ``mean`` / ``inv_std`` (functional/normalization.py:308,362
    meanvarnormdx / meanvarnormdg)."""
    x = dense(tensor1)
    g = dense(grad)
    outer, red, inner, _ = _get_reduce_dims(x.shape, axis)
    if inner != 1:
        raise ValueError("layernorm_backward: the normalised axes must be the trailing ones")
    dx = empty(x.shape, "f32")
    dyxhat = empty(x.shape, "f32")
    check(F.wxx_layernorm_backward(dx.buffer.ptr, dyxhat.buffer.ptr, g.ptr, x.ptr,
                                   dense(mean).ptr, dense(inv_std).ptr, dense(gamma).ptr,
                                   outer, red), "layernorm_backward")
    from .reductions import sum as _sum

    shape = tuple(gamma.shape)
    dgamma = _sum(dyxhat.reshape((outer, red)), 0).reshape(shape)
    dbeta = _sum(g.reshape((outer, red)), 0).reshape(shape)
    return dx, dgamma, dbeta


def meanvarnormdx(grad, tensor1, gamma, mean, var, axis=None):
    return layernorm_backward(grad, tensor1, gamma, mean, var, axis)[0]


def meanvarnormdg(grad, tensor1, mean, var, axis=None):
    from .utils import ones_like

    x = dense(tensor1)
    _, red, _, _ = _get_reduce_dims(x.shape, axis)
    ones = ones_like(x.reshape((-1, red))[0])
    return layernorm_backward(grad, tensor1, ones, mean, var, axis)[1]


def embeddx(tensor1, tensor2, n_token, embed_dim, vocab_size):
    """Embedding weight gradient (functional/layers.py:209): ``tensor1`` the
    upstream gradient (n_token rows of embed_dim), ``tensor2`` the u32 ids;
    returns (vocab_size, embed_dim)."""
    g = dense(tensor1)
    ids = dense(tensor2)
    if ids.type != "u32":
        raise TypeError(f"embeddx expects u32 ids, got {ids.type!r}")
    out = empty((int(vocab_size), int(embed_dim)), "f32")
    check(F.wxx_embedding_backward(out.buffer.ptr, ids.ptr, g.ptr, int(n_token), int(embed_dim),
                                   int(vocab_size)), "embeddx")
    return out


def cceloss(tensor1, tensor2):
    """Softmax cross-entropy of (B, K) logits against (B,) u32 targets
    (functional/loss.py:20, cceloss.wgsl): returns ``(loss (B, 1), grad)``
    with ``grad = softmax(logits) - onehot(target)``.  Targets outside [0, K)
    raise ``ValueError`` before the launch, as in the reference."""
    validation.check_rank(tensor1.shape, min_rank=2, max_rank=2, name="logits")
    validation.check_rank(tensor2.shape, min_rank=1, max_rank=1, name="targets")
    if tensor1.type != "f32":
        raise TypeError(f"cceloss expects f32 logits, got {tensor1.type!r}")
    if tensor2.type != "u32":
        raise TypeError(f"cceloss expects u32 targets, got {tensor2.type!r}")
    B, K = tensor1.shape
    if tensor2.shape[0] != B:
        raise ValueError(f"cceloss expects one target per row, got {tensor2.shape[0]} "
                         f"targets for {B} rows")
    if B < 1 or K < 1:
        raise ValueError(f"cceloss expects non-empty logits, got {(B, K)}")
    t = dense(tensor2)
    from ..graph import capturing

    if not capturing():
        # (while a step is recorded the kernel's own range check reports
        # through the device error word instead)
        top = int(np.asarray(t.numpy()).max())
        if top >= K:
            raise ValueError(f"cceloss targets must be in [0, {K}), got max target {top}")
    z = dense(tensor1)
    loss = empty((B, 1), "f32")
    grad = empty((B, K), "f32")
    check(F.wxx_cceloss(loss.buffer.ptr, grad.buffer.ptr, z.ptr, t.ptr, B, K), "cceloss")
    return loss, grad


def adamw(weight, grad, exp_avg, exp_avg_sq, step, lr, beta1, beta2, eps, weight_decay, bc1,
          bc2):
    """One AdamW step in place (functional/layers.py:21, adamw.wgsl): the moments
    and the weight are updated; ``step`` is the step count (the bias
    corrections ``bc1`` / ``bc2`` come precomputed, as in the reference)."""
    for t, name in ((weight, "weight"), (grad, "grad"), (exp_avg, "exp_avg"),
                    (exp_avg_sq, "exp_avg_sq")):
        if not t.is_dense():
            raise ValueError(f"adamw: {name} must be dense")
        if tuple(t.shape) != tuple(weight.shape):
            raise ValueError(f"adamw: {name} shape {tuple(t.shape)} != {tuple(weight.shape)}")
    check(F.wxx_adamw(weight.ptr, grad.ptr, exp_avg.ptr, exp_avg_sq.ptr,
                      validation.numel(weight.shape), float(lr), float(beta1), float(beta2),
                      float(eps), float(weight_decay), float(bc1), float(bc2)), "adamw")
    for t in (weight, exp_avg, exp_avg_sq):
        mark_written(t)
    return weight
