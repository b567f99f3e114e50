"""Activations and softmax (reference: src/wxx/functional/activations.py)."""

from .. import validation
from ._common import F, check, dense, empty
from .pointwise import _training_only, unary


def relu(tensor1):
    return unary(tensor1, "relu")


def sin(tensor1):
    return unary(tensor1, "sin")


def cos(tensor1):
    return unary(tensor1, "cos")


def gelu(tensor1):
    """Tanh-form GELU with the reference's clamps (x > 10 -> x, x < -10 -> 0)."""
    return unary(tensor1, "gelu")


def sigmoid(tensor1):
    """1 / (1 + exp(-x)) with the input clamped to [-88, 88]."""
    return unary(tensor1, "sigmoid")


def selu(tensor1):
    return unary(tensor1, "selu")


def silu(tensor1):
    """Fused sigmoid(x) * x (the reference's Tensor.silu runs two kernels)."""
    return unary(tensor1, "silu")


def softmax(tensor1, dim):
    """Softmax along ``dim`` (functional/activations.py:126-173): max-shifted,
    ``exp(x - max) / sum``, one read and one write of the tensor."""
    rank = validation.check_rank(tensor1.shape, max_rank=8, name="softmax input")
    dim = validation.normalize_dim(dim, rank, name="dim")
    if tensor1.type != "f32":
        raise TypeError(f"softmax expects f32 input, got {tensor1.type!r}")
    x = dense(tensor1)
    shape = x.shape
    outer = validation.numel(shape[:dim])
    n = shape[dim]
    inner = validation.numel(shape[dim + 1:])
    out = empty(shape, "f32", tensor1.requires_grad)
    check(F.wxx_softmax(out.buffer.ptr, x.ptr, outer, n, inner), "softmax")
    return out


relubackwards = _training_only("relubackwards")
gelubackwards = _training_only("gelubackwards")
sigmoidbackwards = _training_only("sigmoidbackwards")
selubackwards = _training_only("selubackwards")
sinback = _training_only("sinback")
cosback = _training_only("cosback")


def masked_softmax(score, mask):
    """``softmax(score + mask, dim=-1)`` in one pass when ``mask`` is a 2-D
    (S, S) view with unit column stride broadcast over the leading dims of
    ``score`` (the GPT-2 causal mask); any other mask falls back to the
    separate broadcast add and softmax of the reference."""
    from .pointwise import pointwise

    x = dense(score)
    n = x.shape[-1]
    if (len(mask.shape) == 2 and mask.type == "f32" and tuple(mask.shape) == tuple(x.shape[-2:])
            and mask.stride[1] == 1 and 0 < n <= 1024):
        rows = validation.numel(x.shape[:-1])
        out = empty(x.shape, "f32", score.requires_grad)
        check(F.wxx_softmax_masked(out.buffer.ptr, x.ptr, rows, n, mask.ptr, mask.stride[0],
                                   mask.shape[0]), "masked_softmax")
        return out
    return softmax(pointwise(score, mask, 0), -1)
