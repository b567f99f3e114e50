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


def attention_supported(q, n_heads, mask=None):
    """True when ``attention`` can run the fused tcgen05 kernel for these
    operands (TF32 or 3xTF32 mode, head dim 32 or 64, 16-byte aligned rows)."""
    from ._common import get_matmul_mode

    if get_matmul_mode() not in ("tf32", "3xtf32") or len(q.shape) != 3:
        return False
    D = q.shape[-1]
    if D % n_heads or D // n_heads not in (32, 64) or D % 4:
        return False
    if mask is not None and not getattr(mask, "_wxx_causal", False):
        if len(mask.shape) != 2 or mask.type != "f32" or mask.stride[1] != 1:
            return False
    return True


def _attention_rows(t):
    """(t, row stride) for a (B, S, D) operand whose rows are unit-stride,
    16-byte aligned and evenly spaced across the batch (a dense tensor or a
    column block of a wider one); a dense copy otherwise."""
    B, S, D = t.shape
    if t.is_dense():
        return t, D
    st = t.stride
    ld = st[1] if S > 1 else (st[0] if B > 1 else D)
    if (st[2] == 1 and ld >= D and ld % 4 == 0 and t.offset % 4 == 0
            and (B == 1 or st[0] == S * ld)):
        return t, ld
    return dense(t), D


def attention(q, k, v, n_heads, mask=None, causal=False, scale=None, *, feeds_tf32=False):
    """Fused multi-head attention ``softmax(scale * Q K^T + mask) V``.

    ``q`` (B, Sq, D), ``k``/``v`` (B, Sk, D) are the projection outputs with
    heads interleaved along D (head h owns columns h*hd..h*hd+hd-1, as
    ``reshape(b, s, H, hd)`` in nn/module.py:460-495); the result is
    (B, Sq, D) in the same merged layout.  ``causal`` masks keys after the
    query position (what GPT2's -1e9 upper-triangular mask does); ``mask`` is
    an additive (Sq, Sk) view.  Same values as the unfused
    matmul -> scale -> add mask -> softmax -> matmul chain up to rounding:
    TF32 products in tf32 mode, 3xTF32 (fp32-faithful) in 3xtf32 mode.
    ``feeds_tf32``: the result is read only by a TF32 product (the output
    projection), so in tf32 mode it is stored rounded to the nearest TF32
    value."""
    import math

    if len(q.shape) != 3 or len(k.shape) != 3 or len(v.shape) != 3:
        raise ValueError(f"attention: q {q.shape}, k {k.shape}, v {v.shape} must be 3-D")
    B, Sq, D = q.shape
    Sk = k.shape[1]
    if tuple(k.shape) != (B, Sk, D) or tuple(v.shape) != (B, Sk, D):
        raise ValueError(f"attention: q {q.shape}, k {k.shape}, v {v.shape} do not match")
    # Row-strided views (e.g. the q / k / v column blocks of one fused QKV
    # projection) are read in place: the kernel takes a row stride.
    q, q_ld = _attention_rows(q)
    k, k_ld = _attention_rows(k)
    v, v_ld = _attention_rows(v)
    if k_ld != v_ld:
        k, k_ld = dense(k), D
        v, v_ld = dense(v), D
    hd = D // n_heads
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    mptr, mld = None, 0
    if mask is not None and not causal:
        if tuple(mask.shape) != (Sq, Sk):
            raise ValueError(f"attention: mask shape {mask.shape} != {(Sq, Sk)}")
        mptr, mld = mask.ptr, mask.stride[0]
    from ._common import get_matmul_mode

    mode = get_matmul_mode()
    if mode not in ("tf32", "3xtf32"):
        raise ValueError(f"attention: the fused kernel runs in tf32 or 3xtf32 mode, not {mode!r}")
    out = empty((B, Sq, D), "f32", q.requires_grad or k.requires_grad or v.requires_grad)
    check(F.wxx_attention(out.buffer.ptr, q.ptr, k.ptr, v.ptr, B, n_heads, Sq, Sk, hd, q_ld, k_ld, D,
                          float(scale), mptr, mld, int(bool(causal)),
                          int(bool(feeds_tf32) and mode == "tf32"), int(mode == "3xtf32")),
          "attention")
    return out
