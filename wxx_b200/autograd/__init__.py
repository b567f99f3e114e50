"""Autograd function objects (interface: src/wxx/autograd/).

Every class keeps the reference's constructor (the op's input tensors) and
``forward`` signature and runs the forward through ``wxx_b200.functional``.
Under training mode (``backend.context.MODE == 0``) an op whose inputs need
gradients records itself as its output's ``creator``; ``Tensor.backward()``
walks those records in reverse topological order and calls each op's
``backward(grad_output)``, which returns one gradient per constructor input
(``None`` where no gradient flows).

Backward passes exist for the ops a GPT2 training step uses: elementwise
add / sub / mul (with broadcasting), the scalar ops, negate, GELU, matmul and
matmul + bias, reshape / permute / contiguous, softmax, sum / mean,
LayerNorm (``meanvarnorm``), Embedding, Dropout and CrossEntropyLoss.  The
other ops run their forward and raise ``NotImplementedError`` from
``backward``.
"""

import math as _math

from .. import functional
from ..backend import context


class Function:
    """Base of all ops: remembers its inputs and whether each needs a gradient."""

    def __init__(self, *inputs):
        self.inputs = list(inputs)
        self.needs_input_grad = [
            bool(getattr(t, "requires_grad", False)) and context.MODE == 0 for t in inputs
        ]

    def forward(self, *args, **kwargs):
        raise NotImplementedError

    def backward(self, grad_output):
        raise NotImplementedError(
            f"{type(self).__name__}.backward is not implemented in this backend "
            "(backward passes cover the GPT2 training path)")

    def _track(self, out):
        """Marks ``out`` as produced by this op: it requires a gradient when
        any input does (training mode), and then records the op."""
        needs = any(self.needs_input_grad)
        out.requires_grad = needs
        if needs:
            out.creator = self
        return out


def _op(name, fn, doc):
    """A forward-only op (no backward in this backend)."""
    def forward(self, *a, **k):
        return self._track(fn(*a, **k))

    return type(name, (Function,), {"forward": forward, "__doc__": doc})


def _reduce_to(grad, shape):
    """Sums a broadcast gradient back to ``shape`` (leading extra axes and the
    axes where ``shape`` has size 1)."""
    shape = tuple(shape)
    if tuple(grad.shape) == shape:
        return grad
    g = grad
    extra = len(g.shape) - len(shape)
    if extra > 0:
        g = functional.sum(g, tuple(range(extra)) if extra > 1 else 0)
    for axis, n in enumerate(shape):
        if n == 1 and g.shape[axis] != 1:
            g = functional.sum(g, axis, keepdims=True)
    return functional.reshape(g, shape)


def _scale(grad, c):
    return functional.scalarpointwise(grad, float(c), 2)


def _mm(x, y, tx, ty):
    """op(x) @ op(y) (batched, an unbatched side broadcasts)."""
    return functional.matmul_add(x, y, None, transpose_A=tx, transpose_B=ty)


# ------------------------------------------------------------ elementwise

class add(Function):
    def forward(self, a, b):
        self.shapes = (tuple(a.shape), tuple(getattr(b, "shape", ())))
        return self._track(functional.pointwise(a, b, 0))

    def backward(self, grad_output):
        sa, sb = self.shapes
        ga = _reduce_to(grad_output, sa) if self.needs_input_grad[0] else None
        gb = _reduce_to(grad_output, sb) if self.needs_input_grad[1] else None
        return ga, gb


class sub(Function):
    def forward(self, a, b):
        self.shapes = (tuple(a.shape), tuple(b.shape))
        return self._track(functional.pointwise(a, b, 1))

    def backward(self, grad_output):
        sa, sb = self.shapes
        ga = _reduce_to(grad_output, sa) if self.needs_input_grad[0] else None
        gb = _reduce_to(functional.negate(grad_output), sb) if self.needs_input_grad[1] else None
        return ga, gb


class mul(Function):
    def forward(self, a, b):
        if any(self.needs_input_grad):
            self.saved = (a, b)
        return self._track(functional.pointwise(a, b, 2))

    def backward(self, grad_output):
        a, b = self.saved
        self.saved = None
        ga = (_reduce_to(functional.pointwise(grad_output, b, 2), a.shape)
              if self.needs_input_grad[0] else None)
        gb = (_reduce_to(functional.pointwise(grad_output, a, 2), b.shape)
              if self.needs_input_grad[1] else None)
        return ga, gb


class div(Function):
    def forward(self, a, b):
        if any(self.needs_input_grad):
            self.saved = (a, b)
        return self._track(functional.pointwise(a, b, 3))

    def backward(self, grad_output):
        a, b = self.saved
        self.saved = None
        ga = gb = None
        if self.needs_input_grad[0]:
            ga = _reduce_to(functional.pointwise(grad_output, b, 3), a.shape)
        if self.needs_input_grad[1]:
            # d(a/b)/db = -a / b^2
            q = functional.pointwise(functional.pointwise(a, b, 3), b, 3)
            gb = _reduce_to(functional.negate(functional.pointwise(grad_output, q, 2)), b.shape)
        return ga, gb


class addscaler(Function):
    def forward(self, a, c):
        return self._track(functional.scalarpointwise(a, c, 0))

    def backward(self, grad_output):
        return (grad_output,) + (None,) * (len(self.inputs) - 1)


class subscaler(Function):
    def forward(self, a, c):
        return self._track(functional.scalarpointwise(a, c, 1))

    def backward(self, grad_output):
        return (grad_output,) + (None,) * (len(self.inputs) - 1)


class mulscaler(Function):
    def forward(self, a, c):
        self.c = float(c)
        return self._track(functional.scalarpointwise(a, c, 2))

    def backward(self, grad_output):
        return (_scale(grad_output, self.c),) + (None,) * (len(self.inputs) - 1)


class negate(Function):
    def forward(self, a):
        return self._track(functional.negate(a))

    def backward(self, grad_output):
        return functional.negate(grad_output)


class gelu(Function):
    def forward(self, a):
        if any(self.needs_input_grad):
            self.saved = a
        return self._track(functional.gelu(a))

    def backward(self, grad_output):
        x, self.saved = self.saved, None
        return functional.gelu_backward(grad_output, x)


powscaler = _op("powscaler", lambda a, c: functional.scalarpointwise(a, c, 3), "a ** c")
rpowscaler = _op("rpowscaler", lambda a, c: functional.scalarpointwise(a, c, 3, reverse=1),
                 "c ** a")
rdivscaler = _op("rdivscaler", lambda a, c: functional.scalarpointwise(a, c, 4, reverse=1),
                 "c / a")
relu = _op("relu", functional.relu, "relu")
sigmoid = _op("sigmoid", functional.sigmoid, "sigmoid")
selu = _op("selu", functional.selu, "selu")
sin = _op("sin", functional.sin, "sin")
cos = _op("cos", functional.cos, "cos")


class abs(Function):
    def forward(self, a):
        if any(self.needs_input_grad):
            self.saved = a
        return self._track(functional.abs(a))

    def backward(self, grad_output):
        x, self.saved = self.saved, None
        return functional.pointwise(grad_output, functional.sign(x), 2)


sign = _op("sign", functional.sign, "sign")
square = _op("square", functional.square, "x * x")
exp = _op("exp", functional.exp, "exp")
sqrt = _op("sqrt", functional.sqrt, "sqrt")
rsqrt = _op("rsqrt", functional.rsqrt, "rsqrt")
log = _op("log", functional.log, "log")
clamp = _op("clamp", functional.clamp, "clamp")
decay_window = _op("decay_window", functional.decay_window, "exp(-|decay| t)")


# ------------------------------------------------------------ contractions

def _matmul_grads(fn, grad_output, a, b, ta, tb):
    """Gradients of C = op(a) @ op(b) (op = transpose when ta / tb).
    An unbatched weight against a batched input (Linear) is reduced over the
    batch inside one GEMM by folding the batch into the rows."""
    ga = gb = None
    if fn.needs_input_grad[0]:
        # d op(a) = dC op(b)^T ; da = d op(a) or its transpose
        ga = _mm(grad_output, b, False, not tb) if not ta else _mm(b, grad_output, tb, True)
        ga = _reduce_to(ga, a.shape)
    if fn.needs_input_grad[1]:
        if len(b.shape) == 2 and len(a.shape) > 2 and not ta:
            K = a.shape[-1]
            a2 = functional.reshape(a, (-1, K))
            g2 = functional.reshape(grad_output, (-1, grad_output.shape[-1]))
            gb = _mm(a2, g2, True, False) if not tb else _mm(g2, a2, True, False)
        else:
            # d op(b) = op(a)^T dC ; db = d op(b) or its transpose
            gb = _mm(a, grad_output, not ta, False) if not tb else _mm(grad_output, a, True, ta)
            gb = _reduce_to(gb, b.shape)
    return ga, gb


class matmul(Function):
    def forward(self, tensor1, tensor2, transpose_a=False, transpose_b=False):
        self.flags = (bool(transpose_a), bool(transpose_b))
        if any(self.needs_input_grad):
            self.saved = (tensor1, tensor2)
        out = functional.matmul_add(tensor1, tensor2, None, transpose_A=transpose_a,
                                    transpose_B=transpose_b)
        return self._track(out)

    def backward(self, grad_output):
        a, b = self.saved
        self.saved = None
        return _matmul_grads(self, grad_output, a, b, *self.flags)


class matmuladd(Function):
    def forward(self, tensor1, tensor2, tensor3):
        if any(self.needs_input_grad):
            self.saved = (tensor1, tensor2, tuple(tensor3.shape))
        return self._track(functional.matmul_add(tensor1, tensor2, tensor3))

    def backward(self, grad_output):
        a, b, bias_shape = self.saved
        self.saved = None
        ga, gb = _matmul_grads(self, grad_output, a, b, False, False)
        gc = _reduce_to(grad_output, bias_shape) if self.needs_input_grad[2] else None
        return ga, gb, gc


# ------------------------------------------------------------ views

class permute(Function):
    def forward(self, tensor1, axes):
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        self.axes = tuple(axes)
        return self._track(functional.permute(tensor1, *axes))

    def backward(self, grad_output):
        inverse = [0] * len(self.axes)
        for i, a in enumerate(self.axes):
            inverse[a] = i
        return functional.permute(grad_output, *inverse)


class reshape(Function):
    def forward(self, tensor1, shape):
        self.in_shape = tuple(tensor1.shape)
        return self._track(functional.reshape(tensor1, shape))

    def backward(self, grad_output):
        return functional.reshape(grad_output, self.in_shape)


class contiguous(Function):
    def forward(self, tensor1):
        return self._track(functional.contiguous(tensor1))

    def backward(self, grad_output):
        return grad_output


class flatten(Function):
    def forward(self, tensor1, start_dim=0, end_dim=-1):
        self.in_shape = tuple(tensor1.shape)
        return self._track(tensor1.flatten(start_dim, end_dim))

    def backward(self, grad_output):
        return functional.reshape(grad_output, self.in_shape)


narrow = _op("narrow", lambda t, dim, start, length: t.narrow(dim, start, length), "narrow")
squeeze = _op("squeeze", lambda t, dim=None: t.squeeze(dim), "squeeze")
unsqueeze = _op("unsqueeze", lambda t, dim: t.unsqueeze(dim), "unsqueeze")
getitem = _op("getitem", lambda t, index: t._basic_getitem(index), "t[index]")
concat = _op("concat", lambda tensors, dim=-1: functional.concat(tensors, dim), "concat")
diagonal = _op("diagonal", lambda t, offset=0, dim1=0, dim2=1:
               functional.diagonal(t, offset, dim1, dim2), "diagonal")
unfold = _op("unfold", lambda t, dimension, size, step=1:
             functional.unfold(t, dimension, size, step), "unfold")
rfft = _op("rfft", lambda t, n=None: functional.rfft(t, n)[0], "rfft")
irfft = _op("irfft", lambda t, n=None: functional.irfft(t, n), "irfft")
complex_mul = _op("complex_mul", lambda a, b: functional.complex_mul(a, b), "complex_mul")
complex_conj = _op("complex_conj", lambda a: functional.complex_conj(a), "complex_conj")


# ------------------------------------------------------------ reductions

class softmax(Function):
    def forward(self, tensor1, dim=-1):
        out = functional.softmax(tensor1, dim)
        if any(self.needs_input_grad):
            self.saved = (out, dim)
        return self._track(out)

    def backward(self, grad_output):
        out, dim = self.saved
        self.saved = None
        return functional.softmax_backward(grad_output, out, dim)


def _expand_back(fn, grad_output, scale):
    """Gradient of a sum / mean over ``fn.axis``: the output gradient
    broadcast back over the reduced axes (times 1/n for the mean)."""
    shape, axis = fn.in_shape, fn.axis
    rank = len(shape)
    if axis is None:
        kept = (1,) * rank
    else:
        axes = {a % rank for a in ((axis,) if isinstance(axis, int) else axis)}
        kept = tuple(1 if d in axes else n for d, n in enumerate(shape))
    g = functional.reshape(grad_output, kept)
    if scale != 1.0:
        g = _scale(g, scale)
    zeros = functional.scalarpointwise(functional.ones_like(fn.saved_like), 0.0, 2)
    fn.saved_like = None
    return functional.pointwise(zeros, g, 0)


class sum(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        self.in_shape, self.axis, self.saved_like = tuple(tensor1.shape), axis, tensor1
        return self._track(functional.sum(tensor1, axis, keepdims, keepdim=keepdim))

    def backward(self, grad_output):
        return _expand_back(self, grad_output, 1.0)


class mean(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        self.in_shape, self.axis, self.saved_like = tuple(tensor1.shape), axis, tensor1
        return self._track(functional.mean(tensor1, axis, keepdims, keepdim=keepdim))

    def backward(self, grad_output):
        n = _math.prod(self.in_shape)
        if self.axis is not None:
            rank = len(self.in_shape)
            axes = {a % rank for a in ((self.axis,) if isinstance(self.axis, int) else self.axis)}
            n = _math.prod(self.in_shape[a] for a in axes)
        return _expand_back(self, grad_output, 1.0 / n)


var = _op("var", lambda t, axis=None, keepdims=False, *, keepdim=None:
          functional.var(t, axis, keepdims, keepdim=keepdim), "var")
std = _op("std", lambda t, axis=None, keepdims=False, *, keepdim=None:
          functional.std(t, axis, keepdims, keepdim=keepdim), "std")
max = _op("max", lambda t, axis=None, keepdims=False, *, keepdim=None:
          functional.max(t, axis, keepdims, keepdim=keepdim)[0], "max")
min = _op("min", lambda t, axis=None, keepdims=False, *, keepdim=None:
          functional.min(t, axis, keepdims, keepdim=keepdim)[0], "min")
argmax = _op("argmax", lambda t, axis=None, keepdims=False, *, keepdim=None:
             functional.max(t, axis, keepdims, keepdim=keepdim)[1], "argmax")
argmin = _op("argmin", lambda t, axis=None, keepdims=False, *, keepdim=None:
             functional.min(t, axis, keepdims, keepdim=keepdim)[1], "argmin")


# ------------------------------------------------------------ normalisation

class meanvarnorm(Function):
    def forward(self, tensor1, gamma, beta, axis=None):
        y, mu, inv = functional.meanvarnorm(tensor1, gamma, beta, axis)
        if any(self.needs_input_grad):
            self.saved = (tensor1, gamma, mu, inv, axis)
        return self._track(y)

    def backward(self, grad_output):
        x, gamma, mu, inv, axis = self.saved
        self.saved = None
        dx, dgamma, dbeta = functional.layernorm_backward(grad_output, x, gamma, mu, inv, axis)
        need = self.needs_input_grad
        return (dx if need[0] else None, dgamma if need[1] else None,
                dbeta if need[2] else None)


rmsnorm = _op("rmsnorm", lambda t, gamma, axis=None: functional.rmsnorm(t, gamma, axis)[0],
              "rmsnorm")
batchnorm = _op("batchnorm", lambda t, gamma, beta, running_mean, running_var, training=False:
                functional.batchnorm(t, gamma, beta, running_mean, running_var, training)[0],
                "batchnorm")


# ------------------------------------------------------------ convolution / pooling

Conv2D = _op("Conv2D", lambda t, W, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1):
             functional.conv2d(t, W, stride, padding, dilation, bias), "conv2d")
maxpooling2d = _op("maxpooling2d", lambda t, kernel, stride, padding, return_indices=False:
                   functional.maxpool2d(t, kernel, stride, padding, return_indices),
                   "maxpool2d")
adaptive_avgpooling2d = _op("adaptive_avgpooling2d", lambda t, output_size:
                            functional.adaptive_avgpool2d(t, output_size), "adaptive avgpool")
causal_conv1d = _op("causal_conv1d", lambda t, weight, bias:
                    functional.causal_conv1d(t, weight, bias), "causal_conv1d")


# ------------------------------------------------------------ layers and loss

class Embedding(Function):
    def forward(self, tensor1, tensor2, n_token, embed_dim, vocab_size):
        out = functional.embed(tensor1, tensor2, n_token, embed_dim)
        if any(self.needs_input_grad):
            self.saved = (tensor1, int(n_token), int(embed_dim), int(vocab_size))
        return self._track(out)

    def backward(self, grad_output):
        ids, n, d, vocab = self.saved
        self.saved = None
        if not self.needs_input_grad[1]:
            return None, None
        return None, functional.embeddx(grad_output, ids, n, d, vocab)


class Dropout(Function):
    def forward(self, tensor1, p=0.2):
        out, seed = functional.dropout(tensor1, p)
        self.p, self.seed = p, seed
        return self._track(out)

    def backward(self, grad_output):
        return functional.dropoutdx(grad_output, self.p, self.seed)


class CrossEntropyLoss(Function):
    """Per-row softmax cross-entropy of (B, K) logits against (B,) u32
    targets; the output is (B, 1).  The gradient softmax - onehot comes from
    the same kernel as the loss and is scaled by the output gradient."""

    def forward(self, tensor1, tensor2):
        loss, grad = functional.cceloss(tensor1, tensor2)
        if any(self.needs_input_grad):
            self.grad = grad
        return self._track(loss)

    def backward(self, grad_output):
        g, self.grad = self.grad, None
        dz = functional.pointwise(g, grad_output, 2)
        # constructed with the logits alone (nn/loss.py) or with the targets too
        return (dz,) + (None,) * (len(self.inputs) - 1)


def _training_op(name):
    class _T(Function):
        def forward(self, *args, **kwargs):
            raise NotImplementedError(f"{name} is not part of this backend")

    _T.__name__ = name
    return _T


Conv2DTranspose = _training_op("Conv2DTranspose")
avgpooling1d = _training_op("avgpooling1d")
avgpooling2d = _training_op("avgpooling2d")
maxpooling1d = _training_op("maxpooling1d")

__all__ = [name for name in dir() if not name.startswith("_")]
