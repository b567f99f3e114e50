"""Autograd function objects (reference: src/wxx/autograd/).

Every class keeps the reference's constructor (the op's input tensors) and
``forward`` signature and runs the forward through ``wxx_b200.functional``.
This backend implements the inference path: no graph is recorded and
``backward`` raises ``NotImplementedError``.
"""

from .. import functional
from ..backend import context


class Function:
    """Base of all ops: remembers its inputs, exposes ``forward``."""

    def __init__(self, *inputs):
        self.inputs = list(inputs)
        self.needs_input_grad = [
            bool(getattr(t, "requires_grad", False)) and context.MODE == 0 for t in inputs
        ]

    def forward(self, *args, **kwargs):
        raise NotImplementedError

    def backward(self, grad_output):
        raise NotImplementedError(
            f"{type(self).__name__}.backward: training is not part of the B200 inference backend"
        )


def _op(name, fn, doc):
    cls = type(name, (Function,), {"forward": lambda self, *a, **k: fn(*a, **k), "__doc__": doc})
    return cls


def _rg(out, *inputs):
    out.requires_grad = any(getattr(t, "requires_grad", False) for t in inputs)
    return out


add = _op("add", lambda a, b: _rg(functional.pointwise(a, b, 0), a, b), "a + b")
sub = _op("sub", lambda a, b: _rg(functional.pointwise(a, b, 1), a, b), "a - b")
mul = _op("mul", lambda a, b: _rg(functional.pointwise(a, b, 2), a, b), "a * b")
div = _op("div", lambda a, b: _rg(functional.pointwise(a, b, 3), a, b), "a / b")
addscaler = _op("addscaler", lambda a, c: functional.scalarpointwise(a, c, 0), "a + c")
subscaler = _op("subscaler", lambda a, c: functional.scalarpointwise(a, c, 1), "a - c")
mulscaler = _op("mulscaler", lambda a, c: functional.scalarpointwise(a, c, 2), "a * c")
powscaler = _op("powscaler", lambda a, c: functional.scalarpointwise(a, c, 3), "a ** c")
rpowscaler = _op("rpowscaler", lambda a, c: functional.scalarpointwise(a, c, 3, reverse=1),
                 "c ** a")
rdivscaler = _op("rdivscaler", lambda a, c: functional.scalarpointwise(a, c, 4, reverse=1),
                 "c / a")
negate = _op("negate", functional.negate, "-a")
relu = _op("relu", functional.relu, "relu")
gelu = _op("gelu", functional.gelu, "gelu (tanh form)")
sigmoid = _op("sigmoid", functional.sigmoid, "sigmoid")
selu = _op("selu", functional.selu, "selu")
sin = _op("sin", functional.sin, "sin")
cos = _op("cos", functional.cos, "cos")
abs = _op("abs", functional.abs, "abs")
sign = _op("sign", functional.sign, "sign")
square = _op("square", functional.square, "x * x")
exp = _op("exp", functional.exp, "exp")
sqrt = _op("sqrt", functional.sqrt, "sqrt")
rsqrt = _op("rsqrt", functional.rsqrt, "rsqrt")
log = _op("log", functional.log, "log")
clamp = _op("clamp", functional.clamp, "clamp")
decay_window = _op("decay_window", functional.decay_window, "exp(-|decay| t)")


class matmul(Function):
    def forward(self, tensor1, tensor2, transpose_a=False, transpose_b=False):
        out = functional.matmul_add(tensor1, tensor2, None, transpose_A=transpose_a,
                                    transpose_B=transpose_b)
        return _rg(out, tensor1, tensor2)


class matmuladd(Function):
    def forward(self, tensor1, tensor2, tensor3):
        return _rg(functional.matmul_add(tensor1, tensor2, tensor3), tensor1, tensor2, tensor3)


class permute(Function):
    def forward(self, tensor1, axes):
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        return functional.permute(tensor1, *axes)


class reshape(Function):
    def forward(self, tensor1, shape):
        return functional.reshape(tensor1, shape)


class flatten(Function):
    def forward(self, tensor1, start_dim=0, end_dim=-1):
        return tensor1.flatten(start_dim, end_dim)


class narrow(Function):
    def forward(self, tensor1, dim, start, length):
        return tensor1.narrow(dim, start, length)


class squeeze(Function):
    def forward(self, tensor1, dim=None):
        return tensor1.squeeze(dim)


class unsqueeze(Function):
    def forward(self, tensor1, dim):
        return tensor1.unsqueeze(dim)


class getitem(Function):
    def forward(self, tensor1, index):
        return tensor1._basic_getitem(index)


class concat(Function):
    def forward(self, tensors, dim=-1):
        return functional.concat(tensors, dim)


class diagonal(Function):
    def forward(self, tensor1, offset=0, dim1=0, dim2=1):
        return functional.diagonal(tensor1, offset, dim1, dim2)


class unfold(Function):
    def forward(self, tensor1, dimension, size, step=1):
        return functional.unfold(tensor1, dimension, size, step)


class rfft(Function):
    def forward(self, tensor1, n=None):
        return functional.rfft(tensor1, n)[0]


class irfft(Function):
    def forward(self, tensor1, n=None):
        return functional.irfft(tensor1, n)


class complex_mul(Function):
    def forward(self, tensor1, tensor2):
        return functional.complex_mul(tensor1, tensor2)


class complex_conj(Function):
    def forward(self, tensor1):
        return functional.complex_conj(tensor1)


class softmax(Function):
    def forward(self, tensor1, dim=-1):
        return _rg(functional.softmax(tensor1, dim), tensor1)


class sum(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.sum(tensor1, axis, keepdims, keepdim=keepdim)


class mean(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.mean(tensor1, axis, keepdims, keepdim=keepdim)


class var(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.var(tensor1, axis, keepdims, keepdim=keepdim)


class std(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.std(tensor1, axis, keepdims, keepdim=keepdim)


class max(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.max(tensor1, axis, keepdims, keepdim=keepdim)[0]


class min(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.min(tensor1, axis, keepdims, keepdim=keepdim)[0]


class argmax(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.max(tensor1, axis, keepdims, keepdim=keepdim)[1]


class argmin(Function):
    def forward(self, tensor1, axis=None, keepdims=False, *, keepdim=None):
        return functional.min(tensor1, axis, keepdims, keepdim=keepdim)[1]


class meanvarnorm(Function):
    def forward(self, tensor1, gamma, beta, axis=None):
        return _rg(functional.meanvarnorm(tensor1, gamma, beta, axis)[0], tensor1, gamma, beta)


class rmsnorm(Function):
    def forward(self, tensor1, gamma, axis=None):
        return _rg(functional.rmsnorm(tensor1, gamma, axis)[0], tensor1, gamma)


class batchnorm(Function):
    def forward(self, tensor1, gamma, beta, running_mean, running_var, training=False):
        out = functional.batchnorm(tensor1, gamma, beta, running_mean, running_var, training)[0]
        return _rg(out, tensor1, gamma, beta)


class Conv2D(Function):
    def forward(self, tensor1, W, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1)):
        return _rg(functional.conv2d(tensor1, W, stride, padding, dilation, bias), tensor1, W)


class maxpooling2d(Function):
    def forward(self, tensor1, kernel, stride, padding, return_indices=False):
        return functional.maxpool2d(tensor1, kernel, stride, padding, return_indices)


class adaptive_avgpooling2d(Function):
    def forward(self, tensor1, output_size):
        return functional.adaptive_avgpool2d(tensor1, output_size)


class causal_conv1d(Function):
    def forward(self, tensor1, weight, bias):
        return functional.causal_conv1d(tensor1, weight, bias)


class Embedding(Function):
    def forward(self, tensor1, tensor2, n_token, embed_dim, vocab_size):
        return _rg(functional.embed(tensor1, tensor2, n_token, embed_dim), tensor2)


class Dropout(Function):
    def forward(self, tensor1, p=0.2):
        return functional.dropout(tensor1, p)[0]


class CrossEntropyLoss(Function):
    def forward(self, tensor1, tensor2):
        return functional.cceloss(tensor1, tensor2)


def _training_op(name):
    class _T(Function):
        def forward(self, *args, **kwargs):
            raise NotImplementedError(f"{name} is not part of the B200 inference backend")

    _T.__name__ = name
    return _T


Conv2DTranspose = _training_op("Conv2DTranspose")
avgpooling1d = _training_op("avgpooling1d")
avgpooling2d = _training_op("avgpooling2d")
maxpooling1d = _training_op("maxpooling1d")

__all__ = [name for name in dir() if not name.startswith("_")]
