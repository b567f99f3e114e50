"""Module system and layers (reference: src/wxx/nn/module.py).

Same class names, constructor arguments, parameter names (so ``state_dict``
keys and the ``.npz`` format match the reference) and default
initialisations.  ``forward`` runs through ``wxx_b200.autograd`` /
``wxx_b200.functional`` on the GPU.
"""

import math

import numpy as np

from .. import autograd, functional
from ..Tensor import Parameter, Tensor
from ..backend import context
from ..backend.device import get_cmd_buffer
from ..functional.utils import from_numpy, normal


class Module:
    """Base of every layer.  Attributes that are ``Parameter``s or ``Module``s
    are registered (in assignment order) in ``_parameters`` / ``_modules``;
    the dotted names of the parameter tree are the ``state_dict`` keys, the
    same as the reference's (``blocks.0.attn.q.weight`` ...)."""

    def __init__(self):
        object.__setattr__(self, "_parameters", {})
        object.__setattr__(self, "_modules", {})

    def __setattr__(self, name, value):
        registry = None
        if isinstance(value, Parameter):
            registry = self._parameters
        elif isinstance(value, Module):
            registry = self._modules
        elif value is None and name in self._parameters:
            registry = self._parameters      # a parameter slot set to None stays listed
        if registry is not None:
            registry[name] = value
        object.__setattr__(self, name, value)

    def __call__(self, *x):
        return self.forward(*x)

    def forward(self, *args, **kwargs):
        raise NotImplementedError

    # -------------------------------------------------------- the parameter tree
    def _walk(self, prefix="", recurse=True):
        """(dotted name, parameter) for every non-None parameter: this
        module's own first, then each child's subtree, in registration order."""
        own = ((prefix + n, p) for n, p in self._parameters.items() if p is not None)
        yield from own
        if not recurse:
            return
        for child_name, child in self._modules.items():
            if child is not None:
                yield from child._walk(f"{prefix}{child_name}.", True)

    def parameters(self, recurse=True):
        """Yields ``("", parameter)`` pairs -- the pair shape the reference's
        optimisers consume (module.py:39-47)."""
        return (("", p) for _, p in self._walk("", recurse))

    def named_parameters(self, prefix="", recurse=True):
        return self._walk(prefix, recurse)

    def _state_keys(self, prefix=""):
        return [name for name, _ in self._walk(prefix)]

    def state_dict(self, prefix="", destination=None):
        """Parameter name -> host numpy array (a copy)."""
        out = {} if destination is None else destination
        out.update((name, np.array(p.numpy(), copy=True)) for name, p in self._walk(prefix))
        return out

    def load_state_dict(self, state_dict, strict=True):
        """Uploads arrays (or tensors) into the parameters in place.  With
        ``strict`` every parameter must be given and nothing else."""
        uploaders = {"c64": functional.from_numpy_complex,
                     "u32": lambda a: from_numpy(a, dtype=np.uint32)}
        for name, p in self._walk():
            if name not in state_dict:
                if strict:
                    raise KeyError(f"Missing key in state_dict: {name}")
                continue
            src = state_dict[name]
            if not isinstance(src, Tensor):
                src = uploaders.get(p.type, from_numpy)(np.asarray(src))
            if tuple(src.shape) != tuple(p.shape):
                raise ValueError(f"state_dict[{name!r}] has shape {tuple(src.shape)}, "
                                 f"parameter has {tuple(p.shape)}")
            functional.assign(p, src)
        if strict:
            own, given = set(self._state_keys()), set(state_dict)
            if own - given:
                raise RuntimeError(f"Missing keys: {sorted(own - given)}")
            if given - own:
                raise RuntimeError(f"Unexpected keys: {sorted(given - own)}")

    def zero_grad(self, wait=False):
        for _, p in self._walk():
            p.grad = None
        get_cmd_buffer().flush(wait=wait)

    def __repr__(self):
        children = [f"({n}): {c!r}".replace("\n", "\n  ") for n, c in self._modules.items()]
        body = "".join(f"\n  {c}" for c in children)
        return f"{type(self).__name__}({body}\n)"


class _Chain(Module):
    """Children registered under "0", "1", ... and applied in that order."""

    def __init__(self, modules=()):
        super().__init__()
        for m in modules:
            self.append(m)

    def append(self, module):
        setattr(self, str(len(self._modules)), module)
        return self

    def __len__(self):
        return len(self._modules)

    def __iter__(self):
        return iter(list(self._modules.values()))

    def __getitem__(self, idx):
        items = list(self._modules.values())
        return items[idx]

    def forward(self, x, *args, **kwargs):
        for m in self._modules.values():
            x = m(x, *args, **kwargs)
        return x


class ModuleList(_Chain):
    def __init__(self, modules=None):
        super().__init__(() if modules is None else modules)


class Sequential(_Chain):
    def __init__(self, *modules):
        super().__init__(modules)


class Linear(Module):
    """``y = x @ W + b`` with ``W`` of shape (in, out), Kaiming-normal init."""

    def __init__(self, in_features, out_features, bias=True):
        super().__init__()
        self.weight = Parameter(Tensor((in_features, out_features), value=0.0))
        functional._kaiming_normal_init(self.weight, in_features)
        self.bias = Parameter(Tensor((out_features,), value=0.0)) if bias else None

    def forward(self, x):
        if self.bias is None:
            return autograd.matmul(x, self.weight).forward(x, self.weight)
        return autograd.matmuladd(x, self.weight, self.bias).forward(x, self.weight, self.bias)


class Embedding(Module):
    def __init__(self, num_embeddings, embedding_dim, init_std=0.02):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.weight = Parameter(Tensor((num_embeddings, embedding_dim), value=0.0))
        functional.assign(self.weight, normal(0, init_std, (num_embeddings, embedding_dim)))

    def forward(self, x):
        n = x.shape[0] * x.shape[1] if len(x.shape) > 1 else x.shape[0]
        return autograd.Embedding(x, self.weight).forward(
            x, self.weight, n, self.embedding_dim, self.num_embeddings
        )


class Dropout(Module):
    """Inverted dropout in training mode; identity under ``inferenceMode``."""

    def __init__(self, p=0.5):
        super().__init__()
        self.p = p

    def forward(self, x):
        if context.MODE != 0 or self.p == 0:
            return x
        return autograd.Dropout(x).forward(x, self.p)


class LayerNorm(Module):
    """LayerNorm over the trailing ``normalized_shape`` dims.  As in the
    reference the kernel's eps is 1e-5 whatever ``eps`` says."""

    def __init__(self, normalized_shape, eps=1e-5):
        super().__init__()
        if isinstance(normalized_shape, int):
            normalized_shape = (normalized_shape,)
        self.normalized_shape = tuple(normalized_shape)
        self.eps = eps
        self.weightg = Parameter(Tensor(self.normalized_shape, value=1.0))
        self.weightb = Parameter(Tensor(self.normalized_shape, value=0.0))
        # Registered aliases, as in the reference (module.py:207-208): the
        # state_dict carries weightg, weightb, weight and bias.
        self.weight = self.weightg
        self.bias = self.weightb

    def forward(self, x):
        axis = tuple(range(len(x.shape) - len(self.normalized_shape), len(x.shape)))
        axis_arg = axis if len(axis) > 1 else axis[0]
        return autograd.meanvarnorm(x, self.weightg, self.weightb).forward(
            x, self.weightg, self.weightb, axis=axis_arg
        )

    def forward_into_gemm(self, x):
        """``forward(x)`` for an output read only by TF32 products (the
        projection after a pre-LN): under inference mode in tf32 matmul mode
        it is stored rounded to the nearest TF32 value.  Same as ``forward``
        otherwise."""
        if context.MODE == 0:
            return self.forward(x)
        axis = tuple(range(len(x.shape) - len(self.normalized_shape), len(x.shape)))
        return functional.meanvarnorm(x, self.weightg, self.weightb,
                                      axis=axis if len(axis) > 1 else axis[0],
                                      feeds_tf32=True)[0]


class RMSNorm(Module):
    """RMSNorm over the last dim (kernel eps 1e-6, as in the reference)."""

    def __init__(self, d_model, eps=1e-6):
        super().__init__()
        self.d_model = d_model
        self.eps = eps
        self.weight = Parameter(Tensor((d_model,), value=1.0))

    def forward(self, x):
        return autograd.rmsnorm(x, self.weight).forward(x, self.weight, -1)

    def forward_into_gemm(self, x):
        """``forward(x)`` for an output read only by TF32 products: under
        inference mode in tf32 matmul mode it is stored rounded to the
        nearest TF32 value."""
        if context.MODE == 0:
            return self.forward(x)
        return functional.rmsnorm(x, self.weight, -1, feeds_tf32=True)[0]


class BatchNorm(Module):
    """BatchNorm over NCHW.  ``running_std`` holds a variance (reference
    module.py:237-238); running statistics are not in ``state_dict``."""

    def __init__(self, num_features, eps=1e-5, momentum=0.1):
        super().__init__()
        self.num_features = num_features
        self.eps = eps
        self.momentum = momentum
        self.weight = Parameter(Tensor((num_features,), value=1.0))
        self.bias = Parameter(Tensor((num_features,), value=0.0))
        self.running_mean = Tensor((num_features,), value=0.0)
        self.running_std = Tensor((num_features,), value=1.0)

    def forward(self, x):
        training = context.MODE == 0
        return autograd.batchnorm(x, self.weight, self.bias).forward(
            x, self.weight, self.bias, self.running_mean, self.running_std, training
        )


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


class Conv2D(Module):
    def __init__(self, in_channels, out_channels, kernel=3, stride=1, padding=0, dilation=1,
                 bias=True):
        super().__init__()
        kernel = _pair(kernel)
        self.kernel = kernel
        self.stride = _pair(stride)
        self.padding = _pair(padding)
        self.dilation = _pair(dilation)
        self.W = Parameter(Tensor((out_channels, in_channels, kernel[0], kernel[1]), value=0.0))
        functional._kaiming_normal_init(self.W, math.prod(kernel) * in_channels)
        self.bias = Parameter(Tensor((out_channels,), value=0.0)) if bias else None

    def forward(self, x):
        if self.bias is None:
            return autograd.Conv2D(x, self.W).forward(
                x, self.W, None, self.stride, self.padding, self.dilation
            )
        return autograd.Conv2D(x, self.W, self.bias).forward(
            x, self.W, self.bias, self.stride, self.padding, self.dilation
        )


class Conv2DTranspose(Module):
    def __init__(self, *args, **kwargs):
        raise NotImplementedError("Conv2DTranspose is not part of the B200 inference backend")


class MaxPool2d(Module):
    def __init__(self, kernel, stride=None, padding=0, return_indices=False):
        super().__init__()
        kernel = _pair(kernel)
        self.kernel = kernel
        self.stride = kernel if stride is None else _pair(stride)
        self.padding = _pair(padding)
        self.return_indices = return_indices

    def forward(self, x):
        return autograd.maxpooling2d(x).forward(
            x, self.kernel, self.stride, self.padding, self.return_indices
        )


class _UnsupportedPool(Module):
    def __init__(self, *args, **kwargs):
        raise NotImplementedError(
            f"{type(self).__name__} is not on any forward path of the B200 backend"
        )


class MaxPool1d(_UnsupportedPool):
    pass


class AvgPool1d(_UnsupportedPool):
    pass


class AvgPool2d(_UnsupportedPool):
    pass


class AdaptiveAvgPool2d(Module):
    def __init__(self, output_size):
        super().__init__()
        self.output_size = tuple(int(v) for v in _pair(output_size))

    def forward(self, x):
        return autograd.adaptive_avgpooling2d(x).forward(x, self.output_size)


def _source_key(tensors, *extra):
    """Identity of the data in ``tensors``: buffer uid, its write version and
    the view geometry (an in-place write through ``functional.assign`` bumps
    the version)."""
    return tuple((t.buffer.uid, t.buffer.version, t.offset, tuple(t.shape), tuple(t.stride))
                 for t in tensors) + extra


def kmajor_weight(owner, name, linears, round_tf32=False):
    """The weights of ``linears`` (each nn.Linear's (K, N_i)) transposed and
    stacked into one (sum N_i, K) buffer owned by ``owner`` -- the K-major
    operand the tensor-core GEMM reads fastest (``linear(...,
    transpose_weight=True)``), optionally rounded to the nearest TF32 value.

    The copy is made by one launch (``functional.transpose_stack``) and kept:
    it is rebuilt only when a source weight was written since (the buffers'
    write versions) or replaced.  A CUDA graph recorded over a forward that
    reads this copy keeps reading it: after changing weights, record again."""
    K = linears[0].weight.shape[0]
    ns = [lin.weight.shape[1] for lin in linears]
    total = sum(ns)
    key = _source_key([lin.weight for lin in linears], bool(round_tf32))
    entry = owner.__dict__.get(name)
    if entry is not None and entry[1] == key:
        return entry[0]
    buf = entry[0] if entry is not None and tuple(entry[0].shape) == (total, K) else None
    if buf is None:
        buf = Tensor((total, K), value=0.0)
    if not functional.transpose_stack(buf, [lin.weight for lin in linears],
                                      round_tf32=round_tf32):
        row = 0
        for lin, n in zip(linears, ns):
            functional.assign(buf.narrow(0, row, n), lin.weight.transpose(0, 1))
            row += n
        key = key[:-1] + (False,)   # the fallback copy is not rounded
    object.__setattr__(owner, name, (buf, key))
    return buf


def tf32_weight(owner, name, weight):
    """A copy of ``weight`` rounded to the nearest TF32 value, kept and
    rebuilt like ``kmajor_weight``'s (for a weight whose own buffer must stay
    exact, e.g. the embedding that the tied LM head also reads)."""
    from ..backend.lib import F as _F, check as _check

    key = _source_key([weight])
    entry = owner.__dict__.get(name)
    if entry is not None and entry[1] == key:
        return entry[0]
    src = functional.contiguous(weight)
    buf = Tensor._empty(list(weight.shape), "f32")
    _check(_F.wxx_round_tf32(buf.buffer.ptr, src.ptr, int(np.prod(weight.shape))), "round_tf32")
    object.__setattr__(owner, name, (buf, key))
    return buf


class MultiHeadAttention(Module):
    """Multi-head self-attention (module.py:447-495).

    Same parameters and head layout (``reshape(b, s, H, hd).permute(0, 2, 1, 3)``).
    The score path is fused: the 1/sqrt(hd) scale is applied in the QK^T
    GEMM epilogue and the additive mask inside the softmax kernel, so the
    (B*H, S, S) score tensor is written once and read once.
    """

    def __init__(self, d_model, n_heads, dropout=0.0):
        super().__init__()
        assert d_model % n_heads == 0
        self.d_model = d_model
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.q = Linear(d_model, d_model, bias=False)
        self.k = Linear(d_model, d_model, bias=False)
        self.v = Linear(d_model, d_model, bias=False)
        self.out = Linear(d_model, d_model, bias=False)
        self.drop = Dropout(dropout)

    def _heads(self, t, b, seq):
        return (
            t.reshape((b, seq, self.n_heads, self.head_dim))
            .permute(0, 2, 1, 3)
            .reshape((b * self.n_heads, seq, self.head_dim))
        )

    def forward(self, x, mask=None, residual=None, kv_cache=None):
        """``residual`` (shaped like the output) is added by the output
        projection's epilogue: ``residual + attention(x)`` in one pass.
        ``kv_cache``: a (K, V) pair of (batch, max_len, d_model) tensors; the
        keys and values of positions 0..seq-1 are copied into them (the
        prefill of generation, see ``decode``)."""
        b, seq, _ = x.shape
        # the fused kernels record no graph: inference only
        if context.MODE != 0 and functional.attention_supported(x, self.n_heads, mask):
            causal = bool(getattr(mask, "_wxx_causal", False))
            if context.MODE != 0 and self.q.bias is None and self.k.bias is None \
                    and self.v.bias is None:
                # inference: q, k, v from one N = 3D product over a K-major
                # copy of the three weights; attention reads the column
                # blocks of its output in place
                # (the copy, q/k/v and the attention output feed only TF32
                # products: all stored rounded to the nearest TF32 value)
                D = self.d_model
                rnd = functional.get_matmul_mode() == "tf32"
                qkv = functional.linear(x, kmajor_weight(self, "_qkv_t", [self.q, self.k, self.v],
                                                         round_tf32=rnd),
                                        transpose_weight=True, feeds_tf32=True)
                q, k, v = qkv[..., 0:D], qkv[..., D:2 * D], qkv[..., 2 * D:3 * D]
            else:
                q, k, v = self.q(x), self.k(x), self.v(x)
            self._fill_cache(kv_cache, k, v, seq)
            o = functional.attention(q, k, v, self.n_heads,
                                     mask=None if causal else mask, causal=causal,
                                     scale=1.0 / math.sqrt(self.head_dim),
                                     feeds_tf32=context.MODE != 0)
            if context.MODE != 0:
                rnd = functional.get_matmul_mode() == "tf32"
                return functional.linear(o, kmajor_weight(self, "_out_t", [self.out], rnd),
                                         self.out.bias, residual=residual,
                                         transpose_weight=True)
            if residual is not None:
                return functional.linear(o, self.out.weight, self.out.bias, residual=residual)
            return self.out(o)
        q = self._heads(self.q(x), b, seq)
        kx, vx = self.k(x), self.v(x)
        self._fill_cache(kv_cache, kx, vx, seq)
        k = self._heads(kx, b, seq)
        v = self._heads(vx, b, seq)
        if context.MODE != 0:
            # scale in the QK^T epilogue, mask inside the softmax pass
            score = functional.matmul_add(q, k, None, transpose_B=True,
                                          alpha=1.0 / math.sqrt(self.head_dim))
            attn = (functional.masked_softmax(score, mask) if mask is not None
                    else score.softmax(-1))
        else:
            # training: every step recorded for the backward pass
            score = autograd.matmul(q, k).forward(q, k, False, True)
            score = score * (1.0 / math.sqrt(self.head_dim))
            if mask is not None:
                score = score + mask
            attn = score.softmax(-1)
        attn = self.drop(attn)
        out = autograd.matmul(attn, v).forward(attn, v)
        out = (
            out.reshape((b, self.n_heads, seq, self.head_dim))
            .permute(0, 2, 1, 3)
            .reshape((b, seq, self.d_model))
        )
        out = self.out(out)
        return out if residual is None else residual + out

    @staticmethod
    def _fill_cache(kv_cache, k, v, seq):
        if kv_cache is not None:
            functional.assign(kv_cache[0].narrow(1, 0, seq), k)
            functional.assign(kv_cache[1].narrow(1, 0, seq), v)

    def decode(self, x, kv_cache, cur_len, max_len, residual=None, ln=None):
        """One generation step for the newest position of each sequence.

        ``x`` (batch, d_model): the block input of that position; ``kv_cache``
        the (K, V) caches filled by the prefill ``forward`` and earlier steps;
        ``cur_len`` a device int holding the number of tokens so far (the new
        position is cur_len - 1, read on the device, so the same launches serve
        every step and can be replayed from one CUDA graph).  The position's
        key and value are appended to the caches and its query attends over
        positions 0..cur_len-1 (``wxx_decode_attention``, exact fp32).
        ``ln``: a LayerNorm applied to ``x`` first (fused into the q/k/v
        product when the projections have no bias).
        Returns ``residual + out(attention)`` (batch, d_model)."""
        from ..backend.lib import F as _F, check as _check

        B, D = x.shape
        if self.q.bias is None and self.k.bias is None and self.v.bias is None:
            w = kmajor_weight(self, "_qkv_t", [self.q, self.k, self.v],
                              round_tf32=functional.get_matmul_mode() == "tf32")
            if ln is not None:
                qkv = functional.ln_linear(x, ln.weightg, ln.weightb, w)
            else:
                qkv = functional.linear(x, w, transpose_weight=True)
            qp, kp, vp, ld = qkv.ptr, qkv.ptr + 4 * D, qkv.ptr + 8 * D, 3 * D
            keep = (qkv,)
        else:
            if ln is not None:
                x = ln.forward_into_gemm(x)
            q, k, v = self.q(x), self.k(x), self.v(x)
            qp, kp, vp, ld = q.ptr, k.ptr, v.ptr, D
            keep = (q, k, v)
        o = Tensor._empty([B, D], "f32")
        Kc, Vc = kv_cache
        _check(_F.wxx_decode_attention(o.buffer.ptr, D, qp, kp, vp, ld, Kc.ptr, Vc.ptr,
                                       max_len * D, B, self.n_heads, self.head_dim, cur_len.ptr,
                                       max_len, 1.0 / math.sqrt(self.head_dim),
                                       int(functional.get_matmul_mode() == "tf32")),
               "decode_attention")
        del keep
        rnd = functional.get_matmul_mode() == "tf32"
        return functional.linear(o, kmajor_weight(self, "_out_t", [self.out], rnd), self.out.bias,
                                 residual=residual, transpose_weight=True)


class Attention(Module):
    def __init__(self, d_model, n_heads=1):
        super().__init__()
        self.mha = MultiHeadAttention(d_model, n_heads)

    def forward(self, x, mask=None):
        return self.mha(x, mask)


class GELU(Module):
    def forward(self, x):
        return x.gelu()


class Sine(Module):
    """``sin(omega * x)``."""

    def __init__(self, omega=10.0):
        super().__init__()
        self.omega = float(omega)

    def forward(self, x):
        return (x * self.omega).sin()

    def extra_repr(self):
        return f"omega={self.omega}"


class SwiGLU(Module):
    def __init__(self, d_model, hidden_dim=None, mlp_ratio=4):
        super().__init__()
        if hidden_dim is None:
            hidden_dim = int(2 * (mlp_ratio * d_model) / 3)
        self.hidden_dim = hidden_dim
        self.w1 = Linear(d_model, hidden_dim, bias=False)
        self.w2 = Linear(d_model, hidden_dim, bias=False)
        self.w3 = Linear(hidden_dim, d_model, bias=False)

    def forward(self, x, residual=None):
        """``w3(silu(w1 x) * w2 x)`` (+ ``residual``, fused into the last GEMM)."""
        mode = functional.get_matmul_mode()
        d_in = self.w1.weight.shape[0]
        if mode != "fp32" and len(x.shape) >= 2 and (mode == "tf32" or d_in <= 1024):
            return self._forward_fused(x, residual)
        y = self.w3(functional.silu(self.w1(x)) * self.w2(x))
        return y if residual is None else residual + y

    def _forward_fused(self, x, residual):
        """Two GEMMs instead of three plus two elementwise passes: W1 and W2
        interleaved column by column into one weight, whose GEMM epilogue
        writes silu(x W1) * (x W2) directly (``linear(..., "swiglu")``), then
        W3 with the residual add in its epilogue.  The hidden width is rounded
        up to a multiple of 4 so every operand row is 16-byte aligned: the
        extra columns hold zero weights (silu(0) * 0 = 0) and meet zero rows of
        W3.  The weights are copied into buffers owned by the module, and
        copied again only when a source weight was written since (buffer
        write versions, as for ``kmajor_weight``)."""
        h = self.hidden_dim
        hp = (h + 3) // 4 * 4
        d_in = self.w1.weight.shape[0]
        d_out = self.w3.weight.shape[1]
        key = _source_key([self.w1.weight, self.w2.weight, self.w3.weight])
        cache = self.__dict__.get("_glu_cache")
        if cache is None or cache[0] != hp:
            cache = (hp, Tensor((d_in, 2 * hp), value=0.0), Tensor((hp, d_out), value=0.0), None)
        hp_, w12, w3p, done = cache
        if done != key:
            functional.assign(w12[:, 0:2 * h:2], self.w1.weight)
            functional.assign(w12[:, 1:2 * h:2], self.w2.weight)
            functional.assign(w3p.narrow(0, 0, h), self.w3.weight)
            cache = (hp_, w12, w3p, key)
        object.__setattr__(self, "_glu_cache", cache)
        g = functional.linear(x, w12, activation="swiglu", feeds_tf32=context.MODE != 0)
        return functional.linear(g, w3p, residual=residual)


class TiedLinear(Module):
    """Output head sharing an embedding's weight: ``x @ E^T``."""

    def __init__(self, embedding):
        super().__init__()
        object.__setattr__(self, "_embedding", embedding)

    def forward_argmax(self, x):
        """The index of each row's largest logit, ``forward(x).max(-1)[1]``,
        without storing the logits (inference)."""
        w = self._embedding.weight
        if context.MODE != 0 and functional.get_matmul_mode() == "tf32":
            w = tf32_weight(self, "_w_tf32", w)
        ids = functional.linear_argmax(x, w, transpose_weight=True)
        return ids if ids is not None else functional.max(self.forward(x), -1)[1]

    def forward_ln(self, x, ln):
        """``forward(ln(x))`` for a few rows (generation's decode step): the
        LayerNorm and the head product in one launch."""
        w = self._embedding.weight
        if context.MODE != 0 and functional.get_matmul_mode() == "tf32":
            w = tf32_weight(self, "_w_tf32", w)
        return functional.ln_linear(x, ln.weightg, ln.weightb, w)

    def forward(self, x):
        w = self._embedding.weight
        if context.MODE != 0 and functional.get_matmul_mode() == "tf32":
            # the product reads a TF32-rounded copy (the lookup keeps the table)
            w = tf32_weight(self, "_w_tf32", w)
        return autograd.matmul(x, w).forward(x, w, False, True)


class PositionalEncoding(Module):
    """``[t, cos(2 pi k t), sin(2 pi k t)]`` over ``t = linspace(0, 1, L)``."""

    def __init__(self, features=8):
        super().__init__()
        features = int(features)
        if features < 1:
            raise ValueError(f"positional features must be >= 1, got {features}")
        self.features = features
        self.out_features = 2 * features + 1
        self._cache = {}

    def _build(self, length):
        t = np.linspace(0.0, 1.0, int(length), dtype=np.float32)
        k = np.arange(self.features, dtype=np.float32)
        ang = (2.0 * np.pi) * np.outer(t, k)
        return np.concatenate([t[:, None], np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)

    def forward(self, length):
        key = (int(length), self.features)
        pe = self._cache.get(key)
        if pe is None:
            pe = from_numpy(self._build(length))
            self._cache[key] = pe
        return pe

    def extra_repr(self):
        return f"features={self.features}, out_features={self.out_features}"
