"""Hyena language model (reference: src/wxx/nn/hyena.py).

Same modules, parameter names and default initialisation as the reference.
The long convolution ``irfft(rfft(z, n) * rfft(h, n), n)[..., :L]`` runs as
one fused kernel (``functional.fftconv``): each (batch, channel) row is
transformed, multiplied by the filter spectrum and transformed back on chip.
"""

import numpy as np

from .. import autograd, functional
from ..Tensor import Parameter, Tensor
from ..backend import context
from .module import (
    Embedding,
    Linear,
    Module,
    ModuleList,
    PositionalEncoding,
    RMSNorm,
    Sequential,
    Sine,
    SwiGLU,
    TiedLinear,
)


def _next_pow2(n):
    n = int(n)
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


class CausalShortConv1d(Module):
    """Depthwise causal conv ``out[n] = sum_k w[k] x[n-k]`` over (B, D, L)."""

    def __init__(self, d_model, kernel_size=3):
        super().__init__()
        self.d_model = d_model
        self.kernel_size = kernel_size
        self.weight = Parameter(Tensor((d_model, kernel_size), value=0.0))
        self.bias = Parameter(Tensor((d_model,), value=0.0))
        functional.assign(self.weight, functional.normal(0, 0.02, (d_model, kernel_size)))

    def forward(self, x):
        return autograd.causal_conv1d(x, self.weight, self.bias).forward(x, self.weight, self.bias)


class ImplicitFilter(Module):
    """``h(t) = FFN(PositionalEncoding(t))`` returned as (d_model, L)."""

    def __init__(self, d_model, hidden_dim=64, pe_features=8, omega=10.0):
        super().__init__()
        self.d_model = d_model
        self.hidden_dim = hidden_dim
        self.pe_features = pe_features
        self.positional_encoding = PositionalEncoding(pe_features)
        self.mlp = Sequential(
            Linear(self.positional_encoding.out_features, hidden_dim),
            Sine(omega),
            Linear(hidden_dim, d_model),
        )

    def forward(self, L):
        pos = self.positional_encoding(L)
        return self.mlp(pos).transpose(0, 1)


class HyenaOperator(Module):
    def __init__(self, d_model, order=2, fft_size=None, short_conv_kernel=3, filter_hidden=64,
                 pe_features=8, filter_omega=10.0):
        super().__init__()
        if order < 1:
            raise ValueError(f"order must be >= 1, got {order}")
        if short_conv_kernel < 1:
            raise ValueError(f"short_conv_kernel must be >= 1, got {short_conv_kernel}")
        self.d_model = d_model
        self.order = int(order)
        self.fft_size = fft_size
        self.proj_v = Linear(d_model, d_model, bias=False)
        self.proj_x = Linear(d_model, self.order * d_model, bias=False)
        self.out_proj = Linear(d_model, d_model, bias=False)
        self.short_conv = CausalShortConv1d(d_model, kernel_size=short_conv_kernel)
        self.filter_mlp = ModuleList(
            [ImplicitFilter(d_model, hidden_dim=filter_hidden, pe_features=pe_features,
                            omega=filter_omega) for _ in range(self.order)]
        )
        self.decay = Parameter(Tensor((self.order, d_model), value=0.0))
        functional.assign(
            self.decay, functional.from_numpy(np.random.rand(self.order, d_model).astype(np.float32))
        )

    def _fft_size(self, length):
        size = int(self.fft_size) if self.fft_size is not None else _next_pow2(2 * length)
        if size < length:
            size = _next_pow2(length)
        return size

    def fft_conv1d(self, x, h, gate=None):
        """Linear convolution of (B, D, L) with (D, L), fused on the GPU; with
        ``gate`` the result is multiplied by it in the same pass."""
        length = x.shape[-1]
        return functional.fftconv(x, h, self._fft_size(length), out_len=length, gate=gate)

    def _decay_window(self, stage, length):
        return autograd.decay_window(self.decay).forward(self.decay, stage, length)

    def _filters_fused(self, length):
        """Inference: every filter_mlp[i](length) * decay_window(i) of this
        operator from one kernel, as an (order, D, L) tensor; None when the
        filters do not have the plain Linear -> Sine -> Linear form or exceed
        the kernel's limits."""
        lin1, lin2, omegas, pes = [], [], set(), set()
        for filt in self.filter_mlp:
            mods = list(filt.mlp._modules.values())
            if (len(mods) != 3 or not isinstance(mods[0], Linear) or not isinstance(mods[1], Sine)
                    or not isinstance(mods[2], Linear)):
                return None
            lin1.append((mods[0].weight, mods[0].bias))
            lin2.append((mods[2].weight, mods[2].bias))
            omegas.add(mods[1].omega)
            pes.add(filt.positional_encoding.features)
        if len(omegas) != 1 or len(pes) != 1:
            return None
        pe = self.filter_mlp[0].positional_encoding(length)
        return functional.hyena_filters(pe, lin1, lin2, omegas.pop(), self.decay)

    def _filter_spectra(self, length):
        """Inference: the spectra of all this operator's filters at ``length``
        (an (order * D, n/2 + 2) c64 tensor, filter i in rows i*D .. i*D + D),
        made by two launches (the fused filter kernel and one rfft) and kept
        until a filter weight, the decay or the length changes (buffer write
        versions), or None when the fused filter kernel does not apply."""
        from .module import _source_key

        srcs = [self.decay]
        for filt in self.filter_mlp:
            srcs.extend(p for _, p in filt.named_parameters())
        n = self._fft_size(length)
        key = _source_key(srcs, length, n)
        entry = self.__dict__.get("_spectra")
        if entry is not None and entry[1] == key:
            return entry[0]
        hs = self._filters_fused(length)
        if hs is None:
            return None
        spec = functional.filter_spectrum(hs.reshape((self.order * self.d_model, length)), n)
        object.__setattr__(self, "_spectra", (spec, key))
        return spec

    def forward(self, x, residual=None):
        _, length, _ = x.shape
        if context.MODE != 0:
            # inference: each projection, its transpose and the short conv are
            # one GEMM writing (B, channels, L); the gates are channel slices
            conv = self.short_conv
            v = functional.linear_short_conv(x, self.proj_v.weight, self.proj_v.bias,
                                             conv.weight, conv.bias)
            g = functional.linear_short_conv(x, self.proj_x.weight, self.proj_x.bias,
                                             conv.weight, conv.bias)
            D = self.d_model
            gates = [g[:, i * D:(i + 1) * D, :] for i in range(self.order)]
        else:
            v = self.proj_v(x)
            gates = list(self.proj_x(x).chunk(self.order, dim=-1))
            v = v.transpose(1, 2)
            gates = [g.transpose(1, 2) for g in gates]
            v = self.short_conv(v)
            gates = [self.short_conv(g) for g in gates]
        z = v
        spec = self._filter_spectra(length) if context.MODE != 0 else None
        D = self.d_model
        for i in range(self.order):
            if spec is not None:
                # the filter spectra do not depend on the input: kept between calls
                z = functional.fftconv_spectrum(z, spec[i * D:(i + 1) * D],
                                                self._fft_size(length), out_len=length,
                                                gate=gates[i])
                continue
            h = self.filter_mlp[i](length)
            h = h * self._decay_window(i, length)
            z = self.fft_conv1d(z, h, gate=gates[i])
        if residual is not None:
            # the block's residual add rides in the projection's GEMM epilogue
            return functional.linear(z.transpose(1, 2), self.out_proj.weight, self.out_proj.bias,
                                     residual=residual)
        return self.out_proj(z.transpose(1, 2))


class HyenaBlock(Module):
    def __init__(self, d_model, mlp_ratio=4, hidden_dim=None, order=2, short_conv_kernel=3,
                 filter_hidden=64, pe_features=8, filter_omega=10.0):
        super().__init__()
        self.norm1 = RMSNorm(d_model)
        self.mixer = HyenaOperator(d_model, order=order, short_conv_kernel=short_conv_kernel,
                                   filter_hidden=filter_hidden, pe_features=pe_features,
                                   filter_omega=filter_omega)
        self.norm2 = RMSNorm(d_model)
        self.feed_forward = SwiGLU(d_model, hidden_dim=hidden_dim, mlp_ratio=mlp_ratio)

    def forward(self, x):
        if context.MODE != 0:
            # inference: both residual adds ride in GEMM epilogues (same values)
            # (the RMSNorm outputs feed only TF32 products: stored rounded)
            x = self.mixer.forward(self.norm1.forward_into_gemm(x), residual=x)
            return self.feed_forward.forward(self.norm2.forward_into_gemm(x), residual=x)
        x = x + self.mixer(self.norm1(x))
        x = x + self.feed_forward(self.norm2(x))
        return x


class Hyena(Module):
    def __init__(self, vocab_size, d_model=256, n_layers=8, mlp_ratio=4, hidden_dim=None,
                 tie_weights=True, embed_init_std=0.02, order=2, short_conv_kernel=3,
                 filter_hidden=64, pe_features=8, filter_omega=10.0):
        super().__init__()
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.order = order
        self.embed = Embedding(vocab_size, d_model, init_std=embed_init_std)
        self.layers = ModuleList(
            [HyenaBlock(d_model, mlp_ratio=mlp_ratio, hidden_dim=hidden_dim, order=order,
                        short_conv_kernel=short_conv_kernel, filter_hidden=filter_hidden,
                        pe_features=pe_features, filter_omega=filter_omega)
             for _ in range(n_layers)]
        )
        self.norm = RMSNorm(d_model)
        self.head = TiedLinear(self.embed) if tie_weights else Linear(d_model, vocab_size)

    def forward(self, x):
        h = self.embed(x)
        for block in self.layers:
            h = block(h)
        return self.head(self.norm.forward_into_gemm(h))


__all__ = [
    "Sine",
    "PositionalEncoding",
    "CausalShortConv1d",
    "ImplicitFilter",
    "HyenaOperator",
    "SwiGLU",
    "HyenaBlock",
    "TiedLinear",
    "Hyena",
]
