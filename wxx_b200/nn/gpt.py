"""GPT-2 style decoder (reference: src/wxx/nn/gpt.py)."""

import numpy as np

from .. import functional
from ..Tensor import Tensor
from ..backend import context
from ..functional.utils import from_numpy
from .module import (
    GELU,
    kmajor_weight,
    Dropout,
    Embedding,
    LayerNorm,
    Linear,
    Module,
    ModuleList,
    MultiHeadAttention,
    Sequential,
    TiedLinear,
)


class GPT2Block(Module):
    """Pre-LN block: causal self-attention + GELU MLP."""

    def __init__(self, d_model, n_heads, dropout=0.1):
        super().__init__()
        self.ln1 = LayerNorm(d_model)
        self.attn = MultiHeadAttention(d_model, n_heads)
        self.ln2 = LayerNorm(d_model)
        self.mlp = Sequential(Linear(d_model, 4 * d_model), GELU(), Linear(4 * d_model, d_model))
        self.drop = Dropout(dropout)

    def forward(self, x, mask=None, kv_cache=None):
        if context.MODE != 0:
            # Dropout is the identity: the residual adds and the GELU ride in
            # the GEMM epilogues (same values as the unfused lines below).
            # Under inference mode the LayerNorm outputs and the GELU output
            # feed only TF32 products and are stored rounded to TF32.
            h = self.attn.forward(self.ln1.forward_into_gemm(x), mask, residual=x,
                                  kv_cache=kv_cache)
            fc1, act, fc2 = self.mlp._modules.values()
            if isinstance(fc1, Linear) and isinstance(act, GELU) and isinstance(fc2, Linear):
                return self._mlp_inference(h)
            return h + self.mlp(self.ln2(h))
        if kv_cache is not None:
            raise RuntimeError("the K/V cache is filled under inference mode only")
        x = x + self.drop(self.attn(self.ln1(x), mask))
        x = x + self.drop(self.mlp(self.ln2(x)))
        return x

    def _mlp_inference(self, h):
        """h + FC2(GELU(FC1(LN2(h)))) over cached K-major (TF32-rounded in tf32
        mode) weight copies, GELU and the residual in the GEMM epilogues."""
        fc1, _, fc2 = self.mlp._modules.values()
        rnd = functional.get_matmul_mode() == "tf32"
        u = functional.linear(self.ln2.forward_into_gemm(h),
                              kmajor_weight(self, "_fc1_t", [fc1], rnd), fc1.bias,
                              activation="gelu", feeds_tf32=True, transpose_weight=True)
        return functional.linear(u, kmajor_weight(self, "_fc2_t", [fc2], rnd), fc2.bias,
                                 residual=h, transpose_weight=True)

    def decode(self, x, kv_cache, cur_len, max_len):
        """The block for one new position per sequence, ``x`` (batch, d_model)
        (inference mode; see ``MultiHeadAttention.decode``)."""
        h = self.attn.decode(x, kv_cache, cur_len, max_len, residual=x, ln=self.ln1)
        fc1, act, fc2 = self.mlp._modules.values()
        if isinstance(fc1, Linear) and isinstance(act, GELU) and isinstance(fc2, Linear):
            # ln2 -> fc1 + GELU in one few-rows launch, fc2 + residual in another
            rnd = functional.get_matmul_mode() == "tf32"
            u = functional.ln_linear(h, self.ln2.weightg, self.ln2.weightb,
                                     kmajor_weight(self, "_fc1_t", [fc1], rnd), fc1.bias,
                                     activation="gelu", feeds_tf32=True)
            return functional.linear(u, kmajor_weight(self, "_fc2_t", [fc2], rnd), fc2.bias,
                                     residual=h, transpose_weight=True)
        return h + self.mlp(self.ln2(h))


class GPT2(Module):
    def __init__(self, vocab_size, d_model=256, n_heads=8, n_layers=6, max_len=256, dropout=0.1,
                 tie_weights=True):
        super().__init__()
        self.vocab_size = vocab_size
        self.max_len = max_len
        self.tok_emb = Embedding(vocab_size, d_model, init_std=0.02)
        self.pos_emb = Embedding(max_len, d_model, init_std=0.02)
        self.blocks = ModuleList([GPT2Block(d_model, n_heads, dropout) for _ in range(n_layers)])
        self.ln_f = LayerNorm(d_model)
        self.head = TiedLinear(self.tok_emb) if tie_weights else Linear(d_model, vocab_size,
                                                                          bias=False)
        self._gpt2_init()
        object.__setattr__(self, "_causal_mask_cache", None)
        object.__setattr__(self, "_pos_cache", {})

    def _gpt2_init(self):
        """Every >=2-D non-embedding weight ~ N(0, 0.02), biases 0 (gpt.py:66-73)."""
        for name, p in self.named_parameters():
            if name.endswith(("tok_emb.weight", "pos_emb.weight")):
                continue
            if len(p.shape) >= 2:
                functional.assign(p, functional.normal(0, 0.02, p.shape))
            elif name.endswith("bias"):
                functional.assign(p, 0.0)

    def causal_mask(self, seq):
        """Additive (seq, seq) mask, 0 on and below the diagonal, -1e9 above."""
        mask = self._causal_mask_cache
        if mask is None:
            r = np.arange(self.max_len)[:, None]
            c = np.arange(self.max_len)[None, :]
            mask = from_numpy(np.where(c <= r, 0.0, -1e9).astype(np.float32))
            object.__setattr__(self, "_causal_mask_cache", mask)
        # The tag lets MultiHeadAttention skip masked key blocks instead of
        # reading the mask (the values are the same -1e9 upper triangle).
        view = mask if seq == self.max_len else mask.narrow(0, 0, seq).narrow(1, 0, seq)
        view._wxx_causal = True
        return view

    def _positions(self, seq):
        pos = self._pos_cache.get(seq)
        if pos is None:
            pos = from_numpy(np.arange(seq, dtype=np.uint32).reshape(1, seq), dtype=np.uint32)
            self._pos_cache[seq] = pos
        return pos

    def forward(self, x, mask=None):
        b, seq = x.shape
        if seq > self.max_len:
            raise ValueError(f"sequence length {seq} > max_len {self.max_len}")
        if mask is None:
            mask = self.causal_mask(seq)
        h = self.tok_emb(x) + self.pos_emb(self._positions(seq))
        for block in self.blocks:
            h = block(h, mask)
        return self.head(self.ln_f.forward_into_gemm(h))

    def forward_argmax(self, x, mask=None):
        """``forward(x).max(-1)[1]``: the next-token id (u32) of every
        position; with the tied head the logits are never stored (the head's
        GEMM keeps each row's maximum per column tile)."""
        b, seq = x.shape
        if seq > self.max_len:
            raise ValueError(f"sequence length {seq} > max_len {self.max_len}")
        if mask is None:
            mask = self.causal_mask(seq)
        h = self.tok_emb(x) + self.pos_emb(self._positions(seq))
        for block in self.blocks:
            h = block(h, mask)
        h = self.ln_f.forward_into_gemm(h)
        if hasattr(self.head, "forward_argmax"):
            return self.head.forward_argmax(h)
        return functional.max(self.head(h), -1)[1]

    def generate(self, prompt, max_new_tokens=64, temperature=1.0, top_k=None, stop_token=None,
                 rng=None):
        """Samples up to ``max_new_tokens`` ids after ``prompt`` ((batch, seq) or
        (seq,) ids, numpy or a u32 tensor) and returns prompt + new ids as a
        uint32 array: the reference's contract (nn/gpt.py:108-170) --
        ``temperature=0`` is greedy, ``top_k`` keeps the k most likely ids,
        ``stop_token`` ends generation once every row has produced it, at most
        ``max_len`` tokens in total, draws from ``rng`` (numpy Generator).

        Runs on the device with a K/V cache: one prefill forward over the
        prompt, then one decode step per token replayed from a CUDA graph,
        sampling on the device (``wxx_b200.nn.generation``)."""
        from .generation import generate

        return generate(self, prompt, max_new_tokens=max_new_tokens, temperature=temperature,
                        top_k=top_k, stop_token=stop_token, rng=rng)


__all__ = ["GPT2", "GPT2Block"]
