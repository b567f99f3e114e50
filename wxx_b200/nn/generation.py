"""On-device autoregressive generation for GPT2 (interface: src/wxx/nn/gpt.py
``GPT2.generate``, lines 108-170 of the reference).

The reference samples one token per step by re-running the forward over the
whole prefix and copying the (batch, seq, vocab) logits to the host.  Here:

1. prefill: one forward over the prompt under inference mode fills per-layer
   K / V caches of shape (batch, max_len, d_model) and runs the LM head on the
   last position only;
2. every later token is a decode step over the newest position only
   (``GPT2Block.decode``): embedding, per-layer LayerNorm / QKV GEMM / cached
   attention / out projection / MLP, final LayerNorm, LM head, sampler;
3. the token count lives in device memory, so the decode step is the same
   launch sequence every time: it is recorded once as a CUDA graph and
   replayed; the sampler writes the id into the device token buffer and
   advances the count.

The sampler (``wxx_sample_tokens``) follows the reference's rule: temperature 0
takes the first index of the maximum; otherwise logits / temperature in
float64, top-k masking (values below the k-th largest dropped), softmax, and the
first index whose cumulative probability exceeds the row's uniform draw.  The
draws come from the caller's numpy generator, one ``rng.random((batch, 1))``
per step as in the reference, so equal seeds give equal samples.

The host reads the ids back once at the end, or one column per step when a
``stop_token`` is given (to stop when every row has emitted it).
"""

import numpy as np

from ..Tensor import Tensor
from ..backend import context
from ..backend import device as _dev
from ..backend.lib import F, check


class _DecodeState:
    """Device buffers of one generation call: token ids (batch, max_len),
    the token count, the sampler's counter, the draws and the K / V caches."""

    def __init__(self, model, batch):
        D = model.tok_emb.embedding_dim
        L = model.max_len
        self.batch = batch
        self.ids = Tensor._empty([batch, L], "u32")
        self.cur_len = Tensor._empty([1], "u32")      # read as an int on the device
        self.done = Tensor._empty([1], "u32")
        zero = np.zeros(1, np.uint32)
        check(F.wxx_memcpy_h2d(self.done.ptr, zero.ctypes.data, 4), "clear counter")
        self.draws = _dev.DeviceBuffer(8 * max(1, batch), "generate draws")
        self.caches = [(Tensor._empty([batch, L, D], "f32"), Tensor._empty([batch, L, D], "f32"))
                       for _ in model.blocks]

    def set_count(self, n):
        arr = np.array([n], np.uint32)
        check(F.wxx_memcpy_h2d(self.cur_len.ptr, arr.ctypes.data, 4), "upload count")

    def set_draws(self, draws):
        arr = np.ascontiguousarray(draws, np.float64).reshape(-1)
        check(F.wxx_memcpy_h2d(self.draws.ptr, arr.ctypes.data, arr.nbytes), "upload draws")


def _sample(model, state, logits, temperature, top_k):
    """Next id of every row from (batch, vocab) logits (row stride vocab)."""
    V = model.vocab_size
    check(F.wxx_sample_tokens(state.ids.ptr, model.max_len, state.cur_len.ptr, state.done.ptr,
                              logits.ptr, V, state.batch, V, float(temperature),
                              int(top_k), state.draws.ptr, model.max_len), "sample_tokens")


def _prefill(model, state, seq, temperature, top_k):
    ids = state.ids.narrow(1, 0, seq)
    mask = model.causal_mask(seq)
    h = model.tok_emb(ids) + model.pos_emb(model._positions(seq))
    for block, cache in zip(model.blocks, state.caches):
        h = block.forward(h, mask, kv_cache=cache)
    last = h.narrow(1, seq - 1, 1).reshape((state.batch, h.shape[-1]))
    logits = model.head(model.ln_f.forward_into_gemm(last))
    _sample(model, state, logits, temperature, top_k)


def _decode_step(model, state, temperature, top_k):
    B = state.batch
    D = model.tok_emb.embedding_dim
    h = Tensor._empty([B, D], "f32")
    check(F.wxx_decode_embed(h.buffer.ptr, state.ids.ptr, model.max_len, state.cur_len.ptr,
                             model.tok_emb.weight.ptr, model.pos_emb.weight.ptr, B, D,
                             model.vocab_size, model.max_len), "decode_embed")
    for block, cache in zip(model.blocks, state.caches):
        h = block.decode(h, cache, state.cur_len, model.max_len)
    if hasattr(model.head, "forward_ln"):
        logits = model.head.forward_ln(h, model.ln_f)       # ln_f and the head in one launch
    else:
        logits = model.head(model.ln_f.forward_into_gemm(h))
    _sample(model, state, logits, temperature, top_k)
    return logits


def generate(model, prompt, max_new_tokens=64, temperature=1.0, top_k=None, stop_token=None,
             rng=None, use_graph=True):
    """``GPT2.generate``: the prompt plus up to ``max_new_tokens`` sampled ids
    as a (batch, seq + n) uint32 array (see the module docstring)."""
    if isinstance(prompt, Tensor):
        prompt = prompt.numpy()
    ids = np.asarray(prompt)
    if ids.ndim == 1:
        ids = ids.reshape(1, -1)
    if ids.ndim != 2:
        raise ValueError(f"prompt must be 1D or 2D, got shape {ids.shape}")
    ids = np.ascontiguousarray(ids, np.uint32)
    batch, seq = ids.shape
    if seq == 0:
        raise ValueError("prompt must contain at least one token")
    if seq > model.max_len:
        raise ValueError(f"prompt length {seq} > max_len {model.max_len}")
    if temperature < 0:
        raise ValueError("temperature must be non-negative")
    k = 0
    if top_k is not None:
        if int(top_k) < 0:
            raise ValueError("top_k must be non-negative")
        k = min(int(top_k), model.vocab_size)
        k = 0 if k >= model.vocab_size else k
    if rng is None:
        rng = np.random.default_rng()
    n_new = min(int(max_new_tokens), model.max_len - seq)
    if n_new <= 0 or batch == 0:
        return ids

    prev_mode = context.MODE
    context.MODE = 1
    graph = None
    try:
        state = _DecodeState(model, batch)
        check(F.wxx_memcpy_h2d(state.ids.ptr, np.ascontiguousarray(
            np.pad(ids, ((0, 0), (0, model.max_len - seq)))).ctypes.data,
            batch * model.max_len * 4), "upload prompt")
        state.set_count(seq)
        sampling = temperature != 0.0

        def before_step():
            if sampling:
                state.set_draws(rng.random((batch, 1)))

        def stopped(n_done):
            if stop_token is None:
                return False
            col = state.ids.narrow(1, seq + n_done - 1, 1).numpy()
            return bool(np.all(col == np.uint32(stop_token)))

        before_step()
        _prefill(model, state, seq, temperature, k)
        made = 1
        if made < n_new and not stopped(made):
            while made < n_new:
                before_step()
                if graph is None and use_graph and n_new - made >= 3:
                    # capture() runs the step once (this step) and records it
                    from ..graph import capture

                    graph = capture(_decode_step, model, state, temperature, k)
                elif graph is not None:
                    graph.replay()
                else:
                    _decode_step(model, state, temperature, k)
                made += 1
                if stopped(made):
                    break
        out = state.ids.narrow(1, 0, seq + made).numpy()
    finally:
        context.MODE = prev_mode
        if graph is not None:
            graph.close()
    return out
