"""CPU oracle forwards of the reference's models, from a state_dict.

TEST INFRASTRUCTURE ONLY (see oracle/kernels.py).  Each forward follows the
reference module graph op by op (fp32 tensors between ops, float64 inside
each op), so the result is what the reference's WGSL path computes up to the
accumulation order of its kernels:
  GPT2      nn/gpt.py:92-106, nn/module.py:460-495 (heads via reshape(b,s,H,hd).permute(0,2,1,3))
  ResNet18  nn/resnet.py:31-79 (eval BatchNorm with running mean 0 / var 1)
  Hyena     nn/hyena.py:208-316, nn/module.py:541-594
``dtype=np.float32`` selects plain fp32 numpy math instead (used as the timed
CPU baseline, where float64 would only slow the host down).
"""

import numpy as np

from . import kernels as K

F32 = np.float32


class _Ops:
    """float64-accumulating oracle ops, or plain fp32 numpy (fast=True)."""

    def __init__(self, fast=False):
        self.fast = fast

    def mm(self, a, b, bias=None, tb=False):
        if self.fast:
            b = np.swapaxes(b, -1, -2) if tb else b
            out = np.matmul(a, b)
            return out + bias if bias is not None else out
        return K.matmul_add(a, b, bias, transpose_b=tb)

    def layernorm(self, x, g, b):
        if self.fast:
            m = x.mean(-1, keepdims=True)
            v = ((x - m) ** 2).mean(-1, keepdims=True)
            return ((x - m) / np.sqrt(v + F32(1e-5)) * g + b).astype(F32)
        return K.layernorm(x, g, b, axis=-1)[0]

    def rmsnorm(self, x, g):
        if self.fast:
            ms = (x * x).mean(-1, keepdims=True)
            return (x / np.sqrt(ms + F32(1e-6)) * g).astype(F32)
        return K.rmsnorm(x, g, axis=-1)[0]

    def softmax(self, x):
        if self.fast:
            e = np.exp(x - x.max(-1, keepdims=True))
            return (e / e.sum(-1, keepdims=True)).astype(F32)
        return K.softmax(x, -1)

    def gelu(self, x):
        if self.fast:
            u = F32(0.7978845608) * (x + F32(0.044715) * x * x * x)
            y = F32(0.5) * x * (F32(1) + np.tanh(u))
            return np.where(x > 10, x, np.where(x < -10, F32(0), y)).astype(F32)
        return K.gelu(x)

    def fftconv(self, x, h, n, L):
        if self.fast:
            spec = np.fft.rfft(x, n) * np.fft.rfft(h, n)
            return np.fft.irfft(spec, n)[..., :L].astype(F32)
        return K.fftconv(x, h, n, L)


def gpt2_forward(sd, ids, n_heads, n_layers, max_len=None, fast=False):
    """Logits [B, S, V] of GPT2 under inferenceMode (dropout off)."""
    op = _Ops(fast)
    ids = np.asarray(ids)
    B, S = ids.shape
    tok = sd["tok_emb.weight"]
    D = tok.shape[1]
    hd = D // n_heads
    max_len = sd["pos_emb.weight"].shape[0] if max_len is None else max_len
    rows = np.arange(max_len)[:, None]
    cols = np.arange(max_len)[None, :]
    mask = np.where(cols <= rows, 0.0, -1e9).astype(F32)[:S, :S]
    h = (K.embed(ids, tok) + K.embed(np.arange(S)[None, :], sd["pos_emb.weight"])).astype(F32)
    scale = F32(1.0 / np.sqrt(hd))
    for i in range(n_layers):
        p = f"blocks.{i}."
        x = op.layernorm(h, sd[p + "ln1.weightg"], sd[p + "ln1.weightb"])

        def heads(t):
            return t.reshape(B, S, n_heads, hd).transpose(0, 2, 1, 3).reshape(B * n_heads, S, hd)

        q = heads(op.mm(x, sd[p + "attn.q.weight"]))
        k = heads(op.mm(x, sd[p + "attn.k.weight"]))
        v = heads(op.mm(x, sd[p + "attn.v.weight"]))
        score = (op.mm(q, k, tb=True) * scale).astype(F32)
        attn = op.softmax((score + mask).astype(F32))
        o = op.mm(attn, v).reshape(B, n_heads, S, hd).transpose(0, 2, 1, 3).reshape(B, S, D)
        h = (h + op.mm(o, sd[p + "attn.out.weight"])).astype(F32)
        x = op.layernorm(h, sd[p + "ln2.weightg"], sd[p + "ln2.weightb"])
        x = op.gelu(op.mm(x, sd[p + "mlp.0.weight"], sd[p + "mlp.0.bias"]))
        h = (h + op.mm(x, sd[p + "mlp.2.weight"], sd[p + "mlp.2.bias"])).astype(F32)
    x = op.layernorm(h, sd["ln_f.weightg"], sd["ln_f.weightb"])
    return op.mm(x, tok, tb=True).astype(F32)


def resnet18_forward(sd, x, fast=False):
    """Logits [B, num_classes] of ResNet18 in eval mode (running mean 0, var 1)."""
    x = np.asarray(x, F32)

    def bn(t, prefix):
        return K.batchnorm_eval(t, sd[prefix + ".weight"], sd[prefix + ".bias"],
                                np.zeros(t.shape[1], F32), np.ones(t.shape[1], F32))

    def conv(t, key, stride, pad):
        w = sd[key]
        if fast:
            return _conv2d_fast(t, w, stride, pad)
        return K.conv2d(t, w, (stride, stride), (pad, pad))

    out = K.relu(bn(conv(x, "conv1.W", 2, 3), "bn1"))
    out = K.maxpool2d(out, (3, 3), (2, 2), (1, 1))[0]
    cin = 64
    for li, cout in enumerate((64, 128, 256, 512), start=1):
        for bi in range(2):
            p = f"layer{li}.{bi}."
            stride = 2 if (bi == 0 and li > 1) else 1
            y = K.relu(bn(conv(out, p + "conv1.W", stride, 1), p + "bn1"))
            y = bn(conv(y, p + "conv2.W", 1, 1), p + "bn2")
            if bi == 0 and (stride != 1 or cin != cout):
                sc = bn(conv(out, p + "shortcut.0.W", stride, 0), p + "shortcut.1")
            else:
                sc = out
            out = K.relu((y + sc).astype(F32))
            cin = cout
    pooled = K.adaptive_avgpool2d(out, (1, 1)).reshape(out.shape[0], -1)
    if fast:
        return (pooled @ sd["fc.weight"] + sd["fc.bias"]).astype(F32)
    return K.matmul_add(pooled, sd["fc.weight"], sd["fc.bias"])


def _conv2d_fast(x, w, stride, pad):
    """fp32 im2col + BLAS conv (CPU baseline path)."""
    B, C, H, W = x.shape
    O, _, KH, KW = w.shape
    Ho = (H + 2 * pad - KH) // stride + 1
    Wo = (W + 2 * pad - KW) // stride + 1
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    cols = np.empty((B, Ho, Wo, C, KH, KW), F32)
    for i in range(KH):
        for j in range(KW):
            cols[:, :, :, :, i, j] = xp[:, :, i:i + stride * (Ho - 1) + 1:stride,
                                        j:j + stride * (Wo - 1) + 1:stride].transpose(0, 2, 3, 1)
    out = cols.reshape(B * Ho * Wo, -1) @ w.reshape(O, -1).T
    return out.reshape(B, Ho, Wo, O).transpose(0, 3, 1, 2).astype(F32)


def _pe(length, features=8):
    """nn/module.py:575-594 PositionalEncoding._build."""
    t = np.linspace(0.0, 1.0, int(length), dtype=F32)
    k = np.arange(features, dtype=F32)
    ang = (2.0 * np.pi) * np.outer(t, k)
    return np.concatenate([t[:, None], np.cos(ang), np.sin(ang)], axis=1).astype(F32)


def _next_pow2(n):
    return 1 if n <= 1 else 1 << (int(n) - 1).bit_length()


def hyena_forward(sd, ids, n_layers, order, fast=False):
    """Logits [B, L, V] of Hyena (tied head, K = 8 PE features, omega = 10)."""
    op = _Ops(fast)
    ids = np.asarray(ids)
    B, L = ids.shape
    emb = sd["embed.weight"]
    D = emb.shape[1]
    n = _next_pow2(2 * L)
    h = K.embed(ids, emb)
    pe = _pe(L)

    def short_conv(t, p):
        return K.causal_conv1d(t, sd[p + "short_conv.weight"], sd[p + "short_conv.bias"])

    for i in range(n_layers):
        p = f"layers.{i}."
        x = op.rmsnorm(h, sd[p + "norm1.weight"])
        m = p + "mixer."
        v = op.mm(x, sd[m + "proj_v.weight"]).transpose(0, 2, 1)
        gx = op.mm(x, sd[m + "proj_x.weight"])
        gates = [gx[..., j * D:(j + 1) * D].transpose(0, 2, 1) for j in range(order)]
        v = short_conv(v, m)
        gates = [short_conv(g, m) for g in gates]
        z = v
        for s in range(order):
            f = f"{m}filter_mlp.{s}.mlp."
            a = op.mm(pe, sd[f + "0.weight"], sd[f + "0.bias"])
            a = K.unary((a * F32(10.0)).astype(F32), "sin")
            filt = op.mm(a, sd[f + "2.weight"], sd[f + "2.bias"]).T
            filt = (filt * K.decay_window(sd[m + "decay"], s, L)).astype(F32)
            z = (gates[s] * op.fftconv(z, filt, n, L)).astype(F32)
        y = op.mm(np.ascontiguousarray(z.transpose(0, 2, 1)), sd[m + "out_proj.weight"])
        h = (h + y).astype(F32)
        x = op.rmsnorm(h, sd[p + "norm2.weight"])
        ff = p + "feed_forward."
        w1 = op.mm(x, sd[ff + "w1.weight"])
        w2 = op.mm(x, sd[ff + "w2.weight"])
        h = (h + op.mm((K.silu(w1) * w2).astype(F32), sd[ff + "w3.weight"])).astype(F32)
    x = op.rmsnorm(h, sd["norm.weight"])
    return op.mm(x, emb, tb=True).astype(F32)


def gpt2_generate(sd, prompt, n_heads, n_layers, max_new_tokens, temperature=1.0, top_k=None,
                  stop_token=None, rng=None, max_len=None):
    """nn/gpt.py:108-170 GPT2.generate: each step runs the full forward over
    the current ids (float64 logits of the last position), then greedy
    (temperature 0: first index of the maximum) or top-k + temperature
    softmax sampling by inverse CDF with one ``rng.random((batch, 1))`` draw
    per step; stops early once every row emitted ``stop_token``."""
    ids = np.ascontiguousarray(np.asarray(prompt), dtype=np.uint32)
    if ids.ndim == 1:
        ids = ids[None, :]
    max_len = sd["pos_emb.weight"].shape[0] if max_len is None else max_len
    batch, seq = ids.shape
    steps = min(int(max_new_tokens), max_len - seq)
    for _ in range(steps):
        last = gpt2_forward(sd, ids, n_heads, n_layers)[:, -1, :].astype(np.float64)
        if temperature == 0.0:
            nxt = last.argmax(axis=-1)
        else:
            z = last / temperature
            if top_k is not None:
                k = min(int(top_k), z.shape[-1])
                if k < z.shape[-1]:
                    cut = np.partition(z, -k, axis=-1)[:, -k]
                    z[z < cut[:, None]] = -np.inf
            z -= z.max(axis=-1, keepdims=True)
            p = np.exp(z)
            p /= p.sum(axis=-1, keepdims=True)
            u = rng.random((batch, 1))
            nxt = (np.cumsum(p, axis=-1) > u).argmax(axis=-1)
        nxt = nxt.astype(np.uint32)
        ids = np.concatenate([ids, nxt[:, None]], axis=1)
        if stop_token is not None and np.all(nxt == stop_token):
            break
    return ids
