"""CPU oracle for GPT2 training: loss, gradients and one AdamW step.

TEST INFRASTRUCTURE ONLY (see oracle/kernels.py).  float64 numpy, written out
op by op (forward with saved activations, then the chain rule backwards), for
the same graph the reference trains:
  forward        nn/gpt.py:92-106, nn/module.py:460-495 (dropout 0)
  loss           nn/loss.py CCELoss: mean over rows of cceloss.wgsl's
                 log(sum exp z) - z[target]
  backward       autograd/*.py backward methods: matmul (utils.py:40-142),
                 meanvarnorm (normalization.py:35-67), gelu (pointwise.py:328,
                 gelubackwards.wgsl), softmax (reductions.py:11-36), Embedding
                 (layers.py:44-71), CrossEntropyLoss (layers.py:6-20)
  AdamW          nn/optimizer.py:38-84, adamw.wgsl
The tied LM head's weight is the token embedding: its gradient is the sum of
the head's and the lookup's.
"""

import numpy as np

F64 = np.float64


def _ln_fwd(x, g, b, eps=1e-5):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    inv = np.where(var > 0, 1.0 / np.sqrt(var + eps), 0.0)
    xh = (x - mu) * inv
    return xh * g + b, (xh, inv)


def _ln_bwd(dy, cache, g):
    xh, inv = cache
    dxh = dy * g
    dx = inv * (dxh - dxh.mean(-1, keepdims=True) - xh * (dxh * xh).mean(-1, keepdims=True))
    red = tuple(range(dy.ndim - 1))
    return dx, (dy * xh).sum(red), dy.sum(red)


_C = 0.7978845608


def _gelu(x):
    u = _C * (x + 0.044715 * x ** 3)
    y = 0.5 * x * (1.0 + np.tanh(u))
    return np.where(x > 10, x, np.where(x < -10, 0.0, y))


def _gelu_slope(x):
    t = np.tanh(_C * (x + 0.044715 * x ** 3))
    s = 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * _C * (1.0 + 0.134145 * x * x)
    return np.where(x > 10, 1.0, np.where(x < -10, 0.0, s))


def gpt2_loss_and_grads(sd, ids, targets, n_heads, n_layers):
    """(loss, {state-dict key: gradient}) of CCELoss(GPT2(ids)) against
    ``targets`` (one id per position)."""
    P = {k: np.asarray(v, F64) for k, v in sd.items()}
    ids = np.asarray(ids)
    B, S = ids.shape
    tok, pos = P["tok_emb.weight"], P["pos_emb.weight"]
    V, D = tok.shape
    H, hd = n_heads, D // n_heads
    scale = 1.0 / np.sqrt(hd)
    mask = np.where(np.arange(S)[None, :] <= np.arange(S)[:, None], 0.0, -1e9)
    h = tok[ids] + pos[None, :S]
    caches = []
    for i in range(n_layers):
        p = f"blocks.{i}."
        x1, c1 = _ln_fwd(h, P[p + "ln1.weightg"], P[p + "ln1.weightb"])

        def heads(t):
            return t.reshape(B, S, H, hd).transpose(0, 2, 1, 3)

        q, k, v = (heads(x1 @ P[p + f"attn.{w}.weight"]) for w in "qkv")
        s = q @ k.transpose(0, 1, 3, 2) * scale + mask
        s = s - s.max(-1, keepdims=True)
        pr = np.exp(s)
        pr /= pr.sum(-1, keepdims=True)
        o = (pr @ v).transpose(0, 2, 1, 3).reshape(B, S, D)
        h1 = h + o @ P[p + "attn.out.weight"]
        x2, c2 = _ln_fwd(h1, P[p + "ln2.weightg"], P[p + "ln2.weightb"])
        u = x2 @ P[p + "mlp.0.weight"] + P[p + "mlp.0.bias"]
        gu = _gelu(u)
        h_next = h1 + gu @ P[p + "mlp.2.weight"] + P[p + "mlp.2.bias"]
        caches.append((h, x1, c1, q, k, v, pr, o, h1, x2, c2, u, gu))
        h = h_next
    xf, cf = _ln_fwd(h, P["ln_f.weightg"], P["ln_f.weightb"])
    z = (xf @ tok.T).reshape(B * S, V)
    zm = z - z.max(-1, keepdims=True)
    lse = np.log(np.exp(zm).sum(-1))
    t = np.asarray(targets).reshape(-1)
    rows = B * S
    loss = float((lse - zm[np.arange(rows), t]).mean())

    G = {k: np.zeros_like(v) for k, v in P.items()}
    dz = np.exp(zm - lse[:, None])
    dz[np.arange(rows), t] -= 1.0
    dz = (dz / rows).reshape(B, S, V)
    G["tok_emb.weight"] += dz.reshape(rows, V).T @ xf.reshape(rows, D)
    dh, G["ln_f.weightg"], G["ln_f.weightb"] = _ln_bwd(dz @ tok, cf, P["ln_f.weightg"])
    for i in reversed(range(n_layers)):
        p = f"blocks.{i}."
        h, x1, c1, q, k, v, pr, o, h1, x2, c2, u, gu = caches[i]
        df = dh
        G[p + "mlp.2.weight"] = gu.reshape(rows, -1).T @ df.reshape(rows, D)
        G[p + "mlp.2.bias"] = df.sum((0, 1))
        du = (df @ P[p + "mlp.2.weight"].T) * _gelu_slope(u)
        G[p + "mlp.0.weight"] = x2.reshape(rows, D).T @ du.reshape(rows, -1)
        G[p + "mlp.0.bias"] = du.sum((0, 1))
        dx2, G[p + "ln2.weightg"], G[p + "ln2.weightb"] = _ln_bwd(du @ P[p + "mlp.0.weight"].T,
                                                                 c2, P[p + "ln2.weightg"])
        dh1 = dh + dx2
        G[p + "attn.out.weight"] = o.reshape(rows, D).T @ dh1.reshape(rows, D)
        do = (dh1 @ P[p + "attn.out.weight"].T).reshape(B, S, H, hd).transpose(0, 2, 1, 3)
        dp = do @ v.transpose(0, 1, 3, 2)
        dv = pr.transpose(0, 1, 3, 2) @ do
        ds = pr * (dp - (dp * pr).sum(-1, keepdims=True)) * scale
        dq = ds @ k
        dk = ds.transpose(0, 1, 3, 2) @ q

        def merge(t):
            return t.transpose(0, 2, 1, 3).reshape(B, S, D)

        dx1 = np.zeros_like(x1)
        for w, dt in zip("qkv", (dq, dk, dv)):
            dt = merge(dt)
            G[p + f"attn.{w}.weight"] = x1.reshape(rows, D).T @ dt.reshape(rows, D)
            dx1 += dt @ P[p + f"attn.{w}.weight"].T
        dxl, G[p + "ln1.weightg"], G[p + "ln1.weightb"] = _ln_bwd(dx1, c1, P[p + "ln1.weightg"])
        dh = dh1 + dxl
    np.add.at(G["tok_emb.weight"], ids.reshape(-1), dh.reshape(rows, D))
    G["pos_emb.weight"][:S] += dh.sum(0)
    return loss, G


def adamw_step(p, g, m, v, t, lr, beta1, beta2, eps, weight_decay):
    """adamw.wgsl on float64 arrays; returns (p, m, v) after step t (1-based)."""
    p, g, m, v = (np.asarray(a, F64) for a in (p, g, m, v))
    m = beta1 * m + (1 - beta1) * g
    v = beta2 * v + (1 - beta2) * g * g
    step = (m / (1 - beta1 ** t)) / (np.sqrt(v / (1 - beta2 ** t)) + eps)
    return p - lr * (step + weight_decay * p), m, v
