"""Seeded state dicts with the reference's module-default distributions.

TEST INFRASTRUCTURE ONLY (see oracle/kernels.py).  The reference cannot seed
its initialisation (functional/utils.py:644-666 draws from an unseeded
default_rng), so parity runs draw every parameter here and load the same
arrays into the oracle and into wxx_b200 with ``load_state_dict``.  Each
parameter comes from ``default_rng([seed, crc32(name)])`` so the draw does not
depend on enumeration order.  Distributions (reference citations):
  Linear.weight (in, out) ~ N(0, sqrt(2/in)), bias 0       nn/module.py:154-164
  Embedding ~ N(0, init_std)                               nn/module.py:172-178
  GPT2: every >=2-D non-embedding param ~ N(0, 0.02)       nn/gpt.py:66-73
  Conv2D.W ~ N(0, sqrt(2/(Cin*KH*KW)))                     nn/module.py:267-268
  LayerNorm/RMSNorm/BatchNorm gamma 1, beta 0              nn/module.py:198-244
  CausalShortConv1d.weight ~ N(0, 0.02), bias 0            nn/hyena.py:90-96
  Hyena decay ~ U[0, 1)                                    nn/hyena.py:192-197
LayerNorm registers ``weight``/``bias`` as aliases of ``weightg``/``weightb``
(nn/module.py:207-208), so its four keys carry two distinct arrays.
"""

import zlib

import numpy as np

F32 = np.float32


def _rng(seed, name):
    return np.random.default_rng([int(seed), zlib.crc32(name.encode())])


def _normal(seed, name, std, shape):
    return _rng(seed, name).normal(0.0, std, size=shape).astype(F32)


def _layernorm(sd, prefix, d):
    g = np.ones(d, F32)
    b = np.zeros(d, F32)
    sd[prefix + "weightg"] = g
    sd[prefix + "weightb"] = b
    sd[prefix + "weight"] = g.copy()
    sd[prefix + "bias"] = b.copy()


def gpt2_state_dict(seed, vocab_size, d_model, n_heads, n_layers, max_len):
    sd = {}
    sd["tok_emb.weight"] = _normal(seed, "tok_emb.weight", 0.02, (vocab_size, d_model))
    sd["pos_emb.weight"] = _normal(seed, "pos_emb.weight", 0.02, (max_len, d_model))
    for i in range(n_layers):
        p = f"blocks.{i}."
        _layernorm(sd, p + "ln1.", d_model)
        for w in ("q", "k", "v", "out"):
            key = f"{p}attn.{w}.weight"
            sd[key] = _normal(seed, key, 0.02, (d_model, d_model))
        _layernorm(sd, p + "ln2.", d_model)
        sd[p + "mlp.0.weight"] = _normal(seed, p + "mlp.0.weight", 0.02, (d_model, 4 * d_model))
        sd[p + "mlp.0.bias"] = np.zeros(4 * d_model, F32)
        sd[p + "mlp.2.weight"] = _normal(seed, p + "mlp.2.weight", 0.02, (4 * d_model, d_model))
        sd[p + "mlp.2.bias"] = np.zeros(d_model, F32)
    _layernorm(sd, "ln_f.", d_model)
    return sd


def resnet18_state_dict(seed, num_classes=10):
    sd = {}

    def conv(key, cout, cin, k):
        sd[key] = _normal(seed, key, np.sqrt(2.0 / (cin * k * k)), (cout, cin, k, k))

    def bn(prefix, c):
        sd[prefix + "weight"] = np.ones(c, F32)
        sd[prefix + "bias"] = np.zeros(c, F32)

    conv("conv1.W", 64, 3, 7)
    bn("bn1.", 64)
    cin = 64
    for li, cout in enumerate((64, 128, 256, 512), start=1):
        for bi in range(2):
            p = f"layer{li}.{bi}."
            stride = 2 if (bi == 0 and li > 1) else 1
            conv(p + "conv1.W", cout, cin, 3)
            bn(p + "bn1.", cout)
            conv(p + "conv2.W", cout, cout, 3)
            bn(p + "bn2.", cout)
            if bi == 0 and (stride != 1 or cin != cout):
                conv(p + "shortcut.0.W", cout, cin, 1)
                bn(p + "shortcut.1.", cout)
            cin = cout
    sd["fc.weight"] = _normal(seed, "fc.weight", np.sqrt(2.0 / 512), (512, num_classes))
    sd["fc.bias"] = np.zeros(num_classes, F32)
    return sd


def hyena_state_dict(seed, vocab_size, d_model, n_layers, order, mlp_ratio=4, hidden_dim=None,
                     short_conv_kernel=3, filter_hidden=64, pe_features=8):
    sd = {}
    hidden = int(2 * (mlp_ratio * d_model) / 3) if hidden_dim is None else hidden_dim
    pe_out = 2 * pe_features + 1

    def lin(key, fin, fout, bias=False):
        sd[key + ".weight"] = _normal(seed, key + ".weight", np.sqrt(2.0 / fin), (fin, fout))
        if bias:
            sd[key + ".bias"] = np.zeros(fout, F32)

    sd["embed.weight"] = _normal(seed, "embed.weight", 0.02, (vocab_size, d_model))
    for i in range(n_layers):
        p = f"layers.{i}."
        sd[p + "norm1.weight"] = np.ones(d_model, F32)
        m = p + "mixer."
        sd[m + "decay"] = _rng(seed, m + "decay").random((order, d_model)).astype(F32)
        lin(m + "proj_v", d_model, d_model)
        lin(m + "proj_x", d_model, order * d_model)
        lin(m + "out_proj", d_model, d_model)
        sd[m + "short_conv.weight"] = _normal(seed, m + "short_conv.weight", 0.02,
                                              (d_model, short_conv_kernel))
        sd[m + "short_conv.bias"] = np.zeros(d_model, F32)
        for s in range(order):
            f = f"{m}filter_mlp.{s}.mlp."
            lin(f + "0", pe_out, filter_hidden, bias=True)
            lin(f + "2", filter_hidden, d_model, bias=True)
        sd[p + "norm2.weight"] = np.ones(d_model, F32)
        ff = p + "feed_forward."
        lin(ff + "w1", d_model, hidden)
        lin(ff + "w2", d_model, hidden)
        lin(ff + "w3", hidden, d_model)
    sd["norm.weight"] = np.ones(d_model, F32)
    return sd


def token_ids(seed, batch, seq, vocab):
    """Uniform u32 token ids in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, vocab, size=(batch, seq), dtype=np.uint32)
