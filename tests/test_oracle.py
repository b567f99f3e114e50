"""CPU tests: the oracle against the reference's golden vectors and against
independent float64 implementations (no GPU needed)."""

import os

import numpy as np
import pytest

from oracle import init, kernels as K, models

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_golden.npz")


@pytest.fixture(scope="module")
def g():
    with np.load(GOLDEN) as data:
        return {k: data[k] for k in data.files}


# ------------------------------------------------------------ golden vectors

def test_golden_causal_conv1d(g):
    np.testing.assert_allclose(K.causal_conv1d(g["cconv_x"], g["cconv_w"], g["cconv_b"]),
                               g["cconv_out"], rtol=1e-6, atol=1e-6)
    xt = np.transpose(g["cconvT_x_bld"], (0, 2, 1))
    np.testing.assert_allclose(K.causal_conv1d(xt, g["cconvT_w"], g["cconvT_b"]),
                               g["cconvT_out"], rtol=1e-6, atol=1e-6)


def test_golden_embedding_bit_exact(g):
    assert np.array_equal(K.embed(g["emb_ids"], g["emb_w"]), g["emb_out"])


def test_golden_pooling(g):
    for hw in [(1, 1), (3, 4), (5, 5)]:
        np.testing.assert_allclose(K.adaptive_avgpool2d(g["pool_x"], hw),
                                   g[f"apool_{hw[0]}x{hw[1]}"], rtol=1e-6, atol=1e-7)
    v, i = K.maxpool2d(g["pool_x"], (3, 3), (2, 2), (1, 1))
    assert np.array_equal(v, g["mpool_val"]) and np.array_equal(i, g["mpool_idx"])
    v, i = K.maxpool2d(g["mpool_stem_x"], (3, 3), (2, 2), (1, 1))
    assert np.array_equal(v, g["mpool_stem_val"]) and np.array_equal(i, g["mpool_stem_idx"])


def test_golden_activations(g):
    x = g["act_x"]
    assert np.array_equal(K.relu(x), g["act_relu"])
    np.testing.assert_allclose(K.gelu(x), g["act_gelu"], atol=1e-3)       # reference atol
    np.testing.assert_allclose(K.sigmoid(x), g["act_sigmoid"], atol=1e-5)
    s = g["act2_x"]
    for name in ("sin", "cos", "exp"):
        np.testing.assert_allclose(K.unary(s, name), g[f"act2_{name}"], atol=1e-6)
    np.testing.assert_allclose(K.unary(g["act2_logx"], "log"), g["act2_log"], atol=1e-5)
    np.testing.assert_allclose(K.softmax(g["softmax_x"]), g["softmax_out"], atol=1e-5)


def test_golden_reductions(g):
    r = g["red_x"]
    np.testing.assert_allclose(K.reduce(r, None), g["red_sum_all"], atol=1e-4)
    np.testing.assert_allclose(K.reduce(r, 0), g["red_sum_0"], atol=1e-4)
    np.testing.assert_allclose(K.reduce(r, 1, keepdims=True), g["red_sum_1_keep"], atol=1e-4)
    np.testing.assert_allclose(K.reduce(r, -1, mode=1), g["red_mean_last"], atol=1e-4)
    v, i = K.argminmax(g["mm_x"], 1, 0)
    assert np.array_equal(v, g["mm_max1"]) and np.array_equal(i, g["mm_argmax1"])
    v, _ = K.argminmax(g["mm_x"], 0, 1)
    assert np.array_equal(v, g["mm_min0"])


def test_golden_norms(g):
    x = g["ln_x"]
    y, _, _ = K.layernorm(x, np.ones(4, np.float32), np.zeros(4, np.float32), -1)
    np.testing.assert_allclose(y, g["ln_out"], atol=1e-4)
    y, _ = K.rmsnorm(g["rms_x"], np.ones(4, np.float32), -1)
    np.testing.assert_allclose(y, g["rms_out"], atol=1e-4)


def test_golden_positional_encoding(g):
    # tests/common.py:33-39 assert_close: atol=1e-6 with the default rtol=1e-4
    np.testing.assert_allclose(models._pe(8, 4), g["pe_8_4"], atol=1e-6, rtol=1e-4)


# ------------------------------------------------------------ independent float64 checks

def test_matmul_oracle_vs_einsum(rng):
    a = rng.standard_normal((3, 17, 9)).astype(np.float32)
    b = rng.standard_normal((9, 11)).astype(np.float32)
    bias = rng.standard_normal((3, 17, 11)).astype(np.float32)
    ref = np.einsum("bmk,kn->bmn", a.astype(np.float64), b.astype(np.float64)) + bias
    np.testing.assert_allclose(K.matmul_add(a, b, bias), ref, rtol=1e-6, atol=1e-6)
    bt = rng.standard_normal((3, 11, 9)).astype(np.float32)
    ref = np.einsum("bmk,bnk->bmn", a.astype(np.float64), bt.astype(np.float64))
    np.testing.assert_allclose(K.matmul_add(a, bt, None, transpose_b=True), ref, rtol=1e-6,
                               atol=1e-6)


def test_conv2d_oracle_vs_direct_loops(rng):
    x = rng.standard_normal((2, 3, 7, 6)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 3)).astype(np.float32)
    out = K.conv2d(x, w, (2, 1), (1, 2), (1, 2))
    B, C, H, W = x.shape
    Ho = (H + 2 - 2 - 1) // 2 + 1
    Wo = (W + 4 - 4 - 1) // 1 + 1
    ref = np.zeros((2, 4, Ho, Wo))
    for o in range(4):
        for y in range(Ho):
            for xx in range(Wo):
                for c in range(C):
                    for i in range(3):
                        for j in range(3):
                            ih, iw = y * 2 - 1 + i, xx - 2 + 2 * j
                            if 0 <= ih < H and 0 <= iw < W:
                                ref[:, o, y, xx] += x[:, c, ih, iw] * w[o, c, i, j]
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)


def test_fft_oracle_roundtrip_and_linearity(rng):
    x = rng.standard_normal((3, 100))
    X = K.rfft(x, 256)
    np.testing.assert_allclose(K.irfft(X, 256)[:, :100], x, atol=1e-5)
    h = rng.standard_normal((3, 100))
    direct = np.stack([np.convolve(x[i], h[i])[:100] for i in range(3)])
    np.testing.assert_allclose(K.fftconv(x[None], h, 256)[0], direct, atol=1e-4)


def test_argmax_oracle_against_lane_simulation(rng):
    """The vectorised tie rule equals a literal 256-lane simulation."""
    x = rng.integers(0, 4, size=(5, 777)).astype(np.float32)
    v, idx = K.argminmax(x, 1, 0)
    for row in range(5):
        best = [np.float32(-1e38)] * 256
        arg = [0] * 256
        for lane in range(256):
            for r in range(lane, 777, 256):
                if x[row, r] > best[lane]:
                    best[lane], arg[lane] = x[row, r], r
        s = 128
        while s >= 1:
            for t in range(s):
                if best[t + s] > best[t]:
                    best[t], arg[t] = best[t + s], arg[t + s]
            s //= 2
        assert v[row] == best[0] and idx[row] == arg[0]


def test_state_dict_generators_shapes():
    sd = init.gpt2_state_dict(0, 64, 16, 4, 2, 8)
    assert sd["blocks.1.mlp.0.weight"].shape == (16, 64)
    assert np.array_equal(sd["blocks.0.ln1.weight"], sd["blocks.0.ln1.weightg"])
    sd2 = init.gpt2_state_dict(0, 64, 16, 4, 2, 8)
    assert all(np.array_equal(sd[k], sd2[k]) for k in sd)
    r = init.resnet18_state_dict(0, 10)
    assert r["layer2.0.shortcut.0.W"].shape == (128, 64, 1, 1)
    assert "layer1.0.shortcut.0.W" not in r
    h = init.hyena_state_dict(0, 64, 32, 2, 3)
    assert h["layers.0.mixer.proj_x.weight"].shape == (32, 96)
    assert h["layers.1.feed_forward.w1.weight"].shape == (32, int(2 * 4 * 32 / 3))


def _hyena_structural_count(V, D, N, order, k=3, filter_hidden=64, pe_features=8):
    """Hyena's parameter total from its structure (reference
    tests/test_hyena.py:83-113): per block norm1 D, proj_v / proj_x / out_proj
    (2 + order) D^2, the short conv k D + D, order filter MLPs
    (2F+1) h + h + h D + D, the decay order D, norm2 D, SwiGLU 3 D ffn with
    ffn = int(8 D / 3); plus the tied embedding V D and the final norm D."""
    ffn = int(2 * (4 * D) / 3)
    fin = 2 * pe_features + 1
    block = (D + (2 + order) * D * D + (k * D + D)
             + order * (fin * filter_hidden + filter_hidden + filter_hidden * D + D)
             + order * D + D + 3 * D * ffn)
    return N * block + V * D + D


def test_hyena_state_dict_parameter_counts_match_reference():
    """The Hyena state dict holds the reference's parameter total for orders
    1-4 (reference tests/test_hyena.py:116-124) and, for its HyenaLLM
    configuration (vocab 2048, dim 256, depth 6, order 4), the quoted
    6 444 288 plus 6 * 4 * 2 * 8 * 64 for the filters' positional encoding
    (tests/test_hyena.py:126-132).  The GPU model tests load this state dict
    into ``wxx_b200.nn.Hyena`` strictly (every key, no extra key, equal
    shapes), so the product model holds the same total."""
    for order in (1, 2, 3, 4):
        sd = init.hyena_state_dict(0, 32, 16, 2, order)
        assert sum(a.size for a in sd.values()) == _hyena_structural_count(32, 16, 2, order)
    sd = init.hyena_state_dict(0, 2048, 256, 6, 4)
    total = sum(a.size for a in sd.values())
    assert total == _hyena_structural_count(2048, 256, 6, 4)
    assert total == 6_444_288 + 6 * 4 * 2 * 8 * 64


def test_model_oracles_fast_vs_exact():
    sd = init.gpt2_state_dict(0, 64, 32, 4, 2, 16)
    ids = init.token_ids(1, 2, 16, 64)
    a = models.gpt2_forward(sd, ids, 4, 2)
    b = models.gpt2_forward(sd, ids, 4, 2, fast=True)
    assert np.abs(a - b).max() < 1e-4


def test_gpt2_training_oracle_matches_finite_differences():
    """oracle.train's hand-written backward against central differences of its
    own float64 loss on a tiny GPT2 (every parameter kind sampled)."""
    from oracle import init, train

    V, D, H, L, S = 16, 8, 2, 2, 5
    sd = {k: v.astype(np.float64) for k, v in init.gpt2_state_dict(3, V, D, H, L, S).items()}
    rng = np.random.default_rng(0)
    for k in sd:   # non-trivial LayerNorm affine and biases
        if k.endswith(("weightg", "weightb", "bias")):
            sd[k] = sd[k] + 0.1 * rng.standard_normal(sd[k].shape)
    ids = rng.integers(0, V, size=(2, S))
    tgt = rng.integers(0, V, size=(2, S))
    loss, grads = train.gpt2_loss_and_grads(sd, ids, tgt, H, L)
    assert np.isfinite(loss)
    keys = ["tok_emb.weight", "pos_emb.weight", "blocks.0.attn.q.weight", "blocks.1.attn.v.weight",
            "blocks.0.attn.out.weight", "blocks.1.mlp.0.weight", "blocks.0.mlp.0.bias",
            "blocks.1.mlp.2.weight", "blocks.0.mlp.2.bias", "blocks.0.ln1.weightg",
            "blocks.1.ln2.weightb", "ln_f.weightg", "ln_f.weightb"]
    eps = 1e-6
    for key in keys:
        flat = sd[key].reshape(-1)
        for idx in rng.choice(flat.size, size=min(4, flat.size), replace=False):
            old = flat[idx]
            flat[idx] = old + eps
            lp, _ = train.gpt2_loss_and_grads(sd, ids, tgt, H, L)
            flat[idx] = old - eps
            lm, _ = train.gpt2_loss_and_grads(sd, ids, tgt, H, L)
            flat[idx] = old
            fd = (lp - lm) / (2 * eps)
            an = grads[key].reshape(-1)[idx]
            assert abs(fd - an) <= 1e-6 + 1e-5 * abs(fd), (key, idx, fd, an)


def test_adamw_oracle_first_step():
    from oracle import train

    p = np.array([1.0, -2.0, 0.5])
    g = np.array([0.1, -0.2, 0.0])
    z = np.zeros(3)
    p1, m1, v1 = train.adamw_step(p, g, z, z, 1, 1e-2, 0.9, 0.999, 1e-7, 1e-4)
    # at t = 1 the bias-corrected moments are g and g^2: the step is ~ sign(g)
    step = np.where(g != 0, g / (np.abs(g) + 1e-7), 0.0)
    assert np.allclose(p1, p - 1e-2 * (step + 1e-4 * p))
    assert np.allclose(m1, 0.1 * g) and np.allclose(v1, 0.001 * g * g)


def _amax_key(slot):
    """bit-reversed 8-bit slot index (the reduce tree's tie order)."""
    return int(format(slot & 255, "08b")[::-1], 2)


def _tiled_argmax(row):
    """The fused LM-head argmax's rule (per 256-column tile the best column,
    equal values to the smaller key, values must exceed -1e38; then the tiles
    merged in order with the same rule), restated on the host."""
    n = len(row)
    best_v, best_c, best_t = np.float32(-1e38), 0x7FFFFFFF, 0
    for t in range((n + 255) // 256):
        tv, tc = np.float32(-1e38), 0
        for c in range(min(256, n - 256 * t)):
            v = row[256 * t + c]
            if v > tv or (v == tv and tv > np.float32(-1e38) and _amax_key(c) < _amax_key(tc)):
                tv, tc = v, c
        if tv > best_v or (tv == best_v and best_v > np.float32(-1e38)
                           and _amax_key(tc) < _amax_key(best_c)):
            best_v, best_c, best_t = tv, tc, t
    return best_t * 256 + best_c if best_v > np.float32(-1e38) else 0


def test_tiled_argmax_rule_matches_reference_tree():
    """The per-tile maxima merged by bit-reversed slot order give the index of
    reduce_minmax.wgsl's lane tree (ties, NaN, -1e38 included)."""
    rng = np.random.default_rng(5)
    for n in (5, 256, 300, 700, 1500):
        for _ in range(40):
            row = rng.integers(-3, 4, size=n).astype(np.float32)
            row[rng.random(n) < 0.1] = np.nan
            row[rng.random(n) < 0.05] = np.float32(-1e38)
            _, ref = K.argminmax(row[None, :], axis=1)
            assert _tiled_argmax(row) == int(ref[0])
