"""Kernel parity: every wxx_b200.functional op on the GPU against the CPU oracle.

Tolerances (norm-wise: max |got - ref| / max |ref|):
  integer / index / copy / gather work  bit-exact
  fp32 elementwise, reductions, norms   1e-5 (activations with transcendental
                                         functions 2e-6 absolute on unit-scale data)
  matmul / conv2d                       2e-3 in TF32 mode, 1e-5 in 3xTF32 mode
  fused attention (TF32)                4e-3: two chained TF32 products (Q K^T,
                                         then P V), each with truncated operands
  FFT (rfft / irfft / fftconv)          2e-5 of the largest output
"""

import numpy as np
import pytest

from oracle import kernels as K

pytestmark = pytest.mark.gpu


def _w():
    import wxx_b200 as wxx

    return wxx


def up(a, dtype=np.float32):
    return _w().functional.from_numpy(np.asarray(a), dtype=dtype)


def rel(got, ref):
    """max |got - ref| / max |ref|; complex arrays are compared as complex
    numbers (modulus of the difference), so imaginary parts count."""
    cplx = np.iscomplexobj(got) or np.iscomplexobj(ref)
    dt = np.complex128 if cplx else np.float64
    got = np.asarray(got, dt)
    ref = np.asarray(ref, dt)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    scale = max(np.abs(ref).max(), 1e-30) if ref.size else 1.0
    return float(np.abs(got - ref).max() / scale) if ref.size else 0.0


# ------------------------------------------------------------ elementwise / copies

@pytest.mark.parametrize("shape_a,shape_b", [((5, 7), (5, 7)), ((4, 3, 8), (8,)),
                                             ((2, 1, 6), (3, 1)), ((1031,), (1031,)),
                                             ((3, 256, 256), (256, 256))])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_pointwise_broadcast(shape_a, shape_b, op, rng):
    F = _w().functional
    a = rng.standard_normal(shape_a).astype(np.float32)
    b = rng.standard_normal(shape_b).astype(np.float32) + (3.0 if op == 3 else 0.0)
    got = F.pointwise(up(a), up(b), op).numpy()
    assert np.array_equal(got, K.pointwise(a, b, op))


def test_pointwise_strided_views(rng):
    F = _w().functional
    a = rng.standard_normal((4, 6, 8)).astype(np.float32)
    b = rng.standard_normal((8, 6)).astype(np.float32)
    ta = up(a).permute(0, 2, 1)          # (4, 8, 6) strided
    tb = up(b)[1:7:2]                    # (3, 6) strided rows... broadcast below
    got = F.pointwise(ta, up(b), 2).numpy()
    assert np.array_equal(got, np.transpose(a, (0, 2, 1)) * b)
    got2 = F.pointwise(up(a)[:, 1:4, ::2], tb[:, :4], 0).numpy()
    assert np.array_equal(got2, a[:, 1:4, ::2] + b[1:7:2][:, :4])


@pytest.mark.parametrize("op,c,rev", [(0, 1.5, 0), (1, 2.0, 1), (2, -0.5, 0), (4, 3.0, 0),
                                      (4, 2.0, 1), (3, 2.0, 0), (3, 3.0, 0), (3, 0.5, 0),
                                      (3, 2.0, 1)])
def test_scalar_ops(op, c, rev, rng):
    F = _w().functional
    x = rng.standard_normal((37, 11)).astype(np.float32)
    if op == 4 and rev:
        x = x + np.sign(x) * 0.5
    got = F.scalarpointwise(up(x), c, op, reverse=rev).numpy()
    ref = K.scalarpointwise(x, c, op, rev)
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-6, equal_nan=True)


@pytest.mark.parametrize("name", ["relu", "gelu", "sigmoid", "silu", "sin", "cos", "exp",
                                  "abs", "sign", "negate", "square"])
def test_unary(name, rng):
    F = _w().functional
    x = (rng.standard_normal(4099) * 3).astype(np.float32)
    x[:4] = [25.0, -25.0, 0.0, -0.0]
    got = getattr(F, name)(up(x)).numpy()
    ref = K.unary(x, name)
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=2e-6)


def test_contiguous_and_assign_bit_exact(rng):
    F = _w().functional
    a = rng.standard_normal((3, 5, 7, 9)).astype(np.float32)
    t = up(a)
    for view, ref in [(t.permute(3, 1, 0, 2), np.transpose(a, (3, 1, 0, 2))),
                      (t[1:, ::2, 3], a[1:, ::2, 3]),
                      (t.transpose(2, 3), np.swapaxes(a, 2, 3))]:
        assert np.array_equal(F.contiguous(view).numpy(), ref)
    dst = up(np.zeros((4, 6), np.float32))
    F.assign(dst[1:3, 2:5], up(np.arange(6, dtype=np.float32).reshape(2, 3)))
    ref = np.zeros((4, 6), np.float32)
    ref[1:3, 2:5] = np.arange(6).reshape(2, 3)
    assert np.array_equal(dst.numpy(), ref)
    F.assign(dst[:, 0], 7.0)
    ref[:, 0] = 7.0
    assert np.array_equal(dst.numpy(), ref)


@pytest.mark.parametrize("B,S,V,D", [(4, 256, 1024, 256), (8, 300, 64, 32), (2, 5, 7, 3)])
def test_embed_bit_exact(B, S, V, D, rng):
    F = _w().functional
    ids = rng.integers(0, V, size=(B, S)).astype(np.uint32)
    w = rng.standard_normal((V, D)).astype(np.float32)
    got = F.embed(up(ids, np.uint32), up(w), B * S, D).numpy()
    assert got.shape == (B, S, D)
    assert np.array_equal(got, K.embed(ids, w))


def test_causal_conv1d_dense_and_transposed(rng):
    F = _w().functional
    x = rng.standard_normal((3, 5, 40)).astype(np.float32)
    w = rng.standard_normal((5, 3)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    got = F.causal_conv1d(up(x), up(w), up(b)).numpy()
    np.testing.assert_allclose(got, K.causal_conv1d(x, w, b), rtol=1e-5, atol=1e-5)
    xt = rng.standard_normal((2, 70, 37)).astype(np.float32)     # (B, L, D)
    w2 = rng.standard_normal((37, 4)).astype(np.float32)
    b2 = rng.standard_normal(37).astype(np.float32)
    got2 = F.causal_conv1d(up(xt).permute(0, 2, 1), up(w2), up(b2)).numpy()
    np.testing.assert_allclose(got2, K.causal_conv1d(np.transpose(xt, (0, 2, 1)), w2, b2),
                               rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("B,L,D,K_", [(2, 1000, 70, 3), (3, 300, 33, 8), (1, 129, 40, 9),
                                      (2, 8192, 64, 3)])
def test_causal_conv1d_transposed_tiles(B, L, D, K_, rng):
    """Transposed (B, L, D) views: 32 x 128 tiles with ragged edges, K up to
    8 in registers, K = 9 on the generic kernel."""
    F = _w().functional
    xt = rng.standard_normal((B, L, D)).astype(np.float32)
    w = rng.standard_normal((D, K_)).astype(np.float32)
    b = rng.standard_normal(D).astype(np.float32)
    got = F.causal_conv1d(up(xt).permute(0, 2, 1), up(w), up(b)).numpy()
    np.testing.assert_allclose(got, K.causal_conv1d(np.transpose(xt, (0, 2, 1)), w, b),
                               rtol=1e-5, atol=1e-5)


def test_decay_window(rng):
    F = _w().functional
    d = rng.random((4, 33)).astype(np.float32)
    got = F.decay_window(up(d), 2, 100).numpy()
    np.testing.assert_allclose(got, K.decay_window(d, 2, 100), rtol=2e-6, atol=1e-7)


# ------------------------------------------------------------ reductions / norms

@pytest.mark.parametrize("shape,axis", [((4, 5), None), ((4, 5), 0), ((4, 5), 1),
                                        ((37, 4099), 1), ((4099, 37), 0), ((3, 300, 70), 1),
                                        ((2, 3, 4, 5), (1, 2)), ((1024, 1024), 0)])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_reduce(shape, axis, mode, rng):
    F = _w().functional
    x = rng.standard_normal(shape).astype(np.float32)
    fn = [F.sum, F.mean, F.sumsq][mode]
    got = fn(up(x), axis).numpy()
    ref = K.reduce(x, axis, mode)
    # error relative to the l2 norm of the reduced slice (sums can cancel to ~0)
    o, r, i, _ = K.reduce_dims(x.shape, axis)
    scale = np.sqrt((x.reshape(o, r, i).astype(np.float64) ** 2).sum(1)).reshape(ref.shape)
    if mode == 1:
        scale = scale / r
    if mode == 2:
        scale = ref.astype(np.float64)
    assert np.all(np.abs(got.astype(np.float64) - ref) <= 1e-5 * np.maximum(scale, 1e-12))


def test_reduce_keepdims(rng):
    F = _w().functional
    x = rng.standard_normal((4, 5)).astype(np.float32)
    assert F.sum(up(x), 1, keepdims=True).numpy().shape == (4, 1)
    assert F.mean(up(x), None, keepdims=True).numpy().shape == (1, 1)


@pytest.mark.parametrize("shape,axis", [((3, 4), 1), ((3, 4), 0), ((4, 256, 1024), -1),
                                        ((7, 1000, 3), 1), ((5, 70000), 1)])
@pytest.mark.parametrize("op", [0, 1])
def test_argminmax_bit_exact(shape, axis, op, rng):
    F = _w().functional
    x = rng.standard_normal(shape).astype(np.float32)
    vals, idx = (F.max if op == 0 else F.min)(up(x), axis)
    rv, ri = K.argminmax(x, axis, op)
    assert np.array_equal(vals.numpy(), rv)
    assert np.array_equal(idx.numpy(), ri)


def test_argmax_ties_follow_reference_tree(rng):
    """Ties resolved exactly like reduce_minmax.wgsl (not always the lowest index)."""
    F = _w().functional
    x = rng.integers(0, 3, size=(64, 1000)).astype(np.float32)   # heavy ties
    x[5, 128] = 9.0
    x[5, 64] = 9.0                                                 # slot 64 vs 128 -> 128 wins
    vals, idx = F.max(up(x), 1)
    rv, ri = K.argminmax(x, 1, 0)
    assert np.array_equal(idx.numpy(), ri)
    assert ri[5] == 128
    x2 = np.full((2, 10), -np.inf, np.float32)                     # below the -1e38 start
    v2, i2 = F.max(up(x2), 1)
    assert np.array_equal(v2.numpy(), K.argminmax(x2, 1, 0)[0])
    assert np.array_equal(i2.numpy(), np.zeros(2, np.uint32))


@pytest.mark.parametrize("n", [1, 31, 200, 256, 257, 1000, 4096, 5003])
@pytest.mark.parametrize("op", [0, 1])
def test_argminmax_ties_and_nans_all_row_lengths(n, op, rng):
    """Heavy ties and scattered NaNs on row lengths around the 256-slot and
    32-lane boundaries: indices bit-exact against the reference tree."""
    F = _w().functional
    x = rng.integers(0, 4, size=(37, n)).astype(np.float32)
    x[rng.random(x.shape) < 0.02] = np.nan
    vals, idx = (F.max if op == 0 else F.min)(up(x), 1)
    rv, ri = K.argminmax(x, 1, op)
    assert np.array_equal(idx.numpy(), ri)
    assert np.array_equal(vals.numpy(), rv, equal_nan=True)


@pytest.mark.parametrize("shape,dim", [((3, 5), -1), ((32, 256, 256), -1), ((8, 1024), -1),
                                       ((4, 3000), -1), ((6, 9, 5), 1)])
def test_softmax(shape, dim, rng):
    F = _w().functional
    x = (rng.standard_normal(shape) * 3).astype(np.float32)
    got = F.softmax(up(x), dim).numpy()
    np.testing.assert_allclose(got, K.softmax(x, dim), rtol=1e-5, atol=1e-7)


def test_masked_softmax_matches_add_then_softmax(rng):
    F = _w().functional
    x = rng.standard_normal((6, 40, 40)).astype(np.float32)
    m = np.where(np.arange(64)[None, :] <= np.arange(64)[:, None], 0.0, -1e9).astype(np.float32)
    tm = up(m).narrow(0, 0, 40).narrow(1, 0, 40)
    got = F.masked_softmax(up(x), tm).numpy()
    ref = K.softmax((x + m[:40, :40]).astype(np.float32), -1)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("shape,axis", [((2, 3, 4), -1), ((1024, 256), -1), ((8, 1024), -1),
                                        ((3, 2000), -1), ((4, 6, 5), (1, 2)), ((5, 7, 3), 1)])
def test_layernorm_rmsnorm(shape, axis, rng):
    F = _w().functional
    x = rng.standard_normal(shape).astype(np.float32)
    n = K.reduce_dims(shape, axis)[1]
    g = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    y, mean, inv = F.meanvarnorm(up(x), up(g), up(b), axis)
    ry, rm, ri = K.layernorm(x, g, b, axis)
    assert rel(y.numpy(), ry) < 1e-5
    assert rel(mean.numpy(), rm) < 1e-5 and rel(inv.numpy(), ri) < 1e-5
    y2, inv2 = F.rmsnorm(up(x), up(g), axis)
    ry2, ri2 = K.rmsnorm(x, g, axis)
    assert rel(y2.numpy(), ry2) < 1e-5 and rel(inv2.numpy(), ri2) < 1e-5


def test_norm_zero_rows_and_many_rows(rng):
    F = _w().functional
    x = rng.standard_normal((70000, 8)).astype(np.float32)   # > 65535 rows
    x[3] = 0.0
    g = np.ones(8, np.float32)
    y, inv = F.rmsnorm(up(x), up(g), -1)
    ry, ri = K.rmsnorm(x, g, -1)
    assert rel(y.numpy(), ry) < 1e-5
    assert inv.numpy()[3] == 0.0


def test_batchnorm_eval(rng):
    F = _w().functional
    x = rng.standard_normal((4, 6, 5, 5)).astype(np.float32)
    g = rng.standard_normal(6).astype(np.float32)
    b = rng.standard_normal(6).astype(np.float32)
    rm = rng.standard_normal(6).astype(np.float32)
    rv = rng.random(6).astype(np.float32) + 0.5
    y = F.batchnorm(up(x), up(g), up(b), up(rm), up(rv), False)[0].numpy()
    assert rel(y, K.batchnorm_eval(x, g, b, rm, rv)) < 1e-5


# ------------------------------------------------------------ contractions

GEMM_SHAPES = [
    # (batch_a, batch_b, M, N, K)
    ((), (), 1, 1, 1),
    ((), (), 3, 5, 7),
    ((), (), 128, 128, 128),
    ((), (), 127, 129, 33),
    ((), (), 300, 257, 96),
    ((), (), 512, 512, 512),
    ((), (), 256, 1024, 256),
    ((4,), (), 256, 256, 256),
    ((), (3,), 64, 200, 64),
    ((32,), (32,), 256, 256, 32),
    ((2, 3), (2, 3), 70, 40, 24),
    # few tiles, long K: split-K
    ((), (), 128, 256, 4096),
    ((), (), 200, 100, 3000),
    # >= 74 tiles of 256 x 256: SM-pair (cta_group::2) kernel
    ((), (), 2304, 2304, 64),
    ((), (), 2300, 2200, 100),
    ((), (), 2176, 2304, 40),
    ((2,), (2,), 1280, 2048, 96),
    ((), (), 96, 682, 256),
    ((), (), 100, 256, 682),
    ((), (), 256, 10, 512),
    ((), (), 8192 // 16, 64, 17),
]


@pytest.mark.parametrize("shape", GEMM_SHAPES)
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False)])
@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_matmul(shape, ta, tb, mode, rng):
    wxx = _w()
    F = wxx.functional
    ba, bb, M, N, K_ = shape
    a = rng.standard_normal(ba + ((K_, M) if ta else (M, K_))).astype(np.float32)
    b = rng.standard_normal(bb + ((N, K_) if tb else (K_, N))).astype(np.float32)
    F.set_matmul_mode(mode)
    try:
        got = F.matmul_add(up(a), up(b), None, transpose_A=ta, transpose_B=tb).numpy()
    finally:
        F.set_matmul_mode("tf32")
    ref = K.matmul_add(a, b, None, ta, tb)
    tol = 2e-3 if mode == "tf32" else 1e-5
    assert got.shape == ref.shape
    assert rel(got, ref) < tol, rel(got, ref)
    assert _w().backend.device_status() == 0


@pytest.mark.parametrize("bias_kind", ["N", "MN", "BMN"])
def test_matmul_bias_modes(bias_kind, rng):
    F = _w().functional
    a = rng.standard_normal((3, 70, 48)).astype(np.float32)
    b = rng.standard_normal((48, 90)).astype(np.float32)
    bias = {"N": rng.standard_normal(90), "MN": rng.standard_normal((70, 90)),
            "BMN": rng.standard_normal((3, 70, 90))}[bias_kind].astype(np.float32)
    got = F.matmul_add(up(a), up(b), up(bias)).numpy()
    assert rel(got, K.matmul_add(a, b, bias)) < 2e-3


def test_matmul_bias_alpha_pair_tiles(rng):
    """Per-column bias and alpha through the SM-pair kernel's epilogue."""
    F = _w().functional
    a = rng.standard_normal((2304, 64)).astype(np.float32)
    b = rng.standard_normal((64, 2200)).astype(np.float32)
    bias = rng.standard_normal(2200).astype(np.float32)
    got = F.matmul_add(up(a), up(b), up(bias), alpha=0.5).numpy()
    assert rel(got, 0.5 * K.matmul_add(a, b, None) + bias) < 2e-3


def test_matmul_fp32_mode_exact_products(rng):
    F = _w().functional
    a = rng.standard_normal((65, 33)).astype(np.float32)
    b = rng.standard_normal((33, 70)).astype(np.float32)
    F.set_matmul_mode("fp32")
    try:
        got = F.matmul_add(up(a), up(b), None).numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert rel(got, K.matmul_add(a, b)) < 1e-6


def test_matmul_shape_errors():
    F = _w().functional
    with pytest.raises(ValueError):
        F.matmul_add(up(np.zeros((3, 4))), up(np.zeros((5, 6))), None)
    with pytest.raises(ValueError):
        F.matmul_add(up(np.zeros((2, 3, 4))), up(np.zeros((3, 4, 6))), None)


CONV_SHAPES = [
    # B, Cin, H, W, Cout, k, stride, pad, dil
    (2, 2, 8, 8, 3, 3, 1, 1, 1),
    (4, 3, 32, 32, 64, 7, 2, 3, 1),
    (8, 64, 8, 8, 64, 3, 1, 1, 1),
    (8, 64, 8, 8, 128, 3, 2, 1, 1),
    (8, 64, 8, 8, 128, 1, 2, 0, 1),
    (4, 256, 2, 2, 512, 3, 2, 1, 1),
    (3, 5, 11, 13, 7, 3, 2, 2, 2),
    # few output tiles, long K: split-K slices + deterministic reduce
    (16, 256, 4, 4, 512, 3, 1, 1, 1),
    (32, 512, 1, 1, 512, 3, 1, 1, 1),
    (16, 128, 4, 4, 256, 3, 2, 1, 1),
]


@pytest.mark.parametrize("shape", CONV_SHAPES)
@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_conv2d(shape, mode, rng):
    F = _w().functional
    B, C, H, W, O, k, s, p, d = shape
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    w = (rng.standard_normal((O, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    bias = rng.standard_normal(O).astype(np.float32)
    F.set_matmul_mode(mode)
    try:
        got = F.conv2d(up(x), up(w), (s, s), (p, p), (d, d), up(bias)).numpy()
    finally:
        F.set_matmul_mode("tf32")
    ref = K.conv2d(x, w, (s, s), (p, p), (d, d), bias)
    assert got.shape == ref.shape
    assert rel(got, ref) < (2e-3 if mode == "tf32" else 1e-5)


@pytest.mark.parametrize("shape", CONV_SHAPES)
@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
@pytest.mark.parametrize("post", ["bn", "bn_relu", "bn_res_relu"])
def test_conv2d_bn_epilogue(shape, mode, post, rng):
    """conv2d_bn: eval batchnorm (+ residual) (+ relu) in the conv epilogue or
    the split-K reduce, against the separate conv2d / batchnorm / add / relu
    ops on the same inputs (same fp32 operations, so equal up to the
    compiler's choice of fused multiply-adds)."""
    F = _w().functional
    B, C, H, W, O, k, s, p, d = shape
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    w = (rng.standard_normal((O, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    rm = rng.standard_normal(O).astype(np.float32)
    rv = rng.uniform(0.5, 2.0, O).astype(np.float32)
    g = rng.standard_normal(O).astype(np.float32)
    b = rng.standard_normal(O).astype(np.float32)
    rmt, rvt, gt, bt = up(rm), up(rv), up(g), up(b)
    F.set_matmul_mode(mode)
    try:
        y = F.conv2d(up(x), up(w), (s, s), (p, p), (d, d))
        ref, _, _ = F.batchnorm(y, gt, bt, rmt, rvt, False)
        res = None
        if post == "bn_res_relu":
            res = up(rng.standard_normal(tuple(y.shape)).astype(np.float32))
            ref = ref + res
        if post != "bn":
            ref = F.relu(ref)
        got = F.conv2d_bn(up(x), up(w), (s, s), (p, p), (d, d), bn=(rmt, rvt, gt, bt, 1e-5),
                          residual=res, relu=post != "bn").numpy()
    finally:
        F.set_matmul_mode("tf32")
    ref = ref.numpy()
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("B,C,H,W,bias", [(256, 3, 32, 32, False), (3, 3, 17, 23, True),
                                           (2, 1, 1, 5, False), (5, 4, 32, 7, True)])
def test_resnet_stem_matches_separate_ops(B, C, H, W, bias, rng):
    """The fused stem (conv 7x7/2 + bias + eval batchnorm + ReLU + max pool
    3x3/2 + channels-last store) gives the bits of conv2d_bn -> maxpool2d ->
    permute(0, 2, 3, 1), and matches the float64 oracle convolution."""
    F = _w().functional
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    w = (rng.standard_normal((64, C, 7, 7)) * np.sqrt(2.0 / (C * 49))).astype(np.float32)
    bvec = up(rng.standard_normal(64).astype(np.float32)) if bias else None
    rm = up(rng.standard_normal(64).astype(np.float32))
    rv = up(rng.uniform(0.5, 2.0, 64).astype(np.float32))
    g = up(rng.standard_normal(64).astype(np.float32))
    b = up(rng.standard_normal(64).astype(np.float32))
    bn = (rm, rv, g, b, 1e-5)
    got = F.resnet_stem(up(x), up(w), bvec, bn=bn, relu=True)
    assert got is not None
    wp = up(np.ascontiguousarray(w.reshape(64, -1).T))          # (Cin * 49, 64)
    got_packed = F.resnet_stem(up(x), up(w), bvec, bn=bn, relu=True, packed=wp)
    assert np.array_equal(got_packed.numpy(), got.numpy())
    y = F.conv2d_bn(up(x), up(w), (2, 2), (3, 3), (1, 1), bvec, bn=bn, relu=True)
    ref = F.maxpool2d(y, (3, 3), (2, 2), (1, 1)).permute(0, 2, 3, 1).contiguous().numpy()
    got = got.numpy()
    assert got.shape == ref.shape
    assert np.array_equal(got, ref)
    conv = K.conv2d(x, w, (2, 2), (3, 3), (1, 1), None if bvec is None else bvec.numpy())
    inv = 1.0 / np.sqrt(rv.numpy().astype(np.float64) + 1e-5)
    z = (conv - rm.numpy()[None, :, None, None]) * (inv * g.numpy())[None, :, None, None] \
        + b.numpy()[None, :, None, None]
    z = np.maximum(z, 0.0)
    Ho, Wo = z.shape[2], z.shape[3]
    zp = np.full((B, 64, Ho + 2, Wo + 2), -np.inf)
    zp[:, :, 1:-1, 1:-1] = z
    Hp, Wp = (Ho - 1) // 2 + 1, (Wo - 1) // 2 + 1
    pooled = np.full((B, 64, Hp, Wp), -np.inf)
    for dy in range(3):
        for dx in range(3):
            pooled = np.maximum(pooled, zp[:, :, dy:dy + 2 * Hp - 1:2, dx:dx + 2 * Wp - 1:2])
    assert rel(got, pooled.transpose(0, 2, 3, 1)) < 1e-5


def test_resnet_stem_declines_other_shapes(rng):
    F = _w().functional
    x = up(rng.standard_normal((2, 8, 16, 16)).astype(np.float32))     # 8 input channels
    w = up(rng.standard_normal((64, 8, 7, 7)).astype(np.float32))
    assert F.resnet_stem(x, w) is None
    x = up(rng.standard_normal((2, 3, 64, 64)).astype(np.float32))     # too large
    w = up(rng.standard_normal((64, 3, 7, 7)).astype(np.float32))
    assert F.resnet_stem(x, w) is None


NHWC_SHAPES = [
    # B, Cin, H, W, Cout, k, stride, pad, dil
    (8, 64, 8, 8, 64, 3, 1, 1, 1),
    (3, 64, 8, 8, 64, 3, 1, 1, 1),        # partial last tile
    (8, 64, 8, 8, 128, 3, 2, 1, 1),
    (8, 64, 8, 8, 128, 1, 2, 0, 1),
    (4, 256, 2, 2, 512, 3, 2, 1, 1),
    (2, 32, 16, 16, 32, 3, 1, 2, 2),
    (1, 32, 3, 256, 32, 3, 1, 1, 1),       # Wo = 256: one row per tile
    (16, 256, 4, 4, 512, 3, 1, 1, 1),      # split-K
    (32, 512, 1, 1, 512, 3, 1, 1, 1),
    (16, 128, 4, 4, 256, 3, 2, 1, 1),
]


@pytest.mark.parametrize("shape", NHWC_SHAPES)
@pytest.mark.parametrize("mode,tol", [("tf32", 2e-3), ("3xtf32", 1e-5)])
@pytest.mark.parametrize("post", ["none", "bn_relu", "bn_res_relu"])
def test_conv2d_nhwc(shape, mode, tol, post, rng):
    """Channels-last convolution (TMA-box A operand) with its batchnorm /
    residual / ReLU epilogue against the oracle's NCHW convolution."""
    F = _w().functional
    B, C, H, W, O, k, s, p, d = shape
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    w = (rng.standard_normal((O, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    y = K.conv2d(x, w, (s, s), (p, p), (d, d), None).astype(np.float64)
    bn = res_t = None
    if post != "none":
        rm = rng.standard_normal(O).astype(np.float32)
        rv = rng.uniform(0.5, 2.0, O).astype(np.float32)
        g = rng.standard_normal(O).astype(np.float32)
        b = rng.standard_normal(O).astype(np.float32)
        bn = (up(rm), up(rv), up(g), up(b), 1e-5)
        sc = lambda v: v[None, :, None, None]
        y = (y - sc(rm)) / np.sqrt(sc(rv).astype(np.float64) + 1e-5) * sc(g) + sc(b)
        if post == "bn_res_relu":
            r = rng.standard_normal(y.shape).astype(np.float32)
            res_t = up(np.ascontiguousarray(r.transpose(0, 2, 3, 1)))
            y = y + r
        y = np.maximum(y, 0.0)
    xh = up(np.ascontiguousarray(x.transpose(0, 2, 3, 1)))
    F.set_matmul_mode(mode)
    try:
        got = F.conv2d_nhwc(xh, up(w), (s, s), (p, p), (d, d), bn=bn, residual=res_t,
                            relu=post != "none").numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert got.shape == (B, y.shape[2], y.shape[3], O)
    assert rel(got.transpose(0, 3, 1, 2), y) < tol


def test_conv2d_nhwc_rejects_unsupported(rng):
    F = _w().functional
    x = up(rng.standard_normal((2, 7, 7, 64)).astype(np.float32))
    w = up(rng.standard_normal((64, 64, 3, 3)).astype(np.float32))
    assert not F.conv2d_nhwc_supported(64, 64, 7, 7)
    with pytest.raises(ValueError):
        F.conv2d_nhwc(x, w, (1, 1), (1, 1), (1, 1))


def test_pooling(rng):
    F = _w().functional
    x = rng.standard_normal((4, 6, 16, 16)).astype(np.float32)
    out, idx = F.maxpool2d(up(x), (3, 3), (2, 2), (1, 1), return_indices=True)
    rv, ri = K.maxpool2d(x, (3, 3), (2, 2), (1, 1))
    assert np.array_equal(out.numpy(), rv) and np.array_equal(idx.numpy(), ri)
    for hw in [(1, 1), (3, 5), (16, 16)]:
        got = F.adaptive_avgpool2d(up(x), hw).numpy()
        assert rel(got, K.adaptive_avgpool2d(x, hw)) < 1e-6


# ------------------------------------------------------------ FFT

@pytest.mark.parametrize("rows,L,n", [(3, 5, 8), (4, 16, 16), (2, 100, 256), (3, 512, 512),
                                      (5, 1000, 1024), (2, 2047, 2048), (3, 3000, 4096),
                                      (2, 8192, 8192), (2, 8192, 16384), (2, 16384, 32768),
                                      (2, 20, 2), (3, 1, 1), (2, 40000, 65536)])
def test_rfft_irfft(rows, L, n, rng):
    F = _w().functional
    x = rng.standard_normal((rows, L)).astype(np.float32)
    spec, nn = F.rfft(up(x), n)
    assert nn == n
    ref = K.rfft(x, n)
    assert rel(spec.numpy(), ref) < 2e-5
    if n >= 2:
        back = F.irfft(spec, n).numpy()
        assert rel(back, K.irfft(ref, n)) < 2e-5


def test_irfft_truncated_and_padded_spectrum(rng):
    F = _w().functional
    X = (rng.standard_normal((3, 40)) + 1j * rng.standard_normal((3, 40))).astype(np.complex64)
    for n in (32, 128, 2048):
        got = F.irfft(F.from_numpy_complex(X), n).numpy()
        assert rel(got, K.irfft(X, n)) < 2e-5


def _crand(rng, shape):
    return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)


@pytest.mark.parametrize("conj_a,conj_b", [(False, False), (True, False), (False, True),
                                           (True, True)])
def test_complex_mul_broadcast(conj_a, conj_b, rng):
    """complex_mul.wgsl:57-61 with every conj flag: the products are compared
    as complex numbers, so a wrong sign on an imaginary part fails."""
    F = _w().functional
    a = _crand(rng, (3, 4, 9))
    b = _crand(rng, (4, 9))
    got = F.complex_mul(F.from_numpy_complex(a), F.from_numpy_complex(b),
                        conj_a=conj_a, conj_b=conj_b).numpy()
    assert got.dtype == np.complex64
    ref = K.complex_mul(a, b, conj_a=conj_a, conj_b=conj_b)
    assert rel(got, ref) < 1e-6
    assert rel(got.imag, ref.imag) < 1e-6


def test_complex_mul_strided_views(rng):
    """A transposed / sliced c64 view on either side (the reference's strided
    complex operands) against the same product of dense copies."""
    F = _w().functional
    a = _crand(rng, (5, 6, 7))
    b = _crand(rng, (7, 6))
    ta = F.from_numpy_complex(a)[:, 1:5]                      # (5, 4, 7) strided rows
    tb = F.from_numpy_complex(b).permute(1, 0)[1:5]           # (4, 7) transposed view
    got = F.complex_mul(ta, tb, conj_a=True).numpy()
    ref = K.complex_mul(a[:, 1:5], b.T[1:5], conj_a=True)
    assert rel(got, ref) < 1e-6


def test_complex_conj_and_add_inplace(rng):
    F = _w().functional
    a = _crand(rng, (3, 1000))
    b = _crand(rng, (3, 1000))
    assert np.array_equal(F.complex_conj(F.from_numpy_complex(a)).numpy(), np.conj(a))
    acc = F.from_numpy_complex(a)
    F.complex_add_inplace(acc, F.from_numpy_complex(b))
    assert np.array_equal(acc.numpy(), a + b)


@pytest.mark.parametrize("B,D,L", [(2, 3, 64), (2, 3, 200), (3, 2, 300), (3, 4, 1000),
                                   (2, 3, 1001), (2, 3, 1500), (2, 2, 3000), (2, 8, 8192),
                                   (3, 100, 8192), (1, 4, 16384), (1, 2, 40000)])
def test_fftconv_matches_reference_chain(B, D, L, rng):
    F = _w().functional
    x = rng.standard_normal((B, D, L)).astype(np.float32)
    h = rng.standard_normal((D, L)).astype(np.float32)
    n = 1 << (2 * L - 1).bit_length()
    got = F.fftconv(up(x), up(h), n, out_len=L).numpy()
    ref = K.fftconv(x, h, n, L)
    assert rel(got, ref) < 2e-5
    # the unfused reference chain through the public ops gives the same result
    chain = F.irfft(F.complex_mul(F.rfft(up(x), n)[0], F.rfft(up(h), n)[0]), n)
    assert rel(chain.numpy()[..., :L], ref) < 2e-5


@pytest.mark.parametrize("L", [300, 8192])
def test_fftconv_strided_and_unaligned_input(L, rng):
    """x as a (B, L, D) -> (B, D, L) transposed view and as a view starting
    one element into its rows (neither takes the 16-byte vector loads)."""
    F = _w().functional
    B, D = 2, 3
    n = 1 << (2 * L - 1).bit_length()
    h = rng.standard_normal((D, L)).astype(np.float32)
    xt = rng.standard_normal((B, L, D)).astype(np.float32)
    got = F.fftconv(up(xt).permute(0, 2, 1), up(h), n, out_len=L).numpy()
    assert rel(got, K.fftconv(np.ascontiguousarray(xt.transpose(0, 2, 1)), h, n, L)) < 2e-5
    xw = rng.standard_normal((B, D, L + 1)).astype(np.float32)
    got = F.fftconv(up(xw)[:, :, 1:], up(h), n, out_len=L - 5).numpy()
    assert rel(got, K.fftconv(np.ascontiguousarray(xw[:, :, 1:]), h, n, L - 5)) < 2e-5


@pytest.mark.parametrize("B,D,L", [(2, 3, 40), (3, 100, 8192), (2, 3, 1001), (1, 2, 16384),
                                   (1, 2, 40000)])
def test_fftconv_gated(B, D, L, rng):
    """gate * fftconv(x, h) in one pass (Hyena's gates[i] * fft_conv1d(z, h)):
    a dense gate and a transposed (B, L, D) -> (B, D, L) gate view, on the
    small-row, staged, pair, 14-bit and global-memory paths."""
    F = _w().functional
    n = 1 << (2 * L - 1).bit_length()
    x = rng.standard_normal((B, D, L)).astype(np.float32)
    h = rng.standard_normal((D, L)).astype(np.float32)
    g = rng.standard_normal((B, D, L)).astype(np.float32)
    ref = K.fftconv(x, h, n, L) * g
    got = F.fftconv(up(x), up(h), n, out_len=L, gate=up(g)).numpy()
    assert rel(got, ref) < 2e-5
    gt = np.ascontiguousarray(g.transpose(0, 2, 1))
    got = F.fftconv(up(x), up(h), n, out_len=L, gate=up(gt).permute(0, 2, 1)).numpy()
    assert rel(got, ref) < 2e-5


# ------------------------------------------------------------ fused attention

def _attention_ref(q, k, v, H, mask=None, causal=False):
    """Reference chain of nn/module.py:460-495 in float64 (oracle ops)."""
    B, S, D = q.shape
    Sk = k.shape[1]
    hd = D // H

    def heads(t, n):
        return t.reshape(B, n, H, hd).transpose(0, 2, 1, 3).reshape(B * H, n, hd)

    s = K.matmul_add(heads(q, S), heads(k, Sk), None, transpose_b=True) * np.float32(1 / np.sqrt(hd))
    if causal:
        m = np.where(np.arange(Sk)[None, :] <= np.arange(S)[:, None], 0.0, -1e9).astype(np.float32)
        s = s + m
    elif mask is not None:
        s = s + mask
    p = K.softmax(s.astype(np.float32), -1)
    o = K.matmul_add(p, heads(v, Sk))
    return o.reshape(B, H, S, hd).transpose(0, 2, 1, 3).reshape(B, S, D)


@pytest.mark.parametrize("B,S,H,hd,kind", [(2, 256, 4, 64, "causal"), (1, 100, 2, 32, "causal"),
                                           (2, 300, 3, 64, "mask"), (1, 128, 2, 32, "none"),
                                           (3, 200, 2, 64, "none"), (8, 1024, 16, 64, "causal"),
                                           (4, 256, 8, 32, "causal")])
def test_fused_attention(B, S, H, hd, kind, rng):
    F = _w().functional
    D = H * hd
    q = rng.standard_normal((B, S, D)).astype(np.float32)
    k = rng.standard_normal((B, S, D)).astype(np.float32)
    v = rng.standard_normal((B, S, D)).astype(np.float32)
    mask = None
    if kind == "mask":
        mask = np.where(rng.random((S, S)) < 0.3, -1e9, rng.standard_normal((S, S))).astype(np.float32)
        np.fill_diagonal(mask, 0.0)
    got = F.attention(up(q), up(k), up(v), H, mask=None if mask is None else up(mask),
                      causal=(kind == "causal")).numpy()
    ref = _attention_ref(q, k, v, H, mask, kind == "causal")
    assert got.shape == ref.shape
    assert rel(got, ref) < 4e-3, rel(got, ref)
    assert _w().backend.device_status() == 0


def _attention_ref64(q, k, v, H, mask=None, causal=False):
    """nn/module.py:460-495 in float64."""
    B, S, D = q.shape
    Sk = k.shape[1]
    hd = D // H

    def heads(t, n):
        return t.astype(np.float64).reshape(B, n, H, hd).transpose(0, 2, 1, 3)

    s = heads(q, S) @ heads(k, Sk).transpose(0, 1, 3, 2) / np.sqrt(hd)
    if causal:
        s = s + np.where(np.arange(Sk)[None, :] <= np.arange(S)[:, None], 0.0, -1e9)
    elif mask is not None:
        s = s + mask.astype(np.float64)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return (p @ heads(v, Sk)).transpose(0, 2, 1, 3).reshape(B, S, D)


@pytest.mark.parametrize("B,S,H,hd,kind", [(2, 256, 4, 64, "causal"), (1, 100, 2, 32, "causal"),
                                           (2, 300, 3, 64, "mask"), (1, 128, 2, 32, "none"),
                                           (3, 200, 2, 64, "none"), (8, 1024, 16, 64, "causal")])
def test_fused_attention_3xtf32(B, S, H, hd, kind, rng):
    """The 3xTF32 form of the fused kernel is fp32-faithful: 1e-5 of the
    largest output against a float64 restatement."""
    F = _w().functional
    D = H * hd
    q = rng.standard_normal((B, S, D)).astype(np.float32)
    k = rng.standard_normal((B, S, D)).astype(np.float32)
    v = rng.standard_normal((B, S, D)).astype(np.float32)
    mask = None
    if kind == "mask":
        mask = np.where(rng.random((S, S)) < 0.3, -1e9, rng.standard_normal((S, S))).astype(np.float32)
        np.fill_diagonal(mask, 0.0)
    F.set_matmul_mode("3xtf32")
    try:
        got = F.attention(up(q), up(k), up(v), H, mask=None if mask is None else up(mask),
                          causal=(kind == "causal"), feeds_tf32=True).numpy()
    finally:
        F.set_matmul_mode("tf32")
    ref = _attention_ref64(q, k, v, H, mask, kind == "causal")
    assert rel(got, ref) < 1e-5, rel(got, ref)
    tf32 = F.attention(up(q), up(k), up(v), H, mask=None if mask is None else up(mask),
                       causal=(kind == "causal")).numpy()
    assert rel(tf32, ref) > rel(got, ref)     # the TF32 form is the less exact one
    assert _w().backend.device_status() == 0


# ------------------------------------------------------------ fused linear epilogue

@pytest.mark.parametrize("M,K,N", [(100, 64, 96), (8192, 256, 1024), (2304, 64, 2300),
                                   (3, 8, 4)])
@pytest.mark.parametrize("act,res", [("gelu", False), (None, True), (None, False)])
@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_linear_fused_matches_unfused_bits(M, K, N, act, res, mode, rng):
    """GELU / residual fused into the GEMM epilogue: same bits as matmul_add
    followed by gelu / residual add (nn/module.py Linear + GELU, block adds)."""
    F = _w().functional
    x = up(rng.standard_normal((M, K)).astype(np.float32))
    w = up((rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32))
    b = up(rng.standard_normal(N).astype(np.float32))
    r = up(rng.standard_normal((M, N)).astype(np.float32)) if res else None
    F.set_matmul_mode(mode)
    try:
        got = F.linear(x, w, b, activation=act, residual=r).numpy()
        y = F.matmul_add(x, w, b)
        if act == "gelu":
            y = F.gelu(y)
        if r is not None:
            y = F.pointwise(r, y, 0)
        ref = y.numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert np.array_equal(got, ref)
    assert _w().backend.device_status() == 0


def test_linear_fp32_mode_and_ragged_n_fall_back(rng):
    F = _w().functional
    x = rng.standard_normal((2, 5, 16)).astype(np.float32)
    w = rng.standard_normal((16, 7)).astype(np.float32)
    b = rng.standard_normal(7).astype(np.float32)
    got = F.linear(up(x), up(w), up(b), activation="gelu").numpy()        # N % 4 != 0
    ref = K.unary(K.matmul_add(x, w, b), "gelu")
    assert got.shape == (2, 5, 7) and rel(got, ref) < 2e-3
    F.set_matmul_mode("fp32")
    try:
        got32 = F.linear(up(x), up(w), up(b)).numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert rel(got32, K.matmul_add(x, w, b)) < 1e-5


@pytest.mark.parametrize("shape", [(2, 8192, 256, 256), (3, 300, 64, 36), (2, 129, 40, 20)])
@pytest.mark.parametrize("mode,tol", [("tf32", 2e-3), ("3xtf32", 1e-5)])
def test_linear_on_batch_transposed_view(shape, mode, tol, rng):
    """linear(z.transpose(1, 2), W, residual=r) with z (B, K, M) dense: the
    GEMM reads the view as a transposed operand (no copy); Hyena's out
    projection.  Against the oracle and the copied-input path."""
    F = _w().functional
    B, M, Kd, N = shape
    z = rng.standard_normal((B, Kd, M)).astype(np.float32)
    w = (rng.standard_normal((Kd, N)) / np.sqrt(Kd)).astype(np.float32)
    r = rng.standard_normal((B, M, N)).astype(np.float32)
    F.set_matmul_mode(mode)
    try:
        got = F.linear(up(z).transpose(1, 2), up(w), residual=up(r)).numpy()
        copied = F.linear(up(np.ascontiguousarray(z.transpose(0, 2, 1))), up(w),
                          residual=up(r)).numpy()
    finally:
        F.set_matmul_mode("tf32")
    ref = K.matmul_add(np.ascontiguousarray(z.transpose(0, 2, 1)), w, None) + r
    assert got.shape == (B, M, N)
    assert rel(got, ref) < tol
    assert rel(got, copied) < tol


@pytest.mark.parametrize("shape", [(300, 64, 72), (1000, 256, 1376), (4096, 256, 2048),
                                   (130, 40, 200)])
@pytest.mark.parametrize("mode,tol", [("tf32", 2e-3), ("3xtf32", 1e-5)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_linear_swiglu_epilogue(shape, mode, tol, with_bias, rng):
    """linear(x, W, activation='swiglu'): columns 2j, 2j+1 of x @ W (+ bias)
    are (gate, up) and the GEMM epilogue writes silu(gate) * up, against the
    unfused GEMM + silu + product (same GEMM sums, same silu) and the oracle.
    Shapes cover single-SM and SM-pair tiles and ragged M / N edges."""
    F = _w().functional
    M, Kd, N = shape
    x = rng.standard_normal((M, Kd)).astype(np.float32)
    w = (rng.standard_normal((Kd, N)) / np.sqrt(Kd)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32) if with_bias else None
    F.set_matmul_mode(mode)
    try:
        got = F.linear(up(x), up(w), None if b is None else up(b), activation="swiglu").numpy()
        y = F.linear(up(x), up(w), None if b is None else up(b)).numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert got.shape == (M, N // 2)
    g, u = y[:, 0::2], y[:, 1::2]
    gc = np.clip(g, -88, 88)
    unfused = (g * (1.0 / (1.0 + np.exp(-gc)))) * u
    assert rel(got, unfused) < 1e-5
    yr = K.matmul_add(x, w, b)
    gr, ur = yr[:, 0::2], yr[:, 1::2]
    assert rel(got, gr / (1.0 + np.exp(-gr)) * ur) < 4 * tol


@pytest.mark.parametrize("d,hidden", [(64, 170), (256, 682), (64, 128)])
@pytest.mark.parametrize("mode,tol", [("tf32", 2e-3), ("3xtf32", 1e-5)])
def test_swiglu_padded_hidden_matches_plain(d, hidden, mode, tol, rng):
    """SwiGLU through the fused path (W1 and W2 interleaved into one GEMM with
    the paired-GLU epilogue, hidden width padded to a multiple of 4, then W3
    with the residual in its epilogue) against the plain expression.  The
    GEMMs may split K differently, and in TF32 mode the intermediate is then
    truncated to 10 mantissa bits, so the TF32 bound is the matmul one."""
    wxx = _w()
    F = wxx.functional
    wxx.manual_seed(3)
    m = wxx.nn.SwiGLU(d, hidden_dim=hidden)
    x = up(rng.standard_normal((2, 300, d)).astype(np.float32))
    F.set_matmul_mode(mode)
    try:
        got = m(x).numpy()
        ref = m.w3(F.silu(m.w1(x)) * m.w2(x)).numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert got.shape == ref.shape
    assert rel(got, ref) < tol, rel(got, ref)
    # residual fused into the last GEMM
    r = up(rng.standard_normal((2, 300, d)).astype(np.float32))
    F.set_matmul_mode(mode)
    try:
        got_r = m.forward(x, residual=r).numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert rel(got_r, got + r.numpy()) < 1e-5   # split-K vs whole-K sums in the last GEMM
    # the padded copies follow parameter updates
    F.assign(m.w1.weight, F.from_numpy(np.zeros((d, hidden), np.float32)))
    assert np.abs(m(x).numpy()).max() == 0.0


@pytest.mark.parametrize("shape", [((), (), 2304, 2304, 64), ((), (), 2300, 2200, 100),
                                   ((2,), (2,), 1280, 2048, 96), ((), (), 8192, 1024, 4096)])
@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_matmul_stream_k_opt_in(shape, mode, rng, monkeypatch):
    """SM-pair GEMM with the stream-K schedule (WXX_GEMM_STREAMK=1): partial
    tiles handed between pairs through the workspace and per-tile counters."""
    monkeypatch.setenv("WXX_GEMM_STREAMK", "1")
    F = _w().functional
    ba, bb, M, N, K_ = shape
    a = rng.standard_normal(ba + (M, K_)).astype(np.float32)
    b = rng.standard_normal(bb + (K_, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    F.set_matmul_mode(mode)
    try:
        got = F.matmul_add(up(a), up(b), up(bias)).numpy()
    finally:
        F.set_matmul_mode("tf32")
    ref = K.matmul_add(a, b, bias)
    assert rel(got, ref) < (2e-3 if mode == "tf32" else 1e-5)
    assert _w().backend.device_status() == 0


@pytest.mark.parametrize("batch,M,N,kdim", [(1, 2048, 512, 4096), (1, 1024, 256, 16384),
                                            (4, 512, 256, 4096), (1, 8192, 1024, 4096)])
def test_matmul_3xtf32_long_k_stays_fp32_faithful(batch, M, N, kdim, rng):
    """3xTF32 with long K: the product is summed in fp32 over slices of at
    most 1024 K-values per pass, keeping the 1e-5 bar at any K."""
    F = _w().functional
    a = rng.standard_normal(((batch,) if batch > 1 else ()) + (M, kdim)).astype(np.float32)
    b = rng.standard_normal((kdim, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    F.set_matmul_mode("3xtf32")
    try:
        got = F.matmul_add(up(a), up(b), up(bias)).numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert rel(got, K.matmul_add(a, b, bias)) < 1e-5
    assert _w().backend.device_status() == 0


# ------------------------------------------------------------ projection + short conv

def _short_conv_ref(x, w, b, cw, cb):
    """Oracle: y = x @ w (+ b), transposed to (B, N, L), then the causal taps
    of conv row c % C on channel c."""
    y = K.matmul_add(x, w, b)                      # (B, L, N)
    yt = np.ascontiguousarray(y.transpose(0, 2, 1))
    C = cw.shape[0]
    reps = yt.shape[1] // C
    return K.causal_conv1d(yt, np.tile(cw, (reps, 1)), np.tile(cb, reps))


@pytest.mark.parametrize("shape", [(2, 300, 64, 128, 64, 3), (3, 257, 32, 96, 96, 4),
                                   (2, 1000, 256, 1024, 256, 3), (1, 64, 64, 64, 64, 1),
                                   (4, 33, 16, 32, 16, 2), (5, 1, 32, 64, 64, 3),
                                   (2, 8192, 256, 256, 256, 3)])
@pytest.mark.parametrize("mode,tol", [("tf32", 2e-3), ("3xtf32", 1e-5)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_linear_short_conv(shape, mode, tol, with_bias, rng):
    """Hyena's proj -> transpose -> short causal conv as one GEMM whose
    epilogue applies the taps (rows of a tile overlap by taps - 1 so every
    warp holds its own halo): against the composition of the separate GEMM,
    transposed view and causal conv kernels, and the oracle.  Shapes cover
    one and many pair tiles, sequence boundaries inside a warp's rows
    (L = 33, 257, 300), one-position sequences and 1..4 taps."""
    F = _w().functional
    B, L, Kd, N, C, taps = shape
    x = rng.standard_normal((B, L, Kd)).astype(np.float32)
    w = (rng.standard_normal((Kd, N)) / np.sqrt(Kd)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32) if with_bias else None
    cw = rng.standard_normal((C, taps)).astype(np.float32)
    cb = rng.standard_normal(C).astype(np.float32)
    F.set_matmul_mode(mode)
    try:
        bd = None if b is None else up(b)
        got = F.linear_short_conv(up(x), up(w), bd, up(cw), up(cb)).numpy()
        y = F.linear(up(x), up(w), bd).transpose(1, 2)
        parts = [F.causal_conv1d(y[:, i * C:(i + 1) * C, :], up(cw), up(cb)).numpy()
                 for i in range(N // C)]
    finally:
        F.set_matmul_mode("tf32")
    composed = np.concatenate(parts, axis=1)
    ref = _short_conv_ref(x, w, b, cw, cb)
    assert got.shape == (B, N, L)
    assert rel(got, ref) < tol
    assert rel(got, composed) < (1e-5 if mode == "tf32" else 1e-6)
    assert _w().backend.device_status() == 0


def test_linear_short_conv_unaligned_input_falls_back(rng):
    """K = 6 (rows not 16-byte aligned for the tensor memory accelerator): the
    library reports the fused form unsupported and the composition runs."""
    F = _w().functional
    x = rng.standard_normal((2, 40, 6)).astype(np.float32)
    w = rng.standard_normal((6, 8)).astype(np.float32)
    cw = rng.standard_normal((8, 3)).astype(np.float32)
    cb = rng.standard_normal(8).astype(np.float32)
    got = F.linear_short_conv(up(x), up(w), None, up(cw), up(cb)).numpy()
    assert rel(got, _short_conv_ref(x, w, None, cw, cb)) < 2e-3
    assert _w().backend.device_status() == 0


# ------------------------------------------------------------ Hyena implicit filters

def _filters_ref(pe, l1, l2, omega, decay):
    """fp64 restatement of ImplicitFilter.forward (Linear -> Sine -> Linear,
    transposed) times decay_window(decay, i, L) for each filter i."""
    pe = np.asarray(pe, np.float64)
    L = pe.shape[0]
    t = np.arange(L, dtype=np.float64)
    out = []
    for i, ((w1, b1), (w2, b2)) in enumerate(zip(l1, l2)):
        hid = np.sin(omega * (pe @ w1.astype(np.float64) + b1))
        y = (hid @ w2.astype(np.float64) + b2).T
        out.append(y * np.exp(-np.abs(decay[i].astype(np.float64))[:, None] * t[None, :]))
    return np.stack(out)


@pytest.mark.parametrize("L,F,H,D,n", [(8192, 17, 64, 256, 4), (300, 17, 64, 48, 2),
                                       (33, 5, 32, 100, 1), (1, 17, 64, 64, 3),
                                       (1000, 32, 16, 130, 8)])
def test_hyena_filters(L, F, H, D, n, rng):
    """All implicit filters of an operator from one exact-fp32 kernel, written
    (n, D, L): against the fp64 restatement and the composed modules run with
    3xTF32 products (the default TF32 products err by ~1e-2 after the sine's
    omega = 10 scaling)."""
    wxx = _w()
    Fn = wxx.functional
    pe = rng.standard_normal((L, F)).astype(np.float32)
    l1 = [((rng.standard_normal((F, H)) / np.sqrt(F)).astype(np.float32),
           (0.1 * rng.standard_normal(H)).astype(np.float32)) for _ in range(n)]
    l2 = [((rng.standard_normal((H, D)) / np.sqrt(H)).astype(np.float32),
           (0.1 * rng.standard_normal(D)).astype(np.float32)) for _ in range(n)]
    decay = (0.01 * rng.random((n, D))).astype(np.float32)
    got = Fn.hyena_filters(up(pe), [(up(w), up(b)) for w, b in l1],
                           [(up(w), up(b)) for w, b in l2], 10.0, up(decay)).numpy()
    ref = _filters_ref(pe, l1, l2, 10.0, decay)
    assert got.shape == (n, D, L)
    assert rel(got, ref) < 2e-5
    Fn.set_matmul_mode("3xtf32")
    try:
        for i in range(n):
            y = Fn.linear(up(pe), up(l1[i][0]), up(l1[i][1]))
            y = (y * 10.0).sin()                      # Sine(omega), nn/module.py
            y = Fn.linear(y, up(l2[i][0]), up(l2[i][1])).transpose(0, 1)
            comp = (y * Fn.decay_window(up(decay), i, L)).numpy()
            assert rel(got[i], comp) < 2e-4
    finally:
        Fn.set_matmul_mode("tf32")
    assert wxx.backend.device_status() == 0


def test_hyena_filters_outside_limits_returns_none(rng):
    Fn = _w().functional
    pe = up(rng.standard_normal((16, 40)).astype(np.float32))      # F = 40 > 32
    w1 = up(rng.standard_normal((40, 8)).astype(np.float32))
    b1 = up(rng.standard_normal(8).astype(np.float32))
    w2 = up(rng.standard_normal((8, 4)).astype(np.float32))
    b2 = up(rng.standard_normal(4).astype(np.float32))
    assert Fn.hyena_filters(pe, [(w1, b1)], [(w2, b2)], 10.0,
                            up(np.zeros((1, 4), np.float32))) is None


# ------------------------------------------------------------ K-major weights, strided q/k/v

@pytest.mark.parametrize("M,Kd,N", [(300, 64, 72), (4096, 1024, 3072), (130, 40, 200)])
@pytest.mark.parametrize("act,res", [(None, False), ("gelu", False), (None, True)])
@pytest.mark.parametrize("mode,tol", [("tf32", 2e-3), ("3xtf32", 1e-5)])
def test_linear_transposed_weight(M, Kd, N, act, res, mode, tol, rng):
    """linear(x, W^T stored (N, K), transpose_weight=True) -- the K-major
    operand GPT2's inference layers feed the GEMM -- against the (K, N)
    layout and the oracle."""
    F = _w().functional
    x = rng.standard_normal((M, Kd)).astype(np.float32)
    w = (rng.standard_normal((Kd, N)) / np.sqrt(Kd)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32) if res else None
    F.set_matmul_mode(mode)
    try:
        rd = None if r is None else up(r)
        got = F.linear(up(x), up(np.ascontiguousarray(w.T)), up(b), activation=act, residual=rd,
                       transpose_weight=True).numpy()
        plain = F.linear(up(x), up(w), up(b), activation=act, residual=rd).numpy()
    finally:
        F.set_matmul_mode("tf32")
    ref = K.matmul_add(x, w, b)
    if act == "gelu":
        ref = K.unary(ref, "gelu")
    if r is not None:
        ref = ref + r
    assert got.shape == (M, N)
    assert rel(got, ref) < tol
    assert rel(got, plain) < (1e-5 if mode == "tf32" else 1e-6)


@pytest.mark.parametrize("B,S,H,hd", [(2, 256, 4, 64), (3, 100, 2, 32)])
def test_attention_reads_column_blocks_in_place(B, S, H, hd, rng):
    """q, k, v given as column blocks of one (B, S, 3D) projection output
    (row stride 3D): the kernel reads them in place, same bits as dense
    copies."""
    F = _w().functional
    D = H * hd
    qkv = rng.standard_normal((B, S, 3 * D)).astype(np.float32)
    t = up(qkv)
    q, k, v = t[..., 0:D], t[..., D:2 * D], t[..., 2 * D:3 * D]
    got = F.attention(q, k, v, H, causal=True).numpy()
    dq, dk, dv = (up(np.ascontiguousarray(qkv[..., i * D:(i + 1) * D])) for i in range(3))
    ref = F.attention(dq, dk, dv, H, causal=True).numpy()
    assert np.array_equal(got, ref)
    assert _w().backend.device_status() == 0


@pytest.mark.parametrize("n,rows,cols", [(3, 1024, 1024), (2, 100, 70), (1, 33, 5), (8, 64, 96)])
def test_transpose_stack(n, rows, cols, rng):
    """n (rows, cols) weights transposed and stacked into one (n*cols, rows)
    buffer by one launch (the fused QKV operand): bit-exact copies."""
    F = _w().functional
    ws = [rng.standard_normal((rows, cols)).astype(np.float32) for _ in range(n)]
    out = up(np.zeros((n * cols, rows), np.float32))
    assert F.transpose_stack(out, [up(w) for w in ws])
    assert np.array_equal(out.numpy(), np.concatenate([w.T for w in ws], axis=0))


@pytest.mark.parametrize("shape", NHWC_SHAPES)
def test_conv2d_nhwc_packed_weights(shape, rng):
    """Weights reordered for all convolutions in one launch (conv_weight_pack,
    ResNet's channels-last stages) give the same bits as each convolution
    reordering its own; the packed tensor is (Cout, KH, KW, Cin)."""
    F = _w().functional
    B, C, H, W, O, k, s, p, d = shape
    x = rng.standard_normal((B, H, W, C)).astype(np.float32)
    w = rng.standard_normal((O, C, k, k)).astype(np.float32)
    w2 = rng.standard_normal((O // 2 * 2, C, 1, 1)).astype(np.float32)
    pk = up(np.zeros((O, k, k, C), np.float32))
    pk2 = up(np.zeros((w2.shape[0], 1, 1, C), np.float32))
    assert F.conv_weight_pack([up(w), up(w2)], [pk, pk2])
    assert np.array_equal(pk.numpy(), w.transpose(0, 2, 3, 1))
    assert np.array_equal(pk2.numpy(), w2.transpose(0, 2, 3, 1))
    got = F.conv2d_nhwc(up(x), up(w), (s, s), (p, p), (d, d), relu=True, packed=pk).numpy()
    ref = F.conv2d_nhwc(up(x), up(w), (s, s), (p, p), (d, d), relu=True).numpy()
    assert np.array_equal(got, ref)
    assert _w().backend.device_status() == 0
