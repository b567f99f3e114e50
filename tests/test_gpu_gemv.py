"""Few-row products against a K-major weight (the decode step's GEMMs):
``rows_gemv_kernel`` in exact fp32 against a float64 product, with the
epilogue's bias / GELU / residual and the TF32 rounding of the stored value,
and the fused forms equal to the separate ops bit for bit."""

import numpy as np
import pytest

from oracle import train

pytestmark = pytest.mark.gpu


def _F():
    import wxx_b200 as wxx

    return wxx.functional


def up(a):
    return _F().from_numpy(np.asarray(a, np.float32))


def rel(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("M,N,K", [(1, 64, 128), (3, 1000, 1024), (8, 3072, 1024),
                                   (8, 1024, 4096), (13, 257, 1000), (32, 4096, 1024),
                                   (8, 50304, 256)])
def test_rows_gemv_against_float64(M, N, K, rng):
    F = _F()
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    got = F.linear(up(x), up(w), up(b), transpose_weight=True).numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T + b
    assert got.shape == (M, N)
    assert rel(got, ref) < 2e-6


def test_rows_gemv_epilogues_match_separate_ops(rng):
    F = _F()
    M, N, K = 8, 1024, 1024
    x = up(rng.standard_normal((M, K)))
    w = up(rng.standard_normal((N, K)) / 32.0)
    b = up(rng.standard_normal(N))
    r = up(rng.standard_normal((M, N)))
    plain = F.linear(x, w, b, transpose_weight=True)
    fused_gelu = F.linear(x, w, b, activation="gelu", transpose_weight=True).numpy()
    assert np.array_equal(fused_gelu, F.gelu(plain).numpy())
    fused_res = F.linear(x, w, b, residual=r, transpose_weight=True).numpy()
    assert np.array_equal(fused_res, F.pointwise(r, plain, 0).numpy())
    ref = train._gelu(plain.numpy().astype(np.float64))
    assert rel(fused_gelu, ref) < 1e-6


def test_rows_gemv_rounded_store_is_rna_of_plain(rng):
    import wxx_b200 as wxx

    F = _F()
    x = up(rng.standard_normal((5, 512)))
    w = up(rng.standard_normal((300, 512)))
    wxx.set_matmul_mode("tf32")
    plain = F.linear(x, w, transpose_weight=True).numpy()
    rounded = F.linear(x, w, transpose_weight=True, feeds_tf32=True).numpy()
    bits = plain.view(np.uint32).astype(np.uint64)
    rna = ((bits + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)
    assert np.array_equal(rounded, rna)


def test_rows_gemv_batched_rows_fold(rng):
    """A (batch, M, K) input with a shared weight folds into batch * M rows."""
    F = _F()
    x = rng.standard_normal((4, 2, 256)).astype(np.float32)
    w = rng.standard_normal((96, 256)).astype(np.float32)
    got = F.linear(up(x), up(w), transpose_weight=True).numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert rel(got, ref) < 2e-6


def _ln64(x, g, b):
    x = x.astype(np.float64)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + 1e-5) * g + b


@pytest.mark.parametrize("M,N,K,act,res", [(1, 64, 128, None, False), (8, 3072, 1024, None, False),
                                           (8, 4096, 1024, "gelu", False),
                                           (5, 1000, 512, None, True), (32, 256, 256, "gelu", True),
                                           (64, 256, 256, None, True)])
def test_ln_linear_against_float64(M, N, K, act, res, rng):
    """LayerNorm -> linear in one few-rows launch (the decode step's ln1 ->
    q/k/v, ln2 -> fc1, ln_f -> head); 64 rows take the two-launch path."""
    F = _F()
    x = (rng.standard_normal((M, K)) * 3 + 1).astype(np.float32)
    g = rng.standard_normal(K).astype(np.float32)
    b = rng.standard_normal(K).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32) if res else None
    import wxx_b200 as wxx

    wxx.set_matmul_mode("3xtf32")
    try:
        got = F.ln_linear(up(x), up(g), up(b), up(w), up(bias), activation=act,
                          residual=None if r is None else up(r)).numpy()
    finally:
        wxx.set_matmul_mode("tf32")
    ref = _ln64(x, g, b) @ w.astype(np.float64).T + bias
    if act == "gelu":
        ref = train._gelu(ref)
    if r is not None:
        ref = ref + r
    assert got.shape == (M, N)
    assert rel(got, ref) < 1e-5, rel(got, ref)


@pytest.mark.parametrize("M,N,K", [(2048, 4096, 256), (96, 1000, 128), (1, 300, 64)])
def test_linear_argmax_matches_stored_product(M, N, K, rng):
    """The row argmax taken in the SM-pair GEMM's epilogue (large shapes; small
    ones are declined) gives the ids and the tie rule of
    max(linear(x, w), -1)[1] (the argmax kernel's lane tree: ties between
    columns 10 and 265 go to 10, between 40 and 300 to 40)."""
    F = _F()
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.01).astype(np.float32)
    if N > 300:
        w[10] = w[265] = 1.0
        w[40] = w[300] = -1.0
    fused = F.linear_argmax(up(x), up(w), transpose_weight=True)
    ref = F.max(F.linear(up(x), up(w), transpose_weight=True), -1)[1].numpy()
    if M < 2048:
        assert fused is None          # too few output tiles for the SM-pair epilogue
        return
    got = fused.numpy()
    assert got.shape == (M,) and got.dtype == np.uint32
    assert np.array_equal(got, ref)
    if N > 300:
        s = x.sum(1)
        assert np.all(got[s > 1.0] == 10) and np.all(got[s < -1.0] == 40)
