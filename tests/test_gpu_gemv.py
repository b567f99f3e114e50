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
