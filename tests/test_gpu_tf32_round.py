"""Outputs stored rounded to TF32 for consumers that are TF32 products.

A tcgen05 kind::tf32 product reads each fp32 operand by dropping its low 13
mantissa bits.  Where an output feeds only such products (GPT2's LayerNorm ->
QKV, QKV -> attention, attention -> out projection, FC1+GELU -> FC2, the
final LayerNorm -> LM head; Hyena's RMSNorm -> projections, SwiGLU -> W3),
the producing kernel stores it rounded to the nearest TF32 value instead.
Each rounded output must equal the round-to-nearest (ties away from zero) of
the same kernel's unrounded output, bit for bit, and the unrounded path must
be unchanged.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _w():
    import wxx_b200 as wxx

    return wxx


def up(a):
    return _w().functional.from_numpy(np.asarray(a, np.float32))


def rna_tf32(a):
    """Round-to-nearest TF32 (10 explicit mantissa bits, ties away from zero)
    of finite fp32 values, as an fp32 array."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x1000) & 0xFFFFE000).astype(np.uint32)).view(np.float32)


@pytest.mark.parametrize("M,K,N", [(100, 64, 96),        # single-SM tiles, TMA store
                                   (128, 4096, 256),     # split-K (few tiles, long K)
                                   (2304, 64, 2304),     # SM-pair kernel
                                   (3, 8, 4)])
@pytest.mark.parametrize("act,res", [(None, False), ("gelu", False), (None, True)])
def test_linear_rounded_output(M, K, N, act, res, rng):
    F = _w().functional
    x = up(rng.standard_normal((M, K)))
    w = up(rng.standard_normal((K, N)) / np.sqrt(K))
    b = up(rng.standard_normal(N))
    r = up(rng.standard_normal((M, N))) if res else None
    plain = F.linear(x, w, b, activation=act, residual=r).numpy()
    got = F.linear(x, w, b, activation=act, residual=r, feeds_tf32=True).numpy()
    assert np.array_equal(got, rna_tf32(plain))
    assert np.all((got.view(np.uint32) & 0x1FFF) == 0)


def test_linear_rounded_output_kmajor_and_glu(rng):
    F = _w().functional
    x = up(rng.standard_normal((300, 256)))
    wt = up(rng.standard_normal((3 * 256, 256)) / 16)
    plain = F.linear(x, wt, transpose_weight=True).numpy()
    got = F.linear(x, wt, transpose_weight=True, feeds_tf32=True).numpy()
    assert np.array_equal(got, rna_tf32(plain))
    w12 = up(rng.standard_normal((256, 2 * 688)) / 16)
    plain = F.linear(x, w12, activation="swiglu").numpy()
    got = F.linear(x, w12, activation="swiglu", feeds_tf32=True).numpy()
    assert np.array_equal(got, rna_tf32(plain))


def test_rounding_off_outside_tf32_mode(rng):
    F = _w().functional
    x = up(rng.standard_normal((64, 32)))
    w = up(rng.standard_normal((32, 64)))
    F.set_matmul_mode("3xtf32")
    try:
        plain = F.linear(x, w).numpy()
        got = F.linear(x, w, feeds_tf32=True).numpy()
        ln = F.meanvarnorm(x, up(np.ones(32)), up(np.zeros(32)), -1, feeds_tf32=True)[0].numpy()
        ln0 = F.meanvarnorm(x, up(np.ones(32)), up(np.zeros(32)), -1)[0].numpy()
    finally:
        F.set_matmul_mode("tf32")
    assert np.array_equal(got, plain)
    assert np.array_equal(ln, ln0)


@pytest.mark.parametrize("shape", [(37, 256), (5, 1024), (3, 2000), (4, 6, 5)])
def test_norms_rounded_output(shape, rng):
    F = _w().functional
    x = up(rng.standard_normal(shape) * 3)
    n = shape[-1]
    g = up(rng.standard_normal(n))
    b = up(rng.standard_normal(n))
    y0 = F.meanvarnorm(x, g, b, -1)[0].numpy()
    y1 = F.meanvarnorm(x, g, b, -1, feeds_tf32=True)[0].numpy()
    assert np.array_equal(y1, rna_tf32(y0))
    r0 = F.rmsnorm(x, g, -1)[0].numpy()
    r1 = F.rmsnorm(x, g, -1, feeds_tf32=True)[0].numpy()
    assert np.array_equal(r1, rna_tf32(r0))


def test_attention_rounded_output(rng):
    F = _w().functional
    q, k, v = (up(rng.standard_normal((2, 256, 256))) for _ in range(3))
    o0 = F.attention(q, k, v, 4, causal=True).numpy()
    o1 = F.attention(q, k, v, 4, causal=True, feeds_tf32=True).numpy()
    assert np.array_equal(o1, rna_tf32(o0))


def test_transpose_stack_rounded(rng):
    F = _w().functional
    ws = [rng.standard_normal((96, 64)).astype(np.float32) for _ in range(3)]
    out = up(np.zeros((192, 96)))
    assert F.transpose_stack(out, [up(w) for w in ws], round_tf32=True)
    ref = np.concatenate([w.T for w in ws], axis=0)
    assert np.array_equal(out.numpy(), rna_tf32(ref))
    assert F.transpose_stack(out, [up(w) for w in ws])
    assert np.array_equal(out.numpy(), ref)
