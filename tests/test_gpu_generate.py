"""On-device generation (GPT2.generate with a K/V cache and the device sampler)
against the reference's sampling loop (nn/gpt.py:108-170), restated in
``oracle.models.gpt2_generate`` (full float64 forward per step).

Token ids are compared exactly.  The model runs in 3xTF32 mode for the id
comparisons (logits within ~1e-6 of float64, far inside the gaps between the
candidates these seeded models produce); the decode step's logits are also
compared with a full forward of the same prefix.  The sampler kernel is checked
on its own against the numpy rule with the same draws, including ties, top-k
and the no-crossing case.
"""

import ctypes

import numpy as np
import pytest

from oracle import init, models

pytestmark = pytest.mark.gpu


def _wxx():
    import wxx_b200 as wxx

    return wxx


def _model(V, D, H, L, S):
    wxx = _wxx()
    sd = init.gpt2_state_dict(0, V, D, H, L, S)
    m = wxx.nn.GPT2(V, D, H, L, max_len=S)
    m.load_state_dict(sd)
    return m, sd


@pytest.mark.parametrize("V,D,H,L,S,B,P,N", [(128, 64, 2, 2, 48, 3, 7, 30),
                                             (200, 128, 2, 3, 64, 2, 1, 40)])
def test_greedy_matches_reference_loop(V, D, H, L, S, B, P, N):
    wxx = _wxx()
    m, sd = _model(V, D, H, L, S)
    prompt = init.token_ids(4, B, P, V)
    wxx.set_matmul_mode("3xtf32")
    try:
        got = m.generate(prompt, max_new_tokens=N, temperature=0.0)
    finally:
        wxx.set_matmul_mode("tf32")
    ref = models.gpt2_generate(sd, prompt, H, L, N, temperature=0.0)
    assert got.dtype == np.uint32 and got.shape == ref.shape == (B, P + N)
    assert np.array_equal(got, ref)
    assert wxx.backend.device_status() == 0


@pytest.mark.parametrize("temperature,top_k", [(0.8, 10), (1.5, None), (1.0, 1)])
def test_sampling_matches_reference_loop(temperature, top_k):
    wxx = _wxx()
    V, D, H, L, S = 128, 64, 2, 2, 40
    m, sd = _model(V, D, H, L, S)
    prompt = init.token_ids(5, 2, 5, V)
    wxx.set_matmul_mode("3xtf32")
    try:
        got = m.generate(prompt, max_new_tokens=25, temperature=temperature, top_k=top_k,
                         rng=np.random.default_rng(11))
    finally:
        wxx.set_matmul_mode("tf32")
    ref = models.gpt2_generate(sd, prompt, H, L, 25, temperature=temperature, top_k=top_k,
                               rng=np.random.default_rng(11))
    assert np.array_equal(got, ref)


def test_stop_token_and_max_len():
    wxx = _wxx()
    V, D, H, L, S = 128, 64, 2, 2, 24
    m, sd = _model(V, D, H, L, S)
    prompt = init.token_ids(6, 1, 4, V)
    wxx.set_matmul_mode("3xtf32")
    try:
        full = m.generate(prompt, max_new_tokens=100, temperature=0.0)
        assert full.shape == (1, S)                   # capped at max_len tokens
        stop = int(full[0, 4 + 5])
        got = m.generate(prompt, max_new_tokens=100, temperature=0.0, stop_token=stop)
        eager = m.generate(prompt[0], max_new_tokens=100, temperature=0.0)   # 1-D prompt
    finally:
        wxx.set_matmul_mode("tf32")
    ref = models.gpt2_generate(sd, prompt, H, L, 100, temperature=0.0, stop_token=stop)
    assert np.array_equal(got, ref)
    assert got[0, -1] == stop and got.shape[1] <= 4 + 6
    assert np.array_equal(eager, full)
    with pytest.raises(ValueError):
        m.generate(np.zeros((1, S + 1), np.uint32))
    with pytest.raises(ValueError):
        m.generate(prompt, temperature=-1.0)


def test_decode_logits_match_full_forward():
    """The K/V-cache decode step's logits equal the last-position logits of a
    full forward over the same prefix (3xTF32: 1e-5; TF32: 5e-3)."""
    wxx = _wxx()
    from wxx_b200.nn import generation as G

    V, D, H, L, S = 128, 128, 2, 2, 32
    m, _ = _model(V, D, H, L, S)
    prompt = init.token_ids(7, 2, 9, V)
    for mode, tol in (("3xtf32", 1e-5), ("tf32", 5e-3)):
        wxx.set_matmul_mode(mode)
        try:
            with wxx.backend.inferenceMode():
                st = G._DecodeState(m, 2)
                pad = np.zeros((2, S), np.uint32)
                pad[:, :9] = prompt
                wxx.backend.lib.F.wxx_memcpy_h2d(st.ids.ptr, pad.ctypes.data, pad.nbytes)
                st.set_count(9)
                G._prefill(m, st, 9, 0.0, 0)            # writes token 9, count -> 10
                logits = G._decode_step(m, st, 0.0, 0).numpy()   # position 9
                ids = st.ids.numpy()[:, :10]
                full = m(wxx.functional.from_numpy(ids, dtype=np.uint32)).numpy()[:, -1, :]
        finally:
            wxx.set_matmul_mode("tf32")
        assert np.abs(logits - full).max() < tol * max(1.0, np.abs(full).max())


def _numpy_rule(logits, temperature, top_k, draws):
    z = logits.astype(np.float64)
    if temperature == 0.0:
        return z.argmax(-1)
    z = z / temperature
    if top_k:
        k = min(top_k, z.shape[-1])
        if k < z.shape[-1]:
            cut = np.partition(z, -k, axis=-1)[:, -k]
            z[z < cut[:, None]] = -np.inf
    z -= z.max(-1, keepdims=True)
    p = np.exp(z)
    p /= p.sum(-1, keepdims=True)
    return (np.cumsum(p, -1) > draws[:, None]).argmax(-1)


@pytest.mark.parametrize("temperature,top_k", [(0.0, 0), (1.0, 0), (0.7, 50), (2.0, 1),
                                               (1.0, 50303)])
def test_sampler_kernel_rule(temperature, top_k, rng):
    wxx = _wxx()
    F = wxx.functional
    lib = wxx.backend.lib
    B, V, S = 6, 50304, 8
    logits = rng.standard_normal((B, V)).astype(np.float32) * 3
    logits[1, [7, 900, 40000]] = 50.0                 # tie at the maximum: first index
    logits[2] = np.round(logits[2])                   # many ties at the top-k cutoff
    draws = rng.random(B)
    draws[3] = 0.0                                    # the first id with p > 0
    ids = F.from_numpy(np.zeros((B, S), np.uint32), dtype=np.uint32)
    count = F.from_numpy(np.array([3], np.uint32), dtype=np.uint32)
    done = F.from_numpy(np.zeros(1, np.uint32), dtype=np.uint32)
    lg = F.from_numpy(logits)
    dr = wxx.backend.device.DeviceBuffer(8 * B, "draws")
    lib.check(lib.F.wxx_memcpy_h2d(dr.ptr, np.ascontiguousarray(draws).ctypes.data, 8 * B))
    lib.check(lib.F.wxx_sample_tokens(ids.ptr, S, count.ptr, done.ptr, lg.ptr, V, B, V,
                                      float(temperature), int(top_k), dr.ptr, S), "sample")
    got = ids.numpy()[:, 3]
    ref = _numpy_rule(logits, temperature, top_k, draws)
    assert np.array_equal(got, ref.astype(np.uint32)), (got, ref)
    assert count.numpy()[0] == 4 and done.numpy()[0] == 0
    if temperature == 0.0:
        assert got[1] == 7


@pytest.mark.parametrize("hd", [32, 64])
def test_decode_attention_kernel(hd, rng):
    wxx = _wxx()
    F = wxx.functional
    lib = wxx.backend.lib
    B, H, S, p = 3, 4, 40, 17
    D = H * hd
    Kc = rng.standard_normal((B, S, D)).astype(np.float32)
    Vc = rng.standard_normal((B, S, D)).astype(np.float32)
    qkv = rng.standard_normal((B, 3 * D)).astype(np.float32)
    tK, tV, tq = F.from_numpy(Kc), F.from_numpy(Vc), F.from_numpy(qkv)
    out = F.from_numpy(np.zeros((B, D), np.float32))
    count = F.from_numpy(np.array([p + 1], np.uint32), dtype=np.uint32)
    scale = 1.0 / np.sqrt(hd)
    lib.check(lib.F.wxx_decode_attention(out.ptr, D, tq.ptr, tq.ptr + 4 * D, tq.ptr + 8 * D,
                                         3 * D, tK.ptr, tV.ptr, S * D, B, H, hd, count.ptr, S,
                                         scale, 0), "decode_attention")
    Kc[:, p] = qkv[:, D:2 * D]
    Vc[:, p] = qkv[:, 2 * D:]
    assert np.array_equal(tK.numpy(), Kc) and np.array_equal(tV.numpy(), Vc)
    q = qkv[:, :D].reshape(B, H, hd).astype(np.float64)
    k = Kc[:, :p + 1].reshape(B, p + 1, H, hd).astype(np.float64)
    v = Vc[:, :p + 1].reshape(B, p + 1, H, hd).astype(np.float64)
    s = np.einsum("bhd,bjhd->bhj", q, k) * scale
    w = np.exp(s - s.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    ref = np.einsum("bhj,bjhd->bhd", w, v).reshape(B, D)
    assert np.abs(out.numpy() - ref).max() < 1e-5 * np.abs(ref).max()
