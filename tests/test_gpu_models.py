"""Model parity on the GPU: GPT2 / ResNet18 / Hyena forwards through the
unchanged wxx API against the CPU oracle on the same seeded state dict.

Bar: final logits within 1e-3 max-abs.  That bar is
checked in 3xTF32 mode (fp32-faithful contractions), and tighter (1e-4) for
GPT2.  In TF32 mode the tensor cores read each fp32 operand truncated to a
10-bit mantissa (measured on B200: products match truncated operands to fp32
rounding), so the logit error is a property of TF32 arithmetic at this
depth.  Outputs that feed only products are stored rounded to nearest TF32,
which took GPT2 config 0 from 2.7e-3 to 1.5e-3 (measured on B200); it is
bounded at 2.5e-3 there and at 1e-2 relative for ResNet18.
"""

import numpy as np
import pytest

from oracle import init, models

pytestmark = pytest.mark.gpu


def _wxx():
    import wxx_b200 as wxx

    return wxx


def _run(model, ids_or_x, is_ids=True):
    wxx = _wxx()
    F = wxx.functional
    t = F.from_numpy(ids_or_x, dtype=np.uint32) if is_ids else F.from_numpy(ids_or_x)
    with wxx.backend.inferenceMode():
        return model(t).numpy()


@pytest.mark.parametrize("mode,tol", [("tf32", 2.5e-3), ("3xtf32", 1e-4)])
def test_gpt2_config1_logits(mode, tol):
    """GPT2(1024, 256, 8, 6), batch 4, seq 256."""
    wxx = _wxx()
    V, D, H, L, S = 1024, 256, 8, 6, 256
    sd = init.gpt2_state_dict(0, V, D, H, L, S)
    ids = init.token_ids(1, 4, S, V)
    model = wxx.nn.GPT2(V, D, H, L, max_len=S)
    model.load_state_dict(sd)
    wxx.functional.set_matmul_mode(mode)
    try:
        got = _run(model, ids)
    finally:
        wxx.functional.set_matmul_mode("tf32")
    ref = models.gpt2_forward(sd, ids, H, L)
    assert got.shape == (4, S, V)
    assert np.abs(got - ref).max() < tol, np.abs(got - ref).max()


def test_gpt2_causal_and_state_dict_roundtrip(tmp_path):
    wxx = _wxx()
    model = wxx.nn.GPT2(50, 32, 4, 2, max_len=16)
    ids = np.random.default_rng(0).integers(0, 50, size=(2, 16)).astype(np.uint32)
    base = _run(model, ids)
    ids2 = ids.copy()
    ids2[:, 10:] = (ids2[:, 10:] + 7) % 50
    changed = _run(model, ids2)
    assert np.allclose(base[:, :10], changed[:, :10], atol=1e-5)     # causality
    assert not np.allclose(base[:, 10:], changed[:, 10:])
    path = wxx.save(model, str(tmp_path / "gpt2.npz"))
    other = wxx.nn.GPT2(50, 32, 4, 2, max_len=16)
    wxx.load(path, other)
    assert np.array_equal(_run(other, ids), base)
    keys = set(model.state_dict())
    assert "blocks.0.ln1.weightg" in keys and "blocks.0.ln1.weight" in keys


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_resnet18_logits(mode):
    """BASELINE config 2 at a reduced batch: ResNet18(10), eval BatchNorm."""
    wxx = _wxx()
    sd = init.resnet18_state_dict(0, 10)
    x = np.random.default_rng(2).standard_normal((8, 3, 32, 32)).astype(np.float32)
    model = wxx.nn.ResNet18(num_classes=10)
    model.load_state_dict(sd)
    wxx.functional.set_matmul_mode(mode)
    try:
        got = _run(model, x, is_ids=False)
    finally:
        wxx.functional.set_matmul_mode("tf32")
    ref = models.resnet18_forward(sd, x)
    assert got.shape == (8, 10)
    err = np.abs(got - ref).max()
    if mode == "3xtf32":
        assert err < 1e-3, err
    else:
        assert err < 1e-2 * np.abs(ref).max(), err


def test_hyena_logits_small():
    wxx = _wxx()
    V, D, NL, order, B, L = 64, 32, 2, 3, 2, 200
    sd = init.hyena_state_dict(0, V, D, NL, order)
    ids = init.token_ids(3, B, L, V)
    model = wxx.nn.Hyena(V, d_model=D, n_layers=NL, order=order)
    model.load_state_dict(sd)
    got = _run(model, ids)
    ref = models.hyena_forward(sd, ids, NL, order)
    assert got.shape == (B, L, V)
    assert np.abs(got - ref).max() < 1e-3


def test_hyena_causal_and_batch_independent():
    wxx = _wxx()
    model = wxx.nn.Hyena(40, d_model=16, n_layers=1, order=2)
    rng = np.random.default_rng(5)
    ids = rng.integers(0, 40, size=(3, 64)).astype(np.uint32)
    base = _run(model, ids)
    ids2 = ids.copy()
    ids2[0, 40:] = (ids2[0, 40:] + 1) % 40
    out2 = _run(model, ids2)
    assert np.allclose(base[0, :40], out2[0, :40], atol=1e-4)
    assert np.allclose(base[1:], out2[1:], atol=1e-5)


def test_cached_weight_copies_follow_in_place_writes():
    """Inference reads K-major / TF32-rounded copies of the weights, kept
    between calls; a write through the API (assign, load_state_dict) must be
    seen by the next forward."""
    wxx = _wxx()
    F = wxx.functional
    V, D, H, L, S = 128, 64, 4, 2, 32
    sd = init.gpt2_state_dict(0, V, D, H, L, S)
    ids = init.token_ids(1, 2, S, V)
    model = wxx.nn.GPT2(V, D, H, L, max_len=S)
    model.load_state_dict(sd)
    wxx.functional.set_matmul_mode("3xtf32")
    try:
        first = _run(model, ids)
        assert np.abs(first - models.gpt2_forward(sd, ids, H, L)).max() < 1e-4
        sd2 = dict(sd)
        for key in ("blocks.0.mlp.0.weight", "blocks.1.mlp.2.weight", "blocks.0.attn.out.weight",
                    "blocks.1.attn.q.weight", "tok_emb.weight"):
            sd2[key] = (sd[key] * 1.7).astype(np.float32)
            F.assign(dict(model.named_parameters())[key],
                     F.from_numpy(sd2[key]))
        second = _run(model, ids)
        assert np.abs(second - models.gpt2_forward(sd2, ids, H, L)).max() < 1e-4
        model.load_state_dict(sd)
        assert np.abs(_run(model, ids) - first).max() < 1e-6
    finally:
        wxx.functional.set_matmul_mode("tf32")
    # TF32 mode reads the rounded copies; they follow the writes as well
    model.load_state_dict(sd2)
    got = _run(model, ids)
    assert np.abs(got - models.gpt2_forward(sd2, ids, H, L)).max() < 5e-3


@pytest.mark.parametrize("V,D,H,L,S,B", [(1024, 256, 8, 6, 256, 4), (50304, 1024, 16, 2, 1024, 2)])
def test_gpt2_forward_argmax_equals_logits_argmax(V, D, H, L, S, B):
    """GPT2.forward_argmax (the next-token ids straight from the tied head's
    GEMM, the logits never stored) equals max(forward(ids), -1)[1]; the second
    shape (the GPT2-scaled head on 2048 rows) takes the SM-pair epilogue."""
    wxx = _wxx()
    F = wxx.functional
    sd = init.gpt2_state_dict(0, V, D, H, L, S)
    ids = init.token_ids(1, B, S, V)
    model = wxx.nn.GPT2(V, D, H, L, max_len=S)
    model.load_state_dict(sd)
    t = F.from_numpy(ids, dtype=np.uint32)
    with wxx.backend.inferenceMode():
        ref = F.max(model(t), -1)[1].numpy()
        got = model.forward_argmax(t).numpy()
    assert got.shape == (B, S)
    assert np.array_equal(got, ref)


def test_hyena_filter_spectra_follow_writes_and_lengths():
    """Inference keeps each Hyena operator's filter spectra between calls
    (they do not depend on the input); a write to a filter weight or the decay,
    or another sequence length, must give the values of a fresh computation."""
    wxx = _wxx()
    F = wxx.functional
    V, D, NL, order, B = 64, 32, 2, 3, 2
    sd = init.hyena_state_dict(0, V, D, NL, order)
    model = wxx.nn.Hyena(V, d_model=D, n_layers=NL, order=order)
    model.load_state_dict(sd)
    for L in (200, 120, 200):
        ids = init.token_ids(3, B, L, V)
        first = _run(model, ids)
        assert np.array_equal(_run(model, ids), first)
        assert np.abs(first - models.hyena_forward(sd, ids, NL, order)).max() < 1e-3
    sd2 = dict(sd)
    params = dict(model.named_parameters())
    for key in ("layers.0.mixer.decay", "layers.1.mixer.filter_mlp.2.mlp.2.weight",
                "layers.0.mixer.filter_mlp.0.mlp.0.bias"):
        sd2[key] = (sd[key] * 1.5 + 0.1).astype(np.float32)
        F.assign(params[key], F.from_numpy(sd2[key]))
    ids = init.token_ids(4, B, 200, V)
    fresh = wxx.nn.Hyena(V, d_model=D, n_layers=NL, order=order)
    fresh.load_state_dict(sd2)
    assert np.array_equal(_run(model, ids), _run(fresh, ids))
