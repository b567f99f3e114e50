"""Model parity at the benchmarked configurations, against the float64 oracle.

  GPT2-scaled  GPT2(50304, 1024, 16, 24), seq 1024, one sequence (the per-GPU
               shard of the default bench workload holds 8 of them)
  Hyena        Hyena(1024, 256, 6, order 4), one sequence of 8192 (fft 16384)
  ResNet18     ResNet18(10) on a batch of 256 images, eval BatchNorm

Bar (north star): logits within 1e-3 max-abs.  Met in 3xTF32 mode (fp32-faithful
products; measured on B200: 3.0e-5 / 6.1e-6 / 2.8e-4).  TF32 mode reads every
fp32 operand with a 10-bit mantissa; outputs that only feed products are stored
rounded to nearest TF32 (which halves the error against hardware truncation),
but at these depths the logits still drift past 1e-3 (measured: 4.8e-3 on
GPT2-scaled with |logit| <= 3.7, 3.2e-3 on Hyena, 5.7e-3 of the largest logit
on ResNet18); the TF32 bounds below are those measurements with headroom.
"""

import numpy as np
import pytest

from oracle import init, models

pytestmark = pytest.mark.gpu


def _wxx():
    import wxx_b200 as wxx

    return wxx


def _run(model, inp, is_ids, mode):
    wxx = _wxx()
    F = wxx.functional
    F.set_matmul_mode(mode)
    try:
        t = F.from_numpy(inp, dtype=np.uint32) if is_ids else F.from_numpy(inp)
        with wxx.backend.inferenceMode():
            return model(t).numpy()
    finally:
        F.set_matmul_mode("tf32")


@pytest.fixture(scope="module")
def gpt2_scaled():
    wxx = _wxx()
    V, D, H, L, S = 50304, 1024, 16, 24, 1024
    sd = init.gpt2_state_dict(0, V, D, H, L, S)
    ids = init.token_ids(1, 1, S, V)
    model = wxx.nn.GPT2(V, D, H, L, max_len=S)
    model.load_state_dict(sd)
    ref = models.gpt2_forward(sd, ids, H, L)
    del sd
    return model, ids, ref


@pytest.mark.parametrize("mode,tol", [("tf32", 1e-2), ("3xtf32", 1e-3)])
def test_gpt2_scaled_logits(gpt2_scaled, mode, tol):
    model, ids, ref = gpt2_scaled
    got = _run(model, ids, True, mode)
    assert got.shape == ref.shape == (1, 1024, 50304)
    err = float(np.abs(got - ref).max())
    assert err < tol, err
    assert _wxx().backend.device_status() == 0


@pytest.fixture(scope="module")
def hyena_c4():
    wxx = _wxx()
    V, D, NL, O, L = 1024, 256, 6, 4, 8192
    sd = init.hyena_state_dict(0, V, D, NL, O)
    ids = init.token_ids(3, 1, L, V)
    model = wxx.nn.Hyena(V, d_model=D, n_layers=NL, order=O)
    model.load_state_dict(sd)
    return model, ids, models.hyena_forward(sd, ids, NL, O)


@pytest.mark.parametrize("mode,tol", [("tf32", 1e-2), ("3xtf32", 1e-3)])
def test_hyena_config_logits(hyena_c4, mode, tol):
    model, ids, ref = hyena_c4
    got = _run(model, ids, True, mode)
    assert got.shape == ref.shape == (1, 8192, 1024)
    err = float(np.abs(got - ref).max())
    assert err < tol, err


@pytest.fixture(scope="module")
def resnet_b256():
    wxx = _wxx()
    sd = init.resnet18_state_dict(0, 10)
    x = np.random.default_rng(2).standard_normal((256, 3, 32, 32)).astype(np.float32)
    model = wxx.nn.ResNet18(num_classes=10)
    model.load_state_dict(sd)
    return model, x, models.resnet18_forward(sd, x)


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_resnet18_batch256_logits(resnet_b256, mode):
    model, x, ref = resnet_b256
    got = _run(model, x, False, mode)
    assert got.shape == (256, 10)
    err = float(np.abs(got - ref).max())
    if mode == "3xtf32":
        assert err < 1e-3, err
    else:
        assert err < 1.5e-2 * float(np.abs(ref).max()), err
