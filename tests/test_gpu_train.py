"""GPT2 training on the GPU against the float64 oracle (oracle/train.py, itself
checked against finite differences on the CPU).

Per-op backward kernels are compared with their float64 formulas (1e-5 of the
largest value; the embedding gradient's atomic adds only reorder fp32 sums).
The end-to-end step -- GPT2 forward in training mode, CCELoss, backward,
AdamW -- runs its products in 3xTF32 mode and is compared at 1e-4 of each
gradient's largest entry.
"""

import numpy as np
import pytest

from oracle import init, train

pytestmark = pytest.mark.gpu


def _w():
    import wxx_b200 as wxx

    return wxx


def up(a, dtype=np.float32):
    return _w().functional.from_numpy(np.asarray(a), dtype=dtype)


def rel(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


def test_gelu_backward(rng):
    F = _w().functional
    x = (rng.standard_normal(5000) * 4).astype(np.float32)
    x[:4] = [11.0, -11.0, 10.0, -10.0]
    dy = rng.standard_normal(5000).astype(np.float32)
    got = F.gelu_backward(up(dy), up(x)).numpy()
    assert rel(got, dy * train._gelu_slope(x.astype(np.float64))) < 1e-5
    assert rel(F.gelubackwards(up(x)).numpy(), train._gelu_slope(x.astype(np.float64))) < 1e-5


@pytest.mark.parametrize("n", [7, 256, 1000])
def test_softmax_backward(n, rng):
    F = _w().functional
    x = rng.standard_normal((33, n)).astype(np.float32)
    dy = rng.standard_normal((33, n)).astype(np.float32)
    y = F.softmax(up(x), -1)
    got = F.softmax_backward(up(dy), y, -1).numpy()
    yv = y.numpy().astype(np.float64)
    ref = yv * (dy - (dy * yv).sum(-1, keepdims=True))
    assert rel(got, ref) < 1e-5


@pytest.mark.parametrize("shape", [(40, 64), (3, 5, 256), (6, 1000)])
def test_layernorm_backward(shape, rng):
    F = _w().functional
    x = (rng.standard_normal(shape) * 2 + 1).astype(np.float32)
    n = shape[-1]
    g = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    dy = rng.standard_normal(shape).astype(np.float32)
    _, mu, inv = F.meanvarnorm(up(x), up(g), up(b), -1)
    dx, dg, db = F.layernorm_backward(up(dy), up(x), up(g), mu, inv, -1)
    _, cache = train._ln_fwd(x.astype(np.float64), g.astype(np.float64), b.astype(np.float64))
    rdx, rdg, rdb = train._ln_bwd(dy.astype(np.float64), cache, g.astype(np.float64))
    assert rel(dx.numpy(), rdx) < 1e-5
    assert rel(dg.numpy(), rdg) < 1e-5 and rel(db.numpy(), rdb) < 1e-5


def test_embedding_backward(rng):
    F = _w().functional
    V, D, T = 50, 24, 300
    ids = rng.integers(0, V, size=(3, 100)).astype(np.uint32)
    dy = rng.standard_normal((T, D)).astype(np.float32)
    got = F.embeddx(up(dy), up(ids, np.uint32), T, D, V).numpy()
    ref = np.zeros((V, D))
    np.add.at(ref, ids.reshape(-1), dy.astype(np.float64))
    assert rel(got, ref) < 1e-5


def test_cceloss_and_bad_targets(rng):
    F = _w().functional
    z = (rng.standard_normal((17, 300)) * 3).astype(np.float32)
    t = rng.integers(0, 300, size=17).astype(np.uint32)
    loss, grad = F.cceloss(up(z), up(t, np.uint32))
    zd = z.astype(np.float64)
    zm = zd - zd.max(-1, keepdims=True)
    lse = np.log(np.exp(zm).sum(-1))
    assert rel(loss.numpy()[:, 0], lse - zm[np.arange(17), t]) < 1e-5
    sm = np.exp(zm - lse[:, None])
    sm[np.arange(17), t] -= 1.0
    assert rel(grad.numpy(), sm) < 1e-5
    with pytest.raises(ValueError):
        F.cceloss(up(z), up(np.full(17, 300, np.uint32), np.uint32))


def test_adamw_kernel_two_steps(rng):
    F = _w().functional
    p = rng.standard_normal(1000).astype(np.float32)
    m = np.zeros(1000)
    v = np.zeros(1000)
    tp, tm, tv = up(p), up(np.zeros(1000)), up(np.zeros(1000))
    ref = p.astype(np.float64)
    # the kernel takes its hyperparameters as f32: the oracle gets the same values
    # (1 - beta2 in f32 differs from 0.001 by 1.3e-5 relative)
    b1, b2 = float(np.float32(0.9)), float(np.float32(0.999))
    for step in (1, 2):
        g = rng.standard_normal(1000).astype(np.float32)
        F.adamw(tp, up(g), tm, tv, step, 1e-2, b1, b2, 1e-7, 1e-2, 1 - b1 ** step, 1 - b2 ** step)
        ref, m, v = train.adamw_step(ref, g, m, v, step, 1e-2, b1, b2, 1e-7, 1e-2)
    assert rel(tp.numpy(), ref) < 1e-5 and rel(tm.numpy(), m) < 1e-5 and rel(tv.numpy(), v) < 1e-5


def _gpt2(V, D, H, L, S):
    wxx = _w()
    sd = init.gpt2_state_dict(1, V, D, H, L, S)
    rng = np.random.default_rng(4)
    for k in sd:            # non-trivial LayerNorm affine and biases
        if k.endswith(("weightg", "weightb", "bias")):
            sd[k] = (sd[k] + 0.1 * rng.standard_normal(sd[k].shape)).astype(np.float32)
    for k in list(sd):      # LayerNorm aliases carry the same arrays
        if k.endswith("weightg"):
            sd[k[:-1]] = sd[k]
        if k.endswith("weightb"):
            sd[k[:-7] + "bias"] = sd[k]
    model = wxx.nn.GPT2(V, D, H, L, max_len=S, dropout=0.0)
    model.load_state_dict(sd)
    return model, sd


def _loss(model, ids, tgt):
    wxx = _w()
    logits = model(up(ids, np.uint32))
    B, S, V = logits.shape
    return wxx.nn.CCELoss()(logits.reshape((B * S, V)), up(tgt.reshape(-1), np.uint32))


def test_gpt2_training_gradients_match_oracle():
    wxx = _w()
    V, D, H, L, S = 64, 32, 2, 2, 16
    model, sd = _gpt2(V, D, H, L, S)
    rng = np.random.default_rng(9)
    ids = rng.integers(0, V, size=(2, S)).astype(np.uint32)
    tgt = rng.integers(0, V, size=(2, S)).astype(np.uint32)
    wxx.set_matmul_mode("3xtf32")
    try:
        loss = _loss(model, ids, tgt)
        loss.backward()
    finally:
        wxx.set_matmul_mode("tf32")
    ref_loss, ref = train.gpt2_loss_and_grads(sd, ids, tgt, H, L)
    assert abs(float(loss.numpy().reshape(-1)[0]) - ref_loss) < 1e-5 * max(1.0, abs(ref_loss))
    params = dict(model.named_parameters())
    checked = 0
    for name, g_ref in ref.items():
        if name.endswith((".weight", ".bias")) and ("ln" in name.split(".")[-2]):
            continue        # LayerNorm aliases: checked through weightg / weightb
        p = params[name]
        assert p.grad is not None, name
        assert rel(p.grad.numpy(), g_ref) < 1e-4, (name, rel(p.grad.numpy(), g_ref))
        checked += 1
    assert checked >= 4 + 12 * L
    assert wxx.backend.device_status() == 0


def test_gpt2_adamw_training_loss_falls():
    wxx = _w()
    V, D, H, L, S = 64, 32, 2, 2, 16
    model, _ = _gpt2(V, D, H, L, S)
    rng = np.random.default_rng(10)
    ids = rng.integers(0, V, size=(4, S)).astype(np.uint32)
    tgt = np.roll(ids, -1, axis=1)
    opt = wxx.nn.AdamW(model.parameters(), lr=1e-2, weight_decay=0.0)
    losses = []
    for _ in range(30):
        opt.zero_grad()
        loss = _loss(model, ids, tgt)
        loss.backward()
        opt.step()
        losses.append(float(loss.numpy().reshape(-1)[0]))
    assert np.isfinite(losses).all()
    assert losses[-1] < 0.5 * losses[0], losses
    # the inference path reads the trained weights (cached copies rebuilt)
    with wxx.backend.inferenceMode():
        logits = model(up(ids, np.uint32)).numpy()
    z = logits.reshape(-1, V).astype(np.float64)
    zm = z - z.max(-1, keepdims=True)
    infer_loss = float((np.log(np.exp(zm).sum(-1)) - zm[np.arange(z.shape[0]), tgt.reshape(-1)])
                       .mean())
    assert abs(infer_loss - losses[-1]) < 0.2 * losses[0]


def test_gpt2_training_step_replays_from_a_graph():
    """A whole training step (forward, CCELoss, backward, AdamW) recorded as a
    CUDA graph and replayed on new batches ends at the same weights and loss as
    the eager steps (the device step count advances AdamW's bias corrections
    on every replay; the embedding gradient's atomic adds may reorder fp32
    sums, hence a tolerance instead of equal bits)."""
    wxx = _w()
    F = wxx.functional
    V, D, H, L, S, B = 64, 32, 2, 2, 16, 2
    rng = np.random.default_rng(11)
    batches = [rng.integers(0, V, size=(B, S)).astype(np.uint32) for _ in range(5)]

    def make():
        model, _ = _gpt2(V, D, H, L, S)
        opt = wxx.nn.AdamW(model.parameters(), lr=1e-2)
        ids = up(batches[0], np.uint32)
        tgt = up(np.roll(batches[0], -1, axis=1).reshape(-1), np.uint32)

        def step():
            opt.zero_grad()
            logits = model(ids)
            loss = wxx.nn.CCELoss()(logits.reshape((B * S, V)), tgt)
            loss.backward()
            opt.step()
            return loss

        return model, ids, tgt, step

    def load(ids, tgt, k):
        F.assign(ids, up(batches[k], np.uint32))
        F.assign(tgt, up(np.roll(batches[k], -1, axis=1).reshape(-1), np.uint32))

    m_eager, ids, tgt, step = make()
    for k in range(5):
        load(ids, tgt, k)
        last_eager = float(step().numpy().reshape(-1)[0])

    m_graph, ids, tgt, step = make()
    g = wxx.graph.capture(step)                 # its warm-up run is step 1 (batch 0)
    try:
        for k in range(1, 5):
            load(ids, tgt, k)
            out = g.replay()
        last_graph = float(out.numpy().reshape(-1)[0])
        assert abs(last_graph - last_eager) < 1e-4 * max(1.0, abs(last_eager))
        pe = dict(m_eager.named_parameters())
        for name, p in m_graph.named_parameters():
            assert rel(p.numpy(), pe[name].numpy()) < 1e-4, name
    finally:
        g.close()
    assert wxx.backend.device_status() == 0


def test_adamw_module_multi_tensor_matches_oracle(rng):
    """nn.AdamW steps all its parameters with one multi-tensor launch (sizes
    across chunk boundaries, a parameter without a gradient skipped); two
    steps against the float64 oracle with the same f32 hyperparameters."""
    wxx = _w()
    from wxx_b200.Tensor import Parameter

    shapes = [(5000,), (3, 7), (4096,), (1,), (64, 65)]
    host = [rng.standard_normal(s).astype(np.float32) for s in shapes]
    params = [Parameter(up(h)) for h in host]
    b1, b2 = float(np.float32(0.9)), float(np.float32(0.999))
    opt = wxx.nn.AdamW([("", p) for p in params], lr=1e-2, beta1=b1, beta2=b2, eps=1e-7,
                       weight_decay=1e-2)
    ref = [h.astype(np.float64) for h in host]
    mom = [np.zeros(s) for s in shapes]
    vel = [np.zeros(s) for s in shapes]
    for step in (1, 2):
        grads = [rng.standard_normal(s).astype(np.float32) for s in shapes]
        for i, p in enumerate(params):
            p.grad = None if i == 3 else up(grads[i])
        opt.step()
        for i in range(len(shapes)):
            if i == 3:
                continue
            ref[i], mom[i], vel[i] = train.adamw_step(ref[i], grads[i], mom[i], vel[i], step, 1e-2,
                                                      b1, b2, 1e-7, 1e-2)
    for i, p in enumerate(params):
        expect = host[i] if i == 3 else ref[i]
        assert rel(p.numpy(), expect) < 1e-5, i
