"""Generates the golden fixtures in tests/golden/ from the reference's own tests.

The reference (Mo-Ehab/wxx) cannot run here (its wgpu backend needs a
graphics adapter), but its test files carry the expected values as pure-numpy
helpers and formulas.  This script
  * extracts the pure-numpy reference helpers from the reference test files by
    parsing them (ast) and executing only those function definitions:
      ref_causal_conv1d        tests/test_convolution.py:46-52
      _embedding_ref           tests/test_embedding.py:10-11
      ref_adaptive_avgpool2d   tests/test_pooling.py:17-28
      ref_maxpool2d            tests/test_pooling.py:67-94
  * evaluates the known-answer formulas the reference tests compare against
    (restated with the test's inputs and seeds):
      relu / gelu(tanh) / sigmoid  tests/test_activations.py:10-14
      sin / cos / exp / log        tests/test_activations.py:17-25
      softmax                      tests/test_activations.py:28-32
      sum / mean / max / argmax    tests/test_reductions.py:10-25
      LayerNorm / RMSNorm          tests/test_normalization.py:13-31
      Hyena positional encoding    tests/test_hyena.py:246-266
and writes the inputs and expected outputs to tests/golden/reference_golden.npz.
Run it where the reference is mounted:  python tests/golden/make_golden.py REF_ROOT
"""

import ast
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_golden.npz")


def extract(path, names):
    """Executes only the named top-level function definitions of a test file."""
    tree = ast.parse(open(path).read(), filename=path)
    wanted = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = set(names) - {n.name for n in wanted}
    if missing:
        raise SystemExit(f"{path}: missing {sorted(missing)}")
    ns = {"np": np}
    exec(compile(ast.Module(body=wanted, type_ignores=[]), path, "exec"), ns)
    return {n: ns[n] for n in names}


def rng(seed=0):
    # tests/common.py:42-43
    return np.random.default_rng(seed)


def main(ref_root):
    tests = os.path.join(ref_root, "tests")
    conv = extract(os.path.join(tests, "test_convolution.py"), ["ref_causal_conv1d"])
    emb = extract(os.path.join(tests, "test_embedding.py"), ["_embedding_ref"])
    pool = extract(os.path.join(tests, "test_pooling.py"), ["ref_adaptive_avgpool2d", "ref_maxpool2d"])
    g = {}

    # causal conv1d: test_convolution.py:55-92 shapes and seeds
    B, D, L, K = 3, 5, 9, 3
    x = rng(2).standard_normal((B, D, L)).astype(np.float32)
    w = rng(3).standard_normal((D, K)).astype(np.float32)
    b = rng(4).standard_normal((D,)).astype(np.float32)
    g["cconv_x"], g["cconv_w"], g["cconv_b"] = x, w, b
    g["cconv_out"] = conv["ref_causal_conv1d"](x, w, b).astype(np.float32)
    B, D, L, K = 2, 4, 7, 3
    xt = rng(6).standard_normal((B, L, D)).astype(np.float32)
    w2 = rng(7).standard_normal((D, K)).astype(np.float32)
    b2 = rng(8).standard_normal((D,)).astype(np.float32)
    g["cconvT_x_bld"], g["cconvT_w"], g["cconvT_b"] = xt, w2, b2
    g["cconvT_out"] = conv["ref_causal_conv1d"](np.transpose(xt, (0, 2, 1)), w2, b2).astype(np.float32)

    # embedding: test_embedding.py:14-31 (V, D, B, L) = (64, 32, 8, 300), ids from rng(0)
    V, D, B, L = 64, 32, 8, 300
    ids = rng(0).integers(0, V, size=(B, L)).astype(np.uint32)
    wt = rng(11).standard_normal((V, D)).astype(np.float32)
    g["emb_ids"], g["emb_w"] = ids, wt
    g["emb_out"] = emb["_embedding_ref"](wt, ids).astype(np.float32)

    # pooling: test_pooling.py:191-201, 307-318 style inputs
    xp = rng(21).standard_normal((2, 3, 9, 11)).astype(np.float32)
    g["pool_x"] = xp
    for hw in [(1, 1), (3, 4), (5, 5)]:
        g[f"apool_{hw[0]}x{hw[1]}"] = pool["ref_adaptive_avgpool2d"](xp, hw).astype(np.float32)
    mv, mi = pool["ref_maxpool2d"](xp, (3, 3), (2, 2), (1, 1))
    g["mpool_val"], g["mpool_idx"] = mv.astype(np.float32), mi.astype(np.uint32)
    xs = rng(22).standard_normal((2, 64, 16, 16)).astype(np.float32)   # ResNet stem pool shape
    g["mpool_stem_x"] = xs
    sv, si = pool["ref_maxpool2d"](xs, (3, 3), (2, 2), (1, 1))
    g["mpool_stem_val"], g["mpool_stem_idx"] = sv.astype(np.float32), si.astype(np.uint32)

    # activations: test_activations.py:10-32
    a = rng(0).standard_normal((5, 7)).astype(np.float32)
    g["act_x"] = a
    g["act_relu"] = np.maximum(a, 0)
    g["act_gelu"] = (a * 0.5 * (1 + np.tanh(np.sqrt(2 / np.pi) * (a + 0.044715 * a ** 3)))).astype(np.float32)
    g["act_sigmoid"] = (1 / (1 + np.exp(-a))).astype(np.float32)
    s = (rng(1).standard_normal((4, 6)) * 0.5).astype(np.float32)
    g["act2_x"] = s
    g["act2_sin"], g["act2_cos"], g["act2_exp"] = np.sin(s), np.cos(s), np.exp(s)
    pos = (np.abs(rng(2).standard_normal((4, 6))) + 0.5).astype(np.float32)
    g["act2_logx"], g["act2_log"] = pos, np.log(pos)
    sm = rng(3).standard_normal((3, 5)).astype(np.float32)
    g["softmax_x"] = sm
    g["softmax_out"] = (np.exp(sm) / np.exp(sm).sum(axis=-1, keepdims=True)).astype(np.float32)

    # reductions: test_reductions.py:10-25
    r = rng(0).standard_normal((4, 5)).astype(np.float32)
    g["red_x"] = r
    g["red_sum_all"] = np.array([r.sum()], np.float32)
    g["red_sum_0"] = r.sum(axis=0)
    g["red_sum_1_keep"] = r.sum(axis=1, keepdims=True)
    g["red_mean_last"] = r.mean(axis=-1)
    m = rng(1).standard_normal((3, 4)).astype(np.float32)
    g["mm_x"] = m
    g["mm_max1"], g["mm_argmax1"] = m.max(axis=1), m.argmax(axis=1).astype(np.uint32)
    g["mm_min0"] = m.min(axis=0)

    # norms: test_normalization.py:13-31 (gamma 1, beta 0)
    ln = rng(0).standard_normal((2, 3, 4)).astype(np.float32)
    g["ln_x"] = ln
    g["ln_out"] = ((ln - ln.mean(axis=-1, keepdims=True))
                   / np.sqrt(ln.var(axis=-1, keepdims=True) + 1e-5)).astype(np.float32)
    rn = rng(1).standard_normal((2, 4)).astype(np.float32)
    g["rms_x"] = rn
    g["rms_out"] = (rn / np.sqrt((rn ** 2).mean(axis=-1, keepdims=True) + 1e-6)).astype(np.float32)

    # Hyena positional encoding values: test_hyena.py:246-266 (L, K) = (8, 4)
    L, K = 8, 4
    t = np.linspace(0.0, 1.0, L)
    g["pe_8_4"] = np.concatenate(
        [t[:, None]] + [np.cos(2 * np.pi * k * t)[:, None] for k in range(K)]
        + [np.sin(2 * np.pi * k * t)[:, None] for k in range(K)], axis=1).astype(np.float32)

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the wxx reference checkout>")
    main(sys.argv[1])
