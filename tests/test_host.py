"""CPU tests of the host side: the C-ABI library loads and exports every
declared symbol, shape logic, and loud failure without a GPU."""

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "wxx_cuda.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wxx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from wxx_b200.backend import lib

    so = lib.load()
    names = _declared()
    assert len(names) > 40
    for name in names:
        assert hasattr(so, name), name
        assert name in lib.SIGNATURES, f"{name} has no ctypes signature"


def test_ctypes_signatures_cover_only_declared_symbols():
    from wxx_b200.backend import lib

    assert set(lib.SIGNATURES) <= set(_declared())


def test_calls_fail_cleanly_without_init():
    from wxx_b200.backend import lib

    lib.load()
    n = ctypes.c_int(-1)
    assert lib.F.wxx_device_count(ctypes.byref(n)) == 0
    p = ctypes.c_void_p()
    if n.value == 0:
        rc = lib.F.wxx_malloc(ctypes.byref(p), 16)
        assert rc != 0 and "wxx_init" in lib.last_error()


def test_tensor_creation_fails_loudly_without_gpu():
    from wxx_b200.backend import lib

    lib.load()
    n = ctypes.c_int(0)
    lib.F.wxx_device_count(ctypes.byref(n))
    if n.value:
        pytest.skip("a GPU is present")
    import wxx_b200 as wxx

    with pytest.raises(RuntimeError, match="no CPU fallback"):
        wxx.Tensor((2, 3))


def test_reduce_dims_match_reference_rules():
    from wxx_b200.backend.dispatch import _get_reduce_dims, broadcast_shapes

    assert _get_reduce_dims((4096, 4096), 0) == (1, 4096, 4096, (4096,))
    assert _get_reduce_dims((4096, 4096), 1) == (4096, 4096, 1, (4096,))
    assert _get_reduce_dims((2, 3, 4, 5), (1, 2)) == (2, 12, 5, (2, 5))
    assert _get_reduce_dims((2, 3), None) == (1, 6, 1, (1,))
    with pytest.raises(ValueError):
        _get_reduce_dims((2, 3, 4), (0, 2))
    assert broadcast_shapes((4, 1, 3), (5, 1))[0] == (4, 5, 3)
    with pytest.raises(ValueError):
        broadcast_shapes((3,), (4,))


def test_validation_helpers():
    from wxx_b200 import validation as v

    assert v.infer_shape((2, -1), 6) == (2, 3)
    assert v.contiguous_strides((2, 3, 4)) == (12, 4, 1)
    assert v.is_contiguous_layout((2, 1, 4), (4, 99, 1))
    assert not v.is_contiguous_layout((2, 3), (1, 2))
    with pytest.raises(IndexError):
        v.normalize_dim(3, 2)
    with pytest.raises(ValueError):
        v.check_rank((1,) * 7)


def test_functional_api_names_present():
    import wxx_b200.functional as F

    for name in ["matmul_add", "conv2d", "softmax", "sum", "mean", "sumsq", "max", "min",
                 "meanvarnorm", "rmsnorm", "batchnorm", "rfft", "irfft", "complex_mul", "embed",
                 "pointwise", "scalarpointwise", "relu", "gelu", "sigmoid", "sin", "cos",
                 "contiguous", "assign", "causal_conv1d", "decay_window", "maxpool2d",
                 "adaptive_avgpool2d", "from_numpy", "normal", "uniform", "reshape", "permute"]:
        assert callable(getattr(F, name)), name
    with pytest.raises(NotImplementedError):
        F.conv2ddx(None)


def test_matmul_mode_switch():
    import wxx_b200.functional as F

    assert F.get_matmul_mode() in ("tf32", "3xtf32", "fp32")
    F.set_matmul_mode("3xTF32")
    assert F.get_matmul_mode() == "3xtf32"
    F.set_matmul_mode("tf32")
    with pytest.raises(ValueError):
        F.set_matmul_mode("bf16")


def test_oracle_not_imported_by_product():
    pkg = os.path.join(ROOT, "wxx_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f


def test_numpy_available():
    assert np.__version__


def test_validation_contracts():
    from wxx_b200 import validation as v

    assert v.normalize_shape(3) == (3,)
    assert v.normalize_shape((2, -1), allow_infer=True) == (2, -1)
    with pytest.raises(ValueError):
        v.normalize_shape((2, -1))
    with pytest.raises(ValueError):
        v.normalize_shape((-1, -1), allow_infer=True)
    with pytest.raises(TypeError):
        v.normalize_shape((2, 1.5))
    with pytest.raises(TypeError):
        v.normalize_shape((2, True))
    with pytest.raises(ValueError):
        v.infer_shape((4, -1), 6)
    with pytest.raises(ValueError):
        v.infer_shape((0, -1), 0)
    assert v.normalize_dim(-1, 3) == 2
    with pytest.raises(IndexError):
        v.normalize_dim(0, 0)
    with pytest.raises(TypeError):
        v.normalize_dim("1", 2)
    assert v.normalize_dims((-1, 0), 3) == (2, 0)
    with pytest.raises(ValueError):
        v.normalize_dims((1, -2), 3, allow_duplicates=False)
    assert v.check_rank((1, 2), min_rank=2, max_rank=None) == 2
    with pytest.raises(ValueError):
        v.check_rank((1,), min_rank=2, max_rank=2)
    assert v.check_same_shape((2, 3), [2, 3]) == (2, 3)
    with pytest.raises(ValueError):
        v.check_same_shape((2, 3), (3, 2))
    assert v.check_broadcastable((3, 1), (2, 3, 4)) == (2, 3, 4)
    with pytest.raises(ValueError):
        v.check_broadcastable((2, 4), (3, 4))
    assert v.numel(()) == 1 and v.numel((2, 0, 3)) == 0


def test_npz_state_dict_round_trip(tmp_path):
    from wxx_b200 import serialization as s

    state = {"blocks.0.w": np.arange(6, dtype=np.float32).reshape(2, 3),
             "ids": np.array([1, 2], np.uint32)}
    path = s.save(state, tmp_path / "ckpt")
    assert path.endswith(".npz")
    back = s.load(tmp_path / "ckpt")
    assert set(back) == set(state)
    for k in state:
        assert back[k].dtype == state[k].dtype and np.array_equal(back[k], state[k])
    one = s.load(s.save(np.ones(3, np.float32), str(tmp_path / "one.npz")))
    assert list(one) == ["tensor"]


def test_nvtx_wrapping_is_opt_in():
    import subprocess
    import sys

    code = ("import wxx_b200.functional as F;"
            "print(getattr(F.matmul_add, '__wxx_nvtx__', None), getattr(F.fftconv, "
            "'__wxx_nvtx__', None))")
    env = dict(os.environ, WXX_NVTX="1", PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         cwd=ROOT, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split() == ["wxx.matmul_add", "wxx.fftconv"]
    env.pop("WXX_NVTX")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         cwd=ROOT, timeout=300)
    assert out.stdout.split() == ["None", "None"]


def test_check_mode_view_extent():
    import importlib

    T = importlib.import_module("wxx_b200.Tensor")

    class FakeStorage:
        size = 4 * 12          # 12 floats

    old = T._CHECK["views"]
    T._CHECK["views"] = True
    try:
        ok = T.Tensor._wrap([3, 4], FakeStorage())
        assert ok.shape == [3, 4]
        T.Tensor._wrap([2, 2], FakeStorage(), stride=(4, 2), offset=5)     # last element 11
        with pytest.raises(IndexError):
            T.Tensor._wrap([2, 2], FakeStorage(), stride=(4, 2), offset=6)  # element 12
        with pytest.raises(IndexError):
            T.Tensor._wrap([3], FakeStorage(), stride=(-1,), offset=1)      # element -1
    finally:
        T._CHECK["views"] = old
