"""wxx_fftconv_static (allocation-free FFT convolution) against wxx_fftconv.

Both are called through the C ABI.  The allocation-free entry point keeps the
filter spectrum in a fixed device array, so it must give the same result as
wxx_fftconv (which allocates that spectrum) on two calls in a row, must not
touch the library's allocator, and must refuse sizes beyond its fixed limits
without launching anything.  Tolerance: 2e-5 of the largest output, the FFT
tolerance of the kernel parity tests.

The file name sorts last so it also runs after every other GPU test.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WXX_E_ARG = -1
MAX_N = 32768
MAX_SPECTRUM = 256 * (MAX_N // 2 + 2)     # complex values, rows n/2 + 2 apart


def _setup():
    import wxx_b200 as wxx
    from wxx_b200.backend import lib

    lib.load()
    return wxx, lib


def _call(lib, fn, y, x, h, B, D, L, Lh, n, out_len):
    return fn(y.ptr, x.ptr, 0, D * L, L, 1, h.ptr, Lh, Lh, B, D, L, n, out_len)


def _mem_stats(lib):
    out = (lib.ctypes.c_int64 * 6)()
    lib.check(lib.F.wxx_mem_stats(out), "wxx_mem_stats")
    return list(out)


@pytest.mark.parametrize("B,D,L,Lh,n,out_len", [(2, 64, 1024, 1024, 2048, 1024),
                                                (3, 5, 300, 200, 1024, 300),
                                                (2, 8, 100, 100, 256, 100),
                                                (1, 256, 8192, 8192, 16384, 8192),
                                                (1, 256, 16384, 16384, 32768, 16384)])
def test_static_matches_allocating_entry_point(B, D, L, Lh, n, out_len, rng):
    wxx, lib = _setup()
    F = wxx.functional
    x = F.from_numpy(rng.standard_normal((B, D, L)).astype(np.float32))
    h = F.from_numpy((rng.standard_normal((D, Lh)) * 0.05).astype(np.float32))
    y_ref = F.from_numpy(np.zeros((B, D, out_len), np.float32))
    lib.check(_call(lib, lib.F.wxx_fftconv, y_ref, x, h, B, D, L, Lh, n, out_len), "wxx_fftconv")
    ref = y_ref.numpy()
    scale = max(float(np.abs(ref).max()), 1e-30)
    for _ in range(2):
        y = F.from_numpy(np.full((B, D, out_len), np.nan, np.float32))
        lib.check(lib.F.wxx_sync(), "sync")
        before = _mem_stats(lib)
        st = _call(lib, lib.F.wxx_fftconv_static, y, x, h, B, D, L, Lh, n, out_len)
        lib.check(st, "wxx_fftconv_static")
        lib.check(lib.F.wxx_sync(), "sync")
        after = _mem_stats(lib)
        assert after[4] == before[4] and after[5] == before[5], "allocator was used"
        got = y.numpy()
        assert float(np.abs(got - ref).max()) / scale < 2e-5
    assert wxx.backend.device_status() == 0


def test_static_rejects_sizes_beyond_its_limits(rng):
    wxx, lib = _setup()
    F = wxx.functional
    x = F.from_numpy(rng.standard_normal((1, 2, 8)).astype(np.float32))
    h = F.from_numpy(rng.standard_normal((2, 8)).astype(np.float32))
    y = F.from_numpy(np.zeros((1, 2, 8), np.float32))
    count = (lib.ctypes.c_int64 * 1)()
    lib.check(lib.F.wxx_launch_count(count), "launch count")
    launched = count[0]
    # n above the allocation-free limit
    assert _call(lib, lib.F.wxx_fftconv_static, y, x, h, 1, 2, 8, 8, 2 * MAX_N, 8) == WXX_E_ARG
    assert "exceeds" in lib.last_error()
    # D * (n/2 + 1) above the fixed scratch (pointers are never read: the
    # size check comes first and nothing is launched)
    D = MAX_SPECTRUM // (MAX_N // 2 + 2) + 1
    assert _call(lib, lib.F.wxx_fftconv_static, y, x, h, 1, D, 8, 8, MAX_N, 8) == WXX_E_ARG
    assert "static scratch" in lib.last_error()
    # out_len beyond n: refused before the filter transform is launched
    assert _call(lib, lib.F.wxx_fftconv_static, y, x, h, 1, 2, 8, 8, 16, 17) == WXX_E_ARG
    assert "out_len" in lib.last_error()
    # not a power of two
    assert _call(lib, lib.F.wxx_fftconv_static, y, x, h, 1, 2, 8, 8, 24, 8) == WXX_E_ARG
    lib.check(lib.F.wxx_launch_count(count), "launch count")
    assert count[0] == launched
    lib.check(lib.F.wxx_sync(), "sync")
    assert wxx.backend.device_status() == 0
