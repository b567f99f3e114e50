"""Device-side failure detection without a GPU fault.

The tensor-core kernels bound every mbarrier wait with a %globaltimer limit; on
expiry the kernel records WXX_DEV_ERR_MBAR_TIMEOUT (1) in the device error
word, stops waiting and returns, so the context stays usable.
``wxx_wait_probe`` runs that same wait function with a short limit on a
barrier that nothing arrives on (a stalled producer), and with the arrival
made (the normal path).  Nothing here traps, faults or hangs the GPU: the
longest wait is the 0.3 s limit the test sets.
"""

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup():
    import wxx_b200 as wxx
    from wxx_b200.backend import lib

    lib.load()
    return wxx, lib


def _probe(wxx, lib, arrive, limit_ns):
    res = wxx.functional.from_numpy(np.full(1, 7, np.uint32), dtype=np.uint32)
    t0 = time.perf_counter()
    lib.check(lib.F.wxx_wait_probe(int(arrive), int(limit_ns), res.ptr), "wait probe")
    code = wxx.backend.device_status()        # synchronises
    return int(res.numpy()[0]), code, time.perf_counter() - t0


def test_completed_wait_reports_nothing():
    wxx, lib = _setup()
    assert wxx.backend.device_status() == 0
    got, code, _ = _probe(wxx, lib, 1, 1_000_000_000)
    assert got == 1 and code == 0


def test_expired_wait_sets_status_and_context_survives(rng):
    wxx, lib = _setup()
    F = wxx.functional
    got, code, dt = _probe(wxx, lib, 0, 300_000_000)
    assert got == 0
    assert code == 1                           # WXX_DEV_ERR_MBAR_TIMEOUT
    assert 0.25 < dt < 10.0
    assert wxx.backend.device_status() == 0    # read-and-clear
    # the next kernels run normally on the same context
    a = rng.standard_normal((300, 200)).astype(np.float32)
    b = rng.standard_normal((200, 100)).astype(np.float32)
    c = F.matmul_add(F.from_numpy(a), F.from_numpy(b), None).numpy()
    ref = a.astype(np.float64) @ b
    assert np.abs(c - ref).max() < 2e-3 * np.abs(ref).max()
    assert wxx.backend.device_status() == 0


def test_probe_rejects_bad_limits():
    wxx, lib = _setup()
    res = wxx.functional.from_numpy(np.zeros(1, np.uint32), dtype=np.uint32)
    assert lib.F.wxx_wait_probe(0, 0, res.ptr) == -1
    assert lib.F.wxx_wait_probe(0, 20_000_000_000, res.ptr) == -1
    assert wxx.backend.device_status() == 0


def test_check_mode_reports_the_failing_call():
    """WXX_CHECK / set_check_mode: the launching call itself fails, naming the
    device error, instead of a later synchronisation."""
    wxx, lib = _setup()
    from wxx_b200.backend import observe

    F = wxx.functional
    res = F.from_numpy(np.zeros(1, np.uint32), dtype=np.uint32)
    observe.set_check_mode(True)
    try:
        assert observe.check_mode()
        assert lib.F.wxx_wait_probe(0, 200_000_000, res.ptr) == -3      # WXX_E_TIMEOUT
        assert "bounded wait expired" in lib.last_error()
        ids = F.from_numpy(np.array([[1, 99]], np.uint32), dtype=np.uint32)
        table = F.from_numpy(np.ones((8, 4), np.float32))
        with pytest.raises(RuntimeError, match="outside its table"):
            F.embed(ids, table, 2, 4)
        # a correct call still works in check mode
        y = F.embed(F.from_numpy(np.array([[1, 7]], np.uint32), dtype=np.uint32), table, 2, 4)
        assert np.array_equal(y.numpy(), np.ones((1, 2, 4), np.float32))
    finally:
        observe.set_check_mode(False)
    assert wxx.backend.device_status() == 0
    # without check mode the same bad id is reported by the status word
    F.embed(F.from_numpy(np.array([[99]], np.uint32), dtype=np.uint32), table, 1, 4)
    assert wxx.backend.device_status() == 2


def test_nvtx_ranges_leave_results_unchanged(rng):
    wxx, lib = _setup()
    from wxx_b200.backend import observe

    F = wxx.functional
    x = rng.standard_normal((64, 300)).astype(np.float32)
    plain = F.softmax(F.from_numpy(x), -1).numpy()
    ranged_softmax = observe.ranged(F.softmax, "wxx.softmax")
    assert np.array_equal(ranged_softmax(F.from_numpy(x), -1).numpy(), plain)
