"""Record one step (a model forward, a chain of functional ops) as a CUDA graph
and replay it with a single launch.

The reference submits a step's dispatches as one command buffer
(backend/device.py:144-255 GPUCommandBuffer); here the step is recorded once
on the library stream and every later run is one ``cudaGraphLaunch``, so the
host-side cost of a step no longer grows with its kernel count.

    g = wxx_b200.graph.capture(model.forward, ids)   # runs nothing on the GPU
    logits = g.replay()                               # runs the recorded step

Inputs are read from the buffers they occupied during the capture: write new
data into them (``functional.assign`` or an H2D copy) before ``replay``.  The
outputs live in the graph's arena and are overwritten by every replay; they
stay valid until ``close``.  The step must not synchronise with the host
(``numpy()``, ``device_status``), and everything it caches lazily (masks,
position ids, kernel attributes) is created by the untimed warm-up run that
``capture`` performs first.
"""

import ctypes

from .backend import device as _dev
from .backend.lib import F, check

__all__ = ["CapturedGraph", "capture", "capturing"]

_CAPTURING = [False]


def capturing():
    """True while a step is being recorded (host-side checks that would
    synchronise with the device are skipped then; the kernels' own checks
    still report through the device error word)."""
    return _CAPTURING[0]


def _stats():
    out = (ctypes.c_int64 * 6)()
    check(F.wxx_mem_stats(out), "wxx_mem_stats")
    return list(out)


class CapturedGraph:
    """A step recorded by :func:`capture`."""

    def __init__(self, fn, args, kwargs, arena_bytes=None, warmup=True):
        _dev.ensure_init()
        self._handle = None
        self.output = None
        if arena_bytes is None or warmup:
            _dev.synchronize()
            active0 = _stats()[0]
            check(F.wxx_mem_reset_peak(), "wxx_mem_reset_peak")
            out = fn(*args, **kwargs)
            _dev.synchronize()
            need = _stats()[3] - active0
            del out
            if arena_bytes is None:
                # best-fit placement fragments a little more than the pool
                arena_bytes = int(need * 1.25) + (64 << 20)
        last_error = None
        for _ in range(3):
            try:
                self._record(fn, args, kwargs, arena_bytes)
                return
            except RuntimeError as e:
                last_error = e
                if "arena" not in str(e):
                    raise
                arena_bytes *= 2
        raise last_error

    def _record(self, fn, args, kwargs, arena_bytes):
        h = ctypes.c_void_p()
        check(F.wxx_graph_begin(int(arena_bytes), ctypes.byref(h)), "wxx_graph_begin")
        ok = False
        _CAPTURING[0] = True
        try:
            out = fn(*args, **kwargs)
            _CAPTURING[0] = False
            check(F.wxx_graph_end(h), "wxx_graph_end")
            ok = True
        finally:
            _CAPTURING[0] = False
            if not ok:
                out = None
                F.wxx_graph_destroy(h)
        self._handle = h
        self.output = out

    def stats(self):
        """{'arena_bytes', 'peak_bytes', 'kernels'} of the recorded step."""
        out = (ctypes.c_int64 * 3)()
        check(F.wxx_graph_stats(self._handle, out), "wxx_graph_stats")
        return {"arena_bytes": out[0], "peak_bytes": out[1], "kernels": out[2]}

    def replay(self):
        """Enqueues the recorded step on the library stream; returns its output."""
        if self._handle is None:
            raise RuntimeError("graph is closed")
        check(F.wxx_graph_launch(self._handle), "wxx_graph_launch")
        return self.output

    def close(self):
        """Waits for replays in flight and frees the graph and its arena."""
        if self._handle is not None:
            self.output = None
            check(F.wxx_graph_destroy(self._handle), "wxx_graph_destroy")
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def capture(fn, *args, arena_bytes=None, **kwargs):
    """Runs ``fn(*args, **kwargs)`` once eagerly (warm-up, arena sizing), then
    records it as a CUDA graph.  Returns a :class:`CapturedGraph`."""
    return CapturedGraph(fn, args, kwargs, arena_bytes=arena_bytes)
