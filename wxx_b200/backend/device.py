"""CUDA device runtime behind the wxx API (reference: src/wxx/backend/device.py).

The reference creates one WebGPU device, one buffer pool and one command
encoder at import time.  Here the same three roles map onto libwxx_cuda.so:

* ``WebGPUContext``   -> :class:`CudaContext` (device selection, lazy init)
* ``GPUBufferPool``   -> :class:`DeviceBufferPool` over the library's
  stream-ordered caching allocator (blocks freed on the stream are reused by
  later allocations without a device synchronisation)
* ``GPUCommandBuffer``-> :class:`CommandStream`: every kernel is enqueued on
  one CUDA stream in call order; ``flush(wait=True)`` is the stream fence.

The device is chosen from ``WXX_DEVICE``, else ``LOCAL_RANK`` (one process per
GPU under torchrun), else 0.  Initialisation is lazy so that importing the
package on a machine without a GPU works; the first GPU operation there raises.
"""

import ctypes
import itertools
import os
import sys
import weakref

from . import lib
from .lib import F, check


class CudaContext:
    """Device selection and one-time initialisation of the kernel library."""

    def __init__(self):
        self.device = None
        self.ready = False

    def init(self, device=None):
        if self.ready:
            return self
        lib.load()
        if device is None:
            device = int(os.environ.get("WXX_DEVICE", os.environ.get("LOCAL_RANK", "0")))
        count = ctypes.c_int(0)
        F.wxx_device_count(ctypes.byref(count))
        if count.value == 0:
            raise RuntimeError(
                "no CUDA device is visible: wxx_b200 runs its kernels on B200 GPUs "
                "and has no CPU fallback"
            )
        check(F.wxx_init(int(device)), f"wxx_init({device})")
        self.device = int(device)
        self.ready = True
        return self

    def num_sms(self):
        self.init()
        n = ctypes.c_int(0)
        check(F.wxx_num_sms(ctypes.byref(n)))
        return n.value


_ctx = CudaContext()


def ensure_init():
    if not _ctx.ready:
        _ctx.init()


_buffer_uids = itertools.count(1)


class DeviceBuffer:
    """An allocation of the library's device allocator.

    ``ptr`` is the device address, ``size`` the requested byte count.  The
    memory is returned to the allocator (stream-ordered) when the last
    reference to the buffer object goes away, so views keep storage alive by
    holding the same ``DeviceBuffer``.
    """

    # ``uid`` names this allocation for the life of the process (object ids
    # can be reused); ``version`` counts the in-place writes made through the
    # library's API (``functional.assign`` and the other in-place ops), so
    # caches derived from a buffer (K-major weight copies) can tell when it
    # changed.
    __slots__ = ("ptr", "size", "label", "uid", "version", "__weakref__")

    def __init__(self, nbytes, label="Tensor"):
        ensure_init()
        p = ctypes.c_void_p()
        check(F.wxx_malloc(ctypes.byref(p), int(nbytes)), f"wxx_malloc({nbytes})")
        self.ptr = p.value
        self.size = int(nbytes)
        self.label = label
        self.uid = next(_buffer_uids)
        self.version = 0
        _pool._track(self)

    def free(self):
        ptr = self.ptr
        if ptr:
            self.ptr = None
            _pool._untrack(self)
            F.wxx_free(ptr)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def __repr__(self):
        return f"DeviceBuffer(ptr=0x{self.ptr or 0:x}, size={self.size}, label={self.label!r})"


class DeviceBufferPool:
    """Accounting view of the caching allocator (mirrors GPUBufferPool)."""

    def __init__(self):
        self._active = {}

    def _track(self, buf):
        self._active[id(buf)] = weakref.ref(buf)

    def _untrack(self, buf):
        self._active.pop(id(buf), None)

    def create_buffer(self, size, usage=None, label=None):
        if label is None:
            label = sys._getframe(1).f_code.co_name
        return DeviceBuffer(max(4, int(size)), label)

    def release(self, buffer):
        if isinstance(buffer, DeviceBuffer):
            buffer.free()

    def stats(self):
        ensure_init()
        out = (ctypes.c_int64 * 6)()
        check(F.wxx_mem_stats(out))
        return {
            "active_bytes": out[0],
            "active_blocks": out[1],
            "reserved_bytes": out[2],
            "peak_active_bytes": out[3],
            "allocations": out[4],
            "frees": out[5],
        }

    def get_memory_snapshot(self):
        """Same dict shape as the reference (device.py:115-133)."""
        active = []
        for key, ref in list(self._active.items()):
            buf = ref()
            if buf is None or buf.ptr is None:
                self._active.pop(key, None)
            else:
                active.append({"label": buf.label, "size": buf.size})
        st = self.stats() if _ctx.ready else {"active_bytes": 0, "reserved_bytes": 0}
        cached = max(0, st["reserved_bytes"] - st["active_bytes"])
        return {
            "active": active,
            "cached": [{"label": "pool", "size": cached}] if cached else [],
            "active_bytes": sum(b["size"] for b in active),
            "cached_bytes": cached,
        }

    def clear_cache(self):
        if _ctx.ready:
            check(F.wxx_mem_trim())


class CommandStream:
    """Stream-ordered launches; flush(wait=True) synchronises the stream."""

    def flush(self, wait=False):
        if wait and _ctx.ready:
            check(F.wxx_sync(), "wxx_sync")

    def keep_alive(self, buf):
        """No-op: stream-ordered frees already keep buffers valid for queued work."""

    def defer_destroy(self, buf):
        _pool.release(buf)

    def complete_pending(self):
        self.flush(wait=True)


_pool = DeviceBufferPool()
_cmd = CommandStream()


def get_ctx():
    return _ctx


def get_device():
    ensure_init()
    return _ctx.device


def get_buffer_pool():
    return _pool


def get_cmd_buffer():
    return _cmd


def synchronize():
    _cmd.flush(wait=True)


def device_status():
    """Synchronises and returns (then clears) the device error word."""
    ensure_init()
    code = ctypes.c_int(0)
    check(F.wxx_device_status(ctypes.byref(code)))
    return code.value


class Event:
    """A CUDA event recorded on the library stream (for device-side timing)."""

    def __init__(self):
        ensure_init()
        p = ctypes.c_void_p()
        check(F.wxx_event_create(ctypes.byref(p)))
        self.ptr = p.value

    def record(self):
        check(F.wxx_event_record(self.ptr))
        return self

    def elapsed_ms(self, end):
        ms = ctypes.c_float()
        check(F.wxx_event_elapsed_ms(self.ptr, end.ptr, ctypes.byref(ms)))
        return ms.value

    def __del__(self):
        try:
            if self.ptr:
                F.wxx_event_destroy(self.ptr)
        except Exception:
            pass


class PinnedHostBuffer:
    """Page-locked host memory (for timed host<->device copies)."""

    def __init__(self, nbytes):
        ensure_init()
        p = ctypes.c_void_p()
        check(F.wxx_host_alloc(ctypes.byref(p), int(nbytes)))
        self.ptr = p.value
        self.size = int(nbytes)

    def as_numpy(self, dtype, shape):
        import numpy as np

        count = int(np.prod(shape)) if len(shape) else 1
        buf = (ctypes.c_uint8 * self.size).from_address(self.ptr)
        return np.frombuffer(buf, dtype=dtype, count=count).reshape(shape)

    def __del__(self):
        try:
            if self.ptr:
                F.wxx_host_free(self.ptr)
        except Exception:
            pass


def launch_count():
    """Kernels launched by libwxx_cuda.so so far in this process."""
    from .lib import load

    load()
    out = ctypes.c_int64(0)
    check(F.wxx_launch_count(ctypes.byref(out)))
    return out.value
