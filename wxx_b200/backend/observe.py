"""Debugging and tracing switches (no reference counterpart: the reference has
no tracing and no sanitizer mode).

``WXX_NVTX=1`` (read when ``wxx_b200.functional`` is imported) wraps every
public functional operator in an NVTX range named ``wxx.<op>``, so a
profiler's timeline groups the kernels of each call; with no profiler
attached a range costs one library call.

``WXX_CHECK=1`` (read at device initialisation) or ``set_check_mode(True)``
turns on check mode: after every kernel launch the library waits for the
kernel and reads the device error word, so an out-of-table index or an
expired bounded wait is raised by the call that launched the kernel (with its
source line) instead of by a later synchronisation.  Views are also checked on
the host to stay inside their storage.  Check mode serialises the stream; it
is for debugging only.
"""

import functools
import os

from .lib import F, check, load


def nvtx_requested():
    return os.environ.get("WXX_NVTX", "") == "1"


def ranged(fn, label):
    """``fn`` wrapped in an NVTX range called ``label``."""
    name = label.encode()

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        load()
        F.wxx_nvtx_push(name)
        try:
            return fn(*args, **kwargs)
        finally:
            F.wxx_nvtx_pop()

    wrapper.__wxx_nvtx__ = label
    return wrapper


def wrap_namespace(namespace, prefix):
    """Wraps every public function of a module namespace dict in place."""
    import types

    for key, value in list(namespace.items()):
        if key.startswith("_") or not isinstance(value, types.FunctionType):
            continue
        if getattr(value, "__wxx_nvtx__", None):
            continue
        namespace[key] = ranged(value, f"{prefix}.{key}")


def set_check_mode(on):
    import importlib

    # the module (the package attribute of that name is the Tensor class)
    _tensor_module = importlib.import_module("..Tensor", __package__)
    load()
    check(F.wxx_set_check_mode(int(bool(on))), "wxx_set_check_mode")
    _tensor_module._CHECK["views"] = bool(on)


def check_mode():
    import ctypes

    load()
    v = ctypes.c_int(0)
    check(F.wxx_get_check_mode(ctypes.byref(v)), "wxx_get_check_mode")
    return bool(v.value)
