"""ctypes binding of libwxx_cuda.so (the C ABI declared in include/wxx_cuda.h).

The library is built in-tree by ``wxx_b200.csrc.build`` and loaded from
``wxx_b200/lib``.  Every call returns an int status; :func:`call` raises
``RuntimeError`` with the library's message on a non-zero status.  There is
no CPU fallback: when the library or a CUDA device is missing, the first call
that needs the GPU fails loudly.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libwxx_cuda.so")

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_u64 = ctypes.c_uint64
c_u32 = ctypes.c_uint32
c_float = ctypes.c_float
P_i64 = ctypes.POINTER(ctypes.c_int64)
P_int = ctypes.POINTER(ctypes.c_int)
P_float = ctypes.POINTER(ctypes.c_float)
P_void = ctypes.POINTER(ctypes.c_void_p)
P_u8 = ctypes.POINTER(ctypes.c_uint8)

# name -> argument types (all return int unless listed in _RESTYPES)
SIGNATURES = {
    "wxx_last_error": [],
    "wxx_version": [],
    "wxx_launch_count": [P_i64],
    "wxx_device_count": [P_int],
    "wxx_init": [c_int],
    "wxx_current_device": [P_int],
    "wxx_num_sms": [P_int],
    "wxx_malloc": [P_void, c_u64],
    "wxx_free": [c_void_p],
    "wxx_mem_stats": [P_i64],
    "wxx_mem_trim": [],
    "wxx_mem_reset_peak": [],
    "wxx_host_alloc": [P_void, c_u64],
    "wxx_host_free": [c_void_p],
    "wxx_memcpy_h2d": [c_void_p, c_void_p, c_u64],
    "wxx_memcpy_d2h": [c_void_p, c_void_p, c_u64],
    "wxx_memcpy_d2h_async": [c_void_p, c_void_p, c_u64],
    "wxx_memcpy_d2d": [c_void_p, c_void_p, c_u64],
    "wxx_memset": [c_void_p, c_int, c_u64],
    "wxx_sync": [],
    "wxx_get_stream": [],
    "wxx_set_stream": [c_void_p],
    "wxx_device_status": [P_int],
    "wxx_event_create": [P_void],
    "wxx_event_destroy": [c_void_p],
    "wxx_event_record": [c_void_p],
    "wxx_event_elapsed_ms": [c_void_p, c_void_p, P_float],
    "wxx_graph_begin": [c_u64, P_void],
    "wxx_graph_end": [c_void_p],
    "wxx_graph_launch": [c_void_p],
    "wxx_graph_stats": [c_void_p, P_i64],
    "wxx_graph_destroy": [c_void_p],
    "wxx_binary": [c_void_p, c_void_p, c_i64, P_i64, c_void_p, c_i64, P_i64, c_int, P_i64, c_int],
    "wxx_scalar": [c_void_p, c_void_p, c_i64, c_int, c_float, c_int],
    "wxx_clamp": [c_void_p, c_void_p, c_i64, c_float, c_float],
    "wxx_unary": [c_void_p, c_void_p, c_i64, c_int],
    "wxx_strided_copy": [c_void_p, c_i64, P_i64, c_void_p, c_i64, P_i64, c_int, P_i64, c_int],
    "wxx_strided_fill": [c_void_p, c_i64, P_i64, c_int, P_i64, c_u32],
    "wxx_embed": [c_void_p, c_void_p, c_void_p, c_i64, c_int, c_u32],
    "wxx_causal_conv1d": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64, c_void_p, c_void_p,
                          c_int, c_int, c_int, c_int],
    "wxx_decay_window": [c_void_p, c_void_p, c_int, c_int, c_int, c_int],
    "wxx_transpose_stack": [c_void_p, c_void_p, c_int, c_int, c_int, c_int],
    "wxx_round_tf32": [c_void_p, c_void_p, c_i64],
    "wxx_hyena_filters": [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                          c_void_p, c_void_p, c_void_p, c_float, c_void_p],
    "wxx_complex_mul": [c_void_p, c_void_p, c_i64, P_i64, c_void_p, c_i64, P_i64, c_int, P_i64,
                        c_int, c_int],
    "wxx_complex_conj": [c_void_p, c_void_p, c_i64],
    "wxx_complex_add_inplace": [c_void_p, c_void_p, c_i64],
    "wxx_equal": [c_void_p, c_void_p, c_void_p, c_i64, c_int, c_u32],
    "wxx_reduce": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int],
    "wxx_argminmax": [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int],
    "wxx_softmax": [c_void_p, c_void_p, c_i64, c_i64, c_i64],
    "wxx_softmax_masked": [c_void_p, c_void_p, c_i64, c_i64, c_void_p, c_i64, c_i64],
    "wxx_layernorm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64,
                      c_i64, c_float, c_int],
    "wxx_rmsnorm": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_float, c_int],
    "wxx_batchnorm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                      c_void_p, c_int, c_int, c_i64, c_float, c_float, c_int],
    "wxx_matmul": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64, c_i64,
                   c_i64, c_i64, c_i64, c_int, c_int, c_int, c_float, c_int],
    "wxx_linear": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64,
                   c_i64, c_int, c_int, c_float, c_int],
    "wxx_matmul_argmax": [c_void_p, c_void_p, c_void_p, c_void_p] + [c_i64] * 8
                         + [c_int, c_int, c_int],
    "wxx_ln_linear": [c_void_p, c_void_p, c_i64, c_void_p, c_void_p, c_float, c_void_p, c_i64,
                      c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int, c_int],
    "wxx_linear_batched": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64,
                           c_i64, c_i64, c_i64, c_int, c_i64, c_int, c_int, c_float, c_int],
    "wxx_linear_short_conv": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64,
                              c_i64, c_int, c_i64, c_void_p, c_void_p, c_int, c_int, c_int],
    "wxx_conv2d": [c_void_p, c_void_p, c_void_p, c_void_p] + [c_int] * 14,
    "wxx_conv2d_bn": [c_void_p, c_void_p, c_void_p, c_void_p] + [c_int] * 14
                     + [c_void_p] * 4 + [c_float, c_void_p, c_int],
    "wxx_conv2d_nhwc": [c_void_p, c_void_p, c_void_p, c_void_p] + [c_int] * 14
                       + [c_void_p] * 4 + [c_float, c_void_p, c_int],
    "wxx_conv2d_nhwc_packed": [c_void_p, c_void_p, c_void_p, c_void_p] + [c_int] * 14
                              + [c_void_p] * 4 + [c_float, c_void_p, c_int],
    "wxx_conv_weight_pack": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int],
    "wxx_resnet_stem": [c_void_p] * 8 + [c_float] + [c_int] * 6,
    "wxx_attention": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                      c_i64, c_i64, c_i64, c_float, c_void_p, c_i64, c_int, c_int, c_int],
    "wxx_maxpool2d": [c_void_p, c_void_p, c_void_p] + [c_int] * 10,
    "wxx_adaptive_avgpool2d": [c_void_p, c_void_p] + [c_int] * 6,
    "wxx_rfft": [c_void_p, c_i64, c_void_p, c_i64, c_i64, c_i64, c_i64],
    "wxx_irfft": [c_void_p, c_i64, c_void_p, c_i64, c_i64, c_i64, c_i64],
    "wxx_fftconv_spectrum": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64, c_void_p, c_i64,
                             c_int, c_int, c_int, c_i64, c_int],
    "wxx_fftconv_spectrum_gated": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64, c_void_p,
                                   c_i64, c_int, c_int, c_int, c_i64, c_int, c_void_p, c_i64,
                                   c_i64, c_i64, c_i64],
    "wxx_fftconv": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64, c_void_p, c_i64, c_int,
                    c_int, c_int, c_int, c_i64, c_int],
    "wxx_fftconv_gated": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64, c_void_p, c_i64, c_int,
                          c_int, c_int, c_int, c_i64, c_int, c_void_p, c_i64, c_i64, c_i64, c_i64],
    "wxx_fftconv_static": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_i64, c_void_p, c_i64,
                           c_int, c_int, c_int, c_int, c_i64, c_int],
    "wxx_wait_probe": [c_int, c_i64, c_void_p],
    "wxx_set_check_mode": [c_int],
    "wxx_get_check_mode": [P_int],
    "wxx_nvtx_push": [ctypes.c_char_p],
    "wxx_nvtx_pop": [],
    "wxx_decode_embed": [c_void_p, c_void_p, c_i64, c_void_p, c_void_p, c_void_p, c_int, c_int,
                         c_int, c_int],
    "wxx_decode_attention": [c_void_p, c_i64, c_void_p, c_void_p, c_void_p, c_i64, c_void_p,
                             c_void_p, c_i64, c_int, c_int, c_int, c_void_p, c_int, c_float,
                             c_int],
    "wxx_sample_tokens": [c_void_p, c_i64, c_void_p, c_void_p, c_void_p, c_i64, c_int, c_int,
                          c_float, c_int, c_void_p, c_int],
    "wxx_gelu_backward": [c_void_p, c_void_p, c_void_p, c_i64],
    "wxx_softmax_backward": [c_void_p, c_void_p, c_void_p, c_i64, c_i64],
    "wxx_layernorm_backward": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_i64, c_i64],
    "wxx_embedding_backward": [c_void_p, c_void_p, c_void_p, c_i64, c_int, c_int],
    "wxx_cceloss": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_int],
    "wxx_adamw": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64] + [c_float] * 7,
    "wxx_adamw_device": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64] + [c_float] * 5
                        + [c_void_p],
    "wxx_adamw_advance": [c_void_p, c_void_p, ctypes.c_double, ctypes.c_double],
    "wxx_adamw_device_multi": [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
                              + [c_float] * 5 + [c_void_p],
    "wxx_nccl_unique_id": [P_u8],
    "wxx_nccl_init": [P_u8, c_int, c_int],
    "wxx_nccl_allgather": [c_void_p, c_void_p, c_u64],
    "wxx_nccl_allgather_async": [c_void_p, c_void_p, c_u64, c_int],
    "wxx_nccl_wait": [c_int],
    "wxx_nccl_async_error": [P_int],
    "wxx_nccl_destroy": [c_int],
}

_RESTYPES = {
    "wxx_last_error": ctypes.c_char_p,
    "wxx_version": ctypes.c_char_p,
    "wxx_get_stream": c_void_p,
}

_lib = None


class _Funcs:
    """Attribute access to the bound C functions (``F.wxx_matmul(...)``)."""


F = _Funcs()


def load():
    """Loads the library (once) and binds every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing; build it with `python -m wxx_b200.csrc.build` "
            "(wxx_b200 has no CPU fallback)"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, c_int)
        setattr(F, name, fn)
    _lib = lib
    return lib


def last_error():
    load()
    msg = F.wxx_last_error()
    return msg.decode() if msg else ""


def check(status, what=""):
    """Raises RuntimeError for a non-zero library status."""
    if status != 0:
        raise RuntimeError(f"{what or 'wxx call'} failed ({status}): {last_error()}")
    return status


def i64_array(values):
    """A ctypes int64 array (kept alive by the caller for the call's duration)."""
    values = list(values)
    return (ctypes.c_int64 * max(1, len(values)))(*values)
