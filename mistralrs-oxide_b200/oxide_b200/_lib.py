"""ctypes binding of liboxide_b200.so (the C ABI declared in include/oxide_ops.h).

The library is built in-tree by ``make -C mistralrs-oxide_b200`` (or
``__graft_entry__.build()``).  There is no fallback: if the shared library is
missing, :func:`lib` raises, so no op can silently run anywhere but in the
sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_PKG_DIR), "lib", "liboxide_b200.so")

u64, i32, f32, vp = C.c_uint64, C.c_int, C.c_float, C.c_void_p

# name -> (restype, argtypes); every pointer (device, host, stream) is c_void_p.
SIGNATURES: dict[str, tuple] = {
    "oxide_status_string": (C.c_char_p, [i32]),
    "oxide_last_error": (C.c_char_p, []),
    "oxide_version": (C.c_char_p, []),
    "oxide_debug_fail_next": (None, [C.c_char_p]),
    "oxide_selftest_rowdiv": (i32, [vp, u64, vp, u64, vp, vp]),
    "oxide_binary_f32": (i32, [i32, vp, u64, vp, u64, vp, u64, vp]),
    "oxide_binary_bf16": (i32, [i32, vp, u64, vp, u64, vp, u64, vp]),
    "oxide_add_f32": (i32, [vp, vp, vp, u64, vp]),
    "oxide_add_bf16": (i32, [vp, vp, vp, u64, vp]),
    "oxide_sub_f32": (i32, [vp, vp, vp, u64, vp]),
    "oxide_div_f32": (i32, [vp, vp, vp, u64, vp]),
    "oxide_mul_rowbcast_f32": (i32, [vp, vp, vp, u64, u64, vp]),
    "oxide_mul_rowbcast_bf16": (i32, [vp, vp, vp, u64, u64, vp]),
    "oxide_add_mul_rowbcast_f32": (i32, [vp, vp, vp, vp, u64, u64, vp]),
    "oxide_add_mul_rowbcast_bf16": (i32, [vp, vp, vp, vp, u64, u64, vp]),
    "oxide_scale_f32": (i32, [vp, vp, f32, u64, vp]),
    "oxide_scale_bf16": (i32, [vp, vp, f32, u64, vp]),
    "oxide_silu_f32": (i32, [vp, vp, u64, vp]),
    "oxide_silu_bf16": (i32, [vp, vp, u64, vp]),
    "oxide_silu_mul_f32": (i32, [vp, vp, vp, u64, vp]),
    "oxide_silu_mul_bf16": (i32, [vp, vp, vp, u64, vp]),
    "oxide_rms_norm_f32": (i32, [vp, vp, vp, u64, u64, f32, vp]),
    "oxide_rms_norm_bf16": (i32, [vp, vp, vp, u64, u64, f32, vp]),
    "oxide_add_rms_norm_f32": (i32, [vp, vp, vp, vp, vp, u64, u64, f32, vp]),
    "oxide_add_rms_norm_bf16": (i32, [vp, vp, vp, vp, vp, u64, u64, f32, vp]),
    "oxide_softmax_f32": (i32, [vp, vp, u64, u64, u64, vp]),
    "oxide_softmax_bf16": (i32, [vp, vp, u64, u64, u64, vp]),
    "oxide_scale_mask_softmax_f32": (i32, [vp, vp, u64, u64, f32, vp, u64, vp, u64, u64, vp]),
    "oxide_scale_mask_softmax_bf16": (i32, [vp, vp, u64, u64, f32, vp, u64, vp, u64, u64, vp]),
    "oxide_rope_f32": (i32, [vp, vp, u64, vp, vp, u64, vp, vp, u64, vp, u64, u64, i32, vp]),
    "oxide_rope_bf16": (i32, [vp, vp, u64, vp, vp, u64, vp, vp, u64, vp, u64, u64, i32, vp]),
    "oxide_rope_table_host_f32": (i32, [f32, u64, u64, vp, vp]),
    "oxide_argmax_rows_f32": (i32, [vp, u64, u64, vp, vp]),
    "oxide_argmax_rows_bf16": (i32, [vp, u64, u64, vp, vp]),
    "oxide_unary_f32": (i32, [i32, vp, vp, u64, f32, f32, vp]),
    "oxide_unary_bf16": (i32, [i32, vp, vp, u64, f32, f32, vp]),
    "oxide_relu_f32": (i32, [vp, vp, u64, vp]),
    "oxide_gelu_f32": (i32, [vp, vp, u64, vp]),
    "oxide_sigmoid_f32": (i32, [vp, vp, u64, vp]),
    "oxide_tanh_f32": (i32, [vp, vp, u64, vp]),
    "oxide_layer_norm_f32": (i32, [vp, vp, vp, vp, u64, u64, f32, vp]),
    "oxide_layer_norm_bf16": (i32, [vp, vp, vp, vp, u64, u64, f32, vp]),
    "oxide_add_layer_norm_f32": (i32, [vp, vp, vp, vp, vp, u64, u64, f32, vp]),
    "oxide_add_layer_norm_bf16": (i32, [vp, vp, vp, vp, vp, u64, u64, f32, vp]),
    "oxide_decode_weights_f32": (i32, [vp, u64, i32, vp, vp]),
    "oxide_decode_weights_bf16": (i32, [vp, u64, i32, vp, vp]),
    "oxide_repeat_kv_f32": (i32, [vp, vp, u64, u64, u64, u64, u64, vp]),
    "oxide_repeat_kv_bf16": (i32, [vp, vp, u64, u64, u64, u64, u64, vp]),
    "oxide_kv_cache_append_f32": (i32, [vp, vp, vp, vp, u64, u64, u64, u64, u64, u64, vp]),
    "oxide_kv_cache_append_bf16": (i32, [vp, vp, vp, vp, u64, u64, u64, u64, u64, u64, vp]),
    "oxide_decode_attention_workspace_bytes": (u64, [u64, u64, u64, u64]),
    "oxide_debug_decode_attention_path": (None, [i32]),
    "oxide_device_status": (i32, [i32, C.POINTER(C.c_uint32)]),
    "oxide_decode_attention_f32": (i32, [vp, vp, vp, vp, vp, u64, u64, u64, u64, u64, f32, vp, u64, vp]),
    "oxide_decode_attention_bf16": (i32, [vp, vp, vp, vp, vp, u64, u64, u64, u64, u64, f32, vp, u64, vp]),
    "oxide_sample_f32": (i32, [vp, u64, u64, f32, u64, f32, vp, vp, vp, vp]),
    "oxide_sample_bf16": (i32, [vp, u64, u64, f32, u64, f32, vp, vp, vp, vp]),
    "oxide_softmax_with_temperature_f32": (i32, [vp, vp, u64, u64, f32, vp]),
    "oxide_softmax_with_temperature_bf16": (i32, [vp, vp, u64, u64, f32, vp]),
    "oxide_reduce_rows_f32": (i32, [i32, vp, u64, u64, vp, vp]),
    "oxide_reduce_rows_bf16": (i32, [i32, vp, u64, u64, vp, vp]),
    "oxide_reduce_workspace_bytes": (u64, [u64]),
    "oxide_reduce_f32": (i32, [i32, vp, u64, vp, vp, u64, vp]),
    "oxide_reduce_bf16": (i32, [i32, vp, u64, vp, vp, u64, vp]),
    "oxide_reduce_static_f32": (i32, [i32, vp, u64, vp, vp]),
    "oxide_reduce_static_bf16": (i32, [i32, vp, u64, vp, vp]),
    "oxide_pipe_create": (i32, [i32, u64, i32, C.POINTER(C.c_void_p)]),
    "oxide_pipe_destroy": (i32, [vp]),
    "oxide_pipe_binary_f32": (i32, [vp, i32, vp, u64, vp, u64, vp, u64]),
    "oxide_pipe_silu_mul_f32": (i32, [vp, vp, vp, vp, u64]),
    "oxide_pipe_rms_norm_f32": (i32, [vp, vp, vp, vp, u64, u64, f32]),
    "oxide_pipe_defer": (i32, [vp, i32]),
    "oxide_pipe_sync": (i32, [vp]),
    "oxide_pipe_add_mul_rowbcast_f32": (i32, [vp, vp, vp, vp, vp, vp, u64, u64]),
    "oxide_pipe_add_rms_norm_f32": (i32, [vp, vp, vp, vp, vp, vp, u64, u64, f32]),
    "oxide_pipe_add_rms_norm_bf16": (i32, [vp, vp, vp, vp, vp, vp, u64, u64, f32]),
    "oxide_pipe_scale_mask_softmax_f32": (i32, [vp, vp, vp, u64, u64, f32, vp, u64, vp, u64, u64]),
    "oxide_pipe_argmax_rows_f32": (i32, [vp, vp, u64, u64, vp]),
    "oxide_pipe_rope_bf16": (i32, [vp, vp, vp, u64, vp, vp, u64, vp, vp, u64, vp, u64, u64]),
}

# Status codes (oxide_status in include/oxide_ops.h).
OK, ERR_INVALID_ARG, ERR_LAUNCH, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE, ERR_INJECTED, ERR_TIMEOUT = (
    0, -1, -2, -3, -4, -5, -6, -7)
ADD, SUB, MUL, DIV = 0, 1, 2, 3
RELU, GELU, GELU_QUICK, SIGMOID, TANH, EXP, LOG, SQRT, POW, CLAMP, NEG, ABS = range(12)
RED_SUM, RED_MAX, RED_SUMSQ = 0, 1, 2
SAMPLE_INVALID = 0xFFFFFFFF
DEVICE_WAIT_TIMEOUT = 1  # OXIDE_DEVICE_WAIT_TIMEOUT
WDT_F32, WDT_F16, WDT_BF16 = 0, 1, 2

_lock = threading.Lock()
_lib: C.CDLL | None = None


class OxideError(RuntimeError):
    """A non-zero oxide_status, with the library's message for this thread."""

    def __init__(self, status: int, op: str, message: str):
        super().__init__(f"{op}: {message} ({status_name(status)})")
        self.status = status
        self.op = op


def lib() -> C.CDLL:
    """Load liboxide_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"liboxide_b200.so not found at {LIB_PATH}: build it with "
                    "`make -C mistralrs-oxide_b200` (there is no fallback implementation)")
            handle = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_name(status: int) -> str:
    return lib().oxide_status_string(status).decode()


def last_error() -> str:
    return lib().oxide_last_error().decode()


def call(name: str, *args) -> int:
    """Call an entry point; raise OxideError on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        raise OxideError(rc, name, last_error())
    return rc


def raw(name: str, *args):
    """Call an entry point and return its raw result (no status check)."""
    return getattr(lib(), name)(*args)
