"""ctypes binding of libdrift_cuda.so, the library's C ABI (include/drift_*.h).

Loads the in-tree library and nothing else: if it is missing, importing the
ops raises with the command that builds it. There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os

PACKAGE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(PACKAGE, "libdrift_cuda.so")

DRIFT_ERROR_INVALID_ARGUMENT = 1001
DRIFT_ERROR_TIMEOUT = 1002

# Storage types: GGML type ids (runner/src/drift/runner/tensor/DType.scala:151-175).
F32, F16, Q4_0, Q4_1, Q8_0, I32, BF16 = 0, 1, 2, 3, 8, 26, 30
Q4_K, Q6_K = 12, 14  # the K-quants (tensor/KQuants.scala:99, 122)

_p, _i32, _i64, _f32, _sz = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                             ctypes.c_size_t)
_pp = ctypes.POINTER(ctypes.c_void_p)

# name: (restype, argtypes) of every function include/drift_runtime.h and
# include/drift_ops.h declare.
SIGNATURES = {
    # drift_runtime.h
    "drift_init": (_i32, [_i32]),
    "drift_set_device": (_i32, [_i32]),
    "drift_get_device": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "drift_get_device_count": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "drift_set_device_flags": (_i32, [_i32]),
    "drift_device_get_name": (_i32, [ctypes.c_char_p, _i32, _i32]),
    "drift_device_synchronize": (_i32, []),
    "drift_mem_get_info": (_i32, [ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "drift_get_error_string": (ctypes.c_char_p, [_i32]),
    "drift_last_error_message": (ctypes.c_char_p, []),
    "drift_malloc": (_i32, [_pp, _sz]),
    "drift_free": (_i32, [_p]),
    "drift_memset": (_i32, [_p, _i32, _sz]),
    "drift_memcpy": (_i32, [_p, _p, _sz, _i32]),
    "drift_memcpy_async": (_i32, [_p, _p, _sz, _i32, _p]),
    "drift_host_register": (_i32, [_p, _sz, _i32]),
    "drift_host_unregister": (_i32, [_p]),
    "drift_host_get_device_pointer": (_i32, [_pp, _p, _i32]),
    "drift_stream_create": (_i32, [_pp]),
    "drift_stream_destroy": (_i32, [_p]),
    "drift_stream_synchronize": (_i32, [_p]),
    "drift_event_create": (_i32, [_pp]),
    "drift_event_destroy": (_i32, [_p]),
    "drift_event_record": (_i32, [_p, _p]),
    "drift_stream_wait_event": (_i32, [_p, _p]),
    "drift_event_synchronize": (_i32, [_p]),
    "drift_event_elapsed_time": (_i32, [ctypes.POINTER(ctypes.c_float), _p, _p]),
    "drift_module_load_data": (_i32, [_pp, _p]),
    "drift_module_unload": (_i32, [_p]),
    "drift_module_get_function": (_i32, [_pp, _p, ctypes.c_char_p]),
    "drift_module_launch_kernel": (_i32, [_p, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint,
                                          ctypes.c_uint, ctypes.c_uint, ctypes.c_uint,
                                          ctypes.c_uint, _p, _pp, _pp]),
    "drift_kernel_count": (_i32, []),
    "drift_kernel_name": (ctypes.c_char_p, [_i32]),
    # drift_ops.h
    "drift_linear": (_i32, [_i32, _p, _i32, _p, _p, _i64, _i64, _i64, _p]),
    "drift_linears": (_i32, [_i32, _p, _i32, _p, _p, _p, _p, _i64, _i64, _p]),
    "drift_embedding": (_i32, [_i32, _p, _i64, _i64, _p, _i64, _p, _p]),
    "drift_rms_norm": (_i32, [_p, _p, _f32, _f32, _p, _i64, _i64, _p]),
    "drift_add_rms_norm": (_i32, [_p, _p, _p, _f32, _f32, _p, _i64, _i64, _p]),
    "drift_add": (_i32, [_p, _p, _p, _i64, _p]),
    "drift_gated": (_i32, [_i32, _p, _p, _p, _i64, _p]),
    "drift_prepared_x_bytes": (_sz, [_i64, _i64]),
    "drift_causal_conv": (_i32, [_p, _i32, _i32, _p, _i32, _i32, _p, _p, _p, _p]),
    "drift_gated_delta_rule": (_i32, [_p, _i32, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p,
                                      _p]),
    "drift_delta_decode_step": (_i32, [_p, _p, _i32, _i32, _i32, _i32, _i32, _p, _i32, _p, _p, _p,
                                        _p, _p, _p, _p, _p, _f32, _p, _p, _p]),
    "drift_gated_rms_norm": (_i32, [_p, _p, _p, _i32, _f32, _p, _i64, _i64, _i32, _p, _p]),
    "drift_causal_conv_decode": (_i32, [_p, _i32, _i32, _p, _i32, _i32, _p, _p, _p]),
    "drift_gated_delta_rule_decode": (_i32, [_p, _i32, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _p,
                                             _p, _p]),
    "drift_attention_inputs_decode_split": (_i32, [_p, _p, _p, _i32, _i32, _i32, _i32, _p, _p, _f32,
                                                   _f32, _p, _f32, _i32, _i32, _p, _p, _p, _i32,
                                                   _i32, _p, _i32, _p]),
    "drift_attention_decode_gated": (_i32, [_p, _i32, _i32, _p, _p, _i32, _i32, _i32, _i32, _p, _i32,
                                            _p, _i32, _f32, _i32, _f32, _p, _p, _p, _i32, _p, _p]),
    "drift_comm_handle_bytes": (_sz, []),
    "drift_comm_create": (_i32, [_i32, _i32, _sz, _i64, _pp, _p]),
    "drift_comm_open": (_i32, [_p, _p]),
    "drift_comm_slot": (_i32, [_p, _i32, _pp]),
    "drift_comm_destroy": (_i32, [_p]),
    "drift_add_rms_norm_allreduce": (_i32, [_p, _i32, _p, _p, _f32, _f32, _p, _i64, _i64, _p, _p]),
    "drift_add_rms_norm_prepared": (_i32, [_p, _p, _p, _f32, _f32, _p, _i64, _i64, _p, _p]),
    "drift_gated_prepared": (_i32, [_i32, _p, _p, _p, _i64, _i64, _p, _p]),
    "drift_linears_prepared": (_i32, [_i32, _p, _p, _i32, _p, _p, _p, _p, _i64, _i64, _p]),
    "drift_attention_decode_prepared": (_i32, [_p, _i32, _i32, _p, _p, _i32, _i32, _i32, _i32, _p,
                                               _i32, _p, _i32, _f32, _i32, _f32, _p, _p, _p, _p]),
    "drift_rope": (_i32, [_p, _p, _p, _i32, _i32, _i32, _f32, _i32, _i32, _p]),
    "drift_route": (_i32, [_p, _p, _p, _i32, _i32, _i32, _p]),
    "drift_argmax": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p]),
    "drift_argmax_merge": (_i32, [_p, _p, _i64, _i64, _p, _p, _p]),
    "drift_candidates": (_i32, [_p, _i64, _i64, _i64, _i32, _p, _p, _p]),
    "drift_candidates_workspace_bytes": (_sz, [_i64, _i64, _i32]),
    "drift_candidates_merge": (_i32, [_p, _p, _i64, _i64, _i32, _p, _p, _p]),
    "drift_experts_linear_local": (_i32, [_i32, _p, _i64, _i32, _p, _i64, _i64, _i64, _i64, _p,
                                          _i64, _p, _p, _p]),
    "drift_experts_gated_linear_local": (_i32, [_i32, _p, _i64, _i32, _p, _p, _i64, _i64, _i64,
                                                _i64, _p, _i64, _p, _p, _i32, _p]),
    "drift_experts_linear": (_i32, [_i32, _p, _i64, _i32, _p, _i64, _i64, _i64, _p, _i64, _p,
                                    _p]),
    "drift_experts_gated_linear": (_i32, [_i32, _p, _i64, _i32, _p, _p, _i64, _i64, _i64, _p,
                                          _i64, _p, _p]),
    "drift_moe_combine": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p]),
    "drift_moe_combine_norm": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _f32, _f32,
                                      _p, _p]),
    "drift_moe_decode": (_i32, [_i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                _f32, _f32, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "drift_moe_combine_norm_prepared": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _f32,
                                               _f32, _p, _p, _p]),
    "drift_workspace_reserve": (_i32, [_sz]),
    "drift_linear_workspace_bytes": (_sz, [_i64, _i64]),
    "drift_attention_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "drift_device_error_take": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "drift_linear_static": (_i32, [_i32, _p, _i32, _p, _p, _i64, _i64, _i64, _p]),
    "drift_cache_write": (_i32, [_p, _p, _i32, _i32, _i32, _p, _p, _i32, _i32, _p, _i32, _i32, _p]),
    "drift_attention": (_i32, [_p, _i32, _i32, _p, _p, _i32, _i32, _i32, _i32, _p, _i32, _i32, _i32,
                               _f32, _i32, _i32, _f32, _p, _p, _p]),
    "drift_attention_inputs_decode": (_i32, [_p, _p, _p, _i32, _i32, _i32, _i32, _p, _p, _f32, _f32,
                                             _p, _f32, _i32, _i32, _p, _p, _p, _i32, _i32, _p, _i32,
                                             _p]),
    "drift_attention_decode": (_i32, [_p, _i32, _i32, _p, _p, _i32, _i32, _i32, _i32, _p, _i32, _p,
                                      _i32, _f32, _i32, _f32, _p, _p, _p]),
}


class DriftError(RuntimeError):
    """A CUDA failure inside the library (the reference's HipException:
    runner/src/drift/runner/native/HipRuntime.scala:8-9)."""

    def __init__(self, call: str, code: int, message: str):
        super().__init__(f"{call} failed with CUDA error {code}: {message}")
        self.call, self.code = call, code


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library; raises if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIBRARY):
        raise ImportError(
            f"{LIBRARY} is not built: run `python -m drift_b200.build` (nvcc, sm_100a). "
            "drift_b200 has no CPU fallback.")
    lib = ctypes.CDLL(LIBRARY)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def check(call: str, status: int) -> None:
    """Raises for a nonzero status: ValueError for a refused argument (as the
    reference's `require` throws IllegalArgumentException), DriftError for a
    CUDA failure."""
    if status == 0:
        return
    lib = load()
    message = (lib.drift_last_error_message() or b"").decode(errors="replace")
    if status == DRIFT_ERROR_INVALID_ARGUMENT:
        raise ValueError(message)
    if not message:
        message = (lib.drift_get_error_string(status) or b"").decode(errors="replace")
    raise DriftError(call, status, message)
