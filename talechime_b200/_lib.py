"""ctypes binding of libq8lin.so (the C ABI declared in include/q8lin.h).

The library is loaded from the package directory only.  There is no fallback: if
it is missing, importing the operator fails with instructions to build it.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libq8lin.so")

# Status codes (enum q8lin_status).
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_SHAPE = 2
ERR_ALIGNMENT = 3
ERR_CUDA = 4
ERR_NCCL = 5
ERR_OUT_OF_MEMORY = 6
ERR_DEVICE = 7
ERR_WORKSPACE = 8
ERR_FORMAT = 9
ERR_IO = 10
ERR_NOT_FOUND = 11

# q8lin_dispatch_path results (enum q8lin_path)
PATH_STREAM_GEMV = 0
PATH_GEMV = 1
PATH_SMALL_BATCH = 2
PATH_INT8_TC = 3
PATH_F16_TC = 4
PATH_SMALL_BATCH_TC = 5
PATH_NAMES = {PATH_STREAM_GEMV: "stream_gemv", PATH_GEMV: "gemv", PATH_SMALL_BATCH: "small_batch_dp4a",
              PATH_INT8_TC: "int8_tc", PATH_F16_TC: "f16_tc", PATH_SMALL_BATCH_TC: "small_batch_mma"}


class Op(ctypes.Structure):
    """struct q8lin_op (one operation of a persistent decode step)."""
    _fields_ = [("kind", ctypes.c_int32), ("prologue", ctypes.c_int32), ("epilogue", ctypes.c_int32),
                ("argmax", ctypes.c_int32), ("weight", ctypes.c_void_p), ("x", ctypes.c_void_p),
                ("y", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("norm_weight", ctypes.c_void_p),
                ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p), ("cos_t", ctypes.c_void_p),
                ("sin_t", ctypes.c_void_p), ("eps", ctypes.c_float), ("hq", ctypes.c_int32),
                ("hkv", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("max_t", ctypes.c_int32)]


OP_GEMV, OP_ATTENTION, OP_EMBED, OP_ARGMAX = 0, 1, 2, 3
PROLOGUE_NONE, PROLOGUE_RMSNORM, PROLOGUE_SWIGLU = 0, 1, 2
EPILOGUE_NONE, EPILOGUE_SWIGLU = 0, 1

# Every symbol the header declares, with (restype, argtypes).
_c_p = ctypes.c_void_p
_i64 = ctypes.c_int64
SIGNATURES = {
    "q8lin_version": (ctypes.c_int, []),
    "q8lin_last_error": (ctypes.c_char_p, []),
    "q8lin_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "q8lin_weight_create": (ctypes.c_int, [_c_p, _i64, _i64, ctypes.c_int, _c_p, ctypes.POINTER(_c_p)]),
    "q8lin_weight_destroy": (ctypes.c_int, [_c_p]),
    "q8lin_weight_shape": (ctypes.c_int, [_c_p, ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                                          ctypes.POINTER(ctypes.c_int)]),
    "q8lin_weight_device_bytes": (ctypes.c_int, [_c_p, ctypes.POINTER(ctypes.c_size_t)]),
    "q8lin_weight_dequantize": (ctypes.c_int, [_c_p, _c_p, _c_p]),
    "q8lin_weight_export_gguf": (ctypes.c_int, [_c_p, _c_p, _c_p]),
    "q8lin_workspace_size": (ctypes.c_size_t, [_c_p, _i64]),
    "q8lin_dispatch_path": (ctypes.c_int, [_i64, _i64, _i64]),
    "q8lin_forward": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, _c_p]),
    "q8lin_forward_ws": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, _c_p, ctypes.c_size_t, _c_p]),
    "q8lin_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "q8lin_workspace_create": (ctypes.c_int, [ctypes.c_int, _i64, _i64, ctypes.POINTER(_c_p)]),
    "q8lin_workspace_destroy": (ctypes.c_int, [_c_p]),
    "q8lin_workspace_capacity": (ctypes.c_int, [_c_p, ctypes.POINTER(ctypes.c_size_t)]),
    "q8lin_weight_bind_workspace": (ctypes.c_int, [_c_p, _c_p]),
    "q8lin_set_wait_limit_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "q8lin_wait_limit_ns": (ctypes.c_uint64, []),
    "q8lin_quantize_rows": (ctypes.c_int, [_c_p, _i64, _i64, _c_p, _c_p, _c_p]),
    "q8lin_forward_noalloc": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, _c_p]),
    "q8lin_fault_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
    "q8lin_swiglu": (ctypes.c_int, [_c_p, _i64, _i64, _c_p, _c_p]),
    "q8lin_forward_fused": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, ctypes.c_int32, _c_p, ctypes.c_float, _c_p,
                                           _c_p]),
    "q8lin_embed_rows": (ctypes.c_int, [_c_p, _c_p, _i64, _c_p, _c_p]),
    "q8lin_rmsnorm": (ctypes.c_int, [_c_p, _c_p, _i64, _i64, ctypes.c_float, _c_p, _c_p]),
    "q8lin_rope_kv": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_int32, ctypes.c_int32, _c_p, _c_p]),
    "q8lin_attention_workspace_size": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    "q8lin_attention_decode": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, _c_p, ctypes.c_size_t, _c_p, _c_p]),
    "q8lin_rope_attention_decode": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, ctypes.c_int32, ctypes.c_int32,
                                                   ctypes.c_int32, ctypes.c_int32, _c_p, _c_p]),
    "q8lin_rope_attention_decode_ex": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, ctypes.c_int32,
                                                      ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _c_p,
                                                      ctypes.c_uint32, _c_p]),
    "q8lin_add": (ctypes.c_int, [_c_p, _c_p, _i64, _c_p]),
    "q8lin_add_rmsnorm": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, _i64, ctypes.c_float, _c_p, _c_p]),
    "q8lin_rope_kv_rows": (ctypes.c_int, [_c_p, ctypes.c_int32, _i64, ctypes.c_int32, _c_p, _c_p, _c_p, _c_p,
                                          ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _c_p,
                                          _c_p]),
    "q8lin_attention_prefill": (ctypes.c_int, [_c_p, _c_p, _c_p, ctypes.c_int32, _i64, ctypes.c_int32,
                                               ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _c_p,
                                               _c_p]),
    "q8lin_peer_alloc": (ctypes.c_int, [ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(_c_p), _c_p]),
    "q8lin_peer_open": (ctypes.c_int, [ctypes.c_int, _c_p, ctypes.POINTER(_c_p)]),
    "q8lin_peer_close": (ctypes.c_int, [ctypes.c_int, _c_p]),
    "q8lin_peer_free": (ctypes.c_int, [ctypes.c_int, _c_p]),
    "q8lin_allreduce_stage_bytes": (ctypes.c_size_t, [_i64, ctypes.c_int32]),
    "q8lin_allreduce_flag_bytes": (ctypes.c_size_t, [ctypes.c_int32]),
    "q8lin_forward_allreduce": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, _c_p, _c_p, _i64, ctypes.c_int32,
                                                ctypes.c_int32, ctypes.c_uint32, _c_p, _c_p]),
    "q8lin_mlp_tp_create": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, _i64, ctypes.c_int32, ctypes.c_int32, _c_p,
                                           ctypes.c_int, _i64, ctypes.c_uint32, _c_p, ctypes.POINTER(_c_p)]),
    "q8lin_mlp_tp_peer_handle": (ctypes.c_int, [_c_p, _c_p]),
    "q8lin_mlp_tp_connect_peers": (ctypes.c_int, [_c_p, _c_p]),
    "q8lin_mlp_tp_forward": (ctypes.c_int, [_c_p, _c_p, _c_p, _i64, _c_p]),
    "q8lin_mlp_tp_close_peers": (ctypes.c_int, [_c_p]),
    "q8lin_mlp_tp_destroy": (ctypes.c_int, [_c_p]),
    "q8lin_mlp_tp_info": (ctypes.c_int, [_c_p, ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_int32)]),
    "q8lin_mlp_tp_shard": (ctypes.c_int, [_i64, _i64, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(_i64),
                                          ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "q8lin_nccl_available": (ctypes.c_int, []),
    "q8lin_step_create": (ctypes.c_int, [ctypes.POINTER(Op), ctypes.c_int32, _c_p, _c_p, ctypes.c_int,
                                         ctypes.POINTER(_c_p)]),
    "q8lin_step_run": (ctypes.c_int, [_c_p, _c_p]),
    "q8lin_step_destroy": (ctypes.c_int, [_c_p]),
    "q8lin_gguf_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_c_p)]),
    "q8lin_gguf_close": (ctypes.c_int, [_c_p]),
    "q8lin_gguf_version": (ctypes.c_int, [_c_p, ctypes.POINTER(ctypes.c_uint32)]),
    "q8lin_gguf_tensor_count": (_i64, [_c_p]),
    "q8lin_gguf_metadata_count": (_i64, [_c_p]),
    "q8lin_gguf_find_tensor": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "q8lin_gguf_tensor_info": (ctypes.c_int, [_c_p, _i64, ctypes.POINTER(ctypes.c_char_p),
                                              ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32),
                                              ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_uint64)]),
    "q8lin_gguf_tensor_data": (ctypes.c_int, [_c_p, _i64, ctypes.POINTER(_c_p), ctypes.POINTER(ctypes.c_uint64)]),
    "q8lin_gguf_metadata_type": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32)]),
    "q8lin_gguf_metadata_u32": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32)]),
    "q8lin_gguf_metadata_i64": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "q8lin_gguf_metadata_f64": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    "q8lin_gguf_metadata_string": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.POINTER(_c_p),
                                                  ctypes.POINTER(ctypes.c_uint64)]),
    "q8lin_gguf_metadata_array": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                                                 ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_c_p),
                                                 ctypes.POINTER(ctypes.c_uint64)]),
    "q8lin_gguf_weight_create": (ctypes.c_int, [_c_p, ctypes.c_char_p, ctypes.c_int, _c_p, ctypes.POINTER(_c_p)]),
    "q8lin_argmax_workspace_size": (ctypes.c_size_t, []),
    "q8lin_argmax": (ctypes.c_int, [_c_p, _i64, _c_p, ctypes.c_size_t, _c_p, _c_p, _c_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class Q8LinError(RuntimeError):
    """A libq8lin call returned a non-zero status (mirrors candle's Error::Msg)."""

    def __init__(self, status: int, message: str):
        self.status = status
        name = _status_name(status)
        super().__init__(f"{name}: {message}")


def _status_name(status: int) -> str:
    try:
        return lib().q8lin_status_string(status).decode()
    except Exception:  # library unusable: fall back to the number
        return f"status {status}"


def lib() -> ctypes.CDLL:
    """Load libq8lin.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m talechime_b200.build` "
                    "(nvcc, sm_100a).  There is no CPU fallback for the Q8_0 linear.")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().q8lin_last_error().decode(errors="replace")
        raise Q8LinError(status, msg)
