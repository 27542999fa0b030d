"""ctypes binding of ``libmodelc_cuda.so`` (the C ABI in include/modelc_cuda.h).

Loading fails loudly: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# MODELC_CUDA_LIB: another build of the library (a variant built with other
# compile-time settings); the in-tree build otherwise
LIB_PATH = os.environ.get("MODELC_CUDA_LIB") or os.path.join(HERE, "libmodelc_cuda.so")

MC_OK = 0
STATUS = {0: "MC_OK", -1: "MC_E_INVALID", -2: "MC_E_SHAPE", -3: "MC_E_DTYPE", -4: "MC_E_OOM",
          -5: "MC_E_CUDA", -6: "MC_E_NCCL", -7: "MC_E_TIMEOUT", -8: "MC_E_CANCELLED",
          -9: "MC_E_NO_HEAD", -10: "MC_E_CAPACITY"}

DTYPE_F32, DTYPE_I8_TENSOR, DTYPE_I8_ROW, DTYPE_Q4_0 = 0, 1, 2, 3
MEM_HOST, MEM_DEVICE = 0, 1
MODE_REFERENCE, MODE_GENERAL = 0, 1

# Every symbol include/modelc_cuda.h declares.
EXPORTS = [
    "mc_weights_load", "mc_weights_destroy", "mc_weights_bytes", "mc_session_create",
    "mc_session_destroy", "mc_forward", "mc_draft_forward", "mc_kv_len", "mc_kv_truncate",
    "mc_draft", "mc_speculative_generate", "mc_spec_prime", "mc_spec_decode", "mc_spec_read",
    "mc_linear_create", "mc_linear_destroy", "mc_linear_run", "mc_linear_weight_bytes",
    "mc_last_error", "mc_version", "mc_spec_rewind", "mc_spec_verify_launch",
    "mc_session_stream", "mc_session_round_launches", "mc_linear_run_static",
    "mc_spec_set_seed", "mc_tp_unique_id", "mc_session_tp_init", "mc_session_tp_ipc_handle",
    "mc_session_tp_open_peers", "mc_speculative_generate_batch", "mc_spec_prime_batch",
    "mc_spec_read_request", "mc_mlp_draft_create", "mc_mlp_draft", "mc_mlp_draft_destroy",
    "mc_ngram_draft_create", "mc_ngram_draft", "mc_ngram_draft_destroy", "mc_sample_rows",
    "mc_session_set_wait_timeout", "mc_session_create_mlp", "mc_kv_snapshot_take",
    "mc_kv_snapshot_tokens", "mc_kv_snapshot_destroy", "mc_spec_prime_cached",
]


class McError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class ModelCfg(C.Structure):
    _fields_ = [("mode", C.c_int32), ("n_layers", C.c_int32), ("hidden", C.c_int32),
                ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("ffn", C.c_int32), ("vocab", C.c_int32), ("rope_theta", C.c_float),
                ("eps", C.c_float), ("tp_rank", C.c_int32), ("tp_world", C.c_int32)]


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int32), ("location", C.c_int32),
                ("ndim", C.c_int32), ("shape", C.c_int64 * 2), ("data", C.c_void_p),
                ("scales", C.c_void_p)]


class SpecCfg(C.Structure):
    _fields_ = [("gamma", C.c_int32), ("max_context", C.c_int32), ("bonus", C.c_int32),
                ("temperature", C.c_float), ("seed", C.c_uint64),
                ("cancel", C.POINTER(C.c_int32)), ("accept_mode", C.c_int32),
                ("n_requests", C.c_int32), ("top_p", C.c_float), ("min_p", C.c_float),
                ("shift_context", C.c_int32), ("anchor_tokens", C.c_int32),
                ("kv_mode", C.c_int32)]


_lib = None


def use_trace_library() -> None:
    """Load the MC_TRACE build (libmodelc_cuda_trace.so, built on demand)
    instead of the product library; must precede the first lib() call."""
    global LIB_PATH
    if _lib is not None:
        raise RuntimeError("the CUDA library is already loaded")
    from . import build as _build
    LIB_PATH = _build.build(trace=True)


def lib():
    """Load the CUDA library (building it first if the sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    from . import build as _build
    if LIB_PATH == _build.LIB and (not os.path.exists(LIB_PATH) or _build._stale()):
        _build.build()
    L = C.CDLL(LIB_PATH)
    if hasattr(L, "mc_trace_reset"):  # MC_TRACE builds only
        L.mc_trace_reset.restype = C.c_int32
        L.mc_trace_reset.argtypes = []
        L.mc_trace_read.restype = C.c_int32
        L.mc_trace_read.argtypes = [C.POINTER(C.c_ulonglong), C.c_int32]
    vp, i32, i64, u32p = C.c_void_p, C.c_int32, C.c_int64, C.POINTER(C.c_uint32)
    i32p, fp = C.POINTER(C.c_int32), C.POINTER(C.c_float)
    sig = {
        "mc_weights_load": (i32, [C.POINTER(TensorDesc), C.c_size_t, C.POINTER(ModelCfg), i32,
                                  C.POINTER(vp)]),
        "mc_weights_destroy": (i32, [vp]),
        "mc_weights_bytes": (i64, [vp]),
        "mc_session_create": (i32, [vp, vp, C.POINTER(SpecCfg), C.POINTER(vp)]),
        "mc_session_create_mlp": (i32, [vp, vp, C.POINTER(SpecCfg), C.POINTER(vp)]),
        "mc_session_destroy": (i32, [vp]),
        "mc_forward": (i32, [vp, u32p, i32, fp]),
        "mc_draft_forward": (i32, [vp, u32p, i32, fp]),
        "mc_kv_len": (i32, [vp]),
        "mc_kv_truncate": (i32, [vp, i32]),
        "mc_draft": (i32, [vp, u32p, i32, i32, u32p, i32p]),
        "mc_speculative_generate": (i32, [vp, u32p, i32, i32, u32p, i32, i32p, i32p, i32, i32p]),
        "mc_spec_prime": (i32, [vp, u32p, i32]),
        "mc_kv_snapshot_take": (i32, [vp, i32, C.POINTER(vp)]),
        "mc_kv_snapshot_tokens": (i32, [vp, u32p, i32]),
        "mc_kv_snapshot_destroy": (i32, [vp]),
        "mc_spec_prime_cached": (i32, [vp, vp, u32p, i32]),
        "mc_spec_decode": (i32, [vp, i32, i32p]),
        "mc_spec_read": (i32, [vp, u32p, i32, i32p, i32p, i32, i32p]),
        "mc_linear_create": (i32, [C.POINTER(TensorDesc), i32, C.POINTER(vp)]),
        "mc_linear_destroy": (i32, [vp]),
        "mc_linear_run": (i32, [vp, vp, i32, vp, vp]),
        "mc_linear_weight_bytes": (i64, [vp]),
        "mc_linear_run_static": (i32, [vp, vp, i32, vp, vp]),
        "mc_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
        "mc_spec_rewind": (i32, [vp]),
        "mc_spec_verify_launch": (i32, [vp, i32]),
        "mc_spec_set_seed": (i32, [vp, C.c_uint64]),
        "mc_tp_unique_id": (i32, [C.c_char_p]),
        "mc_session_tp_init": (i32, [vp, C.c_char_p, i32, i32]),
        "mc_session_tp_ipc_handle": (i32, [vp, C.c_char_p]),
        "mc_session_tp_open_peers": (i32, [vp, C.c_char_p]),
        "mc_session_set_wait_timeout": (i32, [vp, i32]),
        "mc_speculative_generate_batch": (i32, [vp, u32p, i32p, i32, i32, u32p, i32, i32p, i32p,
                                                i32, i32p]),
        "mc_spec_prime_batch": (i32, [vp, u32p, i32p, i32]),
        "mc_spec_read_request": (i32, [vp, i32, u32p, i32, i32p, i32p, i32, i32p]),
        "mc_mlp_draft_create": (i32, [C.POINTER(TensorDesc), C.c_size_t, i32, C.POINTER(vp)]),
        "mc_mlp_draft": (i32, [vp, u32p, i32, i32, u32p, i32p]),
        "mc_mlp_draft_destroy": (i32, [vp]),
        "mc_ngram_draft_create": (i32, [i32, i32, i32, C.POINTER(vp)]),
        "mc_ngram_draft": (i32, [vp, u32p, i32, i32, u32p, i32p]),
        "mc_ngram_draft_destroy": (i32, [vp]),
        "mc_sample_rows": (i32, [vp, i32, i32, C.c_float, C.c_float, C.c_float, C.c_uint64,
                                 C.c_uint32, vp, vp]),
        "mc_session_stream": (vp, [vp]),
        "mc_session_round_launches": (i32, [vp]),
        "mc_version": (C.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    lib().mc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != MC_OK:
        raise McError(status, last_error())
