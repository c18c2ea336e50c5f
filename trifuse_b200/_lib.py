"""ctypes binding of libtrifuse_b200.so (the C ABI in include/trifuse_b200.h).

The shared library is built in-tree by ``trifuse_b200.build``; importing this
module never falls back to anything else: a missing or unloadable library is
an ImportError-style failure at first use.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libtrifuse_b200.so"

TF_OK = 0
STATUS = {0: "TF_OK", 1: "TF_ERR_INVALID_ARGUMENT", 2: "TF_ERR_SHAPE", 3: "TF_ERR_OUT_OF_MEMORY",
          4: "TF_ERR_CUDA", 5: "TF_ERR_NCCL", 6: "TF_ERR_TIMEOUT", 7: "TF_ERR_CANCELLED",
          8: "TF_ERR_UNSUPPORTED", 9: "TF_ERR_STATE", 10: "TF_ERR_CAPACITY"}
DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 1, 2, 3
HOST_INPUTS, HOST_OUTPUT = 1, 2


class AffineWeight(C.Structure):
    _fields_ = [("q", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("experts", C.c_int32), ("out_features", C.c_int32), ("in_features", C.c_int32),
                ("group_size", C.c_int32), ("bits", C.c_int32)]


class RouterWeight(C.Structure):
    _fields_ = [("dense", C.c_void_p), ("affine", AffineWeight)]


class MoeArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("residual", C.c_void_p), ("out", C.c_void_p),
                ("tokens", C.c_int64), ("hidden", C.c_int32), ("intermediate", C.c_int32),
                ("experts", C.c_int32), ("top_k", C.c_int32), ("act", C.c_int32),
                ("router", RouterWeight), ("gate_proj", AffineWeight), ("up_proj", AffineWeight),
                ("down_proj", AffineWeight), ("logits", C.c_void_p), ("indices", C.c_void_p),
                ("gates", C.c_void_p)]


class OLMoEConfig(C.Structure):
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("heads", C.c_int32),
                ("kv_heads", C.c_int32), ("head_dim", C.c_int32), ("intermediate", C.c_int32),
                ("vocab", C.c_int32), ("experts", C.c_int32), ("top_k", C.c_int32),
                ("capacity", C.c_int32), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("act", C.c_int32)]


P = C.c_void_p
I32, I64, F32, SZ = C.c_int32, C.c_int64, C.c_float, C.c_size_t
PSZ = C.POINTER(C.c_size_t)

# name -> argtypes (restype is int status unless noted); must match the header.
SIGNATURES = {
    "tf_abi_version": [],
    "tf_last_error": [],
    "tf_status_name": [C.c_int],
    "tf_device_check": [C.c_int],
    "tf_rms_norm": [P, I64, I32, P, F32, C.c_int, P, P],
    "tf_affine_qmm": [P, I64, C.POINTER(AffineWeight), C.c_int, P, P],
    "tf_affine_gather_qmm": [P, I64, I32, P, P, I64, C.POINTER(AffineWeight), C.c_int, C.c_int, P, P],
    "tf_affine_embedding": [P, I64, C.POINTER(AffineWeight), C.c_int, P, P],
    "tf_greedy_tokens": [P, I64, I64, P, P],
    "tf_moe_combine": [P, P, P, P, I64, I32, I32, C.c_int, P, P],
    "tf_olmoe_softmax": [P, I64, I32, C.c_int, P, P],
    "tf_olmoe_topk_indices": [P, I64, I32, I32, C.c_int, P, P],
    "tf_take_along_last": [P, I64, I32, P, I32, C.c_int, P, P],
    "tf_olmoe_route": [P, I64, I32, I32, C.c_int, P, P, P],
    "tf_olmoe_router": [P, I64, I32, C.POINTER(RouterWeight), I32, I32, C.c_int, P, P, P, P],
    "tf_moe_route_sort_workspace_size": [I64, I32, I32, PSZ],
    "tf_moe_route_sort": [P, I64, I32, I32, P, P, P, P, SZ, P],
    "tf_moe_workspace_size": [C.POINTER(MoeArgs), PSZ],
    "tf_moe_forward": [C.POINTER(MoeArgs), P, SZ, P],
    "tf_moe_forward_noalloc": [C.POINTER(MoeArgs), P],
    "tf_moe_expert_workspace_size": [I64, I64, I32, I32, I32, C.c_int, PSZ],
    "tf_moe_expert_gpu": [P, I64, I32, P, P, I64, C.c_int, I32, I32, C.POINTER(AffineWeight),
                          C.POINTER(AffineWeight), C.POINTER(AffineWeight), C.c_int, P, P, P, SZ, P],
    "tf_attention_decode_workspace_size": [I32, I32, I32, PSZ],
    "tf_attention_decode": [P, I32, I32, I32, P, P, F32, F32, P, I32, P, P, I32, F32, C.c_int, P, P,
                            SZ, P],
    "tf_model_create": [C.POINTER(OLMoEConfig), C.c_int, C.POINTER(P)],
    "tf_model_bind": [P, C.c_char_p, P, SZ, C.c_int],
    "tf_model_finalize": [P],
    "tf_model_destroy": [P],
    "tf_session_create": [P, I32, I32, I32, C.POINTER(P)],
    "tf_session_destroy": [P],
    "tf_session_kv": [P, I32, C.POINTER(P), C.POINTER(P)],
    "tf_session_set_lengths": [P, P, I32],
    "tf_session_get_lengths": [P, P, I32],
    "tf_session_decode": [P, P, P, I32, P, C.c_int, P],
    "tf_session_decode_greedy": [P, P, P, I32, P, P, C.c_int, P],
    "tf_session_prefill_chunked": [P, I32, P, I64, I32, P, C.c_int, P],
    "tf_session_graphs": [P, C.c_int],
    "tf_session_prefill": [P, P, P, I32, P, P, C.c_int, P],
    "tf_session_cancel": [P],
    "tf_launch_count": [],
    "tf_set_qmm_path": [C.c_int],
    "tf_device_error": [C.c_int],
    "tf_trace_phases": [],
    "tf_trace_phase_name": [C.c_int],
    "tf_session_trace": [P, C.c_int],
    "tf_session_trace_read": [P, C.POINTER(C.c_float), C.POINTER(C.c_int32)],
    "tf_session_reset": [P],
    "tf_session_check": [P, P],
    "tf_moe_expert_gpu_ordered": [P, C.c_int64, C.c_int32, P, P, C.c_int64, C.c_int32, C.c_int32,
                                  C.POINTER(AffineWeight), C.POINTER(AffineWeight), C.POINTER(AffineWeight), C.c_int,
                                  P, P, C.c_size_t, P],
    "tf_gather_rows": [P, C.c_int64, C.c_int32, P, C.c_int32, C.c_int64, C.c_int, P, P],
    "tf_session_capture": [P, P, P, C.c_int64],
    "tf_set_wait_limit": [C.c_int64],
}

_lib = None
_lock = threading.Lock()


class TriFuseError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


def lib():
    """Load the library once; raises if it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(f"{LIB_PATH} is missing; build it with `python -m trifuse_b200.build`")
            L = C.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = C.c_int
            L.tf_last_error.restype = C.c_char_p
            L.tf_status_name.restype = C.c_char_p
            L.tf_trace_phase_name.restype = C.c_char_p
            L.tf_launch_count.restype = C.c_uint64
            _lib = L
    return _lib


def check(status):
    if status != TF_OK:
        msg = lib().tf_last_error().decode(errors="replace")
        if status in (1, 2):
            raise ValueError(msg)
        raise TriFuseError(status, msg)
    return status
