"""ctypes binding of libbell_b200.so (declarations in include/bell.h).

The library is built in-tree (``csrc/build_lib.py``) for sm_100a.  There is no
CPU fallback: if the library is missing, loading raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libbell_b200.so")

BELL_OK = 0
BELL_TILE_IN_OUT = 0
BELL_TILE_OUT_IN = 1
BELL_DTYPE_BF16 = 0
BELL_DTYPE_F32 = 1
BELL_STATUS_COLIDX = 1
BELL_STATUS_TIMEOUT = 2

ERRORS = {-1: "DTYPE", -2: "SHAPE", -3: "ALIGN", -4: "ARCH", -5: "LAUNCH", -6: "TIMEOUT", -7: "COLIDX", -8: "ARG"}


class BellEll(C.Structure):
    _fields_ = [("values", C.c_void_p), ("col_indices", C.c_void_p), ("R", C.c_int32), ("C", C.c_int32),
                ("K", C.c_int32), ("B", C.c_int32), ("layout", C.c_int32), ("flags", C.c_int32)]


BELL_ELL_SAME_COLS_AS_UP = 1


class BellFFNDesc(C.Structure):
    _fields_ = [("T", C.c_int64), ("d_model", C.c_int32), ("d_ff", C.c_int32), ("dtype", C.c_int32),
                ("add_residual", C.c_int32), ("x", C.c_void_p), ("residual", C.c_void_p), ("h", C.c_void_p),
                ("gate_pre", C.c_void_p), ("up_out", C.c_void_p), ("out", C.c_void_p), ("plan", C.c_void_p),
                ("gate", BellEll), ("up", BellEll), ("down", BellEll), ("status", C.c_void_p),
                ("max_ctas", C.c_int32), ("reserved", C.c_int32)]


class BellLinearDesc(C.Structure):
    _fields_ = [("T", C.c_int64), ("dtype", C.c_int32), ("out_dtype", C.c_int32), ("add_residual", C.c_int32),
                ("max_ctas", C.c_int32), ("x", C.c_void_p), ("residual", C.c_void_p), ("out", C.c_void_p),
                ("plan", C.c_void_p), ("w", BellEll), ("status", C.c_void_p), ("residual_row_lo", C.c_int64),
                ("residual_row_hi", C.c_int64)]


class BellTernaryEll(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("col_indices", C.c_void_p), ("R", C.c_int32),
                ("C", C.c_int32), ("K", C.c_int32), ("B", C.c_int32)]


class BellTernaryFFNDesc(C.Structure):
    _fields_ = [("T", C.c_int64), ("d_model", C.c_int32), ("d_ff", C.c_int32), ("add_residual", C.c_int32),
                ("reserved", C.c_int32), ("x", C.c_void_p), ("q_x", C.c_void_p), ("s_x", C.c_void_p),
                ("h", C.c_void_p), ("q_h", C.c_void_p), ("s_h", C.c_void_p), ("gate_pre", C.c_void_p),
                ("up_out", C.c_void_p), ("out", C.c_void_p), ("plan", C.c_void_p), ("gate", BellTernaryEll),
                ("up", BellTernaryEll), ("down", BellTernaryEll), ("status", C.c_void_p)]


class BellLoopDesc(C.Structure):
    _fields_ = [("T", C.c_int64), ("d_model", C.c_int32), ("d_ff", C.c_int32), ("L", C.c_int32),
                ("eps", C.c_float), ("h_in", C.c_void_p), ("h_out", C.c_void_p), ("norm_gain", C.c_void_p),
                ("hn", C.c_void_p), ("h_mid", C.c_void_p), ("plan", C.c_void_p), ("workspace", C.c_void_p),
                ("gate", BellEll), ("up", BellEll), ("down", BellEll), ("status", C.c_void_p),
                ("mode", C.c_int32), ("reserved", C.c_int32)]


BELL_LOOP_AUTO = 0
BELL_LOOP_LAUNCHES = 1
BELL_LOOP_PERSISTENT = 2


class BellDownBwdDesc(C.Structure):
    _fields_ = [("T", C.c_int64), ("grad_out", C.c_void_p), ("gate_pre", C.c_void_p), ("up_out", C.c_void_p),
                ("d_gate_up", C.c_void_p), ("plan", C.c_void_p), ("w_t", BellEll), ("status", C.c_void_p)]


class BellSddmmDesc(C.Structure):
    _fields_ = [("T", C.c_int64), ("a", C.c_void_p), ("b", C.c_void_p), ("lda", C.c_int64), ("ldb", C.c_int64),
                ("col_indices", C.c_void_p), ("R", C.c_int32), ("C", C.c_int32), ("K", C.c_int32),
                ("B", C.c_int32), ("layout", C.c_int32), ("accumulate", C.c_int32), ("grad", C.c_void_p),
                ("grad_bf16", C.c_void_p), ("status", C.c_void_p)]


class BellDenseToEllDesc(C.Structure):
    _fields_ = [("dense", C.c_void_p), ("dtype", C.c_int32), ("out_features", C.c_int32),
                ("in_features", C.c_int32), ("B", C.c_int32), ("K", C.c_int32), ("layout", C.c_int32),
                ("values", C.c_void_p), ("col_indices", C.c_void_p), ("norms", C.c_void_p)]


# every exported symbol of include/bell.h: name -> (restype, argtypes)
SIGNATURES = {
    "bell_abi_version": (C.c_int, []),
    "bell_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "bell_read_status": (C.c_int, [C.POINTER(C.c_int32), C.c_int32, C.c_void_p]),
    "bell_device_info": (C.c_int, [C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "bell_plan_bytes": (C.c_size_t, [C.c_int32] * 5),
    "bell_swiglu_fwd_bf16": (C.c_int, [C.POINTER(BellFFNDesc), C.c_void_p]),
    "bell_gate_up_bf16": (C.c_int, [C.POINTER(BellFFNDesc), C.c_void_p]),
    "bell_down_bf16": (C.c_int, [C.POINTER(BellFFNDesc), C.c_void_p]),
    "bell_swiglu_fwd_bf16_noalloc": (C.c_int, [C.POINTER(BellFFNDesc), C.c_void_p]),
    "bell_noalloc_scratch_bytes": (C.c_size_t, [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                                C.c_int32]),
    "bell_linear_bf16": (C.c_int, [C.POINTER(BellLinearDesc), C.c_void_p]),
    "bell_swiglu_fwd_f32": (C.c_int, [C.POINTER(BellFFNDesc), C.c_void_p]),
    "bell_linear_f32": (C.c_int, [C.POINTER(BellLinearDesc), C.c_void_p]),
    "bell_f32x_slots": (C.c_int32, [C.c_int32, C.c_int32]),
    "bell_f32x_expand_ell": (C.c_int, [C.POINTER(BellEll), C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                       C.c_void_p, C.c_void_p]),
    "bell_f32x_workspace_bytes": (C.c_size_t, [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                               C.c_int32]),
    "bell_swiglu_fwd_f32x": (C.c_int, [C.POINTER(BellFFNDesc), C.c_void_p, C.c_void_p]),
    "bell_f32x_split_rows": (C.c_int, [C.c_int64, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                       C.c_int64, C.c_void_p]),
    "bell_f32x_linear_workspace_bytes": (C.c_size_t, [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "bell_linear_f32x": (C.c_int, [C.POINTER(BellLinearDesc), C.c_void_p, C.c_void_p]),
    "bell_swiglu_fwd_ternary": (C.c_int, [C.POINTER(BellTernaryFFNDesc), C.c_void_p]),
    "bell_loop_fwd_bf16": (C.c_int, [C.POINTER(BellLoopDesc), C.c_void_p]),
    "bell_loop_workspace_bytes": (C.c_size_t, [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "bell_diag_injection_bf16": (C.c_int, [C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p]),
    "bell_inject_rmsnorm_bf16": (C.c_int, [C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p]),
    "bell_rmsnorm_bf16": (C.c_int, [C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p,
                                    C.c_void_p]),
    "bell_rmsnorm_f32": (C.c_int, [C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p,
                                   C.c_void_p]),
    "bell_silu_mul_bwd_bf16": (C.c_int, [C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_int64, C.c_void_p]),
    "bell_down_silu_bwd_bf16": (C.c_int, [C.POINTER(BellDownBwdDesc), C.c_void_p]),
    "bell_sddmm_bf16": (C.c_int, [C.POINTER(BellSddmmDesc), C.c_void_p]),
    "bell_sddmm_f32": (C.c_int, [C.POINTER(BellSddmmDesc), C.c_void_p]),
    "bell_dense_to_ell": (C.c_int, [C.POINTER(BellDenseToEllDesc), C.c_void_p]),
    "bell_sum_slices_bf16": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                       C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int64, C.c_int32,
                                       C.c_int32, C.c_void_p]),
    "bell_memcpy_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "bell_enable_peer_access": (C.c_int, [C.c_int32]),
    "bell_ipc_handle": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_uint64)]),
    "bell_ipc_open": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "bell_ipc_close": (C.c_int, [C.c_void_p]),
    "bell_pin_l2": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p]),
    "bell_unpin_l2": (C.c_int, [C.c_void_p]),
}

_lib = None
_lock = threading.Lock()


def load():
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"libbell_b200.so not found at {LIB_PATH}; build it with "
                                   "`python looped-blockell-tpu_b200/csrc/setup.py` (or __graft_entry__.build())")
            lib = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(512)
    code = load().bell_last_error(buf, 512)
    return f"{ERRORS.get(code, code)}: {buf.value.decode(errors='replace')}"


def check(rc: int, what: str) -> None:
    """Raise RuntimeError with the library's message when rc != 0."""
    if rc != BELL_OK:
        raise RuntimeError(f"{what} failed: {last_error()}")
