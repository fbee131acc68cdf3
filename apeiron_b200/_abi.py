"""ctypes binding of ``libapeiron_cuda.so`` (the C ABI of include/apeiron_cuda.h).

The library is built in place by ``apeiron_b200.build``.  There is no fallback: when the
library is missing or cannot be loaded, importing a projection raises.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libapeiron_cuda.so")

APX_OK = 0
APX_ERR_SHAPE_MISMATCH = 1
APX_ERR_ROW_LENGTH = 2
APX_ERR_SHORT_PAYLOAD = 3
APX_ERR_LENGTH_OVERFLOW = 4
APX_ERR_UNSUPPORTED_QUANT = 5
APX_ERR_NONFINITE_SCALE = 6
APX_ERR_FIXED_OVERFLOW = 7
APX_ERR_ACCUMULATOR_OVERFLOW = 8
APX_ERR_OUTPUT_OVERFLOW = 9
APX_ERR_QUANT_REFUSED = 10
APX_ERR_SWIGLU_REFUSED = 11
APX_ERR_INVALID_ARGUMENT = 20
APX_ERR_LAYOUT_MISMATCH = 21
APX_ERR_CUDA = 22
APX_ERR_OUT_OF_MEMORY = 23
APX_ERR_TOO_LARGE = 24
APX_ERR_DEVICE_TIMEOUT = 25

Q8_0, Q4_K, Q6_K = 8, 12, 14
Q5_0 = 6  # served as Q8_0 (its codes widen exactly at upload)
EXP_ZERO = 0xFF

# Every symbol the header declares (tests/test_abi.py checks the library exports them).
EXPORTS = [
    "apx_open", "apx_close", "apx_version", "apx_tensor_upload", "apx_tensor_free",
    "apx_tensor_device_bytes", "apx_matvec_q8act", "apx_matvec_q8act_chunked",
    "apx_matmat_q8act", "apx_quant_act", "apx_matvec_f32", "apx_debug_block_dots",
    "apx_act_describe_async", "apx_quant_q32_async", "apx_quant_f32_async",
    "apx_matvec_async", "apx_matmat_async", "apx_matmat_f32_async", "apx_act_padded_len", "apx_status_decode", "apx_status_decode_rows",
    "apx_matvec_f32_noalloc", "apx_matmat_f32", "apx_quant_f32_cols_async",
    "apx_peer_alloc", "apx_peer_open", "apx_peer_close", "apx_device_read", "apx_device_write",
    "apx_gather_publish_async", "apx_matvec_gather_async", "apx_matvec_group_async",
    "apx_swiglu_quant_async", "apx_swiglu_quant_cols_async", "apx_swiglu_quant_shard_async", "apx_matmat_f32_group_async", "apx_act_describe_cols_async",
    "apx_ffn_status_decode", "apx_ctx_set_gemm_route", "apx_plan_create", "apx_plan_run_async", "apx_plan_destroy",
]
PLAN_GATE, PLAN_UP = 0, 1
PLAN_MAX_PEERS = 7
PLAN_ACT_UNPADDED = 1
GEMM_AUTO, GEMM_DIGITS, GEMM_FOLD = 0, 1, 2
CARRIER_F32, CARRIER_Q32 = 0, 1

MAX_PEERS = 8
MAX_GATHER_PROJ = 4
PEER_HANDLE_BYTES = 64

NOALLOC_MAX_N_IN = 65536


class ApxErr(C.Structure):
    _fields_ = [
        ("code", C.c_int32),
        ("ggml_type", C.c_uint32),
        ("a", C.c_uint64),
        ("b", C.c_uint64),
        ("row", C.c_uint64),
        ("col", C.c_uint64),
        ("bits", C.c_uint32),
        ("cuda_error", C.c_int32),
    ]


class GatherDesc(C.Structure):
    """Mirror of ``apx_gather_desc`` (include/apeiron_cuda.h)."""

    _fields_ = [
        ("world", C.c_int),
        ("rank", C.c_int),
        ("nproj", C.c_int),
        ("timeout_us", C.c_uint),
        ("peer", C.c_void_p * MAX_PEERS),
        ("out_off", C.c_size_t),
        ("key_off", C.c_size_t),
        ("flag_off", C.c_size_t),
        ("ctr_off", C.c_size_t),
        ("rows_off", C.c_size_t * MAX_GATHER_PROJ),
        ("rows", C.c_size_t * MAX_GATHER_PROJ),
        ("row0", C.c_longlong * MAX_GATHER_PROJ),
        ("nf_key", C.c_longlong * MAX_GATHER_PROJ),
        ("status", C.c_void_p * MAX_GATHER_PROJ),
        ("out_status", C.c_void_p * MAX_GATHER_PROJ),
        ("bytes", C.c_size_t),
        ("desc_off", C.c_size_t),
        ("merged_off", C.c_size_t),
    ]


class CallStatus(C.Structure):
    _fields_ = [("first", C.c_uint64), ("spare", C.c_uint64)]


P = C.c_void_p
class PlanAct(C.Structure):
    _fields_ = [("d_codes", C.c_void_p), ("d_exps", C.c_void_p), ("d_desc", C.c_void_p),
                ("ffn", C.c_int32), ("flags", C.c_int32)]


class PlanProj(C.Structure):
    _fields_ = [("tensor", C.c_uint64), ("n_out", C.c_size_t), ("n_in", C.c_size_t),
                ("act", C.c_int32), ("ffn", C.c_int32), ("role", C.c_int32),
                ("reserved", C.c_int32), ("d_out_q32", C.c_void_p), ("d_out_f32", C.c_void_p),
                ("d_status", C.c_void_p)]


class PlanFfn(C.Structure):
    _fields_ = [("carrier", C.c_int32), ("out_act", C.c_int32), ("d_h", C.c_void_p),
                ("d_status", C.c_void_p), ("n_peers", C.c_int32), ("reserved", C.c_int32),
                ("d_peer_codes", C.c_void_p * PLAN_MAX_PEERS),
                ("d_peer_exps", C.c_void_p * PLAN_MAX_PEERS),
                ("d_peer_desc", C.c_void_p * PLAN_MAX_PEERS)]


SZ = C.c_size_t
U64 = C.c_uint64
EP = C.POINTER(ApxErr)

_SIGS = {
    "apx_open": (P, [C.c_int, EP]),
    "apx_close": (None, [P]),
    "apx_version": (C.c_char_p, []),
    "apx_tensor_upload": (C.c_int, [P, C.c_uint32, P, SZ, SZ, SZ, C.POINTER(U64), EP]),
    "apx_tensor_free": (C.c_int, [P, U64]),
    "apx_tensor_device_bytes": (SZ, [P, U64]),
    "apx_matvec_q8act": (C.c_int, [P, U64, SZ, SZ, P, SZ, P, P, EP]),
    "apx_matvec_q8act_chunked": (C.c_int, [P, U64, SZ, SZ, P, SZ, P, SZ, P, EP]),
    "apx_matmat_q8act": (C.c_int, [P, U64, SZ, SZ, SZ, P, SZ, P, P, EP]),
    "apx_quant_act": (C.c_int, [P, P, SZ, P, P, EP]),
    "apx_matvec_f32": (C.c_int, [P, U64, SZ, SZ, P, P, EP]),
    "apx_debug_block_dots": (C.c_int, [P, U64, SZ, SZ, P, P, EP]),
    "apx_act_describe_async": (C.c_int, [P, P, P, SZ, P, P]),
    "apx_quant_q32_async": (C.c_int, [P, P, SZ, P, P, P, P]),
    "apx_quant_f32_async": (C.c_int, [P, P, SZ, P, P, P, P]),
    "apx_matvec_async": (C.c_int, [P, U64, SZ, SZ, P, P, P, P, P, P, P]),
    "apx_peer_alloc": (C.c_int, [P, SZ, C.POINTER(C.c_void_p), P, EP]),
    "apx_peer_open": (C.c_int, [P, P, C.POINTER(C.c_void_p), EP]),
    "apx_peer_close": (C.c_int, [P, P, C.c_int]),
    "apx_device_read": (C.c_int, [P, P, P, SZ, EP]),
    "apx_device_write": (C.c_int, [P, P, P, SZ, EP]),
    "apx_gather_publish_async": (C.c_int, [P, C.POINTER(GatherDesc), P]),
    "apx_matvec_gather_async": (C.c_int, [P, U64, SZ, SZ, P, P, P, C.POINTER(GatherDesc),
                                          C.c_int, P]),
    "apx_matvec_group_async": (C.c_int, [P, P, C.c_int, SZ, P, P, P, P, P, P, P]),
    "apx_matmat_async": (C.c_int, [P, U64, SZ, SZ, SZ, P, P, P, P, P, P, P]),
    "apx_matmat_f32_async": (C.c_int, [P, U64, SZ, SZ, SZ, P, SZ, P, P, P, P]),
    "apx_act_padded_len": (SZ, [SZ]),
    "apx_status_decode": (C.c_int, [P, U64, C.POINTER(CallStatus), EP]),
    "apx_status_decode_rows": (C.c_int, [P, U64, SZ, C.POINTER(CallStatus), EP]),
    "apx_swiglu_quant_async": (C.c_int, [P, P, P, SZ, C.c_int, P, P, P, P, P, P]),
    "apx_swiglu_quant_cols_async": (C.c_int, [P, P, P, SZ, SZ, C.c_int, P, P, P, P, P, P]),
    "apx_swiglu_quant_shard_async": (C.c_int, [P, P, P, SZ, C.c_int, P, P, P, P, C.c_int, P, P,
                                               P, P, P]),
    "apx_matmat_f32_group_async": (C.c_int, [P, P, C.c_int, SZ, SZ, P, SZ, P, P, P, P]),
    "apx_act_describe_cols_async": (C.c_int, [P, P, P, SZ, SZ, P, P]),
    "apx_ffn_status_decode": (C.c_int, [C.POINTER(CallStatus), EP]),
    "apx_plan_create": (P, [P, C.POINTER(PlanProj), SZ, C.POINTER(PlanAct), SZ,
                            C.POINTER(PlanFfn), SZ, EP]),
    "apx_plan_run_async": (C.c_int, [P, P]),
    "apx_ctx_set_gemm_route": (C.c_int, [P, C.c_int]),
    "apx_plan_destroy": (None, [P]),
    "apx_matvec_f32_noalloc": (C.c_int, [P, U64, SZ, SZ, P, P, P, P]),
    "apx_matmat_f32": (C.c_int, [P, U64, SZ, SZ, SZ, P, P, EP]),
    "apx_quant_f32_cols_async": (C.c_int, [P, P, SZ, SZ, P, P, P, P]),
}

_lib = None


def load(path: str | None = None):
    """Load the backend library (once).  Raises OSError when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise OSError(f"apeiron_b200: CUDA backend library not built: {path} "
                      "(run `python -m apeiron_b200.build`)")
    lib = C.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
