"""ctypes front of the CPU oracle (``liboracle.so``, built from ``apx_oracle.c``).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA backend.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / ``--impl reference`` leg
import this module; the product package ``apeiron_b200`` never does.

Activations use the reference's ``QuantAct`` form (src/engine/chart/mod.rs:67-81):
``scales`` int64 (0 or 2^e) and ``codes`` int8.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

Q8_0, Q4_K, Q6_K = 8, 12, 14
QK = {Q8_0: 32, Q4_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q8_0: 34, Q4_K: 144, Q6_K: 210}


class ApxErr(C.Structure):
    """Mirror of ``apx_err`` (include/apeiron_cuda.h)."""

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

    def as_tuple(self):
        return (self.code, self.a, self.b, self.bits)


def build() -> str:
    """Compile the oracle in place (gcc, see oracle/Makefile)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
SZ = C.c_size_t


def _declare(l):
    l.apxo_f16_to_fixed.argtypes = [C.c_uint16, C.POINTER(C.c_int64)]
    l.apxo_f16_split.argtypes = [C.c_uint16, C.POINTER(C.c_int32), C.POINTER(C.c_uint32)]
    l.apxo_act_scale.argtypes = [C.c_uint64, C.POINTER(C.c_uint64)]
    l.apxo_finish.argtypes = [C.c_int64, C.c_uint32, C.POINTER(C.c_int64)]
    l.apxo_f32_to_q32.argtypes = [C.c_uint32, C.POINTER(C.c_int64)]
    l.apxo_fixed_exp.argtypes = [C.c_int64, C.POINTER(C.c_int64)]
    l.apxo_silu_fixed.argtypes = [C.c_int64, C.POINTER(C.c_int64)]
    l.apxo_exp_f32.argtypes = [C.c_uint32]
    l.apxo_exp_f32.restype = C.c_uint32
    l.apxo_silu_f32.argtypes = [C.c_uint32]
    l.apxo_silu_f32.restype = C.c_uint32
    l.apxo_swiglu.argtypes = [C.c_int64, C.c_int64, C.c_int, C.POINTER(C.c_int64)]
    l.apxo_round_shift_32.argtypes = [C.c_int64, C.c_uint64, C.POINTER(C.c_int64),
                                      C.POINTER(C.c_uint64)]
    l.apxo_quant_act.argtypes = [P, SZ, P, P]
    l.apxo_dequant_act.argtypes = [P, SZ, P, SZ, P]
    l.apxo_dequant_row.argtypes = [C.c_uint32, P, SZ, SZ, P, C.POINTER(ApxErr)]
    l.apxo_matvec_fixed.argtypes = [C.c_uint32, P, SZ, SZ, SZ, P, SZ, P, C.POINTER(ApxErr)]
    l.apxo_matvec_q8act.argtypes = [C.c_uint32, P, SZ, SZ, SZ, P, SZ, P, SZ, P,
                                    C.POINTER(ApxErr)]
    l.apxo_matvec_q8act_chunked.argtypes = [C.c_uint32, P, SZ, SZ, SZ, P, SZ, P, SZ, SZ, P,
                                            C.POINTER(ApxErr)]
    l.apxo_matmat_q8act.argtypes = [C.c_uint32, P, SZ, SZ, SZ, SZ, P, SZ, P, P,
                                    C.POINTER(ApxErr)]
    l.apxo_exact_dot_q8_0.argtypes = [P, SZ, P, P, C.POINTER(C.c_int64)]
    l.apxo_block_dots.argtypes = [C.c_uint32, P, SZ, SZ, P, P]
    l.apxo_matvec_q8act_mt.argtypes = [C.c_uint32, P, SZ, SZ, SZ, P, P, C.c_int, P,
                                       C.POINTER(ApxErr)]
    l.apxo_matmat_q8act_mt.argtypes = [C.c_uint32, P, SZ, SZ, SZ, SZ, P, P, C.c_int, P,
                                       C.POINTER(ApxErr)]
    l.apxo_matvec_q8act_simd_mt.argtypes = l.apxo_matvec_q8act_mt.argtypes
    l.apxo_matmat_q8act_simd_mt.argtypes = l.apxo_matmat_q8act_mt.argtypes
    l.apxo_simd_features.argtypes = []
    l.apxo_gemm_counts.argtypes = [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    l.apxo_q4k_counts.argtypes = [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    l.apxo_q6k_counts.argtypes = [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    l.apxo_kcols_counts.argtypes = [C.POINTER(C.c_uint64)]


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _u8(raw) -> np.ndarray:
    if isinstance(raw, np.ndarray):
        return np.ascontiguousarray(raw, dtype=np.uint8)
    return np.frombuffer(bytes(raw), dtype=np.uint8)


# ---- scalar helpers --------------------------------------------------------------

def f16_to_fixed(h: int):
    v = C.c_int64()
    return None if lib().apxo_f16_to_fixed(h, C.byref(v)) else v.value


def f16_split(h: int):
    m, k = C.c_int32(), C.c_uint32()
    return None if lib().apxo_f16_split(h, C.byref(m), C.byref(k)) else (m.value, k.value)


def act_scale(absmax: int):
    s = C.c_uint64()
    return None if lib().apxo_act_scale(absmax, C.byref(s)) else s.value


def finish(acc: int, s: int):
    v = C.c_int64()
    return None if lib().apxo_finish(acc, s, C.byref(v)) else v.value


def f32_to_q32(bits: int):
    v = C.c_int64()
    return None if lib().apxo_f32_to_q32(bits, C.byref(v)) else v.value


def round_shift_32(v: int) -> int:
    hi, lo = v >> 64, v & ((1 << 64) - 1)
    oh, ol = C.c_int64(), C.c_uint64()
    lib().apxo_round_shift_32(hi, lo, C.byref(oh), C.byref(ol))
    return (oh.value << 64) | ol.value


# ---- the FFN hidden activation (SwiGLU) ------------------------------------------------

FFN_OVERFLOW = 3     # FfnError::Overflow (ops/ffn.rs:23-24)
CARRIER_F32, CARRIER_Q32 = 0, 1


def fixed_exp(x: int):
    """``fixed_exp`` (src/numeric/fixed_exp.rs:176-184): e^x in Q32.32, None out of range."""
    v = C.c_int64()
    return None if lib().apxo_fixed_exp(x, C.byref(v)) else v.value


def silu_fixed(v: int):
    """``silu_fixed`` (src/engine/ops/silu.rs:53): the Q32.32 value, or the FfnError kind as
    ("err", kind)."""
    o = C.c_int64()
    rc = lib().apxo_silu_fixed(v, C.byref(o))
    return ("err", rc) if rc else o.value


def exp_f32(bits: int) -> int:
    """``exp_f32_scalar`` (src/engine/mixer/f32_carrier.rs:291): binary32 bits in and out."""
    return lib().apxo_exp_f32(bits)


def silu_f32(bits: int) -> int:
    """``silu_f32_scalar`` (f32_carrier.rs:372): binary32 bits in and out."""
    return lib().apxo_silu_f32(bits)


def swiglu(gate: int, up: int, carrier: int = CARRIER_F32):
    """``swiglu_one_carrier`` (src/engine/chart/ffn.rs:279): h in Q32.32, or ("err", kind)."""
    o = C.c_int64()
    rc = lib().apxo_swiglu(gate, up, carrier, C.byref(o))
    return ("err", rc) if rc else o.value


def swiglu_quant(gate, up, carrier: int = CARRIER_F32):
    """The SwiGLU and quantization stages of ``fused_ffn_task`` (chart/ffn.rs:1577-1594) over a
    whole hidden vector: ("swiglu", lane, kind) for the lowest refusing lane, ("quant",) when
    quant_act refuses h, else (h, codes, scales)."""
    h = np.zeros(len(gate), dtype=np.int64)
    for i, (g, u) in enumerate(zip(gate, up)):
        r = swiglu(int(g), int(u), carrier)
        if isinstance(r, tuple):
            return ("swiglu", i, r[1])
        h[i] = r
    q = quant_act(h)
    if q is None:
        return ("quant",)
    return (h,) + q


# ---- activations -----------------------------------------------------------------

def quant_act(x):
    """``quant_act`` (chart/mod.rs:258-334): (codes int8, scales int64) or None."""
    x = np.ascontiguousarray(x, dtype=np.int64)
    n = x.size
    codes = np.zeros(n, dtype=np.int8)
    scales = np.zeros((n + 31) // 32, dtype=np.int64)
    if lib().apxo_quant_act(_p(x), n, _p(codes), _p(scales)):
        return None
    return codes, scales


def dequant_act(codes, scales):
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    out = np.zeros(codes.size, dtype=np.int64)
    if lib().apxo_dequant_act(_p(codes), codes.size, _p(scales), scales.size, _p(out)):
        return None
    return out


def scales_to_exps(scales) -> np.ndarray:
    """Scale (0 or 2^e) -> exponent byte (0xFF for zero), the ABI's encoding."""
    s = np.asarray(scales, dtype=np.int64)
    out = np.full(s.shape, 0xFF, dtype=np.uint8)
    nz = s != 0
    out[nz] = np.log2(s[nz].astype(np.float64)).round().astype(np.uint8)
    assert np.all(np.left_shift(np.int64(1), out[nz].astype(np.int64)) == s[nz])
    return out


def exps_to_scales(exps) -> np.ndarray:
    e = np.asarray(exps, dtype=np.uint8)
    out = np.zeros(e.shape, dtype=np.int64)
    nz = e != 0xFF
    out[nz] = np.left_shift(np.int64(1), e[nz].astype(np.int64))
    return out


# ---- projections -----------------------------------------------------------------

def _result(rc, err, out):
    if rc:
        return ("err", err.code, err.a, err.b, err.bits)
    return out


def matvec_fixed(t, raw, n_out, n_in, x):
    raw = _u8(raw)
    x = np.ascontiguousarray(x, dtype=np.int64)
    out = np.zeros(max(n_out, 1), dtype=np.int64)
    err = ApxErr()
    rc = lib().apxo_matvec_fixed(t, _p(raw), raw.size, n_out, n_in, _p(x), x.size, _p(out),
                                 C.byref(err))
    return _result(rc, err, out[:n_out])


def matvec_q8act(t, raw, n_out, n_in, codes, scales):
    raw = _u8(raw)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    out = np.zeros(max(n_out, 1), dtype=np.int64)
    err = ApxErr()
    rc = lib().apxo_matvec_q8act(t, _p(raw), raw.size, n_out, n_in, _p(codes), codes.size,
                                 _p(scales), scales.size, _p(out), C.byref(err))
    return _result(rc, err, out[:n_out])


def matvec_q8act_row(t, raw, n_out, n_in, codes, scales):
    """``matvec_q8act`` with the refusing row: (outputs, None) or (None, ApxErr)."""
    raw = _u8(raw)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    out = np.zeros(max(n_out, 1), dtype=np.int64)
    err = ApxErr()
    rc = lib().apxo_matvec_q8act(t, _p(raw), raw.size, n_out, n_in, _p(codes), codes.size,
                                 _p(scales), scales.size, _p(out), C.byref(err))
    return (None, err) if rc else (out[:n_out], None)


def matvec_q8act_chunked(t, raw, n_out, n_in, codes, scales, chunks):
    raw = _u8(raw)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    out = np.zeros(max(n_out, 1), dtype=np.int64)
    err = ApxErr()
    rc = lib().apxo_matvec_q8act_chunked(t, _p(raw), raw.size, n_out, n_in, _p(codes),
                                         codes.size, _p(scales), scales.size, chunks,
                                         _p(out), C.byref(err))
    return _result(rc, err, out[:n_out])


def matmat_q8act(t, raw, n_out, n_in, codes, scales):
    """codes [k, n_in] int8, scales [k, ceil(n_in/32)] int64 -> out [k, n_out]."""
    raw = _u8(raw)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    k = codes.shape[0]
    out = np.zeros((max(k, 1), max(n_out, 1)), dtype=np.int64)
    err = ApxErr()
    rc = lib().apxo_matmat_q8act(t, _p(raw), raw.size, n_out, n_in, k, _p(codes), n_in,
                                 _p(scales), _p(out), C.byref(err))
    if rc:
        return ("err", err.code, err.a, err.b, err.bits, err.col)
    return out[:k, :n_out]


def matvec_q8act_mt(t, raw, n_out, n_in, codes, scales, threads, simd=False):
    """The fused rows over ``threads`` row chunks; ``simd`` takes the vector rows
    (apx_oracle_x86.c) where the shape allows, with the same results."""
    raw = _u8(raw)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    out = np.zeros(max(n_out, 1), dtype=np.int64)
    err = ApxErr()
    fn = lib().apxo_matvec_q8act_simd_mt if simd else lib().apxo_matvec_q8act_mt
    rc = fn(t, _p(raw), raw.size, n_out, n_in, _p(codes), _p(scales), threads, _p(out),
            C.byref(err))
    return _result(rc, err, out[:n_out])


def matmat_q8act_mt(t, raw, n_out, n_in, codes, scales, threads, simd=False):
    raw = _u8(raw)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    k = codes.shape[0]
    out = np.zeros((k, n_out), dtype=np.int64)
    err = ApxErr()
    fn = lib().apxo_matmat_q8act_simd_mt if simd else lib().apxo_matmat_q8act_mt
    rc = fn(t, _p(raw), raw.size, n_out, n_in, k, _p(codes), _p(scales), threads, _p(out),
            C.byref(err))
    if rc:
        return ("err", err.code, err.a, err.b, err.bits, err.col)
    return out


def gemm_counts():
    """(matmat calls the k-column Q8_0 GEMM completed, (row, group) pairs it sent to the exact
    i128 dot) since the library loaded."""
    a, b = C.c_uint64(), C.c_uint64()
    lib().apxo_gemm_counts(C.byref(a), C.byref(b))
    return a.value, b.value


def q4k_counts():
    """(matmat calls the k-column Q4_K kernel completed, (row, column group) pairs it sent to
    the exact rows) since the library loaded."""
    a, b = C.c_uint64(), C.c_uint64()
    lib().apxo_q4k_counts(C.byref(a), C.byref(b))
    return a.value, b.value


def q6k_counts():
    """The same for the k-column Q6_K kernel."""
    a, b = C.c_uint64(), C.c_uint64()
    lib().apxo_q6k_counts(C.byref(a), C.byref(b))
    return a.value, b.value


def kcols_counts() -> int:
    """Matmat calls the Q8_0 column runs of 16 completed (the path without AVX-VNNI)."""
    a = C.c_uint64()
    lib().apxo_kcols_counts(C.byref(a))
    return a.value


def simd_features() -> dict:
    """What the vector rows use on this host: {"avx2": bool, "avxvnni": bool}."""
    f = lib().apxo_simd_features()
    return {"avx2": bool(f & 1), "avxvnni": bool(f & 2)}


def exact_dot_q8_0(row, blocks, codes, scales):
    row = _u8(row)
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.int64)
    v = C.c_int64()
    if lib().apxo_exact_dot_q8_0(_p(row), blocks, _p(codes), _p(scales), C.byref(v)):
        return None
    return v.value


def block_dots(t, raw, n_out, n_in, codes):
    raw = _u8(raw)
    qk = QK[t]
    blocks = -(-n_in // qk)
    padded = np.zeros(blocks * qk, dtype=np.int8)
    padded[:n_in] = np.asarray(codes, dtype=np.int8)[:n_in]
    per_row = blocks * 16 if t == Q6_K else blocks * (qk // 32)
    dots = np.zeros((max(n_out, 1), max(per_row, 1)), dtype=np.int32)
    rc = lib().apxo_block_dots(t, _p(raw), n_out, n_in, _p(padded), _p(dots))
    assert rc == 0
    return dots[:n_out, :per_row]
