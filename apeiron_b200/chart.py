"""Host-side mirror of apeiron's Q8-activation projection interface over the CUDA backend.

Names, argument meaning and refusals follow the reference:

=====================================  ==================================================
this module                            reference (apeiron tree)
=====================================  ==================================================
``QuantAct``                           src/engine/chart/mod.rs:67-214
``quant_act(x)``                       src/engine/chart/mod.rs:258-334
``Backend.matvec_q8act``               src/engine/chart/mod.rs:1887-1925
``Backend.matvec_q8act_quant_chunked`` src/engine/chart/ffn.rs:667-745
``Backend.matmat_q8act``               src/engine/kern/matmat.rs:92-134
``MatvecError`` and subclasses         src/engine/ops/matvec.rs:11-48
=====================================  ==================================================

Every projection runs on the device through the C ABI; a refusal raises the
``MatvecError`` subclass the reference returns.  Weights are uploaded once per payload
(the engine's resident GGUF slice, src/engine/loader.rs:421-434) and kept on the device.
"""
from __future__ import annotations

import ctypes as C
import hashlib
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _abi

ACT_QK = 32
GEOM = {_abi.Q5_0: (32, 22), _abi.Q8_0: (32, 34), _abi.Q4_K: (256, 144), _abi.Q6_K: (256, 210)}


# ---- refusals (src/engine/ops/matvec.rs:11-48) ---------------------------------------

class MatvecError(Exception):
    """A refused projection.  ``row``/``col`` locate kernel-side refusals."""

    def __init__(self, *args, row=None, col=None):
        super().__init__(*args)
        self.row = row
        self.col = col

    def __eq__(self, other):
        return type(self) is type(other) and self.args == other.args

    def __hash__(self):
        return hash((type(self), self.args))


class ShapeMismatch(MatvecError):
    def __init__(self, x, n_in, **kw):
        super().__init__(x, n_in, **kw)
        self.x, self.n_in = x, n_in


class RowLength(MatvecError):
    pass


class ShortPayload(MatvecError):
    def __init__(self, need, have, **kw):
        super().__init__(need, have, **kw)
        self.need, self.have = need, have


class LengthOverflow(MatvecError):
    pass


class UnsupportedQuant(MatvecError):
    def __init__(self, ggml_type, **kw):
        super().__init__(ggml_type, **kw)
        self.ggml_type = ggml_type


class NonFiniteScale(MatvecError):
    """``MatvecError::Dequant(EngineError::NonFiniteScale { bits })``."""

    def __init__(self, bits, **kw):
        super().__init__(bits, **kw)
        self.bits = bits


class FixedOverflow(MatvecError):
    """``MatvecError::Dequant(EngineError::FixedOverflow)``."""


class AccumulatorOverflow(MatvecError):
    pass


class OutputOverflow(MatvecError):
    pass


class QuantRefused(MatvecError):
    """``quant_act`` / ``f32_to_fixed`` returned None."""


class BackendError(RuntimeError):
    """A backend condition with no reference counterpart (CUDA error, bad handle, ...)."""


def _raise(err: _abi.ApxErr):
    c = err.code
    kw = dict(row=int(err.row), col=int(err.col))
    if c == _abi.APX_ERR_SHAPE_MISMATCH:
        raise ShapeMismatch(int(err.a), int(err.b), **kw)
    if c == _abi.APX_ERR_SHORT_PAYLOAD:
        raise ShortPayload(int(err.a), int(err.b), **kw)
    if c == _abi.APX_ERR_LENGTH_OVERFLOW:
        raise LengthOverflow(**kw)
    if c == _abi.APX_ERR_UNSUPPORTED_QUANT:
        raise UnsupportedQuant(int(err.ggml_type), **kw)
    if c == _abi.APX_ERR_NONFINITE_SCALE:
        raise NonFiniteScale(int(err.bits), **kw)
    if c == _abi.APX_ERR_FIXED_OVERFLOW:
        raise FixedOverflow(**kw)
    if c == _abi.APX_ERR_ACCUMULATOR_OVERFLOW:
        raise AccumulatorOverflow(**kw)
    if c == _abi.APX_ERR_OUTPUT_OVERFLOW:
        raise OutputOverflow(**kw)
    if c == _abi.APX_ERR_ROW_LENGTH:
        raise RowLength(**kw)
    if c == _abi.APX_ERR_QUANT_REFUSED:
        raise QuantRefused(**kw)
    raise BackendError(f"apeiron_b200 backend error {c} (cuda {err.cuda_error})")


# ---- activations (src/engine/chart/mod.rs:67-334) ----------------------------------------

@dataclass
class QuantAct:
    """One scale per 32-lane block (0 or 2^e) and one int8 code per element."""

    scales: np.ndarray  # int64
    codes: np.ndarray   # int8

    @classmethod
    def from_parts(cls, scales, codes) -> "QuantAct":
        return cls(np.ascontiguousarray(scales, dtype=np.int64),
                   np.ascontiguousarray(codes, dtype=np.int8))

    @classmethod
    def from_exps(cls, exps, codes) -> "QuantAct":
        e = np.asarray(exps, dtype=np.uint8)
        s = np.zeros(e.shape, dtype=np.int64)
        nz = e != _abi.EXP_ZERO
        s[nz] = np.left_shift(np.int64(1), e[nz].astype(np.int64))
        return cls(s, np.ascontiguousarray(codes, dtype=np.int8))

    def __len__(self):
        return int(self.codes.size)

    def exps(self) -> np.ndarray:
        """The ABI's exponent bytes; a scale that is not 0 or a power of two <= 2^62
        cannot cross the ABI (quant_act never produces one) and raises ValueError."""
        s = self.scales
        out = np.full(s.shape, _abi.EXP_ZERO, dtype=np.uint8)
        nz = s != 0
        v = s[nz]
        if np.any(v < 0) or np.any(v & (v - 1)):
            raise ValueError("QuantAct scale is not a power of two")
        out[nz] = np.log2(v.astype(np.float64)).round().astype(np.uint8)
        return out

    def dequant(self) -> Optional[np.ndarray]:
        """``QuantAct::dequant`` (chart/mod.rs:188-212): x-hat = S·xq, None when a product
        leaves i64."""
        s = np.repeat(self.scales, ACT_QK)[: len(self)].astype(object)
        v = s * self.codes.astype(object)
        if any(x < -(1 << 63) or x >= (1 << 63) for x in v):
            return None
        return np.array([int(x) for x in v], dtype=np.int64)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Tensor:
    """A weight payload resident on the device (one upload, one repack)."""

    def __init__(self, backend: "Backend", handle: int, ggml_type: int, n_out: int, n_in: int,
                 raw_len: int):
        self.backend, self.handle = backend, handle
        self.ggml_type, self.n_out, self.n_in, self.raw_len = ggml_type, n_out, n_in, raw_len

    def free(self):
        if self.handle:
            self.backend.lib.apx_tensor_free(self.backend.ctx, self.handle)
            self.handle = 0


class Backend:
    """One CUDA backend context (``apx_open``) on ``device``."""

    def __init__(self, device: int = 0):
        self.lib = _abi.load()
        err = _abi.ApxErr()
        self.ctx = self.lib.apx_open(device, C.byref(err))
        if not self.ctx:
            raise BackendError(f"apx_open({device}) failed: code {err.code} cuda {err.cuda_error}")
        self.device = device
        self._cache = {}

    def close(self):
        if self.ctx:
            self.lib.apx_close(self.ctx)
            self.ctx = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    # -- weights ---------------------------------------------------------------------------
    def upload(self, ggml_type: int, raw, n_out: int, n_in: int) -> Tensor:
        buf = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else \
            np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
        h = C.c_uint64()
        err = _abi.ApxErr()
        rc = self.lib.apx_tensor_upload(self.ctx, ggml_type, _ptr(buf), buf.size, n_out, n_in,
                                        C.byref(h), C.byref(err))
        if rc:
            _raise(err)
        return Tensor(self, h.value, ggml_type, n_out, n_in, buf.size)

    def _tensor(self, ggml_type, raw, n_out, n_in) -> Tensor:
        if isinstance(raw, Tensor):
            if raw.ggml_type != ggml_type:
                raise BackendError("tensor was uploaded with another ggml type")
            return raw
        buf = np.ascontiguousarray(raw if isinstance(raw, np.ndarray)
                                   else np.frombuffer(raw, dtype=np.uint8), dtype=np.uint8)
        # keyed by content: the result must follow the bytes passed on this call, as the
        # reference's borrowed-slice interface does, even if a buffer is reused or edited
        digest = hashlib.blake2b(buf.reshape(-1).data, digest_size=16).digest()
        key = (ggml_type, digest, buf.size, n_out, n_in)
        t = self._cache.get(key)
        if t is None:
            t = self.upload(ggml_type, buf, n_out, n_in)
            self._cache[key] = t
        return t

    # -- projections -------------------------------------------------------------------------
    def matvec_q8act(self, ggml_type: int, raw, n_out: int, n_in: int, q: QuantAct) -> np.ndarray:
        """``matvec_q8act`` (chart/mod.rs:1887): the Q32.32 outputs, or raises."""
        t = self._tensor(ggml_type, raw, n_out, n_in)
        codes, exps = q.codes, q.exps()
        out = np.empty(max(n_out, 1), dtype=np.int64)
        err = _abi.ApxErr()
        rc = self.lib.apx_matvec_q8act(self.ctx, t.handle, n_out, n_in, _ptr(codes), codes.size,
                                       _ptr(exps), _ptr(out), C.byref(err))
        if rc:
            _raise(err)
        return out[:n_out]

    def matvec_q8act_quant_chunked(self, ggml_type: int, raw, n_out: int, n_in: int,
                                   q: QuantAct, chunks: int) -> np.ndarray:
        """``matvec_q8act_quant_chunked`` (chart/ffn.rs:667)."""
        t = self._tensor(ggml_type, raw, n_out, n_in)
        codes, exps = q.codes, q.exps()
        out = np.empty(max(n_out, 1), dtype=np.int64)
        err = _abi.ApxErr()
        rc = self.lib.apx_matvec_q8act_chunked(self.ctx, t.handle, n_out, n_in, _ptr(codes),
                                               codes.size, _ptr(exps), chunks, _ptr(out),
                                               C.byref(err))
        if rc:
            _raise(err)
        return out[:n_out]

    def matmat_q8act(self, ggml_type: int, raw, n_out: int, n_in: int,
                     qs: Sequence[QuantAct]) -> list:
        """``matmat_q8act`` (kern/matmat.rs:134): one Q32.32 vector per column."""
        t = self._tensor(ggml_type, raw, n_out, n_in)
        k = len(qs)
        if k == 0:
            return []
        q_len = len(qs[0])
        if any(len(q) != q_len for q in qs):
            # columns of different widths: each column is its own call (per-column contract)
            return [self.matvec_q8act(ggml_type, t, n_out, n_in, q) for q in qs]
        codes = np.ascontiguousarray(np.stack([q.codes for q in qs]), dtype=np.int8)
        exps = np.ascontiguousarray(np.stack([q.exps() for q in qs]), dtype=np.uint8)
        out = np.empty((k, max(n_out, 1)), dtype=np.int64)
        err = _abi.ApxErr()
        rc = self.lib.apx_matmat_q8act(self.ctx, t.handle, n_out, n_in, k, _ptr(codes), q_len,
                                       _ptr(exps), _ptr(out), C.byref(err))
        if rc:
            _raise(err)
        return [out[c, :n_out] for c in range(k)]

    def quant_act(self, x) -> Optional[QuantAct]:
        """``quant_act`` (chart/mod.rs:258) on the device; None where the reference
        returns None."""
        x = np.ascontiguousarray(x, dtype=np.int64)
        n = x.size
        codes = np.empty(max(n, 1), dtype=np.int8)
        exps = np.empty(max((n + 31) // 32, 1), dtype=np.uint8)
        err = _abi.ApxErr()
        rc = self.lib.apx_quant_act(self.ctx, _ptr(x), n, _ptr(codes), _ptr(exps), C.byref(err))
        if rc == _abi.APX_ERR_QUANT_REFUSED:
            return None
        if rc:
            _raise(err)
        return QuantAct.from_exps(exps[: (n + 31) // 32], codes[:n])

    def matvec_f32(self, tensor: Tensor, x) -> np.ndarray:
        """f32 boundary: from_q32(matvec_q8act(W, quant_act(f32_to_fixed(x))))."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(max(tensor.n_out, 1), dtype=np.float32)
        err = _abi.ApxErr()
        rc = self.lib.apx_matvec_f32(self.ctx, tensor.handle, tensor.n_out, tensor.n_in,
                                     _ptr(x), _ptr(y), C.byref(err))
        if rc:
            _raise(err)
        return y[: tensor.n_out]

    def matmat_f32(self, tensor: Tensor, x) -> np.ndarray:
        """f32 boundary of the prefill contract: x is (k, n_in) f32, one token per row; the
        result is (k, n_out) f32, row c equal to ``matvec_f32(tensor, x[c])``."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != tensor.n_in:
            raise ValueError("x must be (k, n_in)")
        k = x.shape[0]
        y = np.empty((max(k, 1), max(tensor.n_out, 1)), dtype=np.float32)
        err = _abi.ApxErr()
        rc = self.lib.apx_matmat_f32(self.ctx, tensor.handle, tensor.n_out, tensor.n_in, k,
                                     _ptr(x), _ptr(y), C.byref(err))
        if rc:
            _raise(err)
        return y[:k, : tensor.n_out]

    def block_dots(self, tensor: Tensor, codes) -> np.ndarray:
        """The exact int32 group dots the kernels form (parity hook)."""
        codes = np.ascontiguousarray(codes, dtype=np.int8)
        qk, _ = GEOM[tensor.ggml_type]
        blocks = -(-tensor.n_in // qk)
        per_row = (-(-tensor.n_in // 32) if tensor.ggml_type == _abi.Q8_0
                   else blocks * (16 if tensor.ggml_type == _abi.Q6_K else 8))
        dots = np.empty((max(tensor.n_out, 1), max(per_row, 1)), dtype=np.int32)
        err = _abi.ApxErr()
        rc = self.lib.apx_debug_block_dots(self.ctx, tensor.handle, tensor.n_out, tensor.n_in,
                                           _ptr(codes), _ptr(dots), C.byref(err))
        if rc:
            _raise(err)
        return dots[: tensor.n_out, :per_row]
