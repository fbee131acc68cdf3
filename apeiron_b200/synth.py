"""Seeded synthetic GGUF payloads and activations with the benchmark's distributions.

The reference ships no weights for this path; the benchmark configurations name seeded
synthetic inputs instead:
  Q8_0: codes uniform in [-127, 127], f16 scale |N(0,1)|·0.02/127;
  Q4_K: nibbles uniform 0..15, 6-bit sub-scales and mins uniform 0..63 (uniform random
        packed bytes give exactly that), f16 d and dmin |N(0,1)|·1e-3;
  Q6_K: 6-bit codes uniform (random ql/qh bytes), int8 sub-scales uniform, f16 d as Q4_K;
  x:    f32 N(0,1).
Block layouts are GGUF's (src/format/quant.rs:52-68): Q8_0 [f16 d][32 i8];
Q4_K [f16 d][f16 dmin][12 B scales][128 B nibbles]; Q6_K [128 B ql][64 B qh][16 i8][f16 d].
"""
from __future__ import annotations

import numpy as np

Q8_0, Q4_K, Q6_K = 8, 12, 14
GEOM = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(-1, 2)


def payload(ggml_type: int, n_out: int, n_in: int, seed: int) -> np.ndarray:
    """Row-major GGUF payload of an n_out x n_in matrix (ragged last block zero-padded)."""
    rng = np.random.default_rng(seed)
    qk, bb = GEOM[ggml_type]
    blocks = -(-n_in // qk)
    nblk = n_out * blocks
    raw = np.empty((nblk, bb), dtype=np.uint8)
    if ggml_type == Q8_0:
        raw[:, 0:2] = _f16_bytes(np.abs(rng.standard_normal(nblk)) * 0.02 / 127)
        raw[:, 2:] = rng.integers(-127, 128, size=(nblk, 32), dtype=np.int8).view(np.uint8)
    elif ggml_type == Q4_K:
        raw[:, 0:2] = _f16_bytes(np.abs(rng.standard_normal(nblk)) * 1e-3)
        raw[:, 2:4] = _f16_bytes(np.abs(rng.standard_normal(nblk)) * 1e-3)
        raw[:, 4:] = rng.integers(0, 256, size=(nblk, 140), dtype=np.uint8)
    else:
        raw[:, 0:208] = rng.integers(0, 256, size=(nblk, 208), dtype=np.uint8)
        raw[:, 208:210] = _f16_bytes(np.abs(rng.standard_normal(nblk)) * 1e-3)
    if n_in % qk:
        # zero the codes past n_in of each row's last block, as a real ragged tensor would
        raw = raw.reshape(n_out, blocks, bb)
        tail = n_in - (blocks - 1) * qk
        if ggml_type == Q8_0:
            raw[:, -1, 2 + tail:] = 0
        # K-quant tails are left random: the contract never reads past n_in
        raw = raw.reshape(nblk, bb)
    return raw.reshape(-1)


def activation_f32(n: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


def f32_to_q32(x: np.ndarray) -> np.ndarray:
    """round(v·2^32), ties away from zero (F32::to_q32, src/engine/num/fp.rs:186-230) for
    finite |v| < 2^31 — exact in float64 because v·2^32 has at most 24 significant bits."""
    v = x.astype(np.float64) * 4294967296.0
    r = np.floor(np.abs(v) + 0.5)
    return (np.sign(v) * r).astype(np.int64)


def quant_act_np(x: np.ndarray):
    """quant_act (src/engine/chart/mod.rs:258-334) for benchmark inputs: codes int8 and
    exponent bytes (0xFF for zero blocks), vectorised with exact integer arithmetic.
    Only for inputs whose scales stay below 2^57 (any f32 activation below 2^24)."""
    x = np.asarray(x, dtype=np.int64)
    n = x.size
    nb = -(-n // 32)
    pad = np.zeros(nb * 32, dtype=np.int64)
    pad[:n] = x
    blk = pad.reshape(nb, 32)
    mag = np.abs(blk).astype(np.uint64)
    absmax = mag.max(axis=1)
    need = absmax // np.uint64(127) + (absmax % np.uint64(127) != 0).astype(np.uint64)
    e = np.zeros(nb, dtype=np.int64)
    big = need > 1
    e[big] = np.ceil(np.log2(need[big].astype(np.float64))).astype(np.int64)
    # fix float rounding of log2 near powers of two: smallest e with 2^e >= need
    e[big] -= ((np.left_shift(np.uint64(1), (e[big] - 1).astype(np.uint64))) >= need[big])
    e[big] += ((np.left_shift(np.uint64(1), e[big].astype(np.uint64))) < need[big])
    assert np.all(e < 57)
    S = np.left_shift(np.uint64(1), e.astype(np.uint64))[:, None]
    q = mag >> e.astype(np.uint64)[:, None]
    r = mag & (S - np.uint64(1))
    code = (q + (np.uint64(2) * r >= S).astype(np.uint64)).astype(np.int64)
    code = np.where(blk < 0, -code, code)
    zero = absmax == 0
    code[zero] = 0
    exps = np.where(zero, 0xFF, e).astype(np.uint8)
    return code.reshape(-1)[:n].astype(np.int8), exps
