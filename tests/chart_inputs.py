"""Seeded input generators restated from the reference's chart tests.

`next_rand` is the xorshift64 of src/engine/chart/tests.rs:14-21; `random_payload`
(:25-70) fills a payload with random bytes and overwrites every block's f16 scale(s);
`random_x` (:73-80) gives Q32.32 activations in [-2048, 2047].
"""
import numpy as np

MASK = (1 << 64) - 1
GEOM = {6: (32, 22), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def next_rand(state):
    s = state
    s ^= (s << 13) & MASK
    s ^= s >> 7
    s ^= (s << 17) & MASK
    return s & MASK


def _stream(seed, n):
    out = np.empty(n, dtype=np.uint64)
    s = seed
    for i in range(n):
        s = next_rand(s)
        out[i] = s
    return out


def random_payload(ggml_type, rows, n_in, d, dmin, seed):
    qk, bb = GEOM[ggml_type]
    blocks = -(-n_in // qk)
    raw = (_stream(seed, rows * blocks * bb) & np.uint64(0xFF)).astype(np.uint8)
    for blk in range(rows * blocks):
        o = blk * bb
        if ggml_type in (6, 8):
            raw[o:o + 2] = (d & 0xFF, d >> 8)
        elif ggml_type == 12:
            raw[o:o + 2] = (d & 0xFF, d >> 8)
            raw[o + 2:o + 4] = (dmin & 0xFF, dmin >> 8)
        elif ggml_type == 14:
            raw[o + 208:o + 210] = (d & 0xFF, d >> 8)
    return raw


def random_x(n, seed):
    s = _stream(seed, n)
    return ((s % np.uint64(4096)).astype(np.int64) - 2048)


def lcg_next(seed):
    return (seed * 6_364_136_223_846_793_005 + 1_442_695_040_888_963_407) & MASK


def _f(bits):
    return np.array(bits, dtype=np.uint32).view(np.float32)


def f32_block_kinds(n, seed):
    """f32 columns of length n for the device quantizer, each stressing one block kind of
    f32_to_fixed + quant_act: subnormals, values that round to zero in Q32.32, values above
    the 32-bit route's 127·2^24, -2^31 (accepted), 2^31, NaN and -inf (refused), a zero
    column, any finite |f| < 2^31, and Q32.32 blocks beside ordinary ones."""
    rng = np.random.default_rng(seed)
    base = rng.standard_normal(n).astype(np.float32)
    cols = [base.copy()]
    cols.append((base * np.float32(1e-12)).astype(np.float32))      # tiny: rounds in Q32.32
    sub = rng.integers(0, 1 << 23, n, dtype=np.uint32) | (rng.integers(0, 2, n, dtype=np.uint32) << 31)
    cols.append(_f(sub))                                              # subnormals
    big = base.copy()
    big[::7] = np.float32(-2.14e9)                                    # above 127·2^24: code -64
    cols.append(big)
    lo = base.copy()
    lo[0] = np.float32(-2147483648.0)                                 # -2^31: i64::MIN, accepted
    cols.append(lo)
    over = base.copy()
    over[n // 2] = np.float32(2147483648.0)                           # 2^31: refused
    cols.append(over)
    nan = base.copy()
    nan[-1] = np.float32(np.nan)
    cols.append(nan)
    inf = base.copy()
    inf[n // 3] = -np.float32(np.inf)
    cols.append(inf)
    cols.append(np.zeros(n, dtype=np.float32))
    edge = base.copy()
    edge[::5] = _f([0x4EFE0000])[0]                                   # exactly 127·2^24
    cols.append(edge)
    above = base.copy()
    above[n // 2] = _f([0x4EFE0001])[0]                               # one ulp above: code 64
    cols.append(above)                                                # leaves i64, refused
    wild = rng.integers(0, 0x4F000000, n, dtype=np.uint32) | (rng.integers(0, 2, n, dtype=np.uint32) << 31)
    cols.append(_f(wild))                                             # any finite |f| < 2^31
    mixed = base.copy()
    mixed[200:232] = np.float32(1.5e9)                                # one Q32.32 block
    mixed[40:72] = np.float32(3e-10)
    cols.append(mixed)
    return np.stack(cols)
