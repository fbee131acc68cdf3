"""Seeded input generators restated from the reference's chart tests.

`next_rand` is the xorshift64 of src/engine/chart/tests.rs:14-21; `random_payload`
(:25-70) fills a payload with random bytes and overwrites every block's f16 scale(s);
`random_x` (:73-80) gives Q32.32 activations in [-2048, 2047].
"""
import numpy as np

MASK = (1 << 64) - 1
GEOM = {8: (32, 34), 12: (256, 144), 14: (256, 210)}


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
        if ggml_type == 8:
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
