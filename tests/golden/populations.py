"""Known-answer populations for the Q8_0 projection, restated from the reference.

The reference's GPU-parity fixture generator (src/engine/kern/native_gpu_probe.rs) builds
14 synthetic populations (`populations`, :247-348) and 12 real-quantizer populations
(`real_quantizer_populations`, :618-813) from closed-form integer formulas, then asserts
properties of their exact outputs: the 14 synthetic cases give 14,678 values and 32
refusals (:373), case 6's first outputs are [1, 0, 2, -1] (:228-233), case 111 cancels to
0 (:766-768), and the quant_act witnesses of :623-697.  The fixture files themselves are
not shipped by the reference, so this module regenerates the inputs with the same
formulas; tests/test_oracle_golden.py checks the oracle against every asserted value and
tests/golden/populations_digest.json pins the full outputs (written by gen_digest.py).

Each case is a dict: id, rows, tokens, blocks, raw (uint8 [rows*blocks*34] GGUF Q8_0
rows), scales (int64 [tokens, blocks]), codes (int8 [tokens, blocks*32]), refusal.
"""
from __future__ import annotations

import numpy as np

ACT_QK = 32
BB = 34


def _case(cid, rows, tokens, blocks, refusal):
    """Case::new (native_gpu_probe.rs:22-47): every weight scale 1.0 (0x3c00), unit
    activation scales, zero codes."""
    raw = np.zeros(rows * blocks * BB, dtype=np.uint8)
    c = dict(id=cid, rows=rows, tokens=tokens, blocks=blocks, raw=raw,
             scales=np.ones((tokens, blocks), dtype=np.int64),
             codes=np.zeros((tokens, blocks * ACT_QK), dtype=np.int8), refusal=refusal)
    for r in range(rows):
        for b in range(blocks):
            set_half(c, r, b, 0x3C00)
    return c


def set_half(c, row, block, half):
    at = (row * c["blocks"] + block) * BB
    c["raw"][at] = half & 0xFF
    c["raw"][at + 1] = half >> 8


def weight(c, row, block, lane, code):
    c["raw"][(row * c["blocks"] + block) * BB + 2 + lane] = np.uint8(code & 0xFF)


def activation(c, token, block, lane, code):
    c["codes"][token, block * ACT_QK + lane] = code


def varied(cid, rows, tokens, blocks):
    """`varied` (native_gpu_probe.rs:62-90)."""
    c = _case(cid, rows, tokens, blocks, False)
    halves = [0x3C00, 0xBC00, 0x3800, 0xB800, 0x0001, 0x8001, 0, 0x8000]
    raw = c["raw"].reshape(rows, blocks, BB)
    r = np.arange(rows)[:, None, None]
    b = np.arange(blocks)[None, :, None]
    lane = np.arange(ACT_QK)[None, None, :]
    hv = np.array(halves, dtype=np.uint16)[(np.arange(rows)[:, None] + np.arange(blocks)[None, :]) % 8]
    raw[:, :, 0] = hv & 0xFF
    raw[:, :, 1] = hv >> 8
    raw[:, :, 2:] = (((r * 29 + b * 17 + lane * 11) % 256) - 128).astype(np.int8).view(np.uint8)
    t = np.arange(tokens)[:, None]
    bb = np.arange(blocks)[None, :]
    c["scales"] = np.where((t + bb) % 11 == 0, 0, np.left_shift(1, (t + 3 * bb) % 11)).astype(np.int64)
    t3 = np.arange(tokens)[:, None, None]
    b3 = np.arange(blocks)[None, :, None]
    c["codes"] = (((t3 * 31 + b3 * 7 + lane * 19) % 255) - 127).astype(np.int8).reshape(tokens, -1)
    return c


def populations():
    """`populations` (native_gpu_probe.rs:247-348), in the reference's order."""
    zero = varied(0, 3, 5, 2)
    zero["scales"][:] = 0
    signed = varied(1, 5, 3, 3)
    subnormal = varied(2, 3, 5, 2)
    for r in range(3):
        for b in range(2):
            set_half(subnormal, r, b, 0x03FF if (r + b) % 2 == 0 else 0x83FF)
    subnormal["scales"][:] = 1 << 18
    signed_zero = varied(3, 3, 5, 2)
    for r in range(3):
        for b in range(2):
            set_half(signed_zero, r, b, 0 if r % 2 == 0 else 0x8000)
    invalid = _case(4, 3, 5, 1, True)
    for r, h in enumerate([0x7C00, 0xFC00, 0x7E01]):
        set_half(invalid, r, 0, h)
    invalid["scales"][:] = 0
    extremes = _case(5, 3, 5, 1, False)
    for r in range(3):
        for lane in range(ACT_QK):
            weight(extremes, r, 0, lane, -128 if r % 2 == 0 else 127)
    extremes["codes"][:] = -127
    ties = _case(6, 4, 5, 1, False)
    for r, code in enumerate([1, -1, 3, -3]):
        set_half(ties, r, 0, 1)
        weight(ties, r, 0, 0, code)
    for t in range(5):
        activation(ties, t, 0, 0, 1)
    ties["scales"][:] = 1 << 23
    high = _case(7, 3, 5, 1, False)
    for r in range(3):
        set_half(high, r, 0, 1 if r % 2 == 0 else 0x8001)
        weight(high, r, 0, 0, 1)
    for t in range(5):
        activation(high, t, 0, 0, 1)
    high["scales"][:] = 1 << 58
    narrow = _case(8, 3, 5, 1, True)
    for r in range(3):
        set_half(narrow, r, 0, 0x7BFF)
        weight(narrow, r, 0, 0, 1)
    for t in range(5):
        activation(narrow, t, 0, 0, 1)
    narrow["scales"][:] = 1 << 58
    overflow_pos = _case(9, 1, 1, 8, True)
    overflow_neg = _case(10, 1, 1, 8, True)
    cancellation = _case(11, 1, 1, 10, False)
    for c in (overflow_pos, overflow_neg, cancellation):
        c["scales"][:] = 1 << 58
        c["codes"][:] = -127
        for b in range(c["blocks"]):
            set_half(c, 0, b, 0xFBFF if (c["id"] == 11 and b % 2 == 1) else 0x7BFF)
            for lane in range(ACT_QK):
                weight(c, 0, b, lane, 127 if c["id"] == 10 else -128)
    return [zero, signed, subnormal, signed_zero, invalid, extremes, ties, high, narrow,
            overflow_pos, overflow_neg, cancellation, varied(12, 257, 31, 64),
            varied(13, 33, 200, 4)]


# ---- real-quantizer populations (native_gpu_probe.rs:618-813) --------------------------

def _real(cid, rows, activations, quant_act):
    n_in = len(activations[0])
    blocks = n_in // ACT_QK
    qs = [quant_act(np.asarray(x, dtype=np.int64)) for x in activations]
    assert all(q is not None for q in qs), cid
    c = _case(cid, rows, len(activations), blocks, False)
    c["codes"] = np.stack([q[0] for q in qs])
    c["scales"] = np.stack([q[1] for q in qs])
    return c


def unit_at(v):
    x = [0] * ACT_QK
    x[0] = v
    return x


def varied_activation(blocks, seed):
    return [((i * 29 + seed * 17) % 63) - 31 for i in range(blocks * ACT_QK)]


def populate_weighted(c, seed):
    for r in range(c["rows"]):
        for b in range(c["blocks"]):
            set_half(c, r, b, [0x3C00, 0x0001, 0xBC00, 0x8000][(r + b + seed) % 4])
    raw = c["raw"].reshape(c["rows"], c["blocks"], BB)
    r = np.arange(c["rows"])[:, None, None]
    b = np.arange(c["blocks"])[None, :, None]
    lane = np.arange(ACT_QK)[None, None, :]
    raw[:, :, 2:] = (((r * 17 + b * 29 + lane * 13 + seed) % 255) - 127).astype(np.int8).view(np.uint8)


def real_quantizer_populations(quant_act):
    """`real_quantizer_boundary_cases` + `real_quantizer_large_cases` (:618-813)."""
    zeros = [0] * ACT_QK
    zero = _real(100, 2, [zeros], quant_act)
    weight(zero, 0, 0, 0, 127)
    boundary = _real(101, 1, [unit_at(v) for v in (127, -127, 128, -128)], quant_act)
    weight(boundary, 0, 0, 0, 1)
    tie_values = [0] * ACT_QK
    tie_values[:3] = [3, -3, 130]
    ties = _real(102, 3, [tie_values], quant_act)
    for r in range(3):
        weight(ties, r, 0, r, 1)
    mixed_x = [0] * (2 * ACT_QK)
    for lane in range(ACT_QK):
        mixed_x[lane] = 127 if lane % 2 == 0 else -127
        mixed_x[ACT_QK + lane] = (63 << 57) if lane % 2 == 0 else -(63 << 57)
    mixed = _real(103, 1, [mixed_x], quant_act)
    weight(mixed, 0, 0, 0, 1)
    weight(mixed, 0, 1, 0, 1)
    high = _real(104, 1, [unit_at(63 << 57), unit_at(-(63 << 57))], quant_act)
    set_half(high, 0, 0, 0x0001)
    weight(high, 0, 0, 0, 1)
    nonfinite = _real(105, 3, [zeros], quant_act)
    set_half(nonfinite, 1, 0, 0x7C00)
    set_half(nonfinite, 2, 0, 0x7E01)
    weight(nonfinite, 0, 0, 0, 1)

    large_acts = []
    for t in range(31):
        a = varied_activation(64, t)
        a[0] = 31
        large_acts.append(a)
    large = _real(106, 257, large_acts, quant_act)
    populate_weighted(large, 0)
    set_half(large, 256, 0, 0x3C00)
    for b in range(large["blocks"]):
        for lane in range(ACT_QK):
            weight(large, 256, b, lane, 0)
    weight(large, 256, 0, 0, 1)
    tail_acts = []
    for t in range(200):
        a = varied_activation(4, t + 31)
        a[0] = 31
        tail_acts.append(a)
    large_tail = _real(107, 33, tail_acts, quant_act)
    populate_weighted(large_tail, 1)
    set_half(large_tail, 32, 0, 0x3C00)
    for b in range(large_tail["blocks"]):
        for lane in range(ACT_QK):
            weight(large_tail, 32, b, lane, 0)
    weight(large_tail, 32, 0, 0, 1)
    narrow = _real(108, 1, [unit_at(63 << 57)], quant_act)
    set_half(narrow, 0, 0, 0x7BFF)
    weight(narrow, 0, 0, 0, 1)
    ov = [63 << 57] * (32 * ACT_QK)
    over_pos = _real(109, 1, [ov], quant_act)
    over_neg = _real(110, 1, [ov], quant_act)
    cancel = _real(111, 1, [[63 << 57] * (64 * ACT_QK)], quant_act)
    for b in range(32):
        set_half(over_pos, 0, b, 0x7BFF)
        set_half(over_neg, 0, b, 0x7BFF)
        for lane in range(ACT_QK):
            weight(over_pos, 0, b, lane, 127)
            weight(over_neg, 0, b, lane, -128)
    for b in range(64):
        set_half(cancel, 0, b, 0x7BFF if b % 2 == 0 else 0xFBFF)
        for lane in range(ACT_QK):
            weight(cancel, 0, b, lane, -128)
    return [zero, boundary, ties, mixed, high, nonfinite, large, large_tail, narrow,
            over_pos, over_neg, cancel]


def exact_outputs(case, exact_dot):
    """The fixture's golden table: exact_dot per (token, row), None for a refusal
    (native_gpu_probe.rs:187-227 order: tokens outer, rows inner)."""
    rows, blocks = case["rows"], case["blocks"]
    out = []
    for t in range(case["tokens"]):
        for r in range(rows):
            row = case["raw"][r * blocks * BB:(r + 1) * blocks * BB]
            out.append(exact_dot(row, blocks, case["codes"][t], case["scales"][t]))
    return out
