"""Pin the CPU oracle to the reference's own known answers (CPU only).

Every expected value below is asserted by a test in the reference tree; the citation on
each test names it.  The oracle is then trusted as the checker of the CUDA backend.
"""
import hashlib
import json
import os
from fractions import Fraction

import numpy as np
import pytest

from oracle import oracle as O
import populations as pop
from chart_inputs import random_payload, random_x, lcg_next

Q5_0, Q8_0, Q4_K, Q6_K = 6, 8, 12, 14
I64_MIN, I64_MAX = -(1 << 63), (1 << 63) - 1
HERE = os.path.dirname(os.path.abspath(__file__))


def test_f16_to_fixed_all_patterns():
    """chart/tests.rs:85-102: the f16 decode on all 65,536 patterns; Inf/NaN refuse.
    Checked against numpy's IEEE half decode, an independent implementation."""
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    vals = h.view(np.float16).astype(np.float64)
    for bits in range(65536):
        got = O.f16_to_fixed(bits)
        v = vals[bits]
        if not np.isfinite(v):
            assert got is None, hex(bits)
        else:
            assert got == int(Fraction(float(v)) * (1 << 32)), hex(bits)


def test_f16_split_matches_f16_to_fixed():
    """pow2.rs:41-64 / gemm.rs:2555 `f16_split_is_f16_to_fixed`."""
    for bits in range(65536):
        s, f = O.f16_split(bits), O.f16_to_fixed(bits)
        if f is None:
            assert s is None
        else:
            m, k = s
            assert abs(m) <= 2047 and 8 <= k <= 37
            assert m * (1 << k) == f


def test_act_scale_is_least_covering_power_of_two():
    """kern/pow2.rs:105-135."""
    samples = [0, 1, 126, 127, 128, 254, 255, 1 << 20, (1 << 20) + 1, 127 << 40,
               (127 << 40) + 1, 127 << 56, (127 << 56) + 1, (1 << 64) - 1]
    for a in samples:
        c = -(-a // 127)
        s = O.act_scale(a)
        if s == 0:
            assert a == 0
        elif s is None:
            assert c > 1 << 62
        else:
            assert s & (s - 1) == 0 and s * 127 >= a
            assert s == 1 or (s // 2) * 127 < a
            assert s < 2 * max(c, 1)


def test_finish_is_round_shift_of_scaled_sum():
    """kern/pow2.rs:137-166."""
    for acc in [0, 1, -1, 3, -3, 1 << 40, -(1 << 40), I64_MAX, I64_MIN, 12_345_678]:
        for s in range(96):
            if s <= 64:
                v = ((acc << s) + (1 << 31)) >> 32
                want = v if I64_MIN <= v <= I64_MAX else None
            else:
                v = acc * (1 << (s - 32))
                want = v if I64_MIN <= v <= I64_MAX else None
            assert O.finish(acc, s) == want, (acc, s)


def _f64_formula(bits):
    """The pre-conversion body of f32_convert.rs:80-97: round(f64(v)*2^32), half away
    from zero, None for non-finite or outside [-2^63, 2^63)."""
    v = np.array([bits], dtype=np.uint32).view(np.float32)[0]
    if not np.isfinite(v):
        return None
    q = Fraction(float(v)) * (1 << 32)
    r = int(abs(q) + Fraction(1, 2))
    r = -r if q < 0 else r
    return r if -(1 << 63) <= r < (1 << 63) else None


def test_f32_to_fixed_equals_f64_formula():
    """f32_convert.rs:106-150 (edges) and fp.rs:640-660, sampled with the same LCG."""
    f = lambda x: int(np.array([x], dtype=np.float32).view(np.uint32)[0])
    edges = [0.0, -0.0, 0.5, -0.5, 2.0**31, -(2.0**31), 2.0**32, -(2.0**32), 2.0**-33,
             -(2.0**-33), np.inf, -np.inf, np.nan]
    edge_bits = [f(e) for e in edges] + [1, 0x80000001, 0x00800000, 0x80800000, 0x007FFFFF,
                                         0x4EFFFFFF, 0xCF000001, 0x7F7FFFFF, 0xFF7FFFFF]
    for b in edge_bits:
        assert O.f32_to_q32(b) == _f64_formula(b), hex(b)
    seed = 0x0BAD5EED00000002
    for _ in range(4000):
        seed = lcg_next(seed)
        anyb = seed >> 32
        assert O.f32_to_q32(anyb) == _f64_formula(anyb), hex(anyb)
        seed = lcg_next(seed)
        e = 100 + seed % 60
        ranged = (anyb & 0x80000000) | (e << 23) | (anyb & 0x007FFFFF)
        assert O.f32_to_q32(ranged) == _f64_formula(ranged), hex(ranged)


def test_quant_act_known_answers():
    """chart/tests.rs:373-416 and native_gpu_probe.rs:623-697."""
    codes, scales = O.quant_act([3, 130, -3])
    assert codes[0] == 2 and codes[2] == -2  # ties away from zero
    codes, scales = O.quant_act(np.zeros(64, dtype=np.int64))
    assert not codes.any() and not scales.any()
    assert O.quant_act([I64_MAX] * 32) is None
    codes, scales = O.quant_act([I64_MIN] * 32)
    assert list(scales) == [1 << 57]
    assert list(O.dequant_act(codes, scales)) == [I64_MIN] * 32
    codes, scales = O.quant_act([127 << 56] * 32)
    assert list(O.dequant_act(codes, scales)) == [127 << 56] * 32
    got = [O.quant_act(pop.unit_at(v)) for v in (127, -127, 128, -128)]
    assert [s[0] for _, s in got] == [1, 1, 2, 2]
    assert [c[0] for c, _ in got] == [127, -127, 64, -64]
    x = [0] * 32
    x[:3] = [3, -3, 130]
    codes, scales = O.quant_act(x)
    assert list(scales) == [2] and list(codes[:3]) == [2, -2, 65]
    mixed = [0] * 64
    for lane in range(32):
        mixed[lane] = 127 if lane % 2 == 0 else -127
        mixed[32 + lane] = (63 << 57) if lane % 2 == 0 else -(63 << 57)
    codes, scales = O.quant_act(mixed)
    assert list(scales) == [1, 1 << 56] and codes[0] == 127 and codes[32] == 126
    for v, c in ((63 << 57, 126), (-(63 << 57), -126)):
        codes, scales = O.quant_act(pop.unit_at(v))
        assert list(scales) == [1 << 56] and codes[0] == c
    assert O.quant_act([I64_MIN, I64_MAX]) is None


def test_quant_act_bounds_and_dequant_contract():
    """chart/tests.rs:373-395: |xq| <= 127, |x - S*xq| <= S/2, zero scale gives zero code."""
    for seed in range(16):
        x = random_x(200, 0x5EED1000 + seed) * 1_000_003
        codes, scales = O.quant_act(x)
        deq = O.dequant_act(codes, scales)
        s = np.repeat(scales, 32)[:200]
        assert np.all(np.abs(codes.astype(np.int64)) <= 127)
        assert np.all(codes[s == 0] == 0)
        assert np.all(2 * np.abs(x - deq) <= s)


def _digest(values):
    v = np.array([0 if x is None else x for x in values], dtype="<i8")
    f = np.array([1 if x is None else 0 for x in values], dtype="<u4")
    return hashlib.sha256(v.tobytes() + f.tobytes()).hexdigest()


def test_native_probe_populations():
    """native_gpu_probe.rs:187-240, 350-373: 14 cases, 4 refusing, 14,678 values and
    32 refusals; case 6's first outputs [1, 0, 2, -1]; per-case refusal flags."""
    cases = pop.populations()
    assert len(cases) == 14 and sum(c["refusal"] for c in cases) == 4
    digests = json.load(open(os.path.join(HERE, "golden", "populations_digest.json")))
    some = refused = 0
    for c, d in zip(cases, digests["synthetic"]):
        vals = pop.exact_outputs(c, O.exact_dot_q8_0)
        assert all((v is None) == c["refusal"] for v in vals), c["id"]
        if c["id"] == 6:
            assert vals[:4] == [1, 0, 2, -1]
        some += sum(v is not None for v in vals)
        refused += sum(v is None for v in vals)
        assert _digest(vals) == d["sha256"], c["id"]
    assert (some, refused) == (14_678, 32)


def test_real_quantizer_populations():
    """native_gpu_probe.rs:696-813: the tails of 106/107 are non-zero values, 108
    narrows past i64, 109/110 overflow the i128 accumulator, 111 cancels to 0, 105
    refuses its non-finite rows."""
    cases = pop.real_quantizer_populations(O.quant_act)
    digests = json.load(open(os.path.join(HERE, "golden", "populations_digest.json")))
    assert len(cases) == 12
    for c, d in zip(cases, digests["real_quantizer"]):
        vals = pop.exact_outputs(c, O.exact_dot_q8_0)
        assert _digest(vals) == d["sha256"], c["id"]
        if c["id"] in (106, 107):
            assert vals[-1] is not None and vals[-1] != 0
        if c["id"] in (108, 109, 110):
            assert vals == [None]
        if c["id"] == 111:
            assert vals == [0]
        if c["id"] == 105:
            assert vals[0] is not None and vals[1] is None and vals[2] is None
    q = cases[9]
    assert np.all(q["scales"] == 1 << 56) and np.all(q["codes"] == 126)


def _fused_equals_fixed(t, raw, rows, n_in, x):
    q = O.quant_act(x)
    assert q is not None
    codes, scales = q
    deq = O.dequant_act(codes, scales)
    a = O.matvec_q8act(t, raw, rows, n_in, codes, scales)
    b = O.matvec_fixed(t, raw, rows, n_in, deq)
    if isinstance(a, tuple) or isinstance(b, tuple):
        assert a == b
    else:
        assert np.array_equal(a, b)
    return a


@pytest.mark.parametrize("t", [Q8_0, Q5_0, Q4_K, Q6_K])
def test_fused_rows_equal_contract_on_random_payloads(t):
    """chart/tests.rs:224-271 (`chart_matches_fixed_on_random_payloads_for_every_family`)."""
    seed = 0x123456789ABCDEF0
    for rows, n_in in [(4, 32), (3, 48), (2, 33), (2, 300), (1, 64), (5, 0), (1, 256),
                       (2, 512), (2, 256)]:
        seed = lcg_next(seed)
        raw = random_payload(t, rows, n_in, 0x3800, 0x3800, seed)
        x = random_x(n_in, seed ^ 0xDEADBEEF)
        _fused_equals_fixed(t, raw, rows, n_in, x)


@pytest.mark.parametrize("t", [Q8_0, Q5_0, Q4_K, Q6_K])
def test_fused_rows_equal_contract_on_extremes_and_ragged(t):
    """chart/tests.rs:273-334: +-127 codes against 0x7BFF scales; ragged widths."""
    raw = random_payload(t, 2, 256, 0x7BFF, 0x7BFF, 0x51FF0000 + t)
    codes = np.array([127 if j % 2 == 0 else -127 for j in range(256)], dtype=np.int8)
    scales = np.ones(8, dtype=np.int64)
    a = O.matvec_q8act(t, raw, 2, 256, codes, scales)
    b = O.matvec_fixed(t, raw, 2, 256, O.dequant_act(codes, scales))
    assert (a == b) if isinstance(a, tuple) else np.array_equal(a, b)
    for n_in in [33, 47, 65, 257, 300, 271]:
        raw = random_payload(t, 2, n_in, 0x3800, 0x3800, 0x7000 + t)
        _fused_equals_fixed(t, raw, 2, n_in, random_x(n_in, 0xABC0 ^ n_in))


def test_zero_activation_blocks():
    """chart/tests.rs:338-370."""
    x = np.zeros(96, dtype=np.int64)
    x[64:] = 1000 - 100 * np.arange(64, 96)
    codes, scales = O.quant_act(x)
    assert not codes[:64].any() and scales[0] == 0 and scales[1] == 0
    for i, t in enumerate([Q8_0, Q4_K, Q6_K]):
        raw = random_payload(t, 1, 96, 0x3800, 0x3800, 0x9000 + i)
        _fused_equals_fixed(t, raw, 1, 96, x)


def test_refusals_follow_the_contract():
    """A non-finite scale refuses with its bits at the first bad row; an output past
    i64 refuses with OutputOverflow (ops/matvec.rs:11-48, chart/mod.rs:1777-1859)."""
    raw = random_payload(Q8_0, 4, 64, 0x3800, 0x3800, 77)
    raw[2 * 68 + 34:2 * 68 + 36] = (0x01, 0x7C)  # row 2, block 1: +Inf
    codes, scales = O.quant_act(random_x(64, 5))
    r = O.matvec_q8act(Q8_0, raw, 4, 64, codes, scales)
    assert r[:2] == ("err", 6) and r[4] == 0x7C01
    big = random_payload(Q8_0, 2, 32, 0x7BFF, 0x7BFF, 3)
    big[2:34] = 127
    c = np.full(32, 127, dtype=np.int8)
    s = np.array([1 << 40], dtype=np.int64)
    r = O.matvec_q8act(Q8_0, big, 2, 32, c, s)
    assert r[:2] == ("err", 9)
    assert O.matvec_fixed(Q8_0, big, 2, 32, O.dequant_act(c, s))[:2] == ("err", 9)
    # ShortPayload is checked before any row (chart/mod.rs:1906-1921).
    assert O.matvec_q8act(Q8_0, big, 3, 32, c, s)[:2] == ("err", 3)


def test_short_payload_and_shape_order():
    """chart/mod.rs:1906-1921 vs ffn.rs:679-697: the chunked entry checks the payload
    before the shape."""
    raw = random_payload(Q8_0, 2, 64, 0x3800, 0x3800, 9)
    codes, scales = O.quant_act(random_x(32, 1))
    assert O.matvec_q8act(Q8_0, raw, 3, 64, codes, scales)[:2] == ("err", 1)
    assert O.matvec_q8act_chunked(Q8_0, raw, 3, 64, codes, scales, 4)[:2] == ("err", 3)
    codes, scales = O.quant_act(random_x(64, 1))
    r = O.matvec_q8act(Q8_0, raw, 3, 64, codes, scales)
    assert r == ("err", 3, 3 * 68, 2 * 68, 0)


@pytest.mark.parametrize("t", [Q8_0, Q5_0, Q4_K, Q6_K])
def test_matmat_and_threads_equal_per_column(t):
    """kern/matmat.rs:92-134: column c equals the per-column call; the threaded CPU
    baseline equals the single-threaded rows."""
    n_in, rows, k = 512, 37, 5
    raw = random_payload(t, rows, n_in, 0x3000, 0x2C00, 1234 + t)
    cs, ss = zip(*[O.quant_act(random_x(n_in, 99 + c) * (c + 1)) for c in range(k)])
    codes, scales = np.stack(cs), np.stack(ss)
    mm = O.matmat_q8act(t, raw, rows, n_in, codes, scales)
    for c in range(k):
        assert np.array_equal(mm[c], O.matvec_q8act(t, raw, rows, n_in, codes[c], scales[c]))
    assert np.array_equal(mm, O.matmat_q8act_mt(t, raw, rows, n_in, codes, scales, 4))
    assert np.array_equal(mm[0], O.matvec_q8act_mt(t, raw, rows, n_in, codes[0], scales[0], 3))


def test_block_dots_rebuild_the_q8_0_value():
    """The exact int32 block dots recombine to exact_dot (gemm.rs:470-486)."""
    raw = random_payload(Q8_0, 3, 128, 0x3800, 0, 5)
    codes, scales = O.quant_act(random_x(128, 8))
    dots = O.block_dots(Q8_0, raw, 3, 128, codes)
    for r in range(3):
        acc = 0
        for b in range(4):
            h = int(raw[r * 136 + b * 34]) | int(raw[r * 136 + b * 34 + 1]) << 8
            acc += O.f16_to_fixed(h) * int(scales[b]) * int(dots[r, b])
        want = O.exact_dot_q8_0(raw[r * 136:(r + 1) * 136], 4, codes, scales)
        assert O.round_shift_32(acc) == want


def test_q5_0_fused_rows_take_the_fast_path_and_equal_the_contract():
    """The Q5_0 fused row (chart/mod.rs:630-712: one pure group per block, w = d·(c − 16))
    against matvec_fixed on the dequantized activation, on whole-block widths under the narrow
    bound (top 16) and on ragged widths, which take the contract."""
    for rows, n_in, seed in [(7, 64, 1), (3, 896, 2), (5, 4864, 3), (4, 33, 4), (2, 300, 5)]:
        raw = random_payload(Q5_0, rows, n_in, 0x3800, 0, 0x5000 + seed)
        for xs in (random_x(n_in, seed), random_x(n_in, seed) << 20):
            _fused_equals_fixed(Q5_0, raw, rows, n_in, xs)
    raw = random_payload(Q5_0, 3, 64, 0x7BFF, 0, 77)
    codes = np.array([127 if j % 3 else -127 for j in range(64)], dtype=np.int8)
    for s in (1, 1 << 40):
        scales = np.full(2, s, dtype=np.int64)
        a = O.matvec_q8act(Q5_0, raw, 3, 64, codes, scales)
        b = O.matvec_fixed(Q5_0, raw, 3, 64, O.dequant_act(codes, scales))
        assert (a == b) if isinstance(a, tuple) else np.array_equal(a, b)
