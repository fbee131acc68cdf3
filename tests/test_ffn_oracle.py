"""The oracle's restatement of the FFN hidden activation (SwiGLU, then quant_act of h) against
the reference's own known answers and its f32-carrier parity test.

Known answers: silu_fixed / fixed_exp (src/engine/tests.rs:946-965,
src/numeric/fixed_exp.rs tests `zero_and_boundaries`, `accuracy_against_f64_exp`), the
hand-computed SwiGLU (src/engine/tests.rs:967-987).  exp_f32_scalar equals the native-f32 body it
replaced on random bit patterns and a sweep (src/engine/mixer/f32_carrier_tests.rs:299-357); that
body is restated here with numpy binary32 arithmetic (one rounding per operation, as in Rust).
"""
import math

import numpy as np

from oracle import oracle as O

ONE = 1 << 32
LN2_Q32 = 2_977_044_472
I64_MIN, I64_MAX = -(1 << 63), (1 << 63) - 1


def test_silu_fixed_known_answers():
    assert O.silu_fixed(0) == 0
    assert O.fixed_exp(-LN2_Q32) == ONE // 2
    assert O.silu_fixed(LN2_Q32) == 1_984_696_315
    assert O.fixed_exp(LN2_Q32) == 2 * ONE
    assert O.silu_fixed(-LN2_Q32) == -992_348_157
    assert O.silu_fixed(16 * ONE) == 16 * ONE
    assert O.silu_fixed(16 * ONE + 1) == 16 * ONE + 1
    assert O.silu_fixed(-21 * ONE) == 0
    assert O.silu_fixed(-21 * ONE - 1) == 0
    assert O.silu_fixed(I64_MIN) == 0
    assert O.silu_fixed(I64_MAX) == I64_MAX


def test_fixed_exp_window_and_accuracy():
    assert O.fixed_exp(0) == ONE
    assert O.fixed_exp(-16 * ONE) is not None and O.fixed_exp(21 * ONE) is not None
    for x in (-16 * ONE - 1, 21 * ONE + 1, I64_MIN, I64_MAX):
        assert O.fixed_exp(x) is None
    # the reference's tolerance (1e-8 relative + 4 ulp of Q32.32), on a coarser grid
    step = ONE // 16
    for x in range(-16 * ONE, 21 * ONE + 1, step):
        want = math.exp(x / ONE)
        got = O.fixed_exp(x) / ONE
        assert abs(got - want) <= 1e-8 * want + 4.0 / ONE, x


def _old_exp(x):
    """The native binary32 body exp_f32_scalar replaced, one numpy float32 rounding per op."""
    f = np.float32
    x = f(x)
    if np.isnan(x):
        return f(np.nan)
    if x < f(-88.0):
        return f(0.0)
    if x > f(88.72284):
        return f(np.inf)
    z = x * f(1.44269504)
    n_flt = f(np.rint(z))
    n_int = int(n_flt)
    r = (x - n_flt * f(0.693359375)) - n_flt * f(-2.1219444e-4)
    r2 = r * r
    p = f(1.9875691e-4)
    for c in (1.3981999e-3, 8.333452e-3, 4.1665796e-2, 1.6666666e-1, 5.0e-1):
        p = p * r + f(c)
    y = (f(1.0) + r) + (r2 * p)
    n1 = n_int >> 1
    n2 = n_int - n1
    s1 = np.array([(n1 + 127) << 23], dtype=np.uint32).view(np.float32)[0]
    s2 = np.array([(n2 + 127) << 23], dtype=np.uint32).view(np.float32)[0]
    return (y * s1) * s2


def _bits(v):
    return int(np.array([v], dtype=np.float32).view(np.uint32)[0])


def test_exp_f32_equals_native_body():
    rng = np.random.default_rng(0x0E57)
    with np.errstate(all="ignore"):
        for b in rng.integers(0, 1 << 32, 4000, dtype=np.uint64):
            want = _old_exp(np.array([b], dtype=np.uint32).view(np.float32)[0])
            got = O.exp_f32(int(b))
            assert got == _bits(want) or (np.isnan(want) and (got & 0x7FFFFFFF) > 0x7F800000), hex(int(b))
        x = np.float32(-90.0)
        while x <= np.float32(90.0):
            assert O.exp_f32(_bits(x)) == _bits(_old_exp(x)), float(x)
            x = np.float32(x + np.float32(0.0137))


def test_swiglu_carriers():
    # the hand-computed SwiGLU: gate = ln 2, up = 1 gives silu(ln 2) (Q32 carrier)
    assert O.swiglu(LN2_Q32, ONE, O.CARRIER_Q32) == 1_984_696_315
    rng = np.random.default_rng(7)
    f = np.float32
    with np.errstate(all="ignore"):
        for g, u in rng.integers(-40 * ONE, 40 * ONE, (500, 2)):
            gf = f(np.float32(int(g))) * f(2.0 ** -32)
            uf = f(np.float32(int(u))) * f(2.0 ** -32)
            s = gf / (f(1.0) + _old_exp(-gf))
            prod = s * uf
            want = O.f32_to_q32(_bits(prod))
            got = O.swiglu(int(g), int(u), O.CARRIER_F32)
            assert got == (want if want is not None else ("err", O.FFN_OVERFLOW)), (g, u)
            # the Q32 carrier agrees with the real function to a few ulp of Q32.32 per unit
            q = O.swiglu(int(g), int(u), O.CARRIER_Q32)
            real = (g / ONE) / (1 + math.exp(-g / ONE)) * (u / ONE)
            assert abs(q / ONE - real) <= 1e-6 * max(1.0, abs(real)), (g, u)
    # |h| >= 2^31 leaves Q32.32: Overflow under both carriers
    assert O.swiglu(30 * ONE, (1 << 61), O.CARRIER_F32) == ("err", O.FFN_OVERFLOW)
    assert O.swiglu(30 * ONE, (1 << 61), O.CARRIER_Q32) == ("err", O.FFN_OVERFLOW)


def test_swiglu_quant_refusal_order():
    gate = np.full(64, ONE, dtype=np.int64)
    up = np.full(64, ONE, dtype=np.int64)
    gate[[9, 5]] = 30 * ONE
    up[[9, 5]] = 1 << 61
    assert O.swiglu_quant(gate, up, O.CARRIER_F32) == ("swiglu", 5, O.FFN_OVERFLOW)
    h, codes, scales = O.swiglu_quant(np.full(40, ONE, np.int64), np.full(40, ONE, np.int64))
    assert h.shape == (40,) and codes.shape == (40,) and scales.shape == (2,)
