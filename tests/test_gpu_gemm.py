"""GPU parity of the prefill contract on the int8 tensor cores (tcgen05 GEMM, Q8_0).

Every multi-column Q8_0 call with at least four columns takes the GEMM; columns the GEMM's
i64 fold cannot take exactly (a code of -128, a wide exponent spread, the reference's call
bound failing) take the checked row path inside the same launch.  Bar: bit-exact Q32.32
outputs against the oracle's per-column contract (src/engine/kern/matmat.rs:92-134),
identical refusals with the lowest refusing column, and f32 outputs identical to the
single-column f32 boundary.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from chart_inputs import random_payload, random_x
from apeiron_b200 import chart, synth
from apeiron_b200.chart import Backend, QuantAct

pytestmark = pytest.mark.gpu

Q8_0 = 8
KIND = {1: chart.ShapeMismatch, 3: chart.ShortPayload, 4: chart.LengthOverflow,
        6: chart.NonFiniteScale, 7: chart.FixedOverflow, 8: chart.AccumulatorOverflow,
        9: chart.OutputOverflow}
THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    yield b
    b.close()


def bench_columns(n_in, k, seed):
    """k benchmark activations (f32 N(0,1) through f32_to_fixed and quant_act)."""
    qs = []
    for c in range(k):
        x = synth.f32_to_q32(synth.activation_f32(n_in, seed + c))
        codes, exps = synth.quant_act_np(x)
        qs.append(QuantAct.from_exps(exps, codes))
    return qs


def stack(qs):
    return (np.stack([q.codes for q in qs]), np.stack([q.scales for q in qs]))


def check_matmat(be, raw, n_out, n_in, qs, threads=1):
    codes, scales = stack(qs)
    if threads > 1:
        want = O.matmat_q8act_mt(Q8_0, raw, n_out, n_in, codes, scales, threads)
    else:
        want = O.matmat_q8act(Q8_0, raw, n_out, n_in, codes, scales)
    try:
        got = be.matmat_q8act(Q8_0, raw, n_out, n_in, qs)
    except chart.MatvecError as e:
        assert isinstance(want, tuple), f"GPU refused {e!r}, oracle gave values"
        assert isinstance(e, KIND[want[1]]), (e, want)
        assert e.col == want[5], (e.col, want)
        return e
    assert not isinstance(want, tuple), f"GPU gave values, oracle refused {want}"
    assert np.array_equal(np.stack(got), want)
    return got


@pytest.mark.parametrize("n_out,n_in", [(4864, 896), (896, 4864)])
def test_prefill_benchmark_shapes_512_tokens(be, n_out, n_in):
    """The prefill configuration: 512 tokens against both Qwen2.5-0.5B FFN shapes."""
    raw = synth.payload(Q8_0, n_out, n_in, 31 + n_out)
    check_matmat(be, raw, n_out, n_in, bench_columns(n_in, 512, 1000), threads=THREADS)


@pytest.mark.parametrize("n_out,n_in,k", [
    (200, 100, 70),     # ragged K (not a multiple of 32), partial row and token tiles
    (130, 1000, 5),
    (1, 32, 4),
    (129, 4000, 65),
    (257, 96, 129),
    (64, 15360, 8),     # the widest K one CTA's exponent table holds
])
def test_ragged_shapes(be, n_out, n_in, k):
    raw = random_payload(Q8_0, n_out, n_in, 0x3000, 0x2C00, n_out * 7 + n_in)
    qs = [_col(n_in, 17 + c, c % 5) for c in range(k)]
    check_matmat(be, raw, n_out, n_in, qs)


def _col(n_in, seed, shift=0):
    c, s = O.quant_act(random_x(n_in, seed) >> shift)
    return QuantAct.from_parts(s, c)


def test_zero_and_sparse_columns(be):
    """All-zero tokens, zero-scale blocks holding stray codes, and a single live block."""
    n_out, n_in, k = 300, 640, 9
    raw = random_payload(Q8_0, n_out, n_in, 0x3400, 0x2800, 5)
    qs = [_col(n_in, 40 + c) for c in range(k)]
    qs[1] = QuantAct.from_parts(np.zeros(n_in // 32, np.int64), np.zeros(n_in, np.int8))
    s = qs[2].scales.copy()
    s[::3] = 0                      # zero scales: their codes must not count
    qs[2] = QuantAct.from_parts(s, qs[2].codes)
    s = np.zeros(n_in // 32, np.int64)
    s[7] = 1 << 20
    qs[3] = QuantAct.from_parts(s, np.full(n_in, 127, np.int8))
    check_matmat(be, raw, n_out, n_in, qs)


def test_checked_route_columns(be):
    """Columns the i64 fold does not take: a -128 code, a 25-exponent activation spread,
    a scale of 2^56 (the reference's call bound fails); their values come from the checked
    rows.  A bound-failing column that overflows refuses like the oracle."""
    n_out, n_in, k = 260, 512, 8
    raw = random_payload(Q8_0, n_out, n_in, 0x3000, 0x2C00, 9)
    qs = [_col(n_in, 60 + c) for c in range(k)]
    c = qs[1].codes.copy()
    c[5] = -128
    qs[1] = QuantAct.from_parts(qs[1].scales, c)
    s = qs[3].scales.copy()
    s[0] = 1 << 2
    s[1] = 1 << 27
    qs[3] = QuantAct.from_parts(s, qs[3].codes)
    s = np.zeros(n_in // 32, np.int64)
    s[4] = 1 << 56
    c = np.zeros(n_in, np.int8)
    c[128:132] = (1, -1, 1, 1)
    qs[6] = QuantAct.from_parts(s, c)
    check_matmat(be, raw, n_out, n_in, qs)
    # the checked list resets itself: the same call again, then a plain call
    check_matmat(be, raw, n_out, n_in, qs)
    check_matmat(be, raw, n_out, n_in, [_col(n_in, 90 + c) for c in range(k)])
    # a bound-failing column large enough to overflow
    qs[5] = QuantAct.from_parts(np.full(n_in // 32, 1 << 57, np.int64), qs[5].codes // 2)
    check_matmat(be, raw, n_out, n_in, qs)


def test_activation_spreads_through_the_fold(be):
    """GEMM columns whose block exponents lie 3..11 above their smallest: the fold shifts each
    block's dot by s before its multiply-add (12 takes the checked rows).  Rows whose codes are
    all -128 or all 127 against codes of ±127 make the shifted dots reach their int32 bound
    (32·128·127·2^11 < 2^31); the other rows hold every code."""
    n_out, n_in, k = 256, 1024, 12
    raw = random_payload(Q8_0, n_out, n_in, 0x3000, 0, 21)
    blk = raw.reshape(n_out, -1, 34)
    blk[:16, :, 2:] = 0x80
    blk[16:32, :, 2:] = 0x7F
    rng = np.random.default_rng(21)
    nb = n_in // 32
    qs = []
    for c in range(k):
        s = np.full(nb, 1 << 8, np.int64)
        s[rng.choice(nb, 5, replace=False)] = 1 << (8 + 3 + c % 10)   # spreads 3..12
        if c % 3 == 2:
            codes = rng.integers(-127, 128, n_in).astype(np.int8)
        else:
            codes = np.full(n_in, 127 if c % 3 else -127, np.int8)
        qs.append(QuantAct.from_parts(s, codes))
    check_matmat(be, raw, n_out, n_in, qs)


def test_weight_spread_bounds_the_activation_shift(be):
    """Rows whose block scales span 2^20 (f16 2^-14 beside 64): the i64 fold then allows an
    activation spread of at most 32 − 20 − log2(nb) = 7 on this tensor, so columns at 6 and 7
    take the GEMM and 8 the checked rows; all equal the oracle."""
    n_out, n_in, k = 192, 1024, 6
    raw = random_payload(Q8_0, n_out, n_in, 0x0400, 0, 22)
    raw.reshape(n_out, -1, 34)[:, 1::2, 0:2] = (0x00, 0x54)
    rng = np.random.default_rng(22)
    nb = n_in // 32
    qs = []
    for spread in (6, 7, 8, 7, 6, 8):
        s = np.full(nb, 1 << 20, np.int64)
        s[rng.choice(nb, 3, replace=False)] = 1 << (20 + spread)
        qs.append(QuantAct.from_parts(s, rng.integers(-127, 128, n_in).astype(np.int8)))
    check_matmat(be, raw, n_out, n_in, qs)


def test_refusals_lowest_column(be):
    """FixedOverflow and OutputOverflow in different columns: the lowest refusing column
    decides, and within it the first row in row order."""
    n_out, n_in, k = 140, 256, 6
    raw = random_payload(Q8_0, n_out, n_in, 0x7BFF, 0, 11)   # every scale 65504
    base = [_col(n_in, 70 + c) for c in range(k)]
    fixed = QuantAct.from_parts(np.full(n_in // 32, 1 << 60, np.int64),
                                np.full(n_in, 127, np.int8))
    c, s = O.quant_act(random_x(n_in, 77) << 30)
    big = QuantAct.from_parts(s, c)
    for pos_fixed, pos_big in [(4, 2), (1, 3), (5, 0)]:
        qs = list(base)
        qs[pos_fixed] = fixed
        qs[pos_big] = big
        e = check_matmat(be, raw, n_out, n_in, qs)
        assert isinstance(e, chart.MatvecError) and e.col == min(pos_fixed, pos_big)


def test_output_overflow_row_order(be):
    """Large weights (every scale 65504) against growing activations: the GEMM's first
    overflowing row in the lowest overflowing column, values where nothing overflows."""
    n_out, n_in, k = 512, 1024, 4
    raw = random_payload(Q8_0, n_out, n_in, 0x7BFF, 0, 12)
    qs = []
    for c, sh in enumerate([0, 10, 30, 20]):
        cc, ss = O.quant_act(random_x(n_in, 80 + c) << sh)
        qs.append(QuantAct.from_parts(ss, cc))
    e = check_matmat(be, raw, n_out, n_in, qs)
    assert isinstance(e, chart.OutputOverflow) and e.col == 2
    check_matmat(be, raw, n_out, n_in, [qs[0], qs[1], qs[0], qs[1]])


def test_wide_weight_spread_and_nonfinite_weights(be):
    """Weights whose scales span subnormal to 65504 (no GEMM view: per-column GEMVs) and a
    non-finite weight scale (column 0 refuses with its bits)."""
    n_out, n_in, k = 96, 512, 5
    raw = synth.payload(Q8_0, n_out, n_in, 13)
    blk = raw.reshape(n_out, -1)[3].reshape(-1, 34)
    blk[0, 0:2] = (0x01, 0x00)   # smallest subnormal
    blk[1, 0:2] = (0xFF, 0x7B)   # 65504
    check_matmat(be, raw, n_out, n_in, [_col(n_in, 85 + c) for c in range(k)])
    raw2 = synth.payload(Q8_0, n_out, n_in, 14)
    raw2.reshape(n_out, -1)[50].reshape(-1, 34)[2, 0:2] = (0x00, 0x7C)   # +Inf
    e = check_matmat(be, raw2, n_out, n_in, [_col(n_in, 86 + c) for c in range(k)])
    assert isinstance(e, chart.NonFiniteScale) and e.col == 0


@pytest.mark.parametrize("n_out,n_in,k", [(4864, 896, 512), (896, 4864, 64), (200, 100, 7)])
def test_f32_boundary_matches_matvec_f32(be, n_out, n_in, k):
    """matmat_f32 (device quantizer + GEMM, f32 epilogue) equals matvec_f32 per column."""
    raw = synth.payload(Q8_0, n_out, n_in, 21 + n_in)
    t = be.upload(Q8_0, raw, n_out, n_in)
    x = np.stack([synth.activation_f32(n_in, 500 + c) for c in range(k)])
    y = be.matmat_f32(t, x)
    for c in range(0, k, max(1, k // 16)):
        assert np.array_equal(y[c], be.matvec_f32(t, x[c])), c


def test_async_columns_match_sync(be):
    """apx_quant_f32_cols_async + apx_matmat_async over device buffers (torch allocates)
    equal the synchronous prefill call, Q32.32 and f32 outputs both."""
    import ctypes as C
    import torch

    from apeiron_b200 import _abi

    lib = be.lib
    n_out, n_in, k = 4864, 896, 96
    raw = synth.payload(Q8_0, n_out, n_in, 23)
    tens = be.upload(Q8_0, raw, n_out, n_in)
    x = np.stack([synth.activation_f32(n_in, 700 + c) for c in range(k)])
    dev = torch.device("cuda:0")
    dx = torch.from_numpy(x).to(dev)
    pad = lib.apx_act_padded_len(n_in)
    codes = torch.zeros(k * pad, dtype=torch.int8, device=dev)
    exps = torch.full((k * pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    descs = torch.zeros(k * 8, dtype=torch.int32, device=dev)
    q32 = torch.zeros(k * n_out, dtype=torch.int64, device=dev)
    f32 = torch.zeros(k * n_out, dtype=torch.float32, device=dev)
    status = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_quant_f32_cols_async(be.ctx, dx.data_ptr(), n_in, k, codes.data_ptr(),
                                        exps.data_ptr(), descs.data_ptr(), stream) == 0
    assert lib.apx_matmat_async(be.ctx, tens.handle, n_out, n_in, k, codes.data_ptr(),
                                exps.data_ptr(), descs.data_ptr(), q32.data_ptr(),
                                f32.data_ptr(), status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    st = status.cpu().numpy()
    for c in range(k):
        word = _abi.CallStatus(int(st[2 * c]) & ((1 << 64) - 1), 0)
        err = _abi.ApxErr()
        assert lib.apx_status_decode(be.ctx, tens.handle, C.byref(word), C.byref(err)) == 0
    qs = []
    for c in range(k):
        cc, ee = synth.quant_act_np(synth.f32_to_q32(x[c]))
        qs.append(QuantAct.from_exps(ee, cc))
    want = np.stack(be.matmat_q8act(Q8_0, tens, n_out, n_in, qs))
    assert np.array_equal(q32.cpu().numpy().reshape(k, n_out), want)
    assert np.array_equal(f32.cpu().numpy().reshape(k, n_out), be.matmat_f32(tens, x))


def _oracle_f32_column(raw, n_out, n_in, col):
    """The reference's f32 prefill of one column: f32_to_fixed, quant_act (None: refused
    with QuantRefused), then matvec_q8act; values or ("err", code, ...)."""
    v = [O.f32_to_q32(int(b)) for b in col.view(np.uint32)]
    if any(t is None for t in v):
        return ("err", 10)
    q = O.quant_act(np.array(v, dtype=np.int64))
    if q is None:
        return ("err", 10)
    codes, scales = q
    r = O.matmat_q8act_mt(Q8_0, raw, n_out, n_in, codes[None, :], scales[None, :], THREADS)
    return r if isinstance(r, tuple) else r[0]


@pytest.mark.parametrize("n_out,n_in,ldx", [(256, 896, 896), (200, 200, 204),
                                            (130, 4864, 4864), (64, 100, 100)])
def test_f32_fused_prep_matches_oracle(be, n_out, n_in, ldx):
    """apx_matmat_f32_async with f32_to_fixed + quant_act fused into the GEMM's prep kernel
    (Q8_0, at least 4 columns, 16-byte aligned rows): every block kind of the device
    quantizer beside ordinary columns, 70 columns so that the last column tile is ragged.
    Bar: Q32.32 outputs equal to the oracle's column by column; refused columns carry the
    oracle's refusal (QuantRefused for a column quant_act refuses); columns that take the
    checked route inside the GEMM (Q32.32 blocks beside tiny ones) are exact too."""
    import ctypes as C
    import torch

    from apeiron_b200 import _abi
    from chart_inputs import f32_block_kinds

    lib = be.lib
    raw = synth.payload(Q8_0, n_out, n_in, 31 + n_in)
    tens = be.upload(Q8_0, raw, n_out, n_in)
    kinds = f32_block_kinds(n_in, 5 + n_in)
    normal = np.stack([synth.activation_f32(n_in, 900 + c) for c in range(70 - len(kinds))])
    x = np.concatenate([normal[:20], kinds, normal[20:]]).astype(np.float32)
    k = x.shape[0]
    xp = np.zeros((k, ldx), dtype=np.float32)
    xp[:, :n_in] = x
    dev = torch.device("cuda:0")
    dx = torch.from_numpy(xp).to(dev)
    q32 = torch.zeros(k * n_out, dtype=torch.int64, device=dev)
    f32 = torch.zeros(k * n_out, dtype=torch.float32, device=dev)
    status = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_matmat_f32_async(be.ctx, tens.handle, n_out, n_in, k, dx.data_ptr(), ldx,
                                    q32.data_ptr(), f32.data_ptr(), status.data_ptr(),
                                    stream) == 0
    torch.cuda.synchronize()
    st = status.cpu().numpy()
    got = q32.cpu().numpy().reshape(k, n_out)
    gotf = f32.cpu().numpy().reshape(k, n_out)
    for c in range(k):
        word = _abi.CallStatus(int(st[2 * c]) & ((1 << 64) - 1), 0)
        err = _abi.ApxErr()
        rc = lib.apx_status_decode(be.ctx, tens.handle, C.byref(word), C.byref(err))
        want = _oracle_f32_column(raw, n_out, n_in, x[c])
        if isinstance(want, tuple):
            assert rc == want[1], (c, rc, want)
            continue
        assert rc == 0, (c, rc)
        assert np.array_equal(got[c], want), c
        assert np.array_equal(gotf[c], be.matvec_f32(tens, x[c])), c


def test_f32_sync_fused_matches_unfused(be):
    """The synchronous f32 prefill on an n_in that allows the fused prep (a multiple of 4)
    and one that does not (quantizer kernel, then the GEMM) both equal matvec_f32."""
    for n_in in (448, 450):
        raw = synth.payload(Q8_0, 192, n_in, 7 + n_in)
        t = be.upload(Q8_0, raw, 192, n_in)
        x = np.stack([synth.activation_f32(n_in, 40 + c) for c in range(9)])
        x[3, 17] = np.float32(np.nan)
        with pytest.raises(chart.MatvecError) as ei:
            be.matmat_f32(t, x)
        assert ei.value.col == 3
        x[3, 17] = 0.5
        y = be.matmat_f32(t, x)
        for c in range(9):
            assert np.array_equal(y[c], be.matvec_f32(t, x[c])), (n_in, c)


@pytest.mark.parametrize("t,n_out,n_in,k", [(Q8_0, 320, 450, 9), (12, 256, 512, 6),
                                            (Q8_0, 128, 256, 3)])
def test_f32_async_off_the_fused_route(be, t, n_out, n_in, k):
    """apx_matmat_f32_async where the fused prep does not apply: a width that is not a multiple
    of 4 (quantizer kernel, then the GEMM), a Q4_K tensor and a 3-column call (quantizer, then
    one GEMV per column).  Each column equals apx_matvec_f32 of it."""
    import torch

    lib = be.lib
    raw = synth.payload(t, n_out, n_in, 90 + n_in)
    tens = be.upload(t, raw, n_out, n_in)
    x = np.stack([synth.activation_f32(n_in, 300 + c) for c in range(k)])
    dev = torch.device("cuda:0")
    dx = torch.from_numpy(x).to(dev)
    f32 = torch.zeros(k * n_out, dtype=torch.float32, device=dev)
    status = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_matmat_f32_async(be.ctx, tens.handle, n_out, n_in, k, dx.data_ptr(), n_in,
                                    None, f32.data_ptr(), status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert bool((status == -1).all().item())
    y = f32.cpu().numpy().reshape(k, n_out)
    for c in range(k):
        assert np.array_equal(y[c], be.matvec_f32(tens, x[c])), c
