"""The timed CPU baseline's vector rows (oracle/apx_oracle_x86.c) equal the scalar fused rows.

The reference tests its AVX2 two-row cores the same way: `tiled2` against the scalar fast row on
every family and extreme payloads (src/engine/chart/x86.rs:1241-1347, chart/tests.rs:108-152).
Both builds run here: AVX-VNNI (when the host has it) and AVX2 (APXO_NO_VNNI=1).
"""
import numpy as np
import pytest

from oracle import oracle as O
from chart_inputs import random_payload, random_x
from apeiron_b200 import synth

Q8_0, Q4_K, Q6_K = O.Q8_0, O.Q4_K, O.Q6_K
Q5_0 = 6

pytestmark = pytest.mark.skipif(not O.simd_features()["avx2"], reason="host has no AVX2")


@pytest.fixture(params=["vnni", "avx2"])
def isa(request, monkeypatch):
    if request.param == "vnni":
        if not O.simd_features()["avxvnni"]:
            pytest.skip("host has no AVX-VNNI")
        monkeypatch.delenv("APXO_NO_VNNI", raising=False)
    else:
        monkeypatch.setenv("APXO_NO_VNNI", "1")
        assert not O.simd_features()["avxvnni"]
    return request.param


def _both(t, raw, rows, n_in, codes, scales, threads):
    a = O.matvec_q8act_mt(t, raw, rows, n_in, codes, scales, threads)
    b = O.matvec_q8act_mt(t, raw, rows, n_in, codes, scales, threads, simd=True)
    if isinstance(a, tuple) or isinstance(b, tuple):
        assert a == b
    else:
        assert np.array_equal(a, b)
    return b


@pytest.mark.parametrize("t,n_in", [(Q8_0, 32), (Q8_0, 96), (Q8_0, 896), (Q8_0, 4864),
                                    (Q4_K, 256), (Q4_K, 1536), (Q4_K, 896), (Q4_K, 64),
                                    (Q4_K, 320), (Q4_K, 448), (Q6_K, 512)])
@pytest.mark.parametrize("rows,threads", [(1, 1), (3, 1), (37, 3), (64, 8)])
def test_vector_rows_equal_scalar_rows(isa, t, n_in, rows, threads):
    raw = synth.payload(t, rows, n_in, seed=rows * 1000 + n_in)
    codes, scales = O.quant_act(synth.f32_to_q32(synth.activation_f32(n_in, seed=n_in)))
    out = _both(t, raw, rows, n_in, codes, scales, threads)
    assert not isinstance(out, tuple)
    # and the contract itself (matvec_fixed on the dequantized activation)
    ref = O.matvec_fixed(t, raw, rows, n_in, O.dequant_act(codes, scales))
    assert np.array_equal(out, ref)


@pytest.mark.parametrize("t", [Q8_0, Q4_K, Q6_K])
def test_vector_rows_on_random_bytes_and_extremes(isa, t):
    """Random header bytes (every Q4_K scale/min pattern), the largest finite scales against
    +-127 codes, and spread activation exponents."""
    for seed, d, dmin in [(11, 0x3800, 0x3800), (12, 0x7BFF, 0x7BFF), (13, 0x0001, 0x8001),
                          (14, 0x3C00, 0xBC00)]:
        raw = random_payload(t, 9, 512, d, dmin, seed)
        x = random_x(512, seed) * (1 << (seed % 5) * 7)
        codes, scales = O.quant_act(x)
        _both(t, raw, 9, 512, codes, scales, 2)
    raw = random_payload(t, 2, 256, 0x7BFF, 0x7BFF, 0x51FF0000 + t)
    codes = np.array([127 if j % 2 == 0 else -127 for j in range(256)], dtype=np.int8)
    _both(t, raw, 2, 256, codes, np.ones(8, dtype=np.int64), 1)


@pytest.mark.parametrize("t", [Q8_0, Q4_K, Q6_K])
def test_vector_rows_refusals(isa, t):
    """A non-finite block scale and an output past i64 refuse exactly as the scalar rows do
    (both redecided by the single-threaded contract)."""
    n_in, rows = 256, 6
    raw = random_payload(t, rows, n_in, 0x3800, 0x3800, 77 + t)
    qk, bb, at = {Q8_0: (32, 34, 0), Q4_K: (256, 144, 0), Q6_K: (256, 210, 208)}[t]
    row_bytes = (n_in // qk) * bb
    bad = raw.copy()
    bad[3 * row_bytes + at:3 * row_bytes + at + 2] = (0x01, 0x7C)  # row 3, block 0: NaN
    codes, scales = O.quant_act(random_x(n_in, 5))
    r = _both(t, bad, rows, n_in, codes, scales, 2)
    assert r[:2] == ("err", 6) and r[4] == 0x7C01
    big = random_payload(t, rows, n_in, 0x7BFF, 0x7BFF, 3)
    c = np.full(n_in, 127, dtype=np.int8)
    s = np.full(n_in // 32, 1 << 40, dtype=np.int64)
    r = _both(t, big, rows, n_in, c, s, 3)
    assert isinstance(r, tuple)


def test_vector_rows_take_minus_128_codes_on_the_scalar_rows(isa):
    """A -128 activation code (outside quant_act's range, but accepted by the C ABI) cannot
    use the |w|·sign(x, w) byte dot; the call takes the scalar rows and agrees."""
    raw = synth.payload(Q8_0, 5, 128, seed=3)
    codes = np.full(128, -128, dtype=np.int8)
    _both(Q8_0, raw, 5, 128, codes, np.ones(4, dtype=np.int64), 2)


@pytest.mark.parametrize("t", [Q8_0, Q4_K])
def test_vector_matmat_equals_per_column(isa, t):
    n_in, rows, k = 512, 21, 4
    raw = synth.payload(t, rows, n_in, seed=99)
    cs, ss = zip(*[O.quant_act(random_x(n_in, 7 + c) * (c + 1)) for c in range(k)])
    codes, scales = np.stack(cs), np.stack(ss)
    a = O.matmat_q8act_mt(t, raw, rows, n_in, codes, scales, 3)
    b = O.matmat_q8act_mt(t, raw, rows, n_in, codes, scales, 3, simd=True)
    assert np.array_equal(a, b)
    for c in range(k):
        assert np.array_equal(b[c], O.matvec_q8act(t, raw, rows, n_in, codes[c], scales[c]))


def _f16(v):
    return np.array([v], dtype=np.float16).view(np.uint8)


@pytest.mark.parametrize("n_out,n_in,k", [(37, 896, 13), (16, 256, 8), (5, 4864, 3),
                                          (64, 1024, 64), (1, 32, 1)])
def test_q8_0_gemm_equals_per_column(n_out, n_in, k):
    """The k-column Q8_0 GEMM of the prefill baseline (kern/gemm.rs:498-580, AVX-VNNI) equals
    the per-column fused rows, on the benchmark distribution."""
    raw = synth.payload(Q8_0, n_out, n_in, seed=n_out + k)
    cs, ss = [], []
    for c in range(k):
        q = O.quant_act(synth.f32_to_q32(synth.activation_f32(n_in, seed=500 + c)))
        cs.append(q[0])
        ss.append(q[1])
    codes, scales = np.stack(cs), np.stack(ss)
    want = O.matmat_q8act(Q8_0, raw, n_out, n_in, codes, scales)
    calls = O.gemm_counts()[0]
    got = O.matmat_q8act_mt(Q8_0, raw, n_out, n_in, codes, scales, 4, simd=True)
    assert np.array_equal(want, got)
    assert O.gemm_counts()[0] == calls + (1 if O.simd_features()["avxvnni"] else 0)


def test_q8_0_gemm_wide_spreads_take_the_exact_dots():
    """Weight exponent spreads (subnormal against 65504 scales) and activation spreads that
    pass the i64 shift limit (29 at 16 blocks) fall to the exact i128 dot per (row, group),
    with the same values; a zero block and an all-zero column fold to zero."""
    n_out, n_in, k = 9, 512, 11
    raw = synth.payload(Q8_0, n_out, n_in, seed=4).reshape(n_out, -1)
    raw[2, 0:2] = _f16(6e-8)                 # subnormal scale in row 2
    raw[2, 34:36] = _f16(60000.0)            # and the largest exponents beside it
    raw[5, 34 * 7:34 * 7 + 2] = _f16(2.0 ** -14)
    raw = raw.reshape(-1)
    cs, ss = [], []
    for c in range(k):
        x = synth.f32_to_q32(synth.activation_f32(n_in, seed=900 + c))
        if c % 3 == 1:
            b = c % 16 + 2                                # away from the 60000 scale
            x[32 * b:32 * b + 32] <<= 15                  # a block 2^15 above the rest
        if c == 4:
            x[64:96] = 0                                  # a zero block
        if c == 7:
            x[:] = 0                                      # an all-zero column
        q = O.quant_act(x)
        cs.append(q[0])
        ss.append(q[1])
    codes, scales = np.stack(cs), np.stack(ss)
    want = O.matmat_q8act(Q8_0, raw, n_out, n_in, codes, scales)
    assert not isinstance(want, tuple)
    calls, exact = O.gemm_counts()
    got = O.matmat_q8act_mt(Q8_0, raw, n_out, n_in, codes, scales, 3, simd=True)
    assert np.array_equal(want, got)
    if O.simd_features()["avxvnni"]:
        now = O.gemm_counts()
        assert now[0] == calls + 1 and now[1] > exact


def test_q8_0_gemm_refusals_fall_to_the_per_column_rows():
    """A non-finite weight scale and an output outside i64 make the GEMM bail; the call then
    refuses exactly as the per-column contract does (lowest column, first row)."""
    n_out, n_in, k = 6, 256, 5
    raw = synth.payload(Q8_0, n_out, n_in, seed=8).reshape(n_out, -1)
    raw[4, 34 * 3:34 * 3 + 2] = (0x00, 0x7C)  # +Inf
    raw = raw.reshape(-1)
    cs, ss = zip(*[O.quant_act(random_x(n_in, 40 + c)) for c in range(k)])
    codes, scales = np.stack(cs), np.stack(ss)
    want = O.matmat_q8act(Q8_0, raw, n_out, n_in, codes, scales)
    got = O.matmat_q8act_mt(Q8_0, raw, n_out, n_in, codes, scales, 2, simd=True)
    assert want == got and want[:2] == ("err", 6)
    big = random_payload(Q8_0, n_out, n_in, 0x7BFF, 0x7BFF, 3)
    c = np.full((k, n_in), 127, dtype=np.int8)
    s = np.full((k, n_in // 32), 1 << 40, dtype=np.int64)
    s[:2] = 1
    want = O.matmat_q8act(Q8_0, big, n_out, n_in, c, s)
    got = O.matmat_q8act_mt(Q8_0, big, n_out, n_in, c, s, 2, simd=True)
    assert want == got and isinstance(want, tuple)


@pytest.mark.parametrize("t,n_in", [(Q6_K, 896), (Q4_K, 300), (Q8_0, 33), (Q6_K, 300)])
@pytest.mark.parametrize("simd", [False, True])
def test_threaded_contract_rows_equal_single_threaded(t, n_in, simd):
    """Widths the fused rows do not take (ragged K-quants, a ragged Q8_0 block) run the contract,
    matvec_fixed on the dequantized activation, over the pool's row chunks, as the reference's
    chunked caller runs every row range on its pool (chart/ffn.rs:705-726); the values equal the
    single-threaded call, and a refusal is still redecided in row order."""
    rows = 29
    raw = random_payload(t, rows, n_in, 0x3800, 0x3800, 0x5150 + n_in)
    codes, scales = O.quant_act(random_x(n_in, 31))
    want = O.matvec_q8act(t, raw, rows, n_in, codes, scales)
    got = O.matvec_q8act_mt(t, raw, rows, n_in, codes, scales, 4, simd=simd)
    assert not isinstance(want, tuple) and np.array_equal(want, got)
    cs, ss = zip(*[O.quant_act(random_x(n_in, 60 + c)) for c in range(3)])
    mm = O.matmat_q8act(t, raw, rows, n_in, np.stack(cs), np.stack(ss))
    assert np.array_equal(mm, O.matmat_q8act_mt(t, raw, rows, n_in, np.stack(cs),
                                                np.stack(ss), 3, simd=simd))
    big = random_payload(t, rows, n_in, 0x7BFF, 0x7BFF, 4)
    c = np.full(n_in, 127, dtype=np.int8)
    s = np.full(-(-n_in // 32), 1 << 45, dtype=np.int64)
    want = O.matvec_q8act(t, big, rows, n_in, c, s)
    got = O.matvec_q8act_mt(t, big, rows, n_in, c, s, 4, simd=simd)
    assert want == got and isinstance(want, tuple)


@pytest.mark.parametrize("n_out,n_in,k", [(37, 1536, 13), (16, 256, 8), (5, 8960, 3),
                                          (64, 1024, 64), (1, 256, 1)])
def test_q4_k_kcols_equals_per_column(isa, n_out, n_in, k):
    """The k-column Q4_K kernel of the prefill baseline (chart/kcols.rs:1406-1464) equals the
    per-column fused rows on the benchmark distribution, in both instruction forms."""
    raw = synth.payload(Q4_K, n_out, n_in, seed=n_out + k)
    cs, ss = [], []
    for c in range(k):
        q = O.quant_act(synth.f32_to_q32(synth.activation_f32(n_in, seed=700 + c)))
        cs.append(q[0])
        ss.append(q[1])
    codes, scales = np.stack(cs), np.stack(ss)
    want = O.matmat_q8act(Q4_K, raw, n_out, n_in, codes, scales)
    assert not isinstance(want, tuple)
    calls = O.q4k_counts()[0]
    got = O.matmat_q8act_mt(Q4_K, raw, n_out, n_in, codes, scales, 4, simd=True)
    assert np.array_equal(want, got)
    assert O.q4k_counts()[0] == calls + 1


def test_q4_k_kcols_random_headers_spreads_and_refusals(isa):
    """Random header bytes (every sub-scale and min pattern, both signs of d and dmin), scale
    spreads past the lane limit (exact rows per (row, group)), zero groups, an all-zero column,
    and a non-finite scale (the call refuses as the per-column contract does)."""
    n_out, n_in, k = 11, 512, 10
    for seed, d, dmin in [(21, 0x3800, 0x3800), (22, 0x0001, 0x7BFF), (23, 0xBC00, 0x3C00)]:
        raw = random_payload(Q4_K, n_out, n_in, d, dmin, seed)
        cs, ss = [], []
        for c in range(k):
            x = random_x(n_in, seed * 100 + c)
            if c % 3 == 1:
                x[32 * (c % 16):32 * (c % 16) + 32] <<= 14
            if c == 4:
                x[64:128] = 0
            if c == 7:
                x[:] = 0
            q = O.quant_act(x)
            cs.append(q[0])
            ss.append(q[1])
        codes, scales = np.stack(cs), np.stack(ss)
        want = O.matmat_q8act(Q4_K, raw, n_out, n_in, codes, scales)
        calls, exact = O.q4k_counts()
        got = O.matmat_q8act_mt(Q4_K, raw, n_out, n_in, codes, scales, 3, simd=True)
        if isinstance(want, tuple):
            assert want == got
        else:
            assert np.array_equal(want, got)
            assert O.q4k_counts()[0] == calls + 1
        if seed == 22:  # subnormal d against the largest dmin: spread 29 > the limit
            assert O.q4k_counts()[1] > exact
    bad = synth.payload(Q4_K, n_out, n_in, seed=5).reshape(n_out, -1)
    bad[6, 144 + 2:144 + 4] = (0x00, 0xFC)  # -Inf dmin in row 6, super-block 1
    cs, ss = zip(*[O.quant_act(random_x(n_in, 90 + c)) for c in range(3)])
    want = O.matmat_q8act(Q4_K, bad.reshape(-1), n_out, n_in, np.stack(cs), np.stack(ss))
    got = O.matmat_q8act_mt(Q4_K, bad.reshape(-1), n_out, n_in, np.stack(cs), np.stack(ss), 2,
                            simd=True)
    assert want == got and want[:2] == ("err", 6)


@pytest.mark.filterwarnings("ignore:This process .* is multi-threaded:DeprecationWarning")
def test_pool_survives_fork():
    """The oracle's host pool is started in this process; a forked child (which has only the
    forking thread) starts its own workers and finishes a threaded call."""
    import os
    import signal
    import time

    raw = synth.payload(Q8_0, 64, 256, seed=1)
    codes, scales = O.quant_act(random_x(256, 2))
    want = O.matvec_q8act_mt(Q8_0, raw, 64, 256, codes, scales, 4, simd=True)
    pid = os.fork()
    if pid == 0:
        got = O.matvec_q8act_mt(Q8_0, raw, 64, 256, codes, scales, 4, simd=True)
        os._exit(0 if np.array_equal(got, want) else 1)
    deadline = time.time() + 30
    while time.time() < deadline:
        done, status = os.waitpid(pid, os.WNOHANG)
        if done:
            assert os.WIFEXITED(status) and os.WEXITSTATUS(status) == 0
            return
        time.sleep(0.05)
    os.kill(pid, signal.SIGKILL)
    os.waitpid(pid, 0)
    raise AssertionError("the forked child's pooled call did not finish")


@pytest.mark.parametrize("n_out,n_in,k", [(37, 1536, 13), (16, 256, 8), (3, 4864, 3),
                                          (64, 1024, 64), (1, 256, 1)])
def test_q6_k_kcols_equals_per_column(isa, n_out, n_in, k):
    """The k-column Q6_K kernel (chart/kcols.rs:1466-1518) equals the per-column fused rows on
    the benchmark distribution, in both instruction forms."""
    raw = synth.payload(Q6_K, n_out, n_in, seed=n_out + k)
    cs, ss = [], []
    for c in range(k):
        q = O.quant_act(synth.f32_to_q32(synth.activation_f32(n_in, seed=800 + c)))
        cs.append(q[0])
        ss.append(q[1])
    codes, scales = np.stack(cs), np.stack(ss)
    want = O.matmat_q8act(Q6_K, raw, n_out, n_in, codes, scales)
    assert not isinstance(want, tuple)
    calls = O.q6k_counts()[0]
    got = O.matmat_q8act_mt(Q6_K, raw, n_out, n_in, codes, scales, 4, simd=True)
    assert np.array_equal(want, got)
    assert O.q6k_counts()[0] == calls + 1


def test_q6_k_kcols_random_bytes_spreads_and_refusals(isa):
    """Random code and sub-scale bytes (negative sub-scales included), weight exponents from
    subnormal to the largest (spreads past the lane limit take the exact rows), zero groups, an
    all-zero column, and a non-finite d (the call refuses as the per-column contract does)."""
    n_out, n_in, k = 13, 512, 10
    for seed, d in [(31, 0x3800), (32, 0x7BFF), (33, 0xBC01)]:
        raw = random_payload(Q6_K, n_out, n_in, d, 0, seed).reshape(n_out, -1)
        if seed == 32:
            raw[3, 208:210] = (0x01, 0x00)  # a subnormal d beside 65504: spread 29
        raw = raw.reshape(-1)
        cs, ss = [], []
        for c in range(k):
            x = random_x(n_in, seed * 100 + c)
            if c % 3 == 1:
                x[32 * (c % 16):32 * (c % 16) + 32] <<= 12
            if c == 4:
                x[64:128] = 0
            if c == 7:
                x[:] = 0
            q = O.quant_act(x)
            cs.append(q[0])
            ss.append(q[1])
        codes, scales = np.stack(cs), np.stack(ss)
        want = O.matmat_q8act(Q6_K, raw, n_out, n_in, codes, scales)
        calls, exact = O.q6k_counts()
        got = O.matmat_q8act_mt(Q6_K, raw, n_out, n_in, codes, scales, 3, simd=True)
        if isinstance(want, tuple):
            assert want == got
        else:
            assert np.array_equal(want, got)
            assert O.q6k_counts()[0] == calls + 1
        if seed == 32:
            assert O.q6k_counts()[1] > exact
    bad = synth.payload(Q6_K, n_out, n_in, seed=6).reshape(n_out, -1)
    bad[9, 210 + 208:210 + 210] = (0x00, 0x7E)  # NaN d in row 9, super-block 1
    cs, ss = zip(*[O.quant_act(random_x(n_in, 95 + c)) for c in range(3)])
    want = O.matmat_q8act(Q6_K, bad.reshape(-1), n_out, n_in, np.stack(cs), np.stack(ss))
    got = O.matmat_q8act_mt(Q6_K, bad.reshape(-1), n_out, n_in, np.stack(cs), np.stack(ss), 2,
                            simd=True)
    assert want == got and want[:2] == ("err", 6)


@pytest.mark.parametrize("t", [Q8_0, Q4_K, Q6_K])
def test_vector_paths_on_degenerate_shapes(t):
    """No rows, one row with more threads than rows, and zero-width activations: the vector
    paths return what the single-threaded rows return."""
    qk = 32 if t == Q8_0 else 256
    for rows, n_in, threads in [(0, qk, 4), (1, qk, 16), (3, 2 * qk, 64), (2, 0, 2)]:
        raw = synth.payload(t, max(rows, 1), max(n_in, 1), seed=rows + n_in)
        if rows == 0:
            raw = raw[:0]
        if n_in == 0:
            raw = raw[:0]
        codes, scales = O.quant_act(random_x(n_in, 3)) if n_in else (
            np.zeros(0, np.int8), np.zeros(0, np.int64))
        want = O.matvec_q8act(t, raw, rows, n_in, codes, scales)
        got = O.matvec_q8act_mt(t, raw, rows, n_in, codes, scales, threads, simd=True)
        if isinstance(want, tuple):
            assert want == got
        else:
            assert np.array_equal(want, got)
        k = 3
        cs = np.stack([codes] * k)
        ss = np.stack([scales] * k)
        want = O.matmat_q8act(t, raw, rows, n_in, cs, ss)
        got = O.matmat_q8act_mt(t, raw, rows, n_in, cs, ss, threads, simd=True)
        if isinstance(want, tuple):
            assert want == got
        else:
            assert np.array_equal(np.asarray(want).reshape(k, rows), got)


@pytest.mark.parametrize("n_out,n_in,k", [(37, 896, 13), (8, 4864, 40), (3, 32, 2)])
def test_q8_0_matmat_without_vnni_runs_column_runs(isa, n_out, n_in, k):
    """Without AVX-VNNI (the AVX2 build) Q8_0 matmats run their columns in runs of 16 per row
    pass (kern/matmat.rs:198-206); with it, the GEMM.  Both equal the per-column rows."""
    raw = synth.payload(Q8_0, n_out, n_in, seed=k)
    cs, ss = zip(*[O.quant_act(synth.f32_to_q32(synth.activation_f32(n_in, seed=40 + c)))
                   for c in range(k)])
    codes, scales = np.stack(cs), np.stack(ss)
    want = O.matmat_q8act(Q8_0, raw, n_out, n_in, codes, scales)
    runs, gemms = O.kcols_counts(), O.gemm_counts()[0]
    got = O.matmat_q8act_mt(Q8_0, raw, n_out, n_in, codes, scales, 3, simd=True)
    assert np.array_equal(want, got)
    if isa == "avx2":
        assert O.kcols_counts() == runs + 1 and O.gemm_counts()[0] == gemms
    else:
        assert O.gemm_counts()[0] == gemms + 1
    # a refusal (an output past i64) is redecided by the per-column contract
    big = random_payload(Q8_0, n_out, n_in, 0x7BFF, 0x7BFF, 3)
    c = np.full((k, n_in), 127, dtype=np.int8)
    s = np.full((k, n_in // 32), 1 << 40, dtype=np.int64)
    assert O.matmat_q8act(Q8_0, big, n_out, n_in, c, s) == \
        O.matmat_q8act_mt(Q8_0, big, n_out, n_in, c, s, 3, simd=True)


@pytest.mark.parametrize("n_in", [32, 64, 896, 4864])
def test_q5_0_vector_rows_equal_scalar_rows(isa, n_in):
    """The Q5_0 vector rows (the fifth bit spread from qh into each lane, c − 16 against the codes)
    equal the scalar fused row and the contract, on random payloads (every qh/qs pattern) and on
    the largest finite scales."""
    for rows, threads, d, seed in [(1, 1, 0x3800, 1), (37, 3, 0x3800, 2), (9, 4, 0x7BFF, 3),
                                   (5, 2, 0xB800, 4)]:
        raw = random_payload(Q5_0, rows, n_in, d, 0, seed + n_in)
        codes, scales = O.quant_act(random_x(n_in, seed) << (seed * 5))
        out = _both(Q5_0, raw, rows, n_in, codes, scales, threads)
        ref = O.matvec_fixed(Q5_0, raw, rows, n_in, O.dequant_act(codes, scales))
        if isinstance(out, tuple):
            assert out[:2] == ref[:2]
        else:
            assert np.array_equal(out, ref)
