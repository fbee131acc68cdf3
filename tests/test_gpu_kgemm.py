"""GPU parity of the prefill contract on the digit-plane tensor-core GEMM, every family.

Multi-column calls (four columns or more) take the digit-plane GEMM (apx_lgemm.cu) whenever the
tensor's weights, over their row's smallest scale exponent, fit four balanced base-256 digits:
Q4_K and Q6_K (the k-column projections the reference runs as gemm_q4_k / gemm_q6_k,
src/engine/chart/kcols.rs:1406-1518, dispatched from matmat_q8act, src/engine/kern/matmat.rs:
158-174) and Q8_0 (gemm_q8_0, src/engine/kern/gemm.rs:498-580).  A Q8_0 tensor whose weights
need more digits keeps the per-block fold GEMM (apx_gemm.cu).  Bar: bit-exact Q32.32 outputs
against the oracle's per-column contract (matmat.rs:92-134), identical refusals with the lowest
refusing column, f32 outputs identical to the single-column f32 boundary.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from chart_inputs import random_payload, random_x
from apeiron_b200 import _abi, chart, synth
from apeiron_b200.chart import Backend, QuantAct

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q6_K = 8, 12, 14
KIND = {1: chart.ShapeMismatch, 3: chart.ShortPayload, 4: chart.LengthOverflow,
        6: chart.NonFiniteScale, 7: chart.FixedOverflow, 8: chart.AccumulatorOverflow,
        9: chart.OutputOverflow}
THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    # this module is about the digit-plane GEMM: Q8_0 calls of every size take it (by default
    # the small ones run the per-block fold GEMM, tested in test_gpu_gemm.py)
    assert b.lib.apx_ctx_set_gemm_route(b.ctx, _abi.GEMM_DIGITS) == 0
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


def _col(n_in, seed, shift=0):
    c, s = O.quant_act(random_x(n_in, seed) >> shift)
    return QuantAct.from_parts(s, c)


def device_bytes(be, t):
    return be.lib.apx_tensor_device_bytes(be.ctx, t.handle)


def digit_plane_bytes(n_out, n_in):
    """Device bytes a digit-plane view adds: three or four int8 planes (three when every scaled
    weight of the tensor fits three digits) and one kmin word per row."""
    m_pad, kp = -(-n_out // 128) * 128, -(-n_in // 64) * 64
    return {d * m_pad * kp + 4 * m_pad for d in (3, 4)}


def check_matmat(be, t, raw, n_out, n_in, qs, threads=1, simd=False):
    """GPU matmat against the oracle's per-column contract; returns the GPU refusal or values."""
    codes = np.stack([q.codes for q in qs])
    scales = np.stack([q.scales for q in qs])
    if threads > 1:
        want = O.matmat_q8act_mt(t, raw, n_out, n_in, codes, scales, threads, simd=simd)
    else:
        want = O.matmat_q8act(t, raw, n_out, n_in, codes, scales)
    try:
        got = be.matmat_q8act(t, raw, n_out, n_in, qs)
    except chart.MatvecError as e:
        assert isinstance(want, tuple), f"GPU refused {e!r}, oracle gave values"
        assert isinstance(e, KIND[want[1]]), (e, want)
        assert e.col == want[5], (e.col, want)
        return e
    assert not isinstance(want, tuple), f"GPU gave values, oracle refused {want}"
    got = np.stack(got)
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        c, r = bad[0]
        raise AssertionError(f"{len(bad)} outputs differ; first col {c} row {r}: "
                             f"gpu {got[c, r]} oracle {want[c, r]}")
    return got


def run_and_check_route(be, t, raw, n_out, n_in, qs, **kw):
    tensor = be._tensor(t, raw, n_out, n_in)
    before = device_bytes(be, tensor)
    out = check_matmat(be, t, raw, n_out, n_in, qs, **kw)
    grown = device_bytes(be, tensor) - before
    return out, grown


@pytest.mark.parametrize("t,n_out,n_in,k", [
    (Q4_K, 1536, 1024, 70),    # whole super-blocks, partial token tile
    (Q4_K, 300, 896, 9),       # 896 wide (the 0.5B FFN width): ragged super-block, fast rows
    (Q4_K, 130, 1000, 5),      # a width outside the fast rows: the contract's values
    (Q6_K, 640, 512, 64),
    (Q6_K, 257, 896, 33),      # ragged rows and width
    (Q8_0, 4864, 896, 512),    # configs[2]: 512 tokens on both Qwen2.5-0.5B FFN shapes
    (Q8_0, 896, 4864, 512),
    (Q8_0, 200, 100, 70),      # ragged K (not a multiple of 32)
])
def test_digit_plane_gemm_equals_oracle(be, t, n_out, n_in, k):
    raw = synth.payload(t, n_out, n_in, 17 + n_out + t)
    qs = bench_columns(n_in, k, 400 + n_in)
    _, grown = run_and_check_route(be, t, raw, n_out, n_in, qs, threads=THREADS)
    assert grown in digit_plane_bytes(n_out, n_in), "the call did not take the digit planes"


@pytest.mark.parametrize("n_out,n_in", [(28672, 8192), (8192, 28672)])
def test_llama70b_ffn_prefill_512_tokens(be, n_out, n_in):
    """configs[4]'s prefill: 512 tokens through the Llama-3-70B-shaped Q4_K FFN matrices, checked
    column by column against the oracle's k-column Q4_K kernel (tested equal to the scalar
    contract rows in test_oracle_x86.py)."""
    raw = synth.payload(Q4_K, n_out, n_in, 70 + n_out)
    qs = bench_columns(n_in, 512, 9000)
    _, grown = run_and_check_route(be, Q4_K, raw, n_out, n_in, qs, threads=THREADS, simd=True)
    assert grown in digit_plane_bytes(n_out, n_in)


def test_kquant_mixed_routes(be):
    """Zero columns, zero-scale blocks, an activation spread of 7 (the GEMM's last) and of 9 and
    a bound-failing scale (both on the checked rows), in one Q4_K and one Q6_K call."""
    for t in (Q4_K, Q6_K):
        n_out, n_in, k = 384, 768, 12
        raw = synth.payload(t, n_out, n_in, 5 + t)
        qs = [_col(n_in, 60 + c) for c in range(k)]
        qs[1] = QuantAct.from_parts(np.zeros(n_in // 32, np.int64), np.zeros(n_in, np.int8))
        s = qs[2].scales.copy()
        s[::3] = 0
        qs[2] = QuantAct.from_parts(s, qs[2].codes)
        for c, spread in ((3, 7), (4, 9)):
            s = qs[c].scales.copy()
            s[0] = s[1] << spread
            qs[c] = QuantAct.from_parts(s, qs[c].codes)
        s = qs[5].scales.copy()
        s[4] = 1 << 56
        c5 = qs[5].codes.copy()
        c5[4 * 32:5 * 32] = np.clip(c5[4 * 32:5 * 32], -1, 1)
        qs[5] = QuantAct.from_parts(s, c5)
        check_matmat(be, t, raw, n_out, n_in, qs)


def test_kquant_refusals(be):
    """OutputOverflow in row order, a non-finite scale before or after it, and the lowest refusing
    column, as the oracle reports them."""
    n_out, n_in, k = 260, 512, 6
    raw = random_payload(Q4_K, n_out, n_in, 0x7BFF, 0x7800, 11)
    big = [QuantAct.from_parts(np.full(n_in // 32, 1 << 40, np.int64),
                               np.full(n_in, 127 - c, np.int8)) for c in range(k)]
    check_matmat(be, Q4_K, raw, n_out, n_in, [_col(n_in, 3 + c) for c in range(2)] + big[:2])
    raw2 = raw.copy()
    raw2[7 * 2 * 144 + 2: 7 * 2 * 144 + 4] = (0x00, 0x7C)  # row 7's dmin = +Inf
    check_matmat(be, Q4_K, raw2, n_out, n_in, [_col(n_in, 3 + c) for c in range(k)])
    check_matmat(be, Q4_K, raw2, n_out, n_in, [_col(n_in, 3 + c) for c in range(3)] + big[:3])
    raw6 = random_payload(Q6_K, n_out, n_in, 0x7BFF, 0, 13)
    check_matmat(be, Q6_K, raw6, n_out, n_in, [_col(n_in, 30 + c) for c in range(3)] + big[:3])


def test_q8_0_wide_weight_spread_keeps_fold_gemm(be):
    """Q8_0 rows whose block scales span 2^-24 .. 1.75 (exponent spread 14) need more than four
    digits: the tensor gets no digit planes and the per-block fold GEMM serves it, bit-exact."""
    n_out, n_in, k = 256, 1024, 16
    raw = synth.payload(Q8_0, n_out, n_in, 41).reshape(-1, 34).copy()
    rng = np.random.default_rng(3)
    f16 = np.where(rng.random(raw.shape[0]) < 0.5, 2.0 ** -24, 1.75)
    raw[:, 0:2] = f16.astype(np.float16).view(np.uint8).reshape(-1, 2)
    raw = raw.reshape(-1)
    qs = bench_columns(n_in, k, 77)
    _, grown = run_and_check_route(be, Q8_0, raw, n_out, n_in, qs)
    assert grown not in digit_plane_bytes(n_out, n_in) and grown > 0


@pytest.mark.parametrize("t,n_out,n_in,k", [(Q4_K, 1536, 1536, 40), (Q6_K, 512, 1024, 9),
                                            (Q8_0, 896, 4864, 24)])
def test_f32_prefill_equals_single_column(be, t, n_out, n_in, k):
    """apx_matmat_f32 on the digit planes (fused quantize-prep) equals apx_matvec_f32 per token."""
    raw = synth.payload(t, n_out, n_in, 90 + t)
    tensor = be.upload(t, raw, n_out, n_in)
    x = np.stack([synth.activation_f32(n_in, 500 + c) for c in range(k)])
    got = be.matmat_f32(tensor, x)
    want = np.stack([be.matvec_f32(tensor, x[c]) for c in range(k)])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    tensor.free()


@pytest.mark.parametrize("t,n_out,n_in,k,e0,spread", [
    (Q4_K, 512, 2816, 8, 34, 4), (Q4_K, 256, 28672, 8, 34, 4), (Q8_0, 384, 1024, 6, 40, 4),
    (Q6_K, 256, 1024, 5, 30, 4),
    (Q4_K, 384, 2816, 100, 30, 9),    # spreads 8..9: the third activation digit's second pass
    (Q8_0, 300, 1024, 70, 30, 14),    # up to 14 (past this tensor's three-digit limit: wide)
    (Q6_K, 256, 1024, 9, 20, 12),
    # spreads past every three-digit limit under the call bound: the wide route
    (Q4_K, 384, 2816, 40, 10, 30), (Q4_K, 256, 28672, 8, 10, 30), (Q4_K, 300, 896, 16, 10, 30),
    (Q6_K, 256, 1024, 12, 10, 24), (Q8_0, 300, 1024, 20, 8, 40),
])
def test_device_descriptors_and_large_exponents(be, t, n_out, n_in, k, e0, spread):
    """apx_matmat_async with descriptors computed on the device (apx_act_describe_cols_async), on
    activations whose scales are 2^e0 .. 2^(e0 + spread) (hidden activations of an FFN, whose
    spread exceeds two activation digits for some tokens), against the oracle column by column;
    a few tokens with a narrow spread ride in the same tiles."""
    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    raw = synth.payload(t, n_out, n_in, 5 + n_in)
    tensor = be._tensor(t, raw, n_out, n_in)
    rng = np.random.default_rng(e0)
    nb = n_in // 32
    pad = lib.apx_act_padded_len(n_in)
    codes = np.zeros((k, pad), np.int8)
    exps = np.full((k, pad // 32), 0xFF, np.uint8)
    for c in range(k):
        codes[c, :n_in] = rng.integers(-127, 128, n_in)
        exps[c, :nb] = e0 + rng.integers(0, 5 if c % 3 == 0 else spread + 1, nb)
        exps[c, 0] = e0  # the spread is reached
    dc, de = torch.from_numpy(codes).to(dev), torch.from_numpy(exps).to(dev)
    dd = torch.zeros(8 * k, dtype=torch.int32, device=dev)
    y = torch.zeros(k * n_out, dtype=torch.int64, device=dev)
    ys = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    assert lib.apx_act_describe_cols_async(be.ctx, dc.data_ptr(), de.data_ptr(), n_in, k,
                                           dd.data_ptr(), stream) == 0
    assert lib.apx_matmat_async(be.ctx, tensor.handle, n_out, n_in, k, dc.data_ptr(),
                                de.data_ptr(), dd.data_ptr(), y.data_ptr(), None, ys.data_ptr(),
                                stream) == 0
    torch.cuda.synchronize()
    got = y.cpu().numpy().reshape(k, n_out)
    sc = [O.exps_to_scales(exps[c, :nb]) for c in range(k)]
    want = O.matmat_q8act(t, raw, n_out, n_in, codes[:, :n_in], np.stack(sc))
    if isinstance(want, tuple):
        assert int(ys[0::2].min().item()) != -1
        return
    assert bool((ys[0::2] == -1).all().item())
    bad = np.argwhere(got != want)
    assert bad.size == 0, (f"{len(bad)} differ; first col {bad[0][0]} row {bad[0][1]}: gpu "
                           f"{got[tuple(bad[0])]} oracle {want[tuple(bad[0])]}")


def test_auto_route_by_call_size(be):
    """APX_GEMM_AUTO: a small Q8_0 call runs the per-block fold GEMM (the tensor gains its fold
    view, not digit planes), a K-quant call the digit planes; both bit-exact; a bad route code is
    refused."""
    assert be.lib.apx_ctx_set_gemm_route(be.ctx, 7) == _abi.APX_ERR_INVALID_ARGUMENT
    assert be.lib.apx_ctx_set_gemm_route(be.ctx, _abi.GEMM_AUTO) == 0
    try:
        n_out, n_in, k = 896, 4864, 64
        raw = synth.payload(Q8_0, n_out, n_in, 123)
        _, grown = run_and_check_route(be, Q8_0, raw, n_out, n_in, bench_columns(n_in, k, 5),
                                       threads=THREADS)
        assert grown > 0 and grown not in digit_plane_bytes(n_out, n_in)
        raw = synth.payload(Q4_K, n_out, n_in, 124)
        _, grown = run_and_check_route(be, Q4_K, raw, n_out, n_in, bench_columns(n_in, 8, 6),
                                       threads=THREADS)
        assert grown in digit_plane_bytes(n_out, n_in)
    finally:
        assert be.lib.apx_ctx_set_gemm_route(be.ctx, _abi.GEMM_DIGITS) == 0


@pytest.mark.parametrize("members,n_in,k", [
    ([(Q8_0, 896), (Q8_0, 128), (Q8_0, 128)], 896, 64),      # q/k/v of the 0.5B model
    ([(Q4_K, 1536), (Q4_K, 256), (Q4_K, 256)], 1536, 40),
    ([(Q6_K, 2048), (Q6_K, 2048)], 1024, 17),                # gate/up
    ([(Q4_K, 512), (Q8_0, 512)], 1024, 8),                   # families differ: member by member
])
def test_grouped_prefill_equals_members(be, members, n_in, k):
    """apx_matmat_f32_group_async: one quantize-and-digits prep for the shared activation, then
    every member's GEMM; each member's Q32.32 and f32 outputs and refusal words equal its own
    apx_matmat_f32_async, a token holding a NaN is refused for every member, and member 0
    equals the oracle."""
    import ctypes as C

    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    raws = [synth.payload(t, n_out, n_in, 800 + i) for i, (t, n_out) in enumerate(members)]
    tens = [be.upload(t, raws[i], n_out, n_in) for i, (t, n_out) in enumerate(members)]
    x = np.stack([synth.activation_f32(n_in, 900 + c) for c in range(k)])
    x[k // 2, 7] = np.nan
    dx = torch.from_numpy(x).to(dev)
    count = len(members)

    def outs():
        return ([torch.zeros(k * n, dtype=torch.int64, device=dev) for _, n in members],
                [torch.zeros(k * n, dtype=torch.float32, device=dev) for _, n in members],
                [torch.full((2 * k,), -1, dtype=torch.int64, device=dev) for _ in members])

    gq, gf, gs = outs()
    P = lambda ts: (C.c_void_p * count)(*[t.data_ptr() for t in ts])
    assert lib.apx_matmat_f32_group_async(be.ctx, (C.c_uint64 * count)(*[t.handle for t in tens]),
                                          count, n_in, k, dx.data_ptr(), n_in, P(gq), P(gf), P(gs),
                                          stream) == 0
    sq, sf, ss = outs()
    for i, (t, n_out) in enumerate(members):
        assert lib.apx_matmat_f32_async(be.ctx, tens[i].handle, n_out, n_in, k, dx.data_ptr(),
                                        n_in, sq[i].data_ptr(), sf[i].data_ptr(),
                                        ss[i].data_ptr(), stream) == 0
    torch.cuda.synchronize()
    for i in range(count):
        assert np.array_equal(gs[i].cpu().numpy(), ss[i].cpu().numpy()), i
        words = gs[i].cpu().numpy()[0::2]
        assert words[k // 2] != -1 and (np.delete(words, k // 2) == -1).all(), i
        ok = [c for c in range(k) if c != k // 2]
        q = gq[i].cpu().numpy().reshape(k, -1)
        assert np.array_equal(q[ok], sq[i].cpu().numpy().reshape(k, -1)[ok]), i
        f = gf[i].cpu().numpy().reshape(k, -1)
        assert np.array_equal(f[ok].view(np.uint32),
                              sf[i].cpu().numpy().reshape(k, -1)[ok].view(np.uint32)), i
    t0, n0 = members[0]
    c0, s0 = O.quant_act(synth.f32_to_q32(x[0]))
    want = O.matvec_q8act_mt(t0, raws[0], n0, n_in, c0, s0, THREADS, simd=True)
    assert np.array_equal(gq[0].cpu().numpy()[:n0], want)
