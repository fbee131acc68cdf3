"""GPU parity: the CUDA backend through the C ABI against the CPU oracle.

Bar: bit-exact Q32.32 outputs and int32 block dots, identical refusals (kind, bits, row,
column), for every family and for the shapes and edge cases the reference's own tests use
(src/engine/chart/tests.rs, src/engine/kern/native_gpu_probe.rs), plus the benchmark shapes.
"""
import numpy as np
import pytest

from oracle import oracle as O
import populations as pop
from chart_inputs import random_payload, random_x, lcg_next
from apeiron_b200 import chart, synth
from apeiron_b200.chart import Backend, QuantAct

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q6_K = 8, 12, 14
FAMILIES = [Q8_0, Q4_K, Q6_K]
KIND = {1: chart.ShapeMismatch, 3: chart.ShortPayload, 4: chart.LengthOverflow,
        6: chart.NonFiniteScale, 7: chart.FixedOverflow, 8: chart.AccumulatorOverflow,
        9: chart.OutputOverflow}


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    yield b
    b.close()


def oracle_q(q: QuantAct):
    return q.codes, q.scales


def check(be, t, raw, n_out, n_in, q: QuantAct, chunks=None):
    """GPU result == oracle result, values or refusal (kind and payload)."""
    if chunks is None:
        want = O.matvec_q8act(t, raw, n_out, n_in, q.codes, q.scales)
    else:
        want = O.matvec_q8act_chunked(t, raw, n_out, n_in, q.codes, q.scales, chunks)
    try:
        if chunks is None:
            got = be.matvec_q8act(t, raw, n_out, n_in, q)
        else:
            got = be.matvec_q8act_quant_chunked(t, raw, n_out, n_in, q, chunks)
    except chart.MatvecError as e:
        assert isinstance(want, tuple), f"GPU refused {e!r}, oracle {want[:4]}"
        assert isinstance(e, KIND[want[1]]), (e, want)
        if want[1] == 6:
            assert e.bits == want[4]
        if want[1] in (1, 3):
            assert e.args == (want[2], want[3])
        return e
    assert not isinstance(want, tuple), f"GPU gave values, oracle refused {want}"
    assert np.array_equal(got, want)
    return got


def qa(x):
    codes, scales = O.quant_act(np.asarray(x, dtype=np.int64))
    return QuantAct.from_parts(scales, codes)


# ---- quant_act ----------------------------------------------------------------------

def test_device_quant_act_known_answers(be):
    q = be.quant_act([3, 130, -3])
    assert q.codes[0] == 2 and q.codes[2] == -2
    assert be.quant_act([(1 << 63) - 1] * 32) is None
    q = be.quant_act([-(1 << 63)] * 32)
    assert list(q.scales) == [1 << 57]
    for v, s, c in ((127, 1, 127), (-127, 1, -127), (128, 2, 64), (-128, 2, -64)):
        q = be.quant_act(pop.unit_at(v))
        assert q.scales[0] == s and q.codes[0] == c
    q = be.quant_act(pop.unit_at(63 << 57))
    assert q.scales[0] == 1 << 56 and q.codes[0] == 126
    assert be.quant_act([-(1 << 63), (1 << 63) - 1]) is None


@pytest.mark.parametrize("n", [1, 31, 32, 33, 200, 896, 8960])
def test_device_quant_act_matches_oracle(be, n):
    for seed in range(4):
        x = random_x(n, 0x5EED0000 + seed + n) * (1 + 999_983 * seed)
        got = be.quant_act(x)
        codes, scales = O.quant_act(x)
        assert np.array_equal(got.codes, codes) and np.array_equal(got.scales, scales)


# ---- the decode contract --------------------------------------------------------------

@pytest.mark.parametrize("t", FAMILIES)
def test_random_payloads_every_family(be, t):
    """chart/tests.rs:224-271 shapes, incl. ragged and zero widths."""
    seed = 0x123456789ABCDEF0
    for rows, n_in in [(4, 32), (3, 48), (2, 33), (2, 300), (1, 64), (5, 0), (1, 256),
                       (2, 512), (2, 256), (37, 896), (33, 1536)]:
        seed = lcg_next(seed)
        raw = random_payload(t, rows, n_in, 0x3800, 0x3800, seed)
        check(be, t, raw, rows, n_in, qa(random_x(n_in, seed ^ 0xDEADBEEF)))


@pytest.mark.parametrize("t", FAMILIES)
def test_extremes_ragged_and_zero_blocks(be, t):
    """chart/tests.rs:273-370."""
    raw = random_payload(t, 2, 256, 0x7BFF, 0x7BFF, 0x51FF0000 + t)
    codes = np.array([127 if j % 2 == 0 else -127 for j in range(256)], dtype=np.int8)
    check(be, t, raw, 2, 256, QuantAct.from_parts(np.ones(8, dtype=np.int64), codes))
    for n_in in [33, 47, 65, 257, 300, 271]:
        raw = random_payload(t, 2, n_in, 0x3800, 0x3800, 0x7000 + t)
        check(be, t, raw, 2, n_in, qa(random_x(n_in, 0xABC0 ^ n_in)))
    x = np.zeros(96, dtype=np.int64)
    x[64:] = 1000 - 100 * np.arange(64, 96)
    raw = random_payload(t, 1, 96, 0x3800, 0x3800, 0x9000 + t)
    check(be, t, raw, 1, 96, qa(x))


@pytest.mark.parametrize("t", FAMILIES)
def test_wide_activation_spreads_and_large_scales(be, t):
    """Activation exponents spread far apart (beyond the fast fold's spread limit) and
    large scales near the call-level bound: the checked path must agree too."""
    rng = np.random.default_rng(7 + t)
    for n_in, spread in [(512, 4), (512, 30), (1024, 40), (256, 55)]:
        x = rng.integers(-(1 << 20), 1 << 20, size=n_in).astype(np.int64)
        blocks = n_in // 32
        shifts = rng.integers(0, spread + 1, size=blocks)
        x = (x.reshape(blocks, 32) << shifts[:, None].astype(np.int64)).reshape(-1)
        raw = random_payload(t, 33, n_in, 0x3000, 0x2000, 99 + spread)
        check(be, t, raw, 33, n_in, qa(x))


def test_refusals(be):
    """Non-finite scale bits at the first bad row, output overflow, accumulator overflow
    on the checked path, unquantizable activation, shape/payload order."""
    for t in FAMILIES:
        raw = random_payload(t, 6, 512, 0x3800, 0x3800, 77 + t)
        qk, bb = O.QK[t], O.BLOCK_BYTES[t]
        rb = (512 // qk) * bb
        off = {Q8_0: 34 + 0, Q4_K: 2, Q6_K: 208}[t]
        raw[3 * rb + off:3 * rb + off + 2] = (0x01, 0x7C)  # row 3: NaN scale
        q = qa(random_x(512, 5))
        e = check(be, t, raw, 6, 512, q)
        assert isinstance(e, chart.NonFiniteScale) and e.bits == 0x7C01 and e.row == 3
        check(be, t, raw, 3, 512, q)  # the bad row is outside the call: values
    big = random_payload(Q8_0, 2, 32, 0x7BFF, 0x7BFF, 3)
    big[2:34] = 127
    qbig = QuantAct.from_parts(np.array([1 << 40]), np.full(32, 127, dtype=np.int8))
    assert isinstance(check(be, Q8_0, big, 2, 32, qbig), chart.OutputOverflow)
    # accumulator overflow: the reference's own witnesses (native_gpu_probe.rs:758-768)
    for c in pop.real_quantizer_populations(O.quant_act)[9:12]:
        qc = QuantAct.from_parts(c["scales"][0], c["codes"][0])
        check(be, Q8_0, c["raw"], 1, c["blocks"] * 32, qc)
    # an activation without a Q32.32 image refuses first, before any shape check
    bad = QuantAct.from_parts(np.array([1 << 58, 1]), np.full(64, 127, dtype=np.int8))
    raw = random_payload(Q8_0, 2, 64, 0x3800, 0x3800, 9)
    assert isinstance(check(be, Q8_0, raw, 2, 64, bad), chart.FixedOverflow)
    short = qa(random_x(32, 1))
    check(be, Q8_0, raw, 2, 64, short)              # ShapeMismatch
    check(be, Q8_0, raw, 2, 64, short, chunks=4)    # ShapeMismatch (payload is long enough)
    check(be, Q8_0, raw, 2, 64, short, chunks=1)


def test_chunked_validation_order(be):
    """ffn.rs:679-697: more than one chunk checks the payload before the shape."""
    raw = random_payload(Q8_0, 2, 64, 0x3800, 0x3800, 9)
    t = be.upload(Q8_0, raw, 2, 64)
    short = qa(random_x(32, 1))
    with pytest.raises(chart.ShapeMismatch):
        be.matvec_q8act(Q8_0, t, 2, 64, short)
    with pytest.raises(chart.ShapeMismatch):
        be.matvec_q8act_quant_chunked(Q8_0, t, 2, 64, short, 4)
    want = O.matvec_q8act_chunked(Q8_0, raw, 3, 64, short.codes, short.scales, 4)
    assert want[1] == 3
    # the backend holds 2 rows; asking 3 with a short activation: ShortPayload first
    with pytest.raises(chart.ShortPayload) as ei:
        be.matvec_q8act_quant_chunked(Q8_0, t, 3, 64, short, 4)
    assert ei.value.args == (want[2], want[3])
    with pytest.raises(chart.ShapeMismatch):
        be.matvec_q8act(Q8_0, t, 3, 64, short)


# ---- prefill contract ------------------------------------------------------------------

@pytest.mark.parametrize("cases", ["synthetic", "real"])
def test_native_probe_populations_matmat(be, cases):
    """Every population of native_gpu_probe.rs as a k-column matmat: equal to the oracle's
    per-column contract (values, refusal and refusing column); where the activation has a
    Q32.32 image and exact_dot gives a value, the values agree with exact_dot."""
    cs = pop.populations() if cases == "synthetic" else pop.real_quantizer_populations(O.quant_act)
    for c in cs:
        n_in = c["blocks"] * 32
        qs = [QuantAct.from_parts(c["scales"][t], c["codes"][t]) for t in range(c["tokens"])]
        want = O.matmat_q8act(Q8_0, c["raw"], c["rows"], n_in, c["codes"], c["scales"])
        if np.any(c["scales"] > (1 << 62)):
            continue
        try:
            got = be.matmat_q8act(Q8_0, c["raw"], c["rows"], n_in, qs)
        except chart.MatvecError as e:
            assert isinstance(want, tuple), (c["id"], e)
            assert isinstance(e, KIND[want[1]]) and e.col == want[5], (c["id"], e, want)
            continue
        assert not isinstance(want, tuple), (c["id"], want)
        assert np.array_equal(np.stack(got), want), c["id"]
        exact = pop.exact_outputs(c, O.exact_dot_q8_0)
        for t in range(c["tokens"]):
            for r in range(c["rows"]):
                v = exact[t * c["rows"] + r]
                if v is not None:
                    assert got[t][r] == v


@pytest.mark.parametrize("t", FAMILIES)
def test_matmat_equals_per_column(be, t):
    n_in, rows, k = 512, 70, 6
    raw = random_payload(t, rows, n_in, 0x3000, 0x2C00, 1234 + t)
    qs = [qa(random_x(n_in, 99 + c) * (c + 1)) for c in range(k)]
    got = be.matmat_q8act(t, raw, rows, n_in, qs)
    want = O.matmat_q8act(t, raw, rows, n_in, np.stack([q.codes for q in qs]),
                          np.stack([q.scales for q in qs]))
    assert np.array_equal(np.stack(got), want)


# ---- block dots, f32 boundary, benchmark shapes ------------------------------------------

@pytest.mark.parametrize("t,n_out,n_in", [(Q8_0, 64, 896), (Q4_K, 64, 1536), (Q4_K, 32, 896),
                                          (Q8_0, 40, 4864), (Q4_K, 48, 8960), (Q6_K, 24, 4096),
                                          (Q6_K, 32, 896), (Q6_K, 33, 512)])
def test_block_dots_bit_exact(be, t, n_out, n_in):
    raw = synth.payload(t, n_out, n_in, 11)
    tens = be.upload(t, raw, n_out, n_in)
    codes, _ = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, 12)))
    qk = O.QK[t]
    padded = np.zeros(-(-n_in // qk) * qk, dtype=np.int8)
    padded[:n_in] = codes
    got = be.block_dots(tens, padded)
    want = O.block_dots(t, raw, n_out, n_in, codes)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("t,n_out,n_in", [
    (Q8_0, 4864, 896),    # config 1 (Qwen2.5-0.5B FFN up)
    (Q4_K, 8960, 1536),   # config 2 (Qwen2.5-1.5B FFN gate/up)
    (Q4_K, 1536, 8960),   # config 2 (Qwen2.5-1.5B FFN down)
    (Q8_0, 896, 4864),    # config 3 down shape
    (Q4_K, 896, 4864),    # config 4 down
    (Q4_K, 128, 896),     # config 4 k/v
    (Q6_K, 4096, 896),    # config 4 LM head, first 4096 vocabulary rows
])
def test_benchmark_shapes_exact(be, t, n_out, n_in):
    raw = synth.payload(t, n_out, n_in, 1000 + n_out + n_in)
    x = synth.activation_f32(n_in, 5)
    codes, exps = synth.quant_act_np(synth.f32_to_q32(x))
    q = QuantAct.from_exps(exps, codes)
    check(be, t, raw, n_out, n_in, q)
    # f32 boundary: device f32_to_fixed + quant_act + exact GEMV, then one rounding to f32
    tens = be.upload(t, raw, n_out, n_in)
    y = be.matvec_f32(tens, x)
    want = O.matvec_q8act(t, raw, n_out, n_in, q.codes, q.scales)
    ref = (want.astype(np.float32) * np.float32(2.0 ** -32)).astype(np.float32)
    assert np.array_equal(y, ref)
    # the scaled f32 outputs against a float64 dequantized reference (tolerance of the
    # benchmark: 1e-5 relative for Q8_0, 1e-4 for K-quants, relative to max |y|)
    xhat = q.dequant().astype(np.float64) / 2.0 ** 32
    w = O.matvec_fixed(t, raw, n_out, n_in, q.dequant())
    tol = 1e-5 if t == Q8_0 else 1e-4
    assert np.max(np.abs(y - w / 2.0 ** 32)) <= tol * np.max(np.abs(w / 2.0 ** 32)) + 1e-30
    del xhat


def test_async_device_path_matches_sync(be):
    """The asynchronous entry points over device buffers (torch for allocation) give the
    synchronous result; the device quantizer feeds the projection without a host trip."""
    import ctypes as C
    import torch

    from apeiron_b200 import _abi

    lib = be.lib
    t, n_out, n_in = Q4_K, 1536, 8960
    raw = synth.payload(t, n_out, n_in, 3)
    tens = be.upload(t, raw, n_out, n_in)
    x = synth.activation_f32(n_in, 4)
    dev = torch.device("cuda:0")
    dx = torch.from_numpy(x).to(dev)
    pad = lib.apx_act_padded_len(n_in)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    out = torch.zeros(n_out, dtype=torch.int64, device=dev)
    status = torch.full((2,), -1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_quant_f32_async(be.ctx, dx.data_ptr(), n_in, codes.data_ptr(),
                                   exps.data_ptr(), desc.data_ptr(), stream) == 0
    assert lib.apx_matvec_async(be.ctx, tens.handle, n_out, n_in, codes.data_ptr(),
                                exps.data_ptr(), desc.data_ptr(), out.data_ptr(), None,
                                status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    st = _abi.CallStatus(int(status[0].item()) & ((1 << 64) - 1), 0)
    err = _abi.ApxErr()
    assert lib.apx_status_decode(be.ctx, tens.handle, C.byref(st), C.byref(err)) == 0
    c, e = synth.quant_act_np(synth.f32_to_q32(x))
    want = be.matvec_q8act(t, tens, n_out, n_in, QuantAct.from_exps(e, c))
    assert np.array_equal(out.cpu().numpy(), want)


def test_async_short_rows_decode(be):
    """A call over the first n_out rows of a tensor with an Inf block scale in a later row
    projects those rows (apx_matvec_q8act decides the same for that n_out):
    apx_status_decode_rows merges the upload-time finding only below n_out."""
    import ctypes as C
    import torch

    from apeiron_b200 import _abi

    lib = be.lib
    t, n_out, n_in = Q8_0, 512, 1024
    raw = synth.payload(t, n_out, n_in, 31).copy()
    bad_row = 200
    off = (bad_row * (n_in // 32) + 5) * 34
    raw[off:off + 2] = (0x00, 0x7C)  # +Inf scale
    tens = be.upload(t, raw, n_out, n_in)
    x = synth.activation_f32(n_in, 32)
    c, e = synth.quant_act_np(synth.f32_to_q32(x))
    dev = torch.device("cuda:0")
    pad = lib.apx_act_padded_len(n_in)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    codes[:n_in] = torch.from_numpy(c).to(dev)
    exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    exps[:e.size] = torch.from_numpy(e).to(dev)
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_act_describe_async(be.ctx, codes.data_ptr(), exps.data_ptr(), n_in,
                                      desc.data_ptr(), stream) == 0
    for rows in (bad_row, bad_row + 1, n_out):
        out = torch.zeros(rows, dtype=torch.int64, device=dev)
        status = torch.full((2,), -1, dtype=torch.int64, device=dev)
        assert lib.apx_matvec_async(be.ctx, tens.handle, rows, n_in, codes.data_ptr(),
                                    exps.data_ptr(), desc.data_ptr(), out.data_ptr(), None,
                                    status.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        st = _abi.CallStatus(int(status[0].item()) & ((1 << 64) - 1), 0)
        err = _abi.ApxErr()
        rc = lib.apx_status_decode_rows(be.ctx, tens.handle, rows, C.byref(st), C.byref(err))
        if rows <= bad_row:
            assert rc == _abi.APX_OK
            want = O.matvec_q8act(t, raw[:rows * (n_in // 32) * 34], rows, n_in, c,
                                  O.exps_to_scales(e))
            assert np.array_equal(out.cpu().numpy(), want)
        else:
            assert rc == _abi.APX_ERR_NONFINITE_SCALE and err.row == bad_row
    err = _abi.ApxErr()
    assert lib.apx_status_decode_rows(be.ctx, tens.handle, n_out + 1, C.byref(st),
                                      C.byref(err)) == _abi.APX_ERR_INVALID_ARGUMENT


# ---- matrices beyond one resident wave: the persistent streaming kernel --------------------

@pytest.mark.parametrize("t,n_out,n_in", [
    (Q8_0, 16384, 4096),
    (Q8_0, 20000, 1000),    # ragged last block, padded final row tile
    (Q4_K, 14336, 4096),
    (Q4_K, 8200, 2304),
    (Q6_K, 151936, 896),    # config 4 LM head, whole vocabulary
])
def test_streaming_shapes_exact(be, t, n_out, n_in):
    raw = synth.payload(t, n_out, n_in, 77 + n_out)
    c, e = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, 9)))
    check(be, t, raw, n_out, n_in, QuantAct.from_exps(e, c))


def test_streaming_checked_path_and_refusals(be):
    """The streaming kernel's checked path (a wide exponent spread) and an output overflow
    in a late row."""
    rng = np.random.default_rng(3)
    n_out, n_in = 8192, 4096
    raw = synth.payload(Q4_K, n_out, n_in, 5)
    x = rng.integers(-(1 << 20), 1 << 20, size=n_in).astype(np.int64)
    shifts = rng.integers(0, 31, size=n_in // 32)
    x = (x.reshape(-1, 32) << shifts[:, None].astype(np.int64)).reshape(-1)
    check(be, Q4_K, raw, n_out, n_in, qa(x))
    big = synth.payload(Q8_0, 16384, 4096, 6)
    row = 12345
    blk = big.reshape(16384, -1)[row].reshape(-1, 34)
    blk[:, 0:2] = (0xFF, 0x7B)   # 65504 scales
    blk[:, 2:] = 127
    q = QuantAct.from_parts(np.full(128, 1 << 40, dtype=np.int64), np.full(4096, 127, dtype=np.int8))
    e = check(be, Q8_0, big, 16384, 4096, q)
    assert isinstance(e, chart.OutputOverflow)
