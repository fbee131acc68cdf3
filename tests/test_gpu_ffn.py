"""GPU parity of the FFN hidden activation (apx_swiglu_quant_async): h = SwiGLU(gate, up) under
both carriers, then quant_act(h) for the down projection (src/engine/chart/ffn.rs:1577-1594,
swiglu_one_carrier :246-284).  Bar: h, codes, exponent bytes and descriptor identical to the
oracle's restatement; the lowest refusing lane and its FfnError kind; a quant_act refusal with
no SwiGLU refusal.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

from apeiron_b200 import _abi, synth
from apeiron_b200.chart import Backend

pytestmark = pytest.mark.gpu

ONE = 1 << 32
LN2_Q32 = 2_977_044_472


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    yield b
    b.close()


def hidden(n, seed):
    """gate across both SiLU saturation windows, up of either sign, and the edge lanes."""
    rng = np.random.default_rng(seed)
    gate = rng.integers(-24 * ONE, 24 * ONE, n, dtype=np.int64)
    up = rng.integers(-8 * ONE, 8 * ONE, n, dtype=np.int64)
    edges = [16 * ONE, 16 * ONE - 1, -21 * ONE, -21 * ONE + 1, 0, 1, -1, LN2_Q32, -LN2_Q32,
             (1 << 63) - 1, -(1 << 63)]
    m = min(n, len(edges))
    gate[:m] = edges[:m]
    up[:m] = [ONE, 3, -ONE, 5 * ONE, 7, ONE, -ONE, ONE, 2 * ONE, 0, 12345][:m]
    return gate, up


def run(be, gate, up, carrier):
    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    n = gate.size
    pad = max(lib.apx_act_padded_len(n), 32)
    dg = torch.from_numpy(gate).to(dev)
    du = torch.from_numpy(up).to(dev)
    h = torch.zeros(max(n, 1), dtype=torch.int64, device=dev)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    exps = torch.full((pad // 32,), 0xEE, dtype=torch.uint8, device=dev)
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    status = torch.full((2,), -1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_swiglu_quant_async(be.ctx, dg.data_ptr(), du.data_ptr(), n, carrier,
                                      h.data_ptr(), codes.data_ptr(), exps.data_ptr(),
                                      desc.data_ptr(), status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    st = status.cpu().numpy()
    err = _abi.ApxErr()
    word = _abi.CallStatus(int(st[0]) & ((1 << 64) - 1), 0)
    rc = lib.apx_ffn_status_decode(C.byref(word), C.byref(err))
    return (h.cpu().numpy()[:n], codes.cpu().numpy(), exps.cpu().numpy(), desc.cpu().numpy(),
            (rc, err.row, err.bits))


@pytest.mark.parametrize("carrier", [_abi.CARRIER_F32, _abi.CARRIER_Q32])
@pytest.mark.parametrize("n", [32, 100, 896, 4864, 8960])
def test_swiglu_quant_matches_oracle(be, carrier, n):
    gate, up = hidden(n, 11 + n)
    h, codes, exps, desc, (rc, _, _) = run(be, gate, up, carrier)
    want = O.swiglu_quant(gate, up, carrier)
    assert isinstance(want[0], np.ndarray), want
    wh, wc, ws = want
    assert rc == _abi.APX_OK
    assert np.array_equal(h, wh)
    assert np.array_equal(codes[:n], wc) and not codes[n:].any()
    we = O.scales_to_exps(ws)
    nb = (n + 31) // 32
    assert np.array_equal(exps[:nb], we)
    nz = we != 0xFF
    assert desc[0] == 0 and desc[3] == n and desc[4] == nz.sum()
    if nz.any():
        assert (desc[1], desc[2]) == (we[nz].min(), we[nz].max())


@pytest.mark.parametrize("carrier", [_abi.CARRIER_F32, _abi.CARRIER_Q32])
def test_swiglu_refusals(be, carrier):
    """Overflowing lanes at 400, 77 and 512: the call reports lane 77 (FfnError::Overflow) and
    the descriptor refuses the activation."""
    gate, up = hidden(600, 5)
    gate[[400, 77, 512]] = 30 * ONE
    up[[400, 77, 512]] = 1 << 61
    want = O.swiglu_quant(gate, up, carrier)
    assert want == ("swiglu", 77, O.FFN_OVERFLOW)
    _, _, _, desc, (rc, row, bits) = run(be, gate, up, carrier)
    assert (rc, row, bits) == (_abi.APX_ERR_SWIGLU_REFUSED, 77, O.FFN_OVERFLOW)
    assert desc[0] == _abi.APX_ERR_QUANT_REFUSED


def test_quant_refusal_without_swiglu_refusal(be):
    """Q32 carrier: h = 2^63 − 2^54 in one lane is a valid SwiGLU value whose block needs a
    scale above 2^56, so quant_act refuses h (QuantRefused) with no lane refused."""
    gate, up = hidden(96, 9)
    gate[40] = 16 * ONE
    up[40] = (1 << 59) - (1 << 50)
    assert O.swiglu_quant(gate, up, _abi.CARRIER_Q32) == ("quant",)
    _, _, _, desc, (rc, _, _) = run(be, gate, up, _abi.CARRIER_Q32)
    assert rc == _abi.APX_OK and desc[0] == _abi.APX_ERR_QUANT_REFUSED


@pytest.mark.parametrize("t,n_embd,n_ff,carrier", [(12, 896, 4864, _abi.CARRIER_F32),
                                                    (8, 512, 1024, _abi.CARRIER_Q32)])
def test_decode_ffn_chain_on_device(be, t, n_embd, n_ff, carrier):
    """One decode FFN with nothing on the host between its stages: quant_act of x on the
    device, gate and up as one grouped launch (Q32.32 outputs), SwiGLU + quant_act of h, then
    the down projection reading that activation.  y equals the reference's chain
    (matvec_q8act, swiglu_one_carrier, quant_act, matvec_q8act) computed by the oracle."""
    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    shapes = [(n_ff, n_embd), (n_ff, n_embd), (n_embd, n_ff)]
    raws = [synth.payload(t, o, i, 60 + k) for k, (o, i) in enumerate(shapes)]
    tens = [be.upload(t, r, o, i) for r, (o, i) in zip(raws, shapes)]
    x = synth.activation_f32(n_embd, 3)
    pad = lib.apx_act_padded_len(n_embd)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    dx = torch.from_numpy(x).to(dev)
    assert lib.apx_quant_f32_async(be.ctx, dx.data_ptr(), n_embd, codes.data_ptr(),
                                   exps.data_ptr(), desc.data_ptr(), stream) == 0
    gu = [torch.zeros(n_ff, dtype=torch.int64, device=dev) for _ in range(2)]
    gs = [torch.full((2,), -1, dtype=torch.int64, device=dev) for _ in range(2)]
    handles = (C.c_uint64 * 2)(tens[0].handle, tens[1].handle)
    optr = (C.c_void_p * 2)(*[o.data_ptr() for o in gu])
    sptr = (C.c_void_p * 2)(*[s_.data_ptr() for s_ in gs])
    assert lib.apx_matvec_group_async(be.ctx, handles, 2, n_embd, codes.data_ptr(),
                                      exps.data_ptr(), desc.data_ptr(), optr, None, sptr,
                                      stream) == 0
    padh = lib.apx_act_padded_len(n_ff)
    hc = torch.zeros(padh, dtype=torch.int8, device=dev)
    he = torch.full((padh // 32,), 0xFF, dtype=torch.uint8, device=dev)
    hd = torch.zeros(8, dtype=torch.int32, device=dev)
    fs = torch.full((2,), -1, dtype=torch.int64, device=dev)
    assert lib.apx_swiglu_quant_async(be.ctx, gu[0].data_ptr(), gu[1].data_ptr(), n_ff, carrier,
                                      None, hc.data_ptr(), he.data_ptr(), hd.data_ptr(),
                                      fs.data_ptr(), stream) == 0
    y = torch.zeros(n_embd, dtype=torch.int64, device=dev)
    ys = torch.full((2,), -1, dtype=torch.int64, device=dev)
    assert lib.apx_matvec_async(be.ctx, tens[2].handle, n_embd, n_ff, hc.data_ptr(),
                                he.data_ptr(), hd.data_ptr(), y.data_ptr(), None, ys.data_ptr(),
                                stream) == 0
    torch.cuda.synchronize()
    for st in gs + [fs, ys]:
        assert int(st[0].item()) == -1
    c, sc = O.quant_act(synth.f32_to_q32(x))
    g = O.matvec_q8act(t, raws[0], n_ff, n_embd, c, sc)
    u = O.matvec_q8act(t, raws[1], n_ff, n_embd, c, sc)
    assert np.array_equal(gu[0].cpu().numpy(), g) and np.array_equal(gu[1].cpu().numpy(), u)
    h, hcodes, hscales = O.swiglu_quant(g, u, carrier)
    want = O.matvec_q8act(t, raws[2], n_embd, n_ff, hcodes, hscales)
    assert np.array_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("n,k,carrier", [(4864, 9, _abi.CARRIER_F32), (1000, 5, _abi.CARRIER_Q32),
                                         (96, 3, _abi.CARRIER_F32)])
def test_swiglu_columns_equal_single_column(be, n, k, carrier):
    """apx_swiglu_quant_cols_async over k columns (one launch) equals apx_swiglu_quant_async of
    every column: h, codes, exponent bytes, descriptor and status word, refusing columns
    included."""
    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    cols = [hidden(n, 100 + c) for c in range(k)]
    if k > 2:  # one column with a lane the carrier refuses, one whose h quant_act refuses
        cols[1][0][5], cols[1][1][5] = 16 * ONE, (1 << 62)
        cols[2][0][40], cols[2][1][40] = 16 * ONE, (1 << 59) - (1 << 50)
    gate = np.concatenate([c[0] for c in cols])
    up = np.concatenate([c[1] for c in cols])
    pad = lib.apx_act_padded_len(n)
    dg, du = torch.from_numpy(gate).to(dev), torch.from_numpy(up).to(dev)
    h = torch.zeros(k * n, dtype=torch.int64, device=dev)
    codes = torch.zeros(k * pad, dtype=torch.int8, device=dev)
    exps = torch.full((k * pad // 32,), 0xEE, dtype=torch.uint8, device=dev)
    descs = torch.zeros(8 * k, dtype=torch.int32, device=dev)
    status = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    assert lib.apx_swiglu_quant_cols_async(be.ctx, dg.data_ptr(), du.data_ptr(), n, k, carrier,
                                           h.data_ptr(), codes.data_ptr(), exps.data_ptr(),
                                           descs.data_ptr(), status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    hh, cc, ee = h.cpu().numpy(), codes.cpu().numpy(), exps.cpu().numpy()
    dd, ss = descs.cpu().numpy(), status.cpu().numpy()
    nb = -(-n // 32)
    for c in range(k):
        h1, c1, e1, d1, _ = run(be, cols[c][0], cols[c][1], carrier)
        st1 = torch.full((2,), -1, dtype=torch.int64, device=dev)
        # the single-column call's raw status word, for an exact comparison
        g1, u1 = torch.from_numpy(cols[c][0]).to(dev), torch.from_numpy(cols[c][1]).to(dev)
        tmp_c = torch.zeros(pad, dtype=torch.int8, device=dev)
        tmp_e = torch.full((pad // 32,), 0xEE, dtype=torch.uint8, device=dev)
        tmp_d = torch.zeros(8, dtype=torch.int32, device=dev)
        assert lib.apx_swiglu_quant_async(be.ctx, g1.data_ptr(), u1.data_ptr(), n, carrier, None,
                                          tmp_c.data_ptr(), tmp_e.data_ptr(), tmp_d.data_ptr(),
                                          st1.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        assert np.array_equal(hh[c * n:(c + 1) * n], h1), c
        assert np.array_equal(cc[c * pad:c * pad + n], c1[:n]), c
        assert np.array_equal(ee[c * pad // 32:c * pad // 32 + nb], e1[:nb]), c
        assert np.array_equal(dd[8 * c:8 * c + 8], d1), c
        assert ss[2 * c] == int(st1[0].item()), c


def test_prefill_ffn_chain_on_device(be):
    """A prefill FFN over 48 tokens with nothing on the host between its stages: gate and up on
    the tensor cores (Q32.32 outputs, column-major), SwiGLU + quant_act of every token's h in
    one launch, then the down projection of all tokens reading those codes.  Every token's y
    equals the reference's chain computed by the oracle."""
    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    t, n_embd, n_ff, k, carrier = 12, 1024, 2816, 48, _abi.CARRIER_F32
    shapes = [(n_ff, n_embd), (n_ff, n_embd), (n_embd, n_ff)]
    raws = [synth.payload(t, o, i, 80 + j) for j, (o, i) in enumerate(shapes)]
    tens = [be.upload(t, r, o, i) for r, (o, i) in zip(raws, shapes)]
    x = np.stack([synth.activation_f32(n_embd, 30 + c) for c in range(k)])
    dx = torch.from_numpy(x).to(dev)
    gu = [torch.zeros(k * n_ff, dtype=torch.int64, device=dev) for _ in range(2)]
    gs = [torch.full((2 * k,), -1, dtype=torch.int64, device=dev) for _ in range(2)]
    for j in range(2):
        assert lib.apx_matmat_f32_async(be.ctx, tens[j].handle, n_ff, n_embd, k, dx.data_ptr(),
                                        n_embd, gu[j].data_ptr(), None, gs[j].data_ptr(),
                                        stream) == 0
    padh = lib.apx_act_padded_len(n_ff)
    hc = torch.zeros(k * padh, dtype=torch.int8, device=dev)
    he = torch.full((k * padh // 32,), 0xFF, dtype=torch.uint8, device=dev)
    hd = torch.zeros(8 * k, dtype=torch.int32, device=dev)
    fs = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    assert lib.apx_swiglu_quant_cols_async(be.ctx, gu[0].data_ptr(), gu[1].data_ptr(), n_ff, k,
                                           carrier, None, hc.data_ptr(), he.data_ptr(),
                                           hd.data_ptr(), fs.data_ptr(), stream) == 0
    y = torch.zeros(k * n_embd, dtype=torch.int64, device=dev)
    ys = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    assert lib.apx_matmat_async(be.ctx, tens[2].handle, n_embd, n_ff, k, hc.data_ptr(),
                                he.data_ptr(), hd.data_ptr(), y.data_ptr(), None, ys.data_ptr(),
                                stream) == 0
    torch.cuda.synchronize()
    for st in gs + [fs, ys]:
        assert bool((st[0::2] == -1).all().item())
    g_all, u_all = gu[0].cpu().numpy().reshape(k, n_ff), gu[1].cpu().numpy().reshape(k, n_ff)
    y_all = y.cpu().numpy().reshape(k, n_embd)
    for c in range(k):
        cx, sx = O.quant_act(synth.f32_to_q32(x[c]))
        g = O.matvec_q8act(t, raws[0], n_ff, n_embd, cx, sx)
        u = O.matvec_q8act(t, raws[1], n_ff, n_embd, cx, sx)
        assert np.array_equal(g_all[c], g) and np.array_equal(u_all[c], u), c
        _, hcodes, hscales = O.swiglu_quant(g, u, carrier)
        want = O.matvec_q8act(t, raws[2], n_embd, n_ff, hcodes, hscales)
        assert np.array_equal(y_all[c], want), c


@pytest.mark.parametrize("n,peers", [(4864, 3), (1000, 7), (64, 1)])
def test_swiglu_shard_copies_equal_single_call(be, n, peers):
    """apx_swiglu_quant_shard_async: the slice's codes, exponent bytes and descriptor, and every
    copy of them, equal apx_swiglu_quant_async's (device buffers on this GPU stand in for the
    other ranks'); a bad peer count is refused."""
    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    gate, up = hidden(n, 77 + n)
    h0, c0, e0, d0, s0 = run(be, gate, up, _abi.CARRIER_F32)
    dg = torch.from_numpy(gate).to(dev)
    du = torch.from_numpy(up).to(dev)
    pad = max(lib.apx_act_padded_len(n), 32)
    bufs = [(torch.zeros(pad, dtype=torch.int8, device=dev),
             torch.full((pad // 32,), 0xEE, dtype=torch.uint8, device=dev),
             torch.zeros(8, dtype=torch.int32, device=dev)) for _ in range(peers + 1)]
    own, rest = bufs[0], bufs[1:]
    pc = (C.c_void_p * peers)(*[b[0].data_ptr() for b in rest])
    pe = (C.c_void_p * peers)(*[b[1].data_ptr() for b in rest])
    pd = (C.c_void_p * peers)(*[b[2].data_ptr() for b in rest])
    status = torch.full((2,), -1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_swiglu_quant_shard_async(be.ctx, dg.data_ptr(), du.data_ptr(), n, 0, None,
                                            own[0].data_ptr(), own[1].data_ptr(),
                                            own[2].data_ptr(), peers, pc, pe, pd,
                                            status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    nb = (n + 31) // 32
    for b in bufs:
        assert np.array_equal(b[0].cpu().numpy()[:n], c0[:n])
        assert np.array_equal(b[1].cpu().numpy()[:nb], e0[:nb])
        assert np.array_equal(b[2].cpu().numpy(), d0)
    assert lib.apx_swiglu_quant_shard_async(be.ctx, dg.data_ptr(), du.data_ptr(), n, 0, None,
                                            own[0].data_ptr(), own[1].data_ptr(),
                                            own[2].data_ptr(), 8, pc, pe, pd,
                                            status.data_ptr(), stream) == \
        _abi.APX_ERR_INVALID_ARGUMENT


def test_hidden_gather_one_rank_merges_descriptor(be):
    """shard.HiddenGather at world 1: the slice stored by apx_swiglu_quant_shard_async into the
    gather buffer, one publication (flags, keys, the descriptor merge), and the whole h read
    back equal to apx_swiglu_quant_async's, parity after parity."""
    import torch

    from apeiron_b200 import shard

    lib = be.lib
    dev = torch.device("cuda:0")
    n, n_in = 4096, 512
    raw = synth.payload(12, n, n_in, 5)
    gsh = shard.RowShard(be, 12, raw, n, n_in, 0, 1, None, "cuda:0")
    ush = shard.RowShard(be, 12, raw, n, n_in, 0, 1, None, "cuda:0")
    hg = shard.HiddenGather(lib, be.ctx, gsh, ush)
    st = torch.full((2, 2), -1, dtype=torch.int64, device=dev)
    merged = torch.full((2, 2), -1, dtype=torch.int64, device=dev)
    fst = torch.full((2,), -1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for step in range(4):
            gate, up = hidden(n, 300 + step)
            _, c0, e0, d0, _ = run(be, gate, up, _abi.CARRIER_F32)
            dg = torch.from_numpy(gate).to(dev)
            du = torch.from_numpy(up).to(dev)
            par = hg.next_parity()
            oc, oe, od = hg.slice_dest(par, 0)
            assert lib.apx_swiglu_quant_shard_async(be.ctx, dg.data_ptr(), du.data_ptr(), n, 0,
                                                    None, oc, oe, od, 0, None, None, None,
                                                    fst.data_ptr(), stream) == 0
            assert hg.publish(st, merged, stream) == par
            torch.cuda.synchronize()
            codes, exps, desc = hg.read(par)
            assert np.array_equal(codes, c0[:n]) and np.array_equal(exps, e0[:n // 32])
            assert np.array_equal(desc, d0), (desc, d0)
            assert bool((merged[:, 0] == -1).all().item())
    finally:
        torch.cuda.synchronize()
        hg.close()
