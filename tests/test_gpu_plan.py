"""Step plans (apx_plan_*): many projections, and FFNs whose gate/up finish runs SwiGLU +
quant_act, in one persistent launch.  Every output, activation and refusal word must equal the
per-call path (apx_matvec_async, apx_swiglu_quant_async) on the same inputs, and the oracle."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from apeiron_b200 import _abi, synth

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q6_K = 8, 12, 14


@pytest.fixture(scope="module")
def be():
    from apeiron_b200.chart import Backend
    b = Backend(0)
    yield b
    b.close()


def _torch():
    import torch
    return torch


class DevAct:
    """A resident activation (codes, exponent bytes, descriptor on the device)."""

    def __init__(self, lib, ctx, n, seed=None, x=None, scale=1.0):
        torch = _torch()
        dev = torch.device("cuda:0")
        self.n = n
        pad = lib.apx_act_padded_len(n)
        self.codes = torch.zeros(pad, dtype=torch.int8, device=dev)
        self.exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
        self.desc = torch.zeros(8, dtype=torch.int32, device=dev)
        if x is None:
            x = synth.activation_f32(n, seed) * np.float32(scale)
        self.x = x
        dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev)
        st = torch.cuda.current_stream().cuda_stream
        assert lib.apx_quant_f32_async(ctx, dx.data_ptr(), n, self.codes.data_ptr(),
                                       self.exps.data_ptr(), self.desc.data_ptr(), st) == 0
        torch.cuda.synchronize()

    def rec(self, ffn=-1):
        return _abi.PlanAct(self.codes.data_ptr(), self.exps.data_ptr(), self.desc.data_ptr(),
                            ffn, 0)


class Out:
    def __init__(self, n):
        torch = _torch()
        dev = torch.device("cuda:0")
        self.q32 = torch.zeros(max(n, 1), dtype=torch.int64, device=dev)
        self.f32 = torch.zeros(max(n, 1), dtype=torch.float32, device=dev)
        self.status = torch.full((2,), -1, dtype=torch.int64, device=dev)
        self.n = n

    def reset(self):
        self.status.fill_(-1)


def _word(status):
    return _abi.CallStatus(int(status[0].item()) & ((1 << 64) - 1), 0)


def _decode(lib, ctx, tensor, n_out, status):
    err = _abi.ApxErr()
    rc = lib.apx_status_decode_rows(ctx, tensor.handle, n_out, C.byref(_word(status)),
                                    C.byref(err))
    return rc, (err.row if rc else None)


def _single(lib, ctx, tensor, n_out, n_in, codes, exps, desc):
    """apx_matvec_async on the same device activation: (q32, f32, rc, row)."""
    o = Out(n_out)
    torch = _torch()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.apx_matvec_async(ctx, tensor.handle, n_out, n_in, codes, exps, desc,
                                o.q32.data_ptr(), o.f32.data_ptr(), o.status.data_ptr(), st) == 0
    torch.cuda.synchronize()
    rc, row = _decode(lib, ctx, tensor, n_out, o.status)
    return o.q32.cpu().numpy()[:n_out], o.f32.cpu().numpy()[:n_out], rc, row


def _plan(lib, ctx, projs, acts, ffns=()):
    P = (_abi.PlanProj * len(projs))(*projs)
    A = (_abi.PlanAct * len(acts))(*acts)
    F = (_abi.PlanFfn * max(len(ffns), 1))(*ffns)
    err = _abi.ApxErr()
    plan = lib.apx_plan_create(ctx, P, len(projs), A, len(acts), F, len(ffns), C.byref(err))
    return plan, err.code


def _run(lib, plan):
    torch = _torch()
    assert lib.apx_plan_run_async(plan, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()


def _proj(tensor, n_out, n_in, act, out, ffn=-1, role=0, q32=True):
    return _abi.PlanProj(tensor.handle, n_out, n_in, act, ffn, role, 0,
                         out.q32.data_ptr() if q32 else None, out.f32.data_ptr(),
                         out.status.data_ptr())


# every layout the plan reads: one-wave L = 1 / 2 / 4, the streaming layout in one piece and in
# several, ragged widths, short row counts
SHAPES_Q4K = [(4864, 896, 4864), (896, 896, 896), (128, 896, 100), (896, 4864, 896),
              (1536, 8960, 1536), (16384, 4096, 16384), (8192, 8192, 8000), (600, 2304, 600)]


@pytest.mark.parametrize("t,shapes", [
    (Q4_K, SHAPES_Q4K),
    (Q8_0, [(4864, 896, 4864), (896, 4864, 896), (20000, 1000, 20000), (130, 96, 130),
            (8192, 8192, 8192)]),
    (Q6_K, [(2048, 896, 2048), (896, 4864, 896), (30000, 896, 29999)]),
])
def test_plan_independent_projections_equal_single_calls(be, t, shapes):
    lib, ctx = be.lib, be.ctx
    tens, acts, outs, projs = [], {}, [], []
    for i, (n_out, n_in, rows) in enumerate(shapes):
        tens.append(be.upload(t, synth.payload(t, n_out, n_in, 500 + i), n_out, n_in))
        if n_in not in acts:
            acts[n_in] = (len(acts), DevAct(lib, ctx, n_in, seed=600 + n_in))
        outs.append(Out(rows))
        projs.append(_proj(tens[i], rows, n_in, acts[n_in][0], outs[i]))
    act_list = [a for _, a in sorted(acts.values(), key=lambda p: p[0])]
    plan, rc = _plan(lib, ctx, projs, [a.rec() for a in act_list])
    assert plan, rc
    try:
        for rep in range(3):  # the counters reset themselves between launches
            for o in outs:
                o.reset()
            _run(lib, plan)
            for i, (n_out, n_in, rows) in enumerate(shapes):
                a = acts[n_in][1]
                q, f, rc1, row1 = _single(lib, ctx, tens[i], rows, n_in, a.codes.data_ptr(),
                                          a.exps.data_ptr(), a.desc.data_ptr())
                assert _decode(lib, ctx, tens[i], rows, outs[i].status) == (rc1, row1)
                assert rc1 == _abi.APX_OK
                assert np.array_equal(outs[i].q32.cpu().numpy()[:rows], q), (rep, i)
                assert np.array_equal(outs[i].f32.cpu().numpy()[:rows].view(np.uint32),
                                      f.view(np.uint32)), (rep, i)
        # the oracle on the first and the last projection
        for i in (0, len(shapes) - 1):
            n_out, n_in, rows = shapes[i]
            a = acts[n_in][1]
            c, e = synth.quant_act_np(synth.f32_to_q32(a.x))
            want = O.matvec_q8act_mt(t, synth.payload(t, n_out, n_in, 500 + i), n_out, n_in, c,
                                     O.exps_to_scales(e), 8, simd=True)
            assert np.array_equal(outs[i].q32.cpu().numpy()[:rows], want[:rows])
    finally:
        lib.apx_plan_destroy(plan)


def _ffn_layers(be, t, n_embd, n_ff, layers, carrier, seed):
    """`layers` FFNs (gate/up -> SwiGLU + quant_act -> down) in one plan, plus the separate
    per-call chain on the same inputs for comparison."""
    torch = _torch()
    dev = torch.device("cuda:0")
    lib, ctx = be.lib, be.ctx
    projs, acts, ffns, keep = [], [], [], []
    for layer in range(layers):
        s0 = seed + 10 * layer
        tg = be.upload(t, synth.payload(t, n_ff, n_embd, s0), n_ff, n_embd)
        tu = be.upload(t, synth.payload(t, n_ff, n_embd, s0 + 1), n_ff, n_embd)
        td = be.upload(t, synth.payload(t, n_embd, n_ff, s0 + 2), n_embd, n_ff)
        x = DevAct(lib, ctx, n_embd, seed=s0 + 3)
        h = DevAct(lib, ctx, n_ff, x=np.zeros(n_ff, np.float32))  # buffers the FFN writes
        h_q32 = torch.zeros(n_ff, dtype=torch.int64, device=dev)
        f_status = torch.full((2,), -1, dtype=torch.int64, device=dev)
        og, ou, od = Out(n_ff), Out(n_ff), Out(n_embd)
        ax = len(acts)
        acts.append(x.rec())
        ah = len(acts)
        acts.append(h.rec(ffn=layer))
        projs.append(_proj(tg, n_ff, n_embd, ax, og, ffn=layer, role=_abi.PLAN_GATE,
                           q32=layer % 2 == 0))  # odd layers: plan-owned gate/up Q32 buffers
        projs.append(_proj(tu, n_ff, n_embd, ax, ou, ffn=layer, role=_abi.PLAN_UP,
                           q32=layer % 2 == 0))
        projs.append(_proj(td, n_embd, n_ff, ah, od))
        ffns.append(_abi.PlanFfn(carrier, ah, h_q32.data_ptr(), f_status.data_ptr()))
        keep.append(dict(tg=tg, tu=tu, td=td, x=x, h=h, h_q32=h_q32, f_status=f_status, og=og,
                         ou=ou, od=od, seeds=(s0, s0 + 1, s0 + 2)))
    return projs, acts, ffns, keep


def _separate_chain(be, k, n_embd, n_ff, carrier):
    """The same FFN by the per-call entry points: gate, up, SwiGLU + quant_act, down."""
    torch = _torch()
    dev = torch.device("cuda:0")
    lib, ctx = be.lib, be.ctx
    x = k["x"]
    g = _single(lib, ctx, k["tg"], n_ff, n_embd, x.codes.data_ptr(), x.exps.data_ptr(),
                x.desc.data_ptr())
    u = _single(lib, ctx, k["tu"], n_ff, n_embd, x.codes.data_ptr(), x.exps.data_ptr(),
                x.desc.data_ptr())
    dg = torch.from_numpy(g[0].copy()).to(dev)
    du = torch.from_numpy(u[0].copy()).to(dev)
    pad = lib.apx_act_padded_len(n_ff)
    hc = torch.zeros(pad, dtype=torch.int8, device=dev)
    he = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    hd = torch.zeros(8, dtype=torch.int32, device=dev)
    hq = torch.zeros(n_ff, dtype=torch.int64, device=dev)
    fs = torch.full((2,), -1, dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    assert lib.apx_swiglu_quant_async(ctx, dg.data_ptr(), du.data_ptr(), n_ff, carrier,
                                      hq.data_ptr(), hc.data_ptr(), he.data_ptr(), hd.data_ptr(),
                                      fs.data_ptr(), st) == 0
    torch.cuda.synchronize()
    y = _single(lib, ctx, k["td"], n_embd, n_ff, hc.data_ptr(), he.data_ptr(), hd.data_ptr())
    return dict(g=g, u=u, hc=hc.cpu().numpy(), he=he.cpu().numpy(), hd=hd.cpu().numpy(),
                hq=hq.cpu().numpy(), fs=int(fs[0].item()), y=y)


@pytest.mark.parametrize("t,n_embd,n_ff,layers,carrier", [
    (Q4_K, 896, 4864, 2, 0),
    (Q4_K, 896, 4864, 1, 1),
    (Q8_0, 1024, 2816, 3, 0),
    (Q4_K, 2048, 5632, 1, 0),
    (Q4_K, 8192, 1024, 1, 0),   # gate/up in 8-row tiles (L = 4): four per block of h
    (Q8_0, 4096, 1000, 1, 1),   # L = 4 and a ragged last block of h (one 8-row tile)
])
def test_plan_ffn_chain_equals_separate_calls(be, t, n_embd, n_ff, layers, carrier):
    lib, ctx = be.lib, be.ctx
    projs, acts, ffns, keep = _ffn_layers(be, t, n_embd, n_ff, layers, carrier, 900)
    plan, rc = _plan(lib, ctx, projs, acts, ffns)
    assert plan, rc
    try:
        want = [_separate_chain(be, k, n_embd, n_ff, carrier) for k in keep]
        for rep in range(3):
            for k in keep:
                for o in (k["og"], k["ou"], k["od"]):
                    o.reset()
                k["f_status"].fill_(-1)
            _run(lib, plan)
            for layer, (k, w) in enumerate(zip(keep, want)):
                assert int(k["f_status"][0].item()) == w["fs"] == -1
                assert np.array_equal(k["h_q32"].cpu().numpy(), w["hq"]), (rep, layer)
                assert np.array_equal(k["h"].codes.cpu().numpy(), w["hc"]), (rep, layer)
                assert np.array_equal(k["h"].exps.cpu().numpy(), w["he"]), (rep, layer)
                assert np.array_equal(k["h"].desc.cpu().numpy(), w["hd"]), (rep, layer)
                for o, (q, f, rc1, _) in ((k["og"], w["g"]), (k["ou"], w["u"]), (k["od"], w["y"])):
                    assert rc1 == _abi.APX_OK
                    assert int(o.status[0].item()) == -1
                    assert np.array_equal(o.f32.cpu().numpy()[:o.n].view(np.uint32),
                                          f.view(np.uint32)), (rep, layer)
                assert np.array_equal(k["od"].q32.cpu().numpy()[:n_embd], w["y"][0])
        # the oracle's chain for the first layer (matvec_q8act, swiglu_quant, matvec_q8act)
        k = keep[0]
        c, e = synth.quant_act_np(synth.f32_to_q32(k["x"].x))
        s0, s1, s2 = k["seeds"]
        g = O.matvec_q8act_mt(t, synth.payload(t, n_ff, n_embd, s0), n_ff, n_embd, c,
                              O.exps_to_scales(e), 8, simd=True)
        u = O.matvec_q8act_mt(t, synth.payload(t, n_ff, n_embd, s1), n_ff, n_embd, c,
                              O.exps_to_scales(e), 8, simd=True)
        _, hcodes, hscales = O.swiglu_quant(g, u, carrier)
        y = O.matvec_q8act_mt(t, synth.payload(t, n_embd, n_ff, s2), n_embd, n_ff, hcodes,
                              hscales, 8, simd=True)
        assert np.array_equal(k["od"].q32.cpu().numpy()[:n_embd], y)
    finally:
        lib.apx_plan_destroy(plan)


def test_plan_refusals_match_single_calls(be):
    """A refused activation, a wide activation on the checked rows, and an FFN whose gate
    holds an Inf scale below its width: each projection's refusal equals the per-call one, and
    the FFN's reader refuses."""
    torch = _torch()
    dev = torch.device("cuda:0")
    lib, ctx = be.lib, be.ctx
    t, n_embd, n_ff = Q4_K, 1024, 2048
    x_bad = synth.activation_f32(n_embd, 41)
    x_bad[17] = np.nan
    a_bad = DevAct(lib, ctx, n_embd, x=x_bad)
    x_wide = synth.activation_f32(n_embd, 42)
    x_wide[:256] *= np.float32(2.0 ** -28)  # an exponent spread past the fast fold (23)
    a_wide = DevAct(lib, ctx, n_embd, x=x_wide)
    a_ok = DevAct(lib, ctx, n_embd, seed=43)
    t1 = be.upload(t, synth.payload(t, 3000, n_embd, 44), 3000, n_embd)
    raw_g = synth.payload(t, n_ff, n_embd, 45).copy()
    row_bytes = (n_embd // 256) * 144
    raw_g[700 * row_bytes + 144 * 2: 700 * row_bytes + 144 * 2 + 2] = (0x00, 0x7C)  # d = +Inf
    tg = be.upload(t, raw_g, n_ff, n_embd)
    tu = be.upload(t, synth.payload(t, n_ff, n_embd, 46), n_ff, n_embd)
    td = be.upload(t, synth.payload(t, n_embd, n_ff, 47), n_embd, n_ff)
    h = DevAct(lib, ctx, n_ff, x=np.zeros(n_ff, np.float32))
    fs = torch.full((2,), -1, dtype=torch.int64, device=dev)
    o_bad, o_wide, o_g, o_u, o_d = Out(3000), Out(3000), Out(n_ff), Out(n_ff), Out(n_embd)
    acts = [a_bad.rec(), a_wide.rec(), a_ok.rec(), h.rec(ffn=0)]
    projs = [_proj(t1, 3000, n_embd, 0, o_bad), _proj(t1, 3000, n_embd, 1, o_wide),
             _proj(tg, n_ff, n_embd, 2, o_g, ffn=0, role=_abi.PLAN_GATE),
             _proj(tu, n_ff, n_embd, 2, o_u, ffn=0, role=_abi.PLAN_UP),
             _proj(td, n_embd, n_ff, 3, o_d)]
    plan, rc = _plan(lib, ctx, projs, acts, [_abi.PlanFfn(0, 3, None, fs.data_ptr())])
    assert plan, rc
    try:
        _run(lib, plan)
        for o, a in ((o_bad, a_bad), (o_wide, a_wide)):
            q, f, rc1, row1 = _single(lib, ctx, t1, 3000, n_embd, a.codes.data_ptr(),
                                      a.exps.data_ptr(), a.desc.data_ptr())
            assert _decode(lib, ctx, t1, 3000, o.status) == (rc1, row1)
            if rc1 == _abi.APX_OK:
                assert np.array_equal(o.q32.cpu().numpy(), q)
        assert _decode(lib, ctx, t1, 3000, o_bad.status)[0] == _abi.APX_ERR_QUANT_REFUSED
        assert _decode(lib, ctx, t1, 3000, o_wide.status)[0] == _abi.APX_OK
        assert _decode(lib, ctx, tg, n_ff, o_g.status) == (_abi.APX_ERR_NONFINITE_SCALE, 700)
        assert int(h.desc[0].item()) == _abi.APX_ERR_QUANT_REFUSED
        assert _decode(lib, ctx, td, n_embd, o_d.status)[0] == _abi.APX_ERR_QUANT_REFUSED
    finally:
        lib.apx_plan_destroy(plan)


def test_plan_create_refuses_bad_records(be):
    lib, ctx = be.lib, be.ctx
    a = DevAct(lib, ctx, 896, seed=3)
    t4 = be.upload(Q4_K, synth.payload(Q4_K, 512, 896, 4), 512, 896)
    t8 = be.upload(Q8_0, synth.payload(Q8_0, 512, 896, 5), 512, 896)
    o1, o2 = Out(512), Out(512)
    # families differ
    plan, rc = _plan(lib, ctx, [_proj(t4, 512, 896, 0, o1), _proj(t8, 512, 896, 0, o2)],
                     [a.rec()])
    assert not plan and rc == _abi.APX_ERR_INVALID_ARGUMENT
    # a width that is not the tensor's
    plan, rc = _plan(lib, ctx, [_proj(t4, 512, 800, 0, o1)], [a.rec()])
    assert not plan and rc == _abi.APX_ERR_LAYOUT_MISMATCH
    # an FFN reader before its FFN, and an FFN with two gates
    torch = _torch()
    fs = torch.full((2,), -1, dtype=torch.int64, device=torch.device("cuda:0"))
    tg = be.upload(Q4_K, synth.payload(Q4_K, 1024, 896, 6), 1024, 896)
    td = be.upload(Q4_K, synth.payload(Q4_K, 896, 1024, 7), 896, 1024)
    h = DevAct(lib, ctx, 1024, x=np.zeros(1024, np.float32))
    og, ou, od = Out(1024), Out(1024), Out(896)
    acts = [a.rec(), h.rec(ffn=0)]
    ffn = [_abi.PlanFfn(0, 1, None, fs.data_ptr())]
    good = [_proj(tg, 1024, 896, 0, og, 0, _abi.PLAN_GATE), _proj(tg, 1024, 896, 0, ou, 0,
                                                                  _abi.PLAN_UP),
            _proj(td, 896, 1024, 1, od)]
    plan, rc = _plan(lib, ctx, good, acts, ffn)
    assert plan, rc
    lib.apx_plan_destroy(plan)
    plan, rc = _plan(lib, ctx, [good[2], good[0], good[1]], acts, ffn)
    assert not plan and rc == _abi.APX_ERR_INVALID_ARGUMENT
    plan, rc = _plan(lib, ctx, [good[0], _proj(tg, 1024, 896, 0, ou, 0, _abi.PLAN_GATE),
                                good[2]], acts, ffn)
    assert not plan and rc == _abi.APX_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("t,n_embd,n_ff", [(Q4_K, 896, 4864), (Q4_K, 8192, 1024)])
def test_plan_ffn_peer_destinations(be, t, n_embd, n_ff):
    """An FFN's peer destinations (apx_plan_ffn.n_peers: where a row shard's SwiGLU + quant_act
    blocks and its slice descriptor also go, one per other rank) hold exactly what the FFN writes
    into its own activation, on every launch; the chain's down is unchanged.  Here the
    destinations are other buffers of the same GPU (L = 1 gate/up rows, and L = 4)."""
    torch = _torch()
    dev = torch.device("cuda:0")
    lib, ctx = be.lib, be.ctx
    projs, acts, ffns, keep = _ffn_layers(be, t, n_embd, n_ff, 1, 0, 950)
    pad = lib.apx_act_padded_len(n_ff)
    peers = [(torch.zeros(pad, dtype=torch.int8, device=dev),
              torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev),
              torch.zeros(8, dtype=torch.int32, device=dev)) for _ in range(3)]
    f = ffns[0]
    f.n_peers = len(peers)
    for i, (pc, pe, pd) in enumerate(peers):
        f.d_peer_codes[i] = pc.data_ptr()
        f.d_peer_exps[i] = pe.data_ptr()
        f.d_peer_desc[i] = pd.data_ptr()
    plan, rc = _plan(lib, ctx, projs, acts, ffns)
    assert plan, rc
    try:
        want = _separate_chain(be, keep[0], n_embd, n_ff, 0)
        k = keep[0]
        for rep in range(2):
            for o in (k["og"], k["ou"], k["od"]):
                o.reset()
            k["f_status"].fill_(-1)
            for pc, pe, pd in peers:
                pc.zero_()
                pe.fill_(0xFF)
                pd.zero_()
            _run(lib, plan)
            assert int(k["f_status"][0].item()) == -1
            hc = k["h"].codes.cpu().numpy()
            he = k["h"].exps.cpu().numpy()
            hd = k["h"].desc.cpu().numpy()
            assert np.array_equal(hc, want["hc"]) and np.array_equal(he, want["he"])
            assert np.array_equal(hd, want["hd"])
            for pc, pe, pd in peers:
                assert np.array_equal(pc.cpu().numpy()[:n_ff], hc[:n_ff]), rep
                assert np.array_equal(pe.cpu().numpy()[:(n_ff + 31) // 32],
                                      he[:(n_ff + 31) // 32]), rep
                assert np.array_equal(pd.cpu().numpy(), hd), rep
            assert np.array_equal(k["od"].q32.cpu().numpy()[:n_embd], want["y"][0])
    finally:
        lib.apx_plan_destroy(plan)
