"""Grouped projections over one activation (apx_matvec_group_async): q/k/v and gate/up of a
decode step in one launch.  Each member's Q32.32 outputs and refusal word equal its own
matvec_q8act (src/engine/chart/mod.rs:1887-1925) on the same activation."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from apeiron_b200 import _abi, synth
from apeiron_b200.chart import Backend

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    yield b
    b.close()


def _run(be, tens, n_in, x_seed=11, nonfinite_act=False):
    import torch

    lib = be.lib
    dev = torch.device("cuda:0")
    x = synth.activation_f32(n_in, x_seed)
    c, e = synth.quant_act_np(synth.f32_to_q32(x))
    pad = lib.apx_act_padded_len(n_in)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    codes[:n_in] = torch.from_numpy(c).to(dev)
    exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    exps[:e.size] = torch.from_numpy(e).to(dev)
    if nonfinite_act:
        exps[0] = 63  # an exponent byte no quant_act produces: the activation is refused
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_act_describe_async(be.ctx, codes.data_ptr(), exps.data_ptr(), n_in,
                                      desc.data_ptr(), stream) == 0
    outs = [torch.zeros(t.n_out, dtype=torch.int64, device=dev) for t in tens]
    stats = [torch.full((2,), -1, dtype=torch.int64, device=dev) for _ in tens]
    k = len(tens)
    handles = (C.c_uint64 * k)(*[t.handle for t in tens])
    optr = (C.c_void_p * k)(*[o.data_ptr() for o in outs])
    sptr = (C.c_void_p * k)(*[s_.data_ptr() for s_ in stats])
    assert lib.apx_matvec_group_async(be.ctx, handles, k, n_in, codes.data_ptr(), exps.data_ptr(),
                                      desc.data_ptr(), optr, None, sptr, stream) == 0
    torch.cuda.synchronize()
    return c, e, [o.cpu().numpy() for o in outs], [int(s_[0].item()) for s_ in stats]


@pytest.mark.parametrize("shapes", [
    [(12, 896, 896), (12, 128, 896), (12, 128, 896)],      # q, k, v
    [(12, 4864, 896), (12, 4864, 896)],                    # gate, up
    [(8, 4864, 896), (8, 896, 896), (8, 64, 896), (8, 33, 896)],
    [(14, 300, 512), (14, 64, 512)],
    [(12, 8960, 1536), (12, 1536, 1536)],
    [(12, 20000, 4096), (12, 128, 4096)],                  # a streaming member: one launch each
    [(8, 100, 256), (12, 100, 256)],                       # mixed families: one launch each
])
def test_group_equals_members(be, shapes):
    raws = [synth.payload(t, n_out, n_in, 40 + i) for i, (t, n_out, n_in) in enumerate(shapes)]
    tens = [be.upload(t, r, n_out, n_in) for (t, n_out, n_in), r in zip(shapes, raws)]
    n_in = shapes[0][2]
    c, e, outs, words = _run(be, tens, n_in)
    for (t, n_out, _), r, o, w in zip(shapes, raws, outs, words):
        want = O.matvec_q8act(t, r, n_out, n_in, c, O.exps_to_scales(e))
        assert w == -1 and np.array_equal(o, want), (t, n_out)


def test_group_refusals_stay_with_their_member(be):
    shapes = [(12, 896, 896), (12, 128, 896), (12, 128, 896)]
    raws = [synth.payload(t, n_out, n_in, 50 + i).copy() for i, (t, n_out, n_in) in
            enumerate(shapes)]
    rb = 4 * 144
    raws[1][70 * rb: 70 * rb + 2] = (0x00, 0x7C)  # +Inf d in row 70 of k: found at upload
    tens = [be.upload(t, r, n_out, n_in) for (t, n_out, n_in), r in zip(shapes, raws)]
    c, e, outs, words = _run(be, tens, 896)
    for i, ((t, n_out, n_in), r, o, w) in enumerate(zip(shapes, raws, outs, words)):
        word = _abi.CallStatus(w & ((1 << 64) - 1), 0)
        err = _abi.ApxErr()
        rc = be.lib.apx_status_decode(be.ctx, tens[i].handle, C.byref(word), C.byref(err))
        if i == 1:
            assert rc == _abi.APX_ERR_NONFINITE_SCALE and err.row == 70
        else:
            want = O.matvec_q8act(t, r, n_out, n_in, c, O.exps_to_scales(e))
            assert rc == 0 and np.array_equal(o, want)
    # an activation the descriptor refuses: every member's word says so
    _, _, _, words = _run(be, tens, 896, nonfinite_act=True)
    assert all(w != -1 and ((w >> 16) & 0xFF) == _abi.APX_ERR_INVALID_ARGUMENT for w in words)
