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

from apeiron_b200 import _abi
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
