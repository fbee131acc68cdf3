"""GPU parity of the column quantizer (apx_quant_f32_cols_async): f32_to_fixed then
quant_act per column (src/engine/num/f32_convert.rs:44-49, src/engine/chart/mod.rs:258-334).

The device kernel has a 32-bit route on the f32 fields for blocks whose absmax is at most
127·2^24 and the Q32.32 route for the rest; the columns below put every block kind beside
ordinary ones (huge but accepted values, -2^31, values refused by f32_to_fixed or by
act_scale, subnormals, values that round to zero in Q32.32).  Bar: codes, exponent bytes and
descriptor identical to the oracle's restatement, refusal where it returns None.
"""
import numpy as np
import pytest

from oracle import oracle as O

from apeiron_b200.chart import Backend
from chart_inputs import f32_block_kinds as columns

pytestmark = pytest.mark.gpu

REFUSED = 10


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    yield b
    b.close()


def expected(col):
    bits = col.view(np.uint32)
    v = [O.f32_to_q32(int(b)) for b in bits]
    if any(t is None for t in v):
        return None
    return O.quant_act(np.array(v, dtype=np.int64))


@pytest.mark.parametrize("n", [1, 37, 128, 200, 896, 4864])
def test_quant_cols_matches_oracle(be, n):
    import torch

    lib = be.lib
    x = columns(n, 77 + n)
    k = x.shape[0]
    dev = torch.device("cuda:0")
    dx = torch.from_numpy(x).to(dev)
    pad = lib.apx_act_padded_len(n)
    codes = torch.zeros(k * pad, dtype=torch.int8, device=dev)
    exps = torch.full((k * pad // 32,), 0xEE, dtype=torch.uint8, device=dev)
    descs = torch.zeros(k * 8, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.apx_quant_f32_cols_async(be.ctx, dx.data_ptr(), n, k, codes.data_ptr(),
                                        exps.data_ptr(), descs.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    codes = codes.cpu().numpy().reshape(k, pad)
    exps = exps.cpu().numpy().reshape(k, pad // 32)
    descs = descs.cpu().numpy().reshape(k, 8)
    nb = (n + 31) // 32
    for c in range(k):
        want = expected(x[c])
        if want is None:
            assert descs[c, 0] == REFUSED, c
            continue
        wc, ws = want
        we = O.scales_to_exps(ws)
        assert descs[c, 0] == 0, c
        assert np.array_equal(codes[c, :n], wc), c
        assert np.array_equal(exps[c, :nb], we), c
        nz = we != 0xFF
        assert descs[c, 4] == nz.sum(), c
        assert descs[c, 3] == n, c
        if nz.any():
            assert (descs[c, 1], descs[c, 2]) == (we[nz].min(), we[nz].max()), c
        else:
            assert descs[c, 2] == -1, c
