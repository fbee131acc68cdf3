"""Q5_0 weights (quant.rs:261-299): served by widening each block's five-bit codes (offset by
-16) into the Q8_0 layout at upload, which leaves every dequantized weight d·code unchanged.
Bar: Q32.32 outputs and refusals equal to the oracle's restatement of the reference's Q5_0
dequantization (num/dequant.rs:137-145, 357-390) under the matvec_q8act / matmat_q8act
contracts, on the GEMV and on the tcgen05 GEMM."""
import numpy as np
import pytest

from oracle import oracle as O
from chart_inputs import random_payload
from apeiron_b200 import chart, synth
from apeiron_b200.chart import Backend, QuantAct

pytestmark = pytest.mark.gpu

Q5_0 = 6


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    yield b
    b.close()


def _col(n_in, seed):
    c, e = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, seed)))
    return QuantAct.from_exps(e, c)


@pytest.mark.parametrize("n_out,n_in", [(896, 896), (4864, 896), (896, 4864), (300, 100),
                                        (151, 32), (40, 8192)])
def test_q5_0_gemv_matches_oracle(be, n_out, n_in):
    raw = random_payload(Q5_0, n_out, n_in, 0x2100, 0, 3 + n_in)
    q = _col(n_in, 7 + n_out)
    got = be.matvec_q8act(Q5_0, raw, n_out, n_in, q)
    want = O.matvec_q8act(Q5_0, raw, n_out, n_in, q.codes, q.scales)
    assert np.array_equal(got, want)


def test_q5_0_gemm_matches_oracle(be):
    n_out, n_in, k = 640, 896, 12
    raw = random_payload(Q5_0, n_out, n_in, 0x2400, 0, 31)
    qs = [_col(n_in, 50 + c) for c in range(k)]
    got = np.stack(be.matmat_q8act(Q5_0, raw, n_out, n_in, qs))
    want = O.matmat_q8act(Q5_0, raw, n_out, n_in, np.stack([q.codes for q in qs]),
                          np.stack([q.scales for q in qs]))
    assert np.array_equal(got, want)


def test_q5_0_refusals(be):
    n_out, n_in = 64, 256
    raw = random_payload(Q5_0, n_out, n_in, 0x2100, 0, 9)
    bad = raw.copy()
    bad[(5 * (n_in // 32) + 3) * 22: (5 * (n_in // 32) + 3) * 22 + 2] = (0x00, 0x7C)   # +Inf, row 5
    q = _col(n_in, 3)
    with pytest.raises(chart.NonFiniteScale) as e:
        be.matvec_q8act(Q5_0, bad, n_out, n_in, q)
    want = O.matvec_q8act(Q5_0, bad, n_out, n_in, q.codes, q.scales)
    assert isinstance(want, tuple) and e.value.bits == want[4]
    with pytest.raises(chart.ShortPayload) as e:
        be.matvec_q8act(Q5_0, raw[:-1], n_out, n_in, q)
    assert (e.value.need, e.value.have) == (n_out * (n_in // 32) * 22, raw.size - 1)
