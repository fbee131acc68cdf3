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

pytestmark = pytest.mark.gpu

REFUSED = 10


@pytest.fixture(scope="module")
def be():
    b = Backend(0)
    yield b
    b.close()


def _f(bits):
    return np.array(bits, dtype=np.uint32).view(np.float32)


def columns(n, seed):
    """Columns of length n, each stressing one block kind (index 0 in every block-sized
    stretch where the kind is a single value)."""
    rng = np.random.default_rng(seed)
    base = rng.standard_normal(n).astype(np.float32)
    cols = [base.copy()]
    cols.append((base * np.float32(1e-12)).astype(np.float32))      # tiny: rounds in Q32.32
    sub = rng.integers(0, 1 << 23, n, dtype=np.uint32) | (rng.integers(0, 2, n, dtype=np.uint32) << 31)
    cols.append(_f(sub))                                              # subnormals
    big = base.copy()
    big[::7] = np.float32(-2.14e9)                                    # above 127·2^24: code -64
    cols.append(big)
    lo = base.copy()
    lo[0] = np.float32(-2147483648.0)                                 # -2^31: i64::MIN, accepted
    cols.append(lo)
    over = base.copy()
    over[n // 2] = np.float32(2147483648.0)                           # 2^31: refused
    cols.append(over)
    nan = base.copy()
    nan[-1] = np.float32(np.nan)
    cols.append(nan)
    inf = base.copy()
    inf[n // 3] = -np.float32(np.inf)
    cols.append(inf)
    cols.append(np.zeros(n, dtype=np.float32))
    edge = base.copy()
    edge[::5] = _f([0x4EFE0000])[0]                                   # exactly 127·2^24
    cols.append(edge)
    above = base.copy()
    above[n // 2] = _f([0x4EFE0001])[0]                               # one ulp above: code 64
    cols.append(above)                                                # leaves i64, refused
    wild = rng.integers(0, 0x4F000000, n, dtype=np.uint32) | (rng.integers(0, 2, n, dtype=np.uint32) << 31)
    cols.append(_f(wild))                                             # any finite |f| < 2^31
    mixed = base.copy()
    mixed[200:232] = np.float32(1.5e9)                                # one Q32.32 block
    mixed[40:72] = np.float32(3e-10)
    cols.append(mixed)
    return np.stack(cols)


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
