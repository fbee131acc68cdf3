"""Activations whose exponent spread is past the fast fold's limit (Q4_K 23, Q6_K 22) while the
call bound still holds (chart/mod.rs:362-383) take the wide fold: the fast fold on exponents
relative to each super-block's own smallest, or one 128-bit term per group when the spread
inside a super-block is wide too.  Both must equal the oracle's matvec_fixed bit for bit, in
the one-wave kernel, the streaming kernel and a step plan.

The one-wave kernel splits the units of a long row tile over up to 8 CTAs of one thread-block
cluster (partial sums meeting in distributed shared memory), over more through global scratch
and an arrival counter; shapes of both are checked here as well."""
import numpy as np
import pytest

from oracle import oracle as O
from apeiron_b200 import _abi, synth
from apeiron_b200.chart import QuantAct

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q6_K = 8, 12, 14


@pytest.fixture(scope="module")
def be():
    from apeiron_b200.chart import Backend
    b = Backend(0)
    yield b
    b.close()


def wide_x(n_in, seed, pattern, shift=28):
    """f32 activations ~N(0,1) with some 32-element blocks scaled by 2^-shift:
    "super" scales whole 256-element super-blocks (every other one), so each super-block is
    narrow and the call is wide; "blocks" scales every other 32-element block, so every
    super-block is wide too."""
    x = synth.activation_f32(n_in, seed).astype(np.float32)
    nb = (n_in + 31) // 32
    for b in range(nb):
        hit = (b // 8) % 2 == 1 if pattern == "super" else b % 2 == 1
        if hit:
            x[32 * b:32 * b + 32] *= np.float32(2.0 ** -shift)
    return x


def quant(x):
    codes, scales = O.quant_act(synth.f32_to_q32(x))
    return QuantAct.from_parts(scales, codes)


def spread(q):
    ex = q.exps()
    e = ex[ex != 0xFF].astype(int)
    return int(e.max() - e.min())


def check(be, t, raw, n_out, n_in, q):
    want = O.matvec_q8act(t, raw, n_out, n_in, q.codes, q.scales)
    assert not isinstance(want, tuple), want
    got = be.matvec_q8act(t, raw, n_out, n_in, q)
    assert np.array_equal(got, want)


# one-wave L = 1, one-wave L = 4 (long rows), the streaming kernel
WIDE_SHAPES = [(300, 2048), (64, 8960), (20000, 4096)]


@pytest.mark.parametrize("t", [Q4_K, Q6_K, Q8_0])
@pytest.mark.parametrize("pattern", ["super", "blocks"])
@pytest.mark.parametrize("n_out,n_in", WIDE_SHAPES)
def test_wide_spread_matvec(be, t, pattern, n_out, n_in):
    q = quant(wide_x(n_in, 31 + n_in, pattern))
    assert spread(q) > 23, spread(q)  # past every family's fast fold
    raw = synth.payload(t, n_out, n_in, 900 + n_out)
    check(be, t, raw, n_out, n_in, q)


@pytest.mark.parametrize("t", [Q4_K, Q6_K])
def test_wide_spread_extremes(be, t):
    """Spreads of about 44 (blocks scaled up by 2^16 and down by 2^-28, the largest exponent
    still inside the call bound for this width), in whole super-blocks and inside one, and a
    super-block whose groups reach both ends."""
    n_out, n_in = 257, 1024
    raw = synth.payload(t, n_out, n_in, 77)
    for pattern in ("super", "blocks"):
        x = wide_x(n_in, 11, pattern).reshape(-1, 32)
        x[::3] *= np.float32(2.0 ** 16)  # every third 32-element block scaled up
        x = x.reshape(-1)
        q = quant(x)
        assert spread(q) > 40, spread(q)
        check(be, t, raw, n_out, n_in, q)
    x = synth.activation_f32(n_in, 5).astype(np.float32)
    x[32:64] *= np.float32(2.0 ** -28)
    x[64:96] *= np.float32(2.0 ** 16)
    x[700:732] *= np.float32(2.0 ** -20)
    check(be, t, raw, n_out, n_in, quant(x))


@pytest.mark.parametrize("t,n_out,n_in", [
    (Q4_K, 1024, 28672),  # 128 row tiles of 28 units: clusters of 3 CTAs
    (Q8_0, 600, 30000),   # ragged K: 59 units a row tile, clusters of 5
    (Q6_K, 64, 20480),    # clusters of 2
    (Q4_K, 40, 131072),   # 128 units a row tile: 11 CTAs, global scratch and counters
    (Q4_K, 1536, 8960),   # no split (192 CTAs of 9 warps)
    (Q4_K, 3584, 8192),   # 448 CTAs of 8 warps: weights in shared memory (64 registers)
    (Q8_0, 2048, 8192),   # shared-memory weights and clusters of 2
])
def test_cluster_split_shapes(be, t, n_out, n_in):
    x = synth.activation_f32(n_in, 3 + n_in)
    q = quant(x)
    raw = synth.payload(t, n_out, n_in, 40 + n_out)
    for _ in range(2):  # a second call on the same tensor
        check(be, t, raw, n_out, n_in, q)


@pytest.mark.parametrize("t", [Q4_K, Q6_K])
def test_wide_spread_plan(be, t):
    """Wide activations read by a step plan (staged through its shared-memory ring), with a
    narrow one in the same plan: every projection equals the oracle."""
    import ctypes as C
    import torch
    lib, ctx = be.lib, be.ctx
    dev = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    n_in = 2048
    xs = [wide_x(n_in, 71, "super"), wide_x(n_in, 72, "blocks"), synth.activation_f32(n_in, 73)]
    acts, recs = [], []
    for x in xs:
        pad = lib.apx_act_padded_len(n_in)
        dc = torch.zeros(pad, dtype=torch.int8, device=dev)
        de = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
        dd = torch.zeros(8, dtype=torch.int32, device=dev)
        dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev)
        assert lib.apx_quant_f32_async(ctx, dx.data_ptr(), n_in, dc.data_ptr(), de.data_ptr(),
                                       dd.data_ptr(), st) == 0
        acts.append((dc, de, dd, dx))
        recs.append(_abi.PlanAct(dc.data_ptr(), de.data_ptr(), dd.data_ptr(), -1, 0))
    shapes = [(3000, 0), (700, 1), (4096, 2), (20000, 1)]
    raws = [synth.payload(t, n, n_in, 80 + i) for i, (n, _) in enumerate(shapes)]
    tens = [be.upload(t, r, n, n_in) for r, (n, _) in zip(raws, shapes)]
    outs = [(torch.zeros(n, dtype=torch.int64, device=dev),
             torch.zeros(n, dtype=torch.float32, device=dev),
             torch.full((2,), -1, dtype=torch.int64, device=dev)) for n, _ in shapes]
    projs = [_abi.PlanProj(tn.handle, n, n_in, a, -1, 0, 0, o[0].data_ptr(), o[1].data_ptr(),
                           o[2].data_ptr()) for tn, (n, a), o in zip(tens, shapes, outs)]
    P = (_abi.PlanProj * len(projs))(*projs)
    A = (_abi.PlanAct * len(recs))(*recs)
    F = (_abi.PlanFfn * 1)()
    err = _abi.ApxErr()
    plan = lib.apx_plan_create(ctx, P, len(projs), A, len(recs), F, 0, C.byref(err))
    assert plan, err.code
    try:
        torch.cuda.synchronize()
        for _ in range(2):
            for o in outs:
                o[2].fill_(-1)
            assert lib.apx_plan_run_async(plan, st) == 0
            torch.cuda.synchronize()
            for raw, (n, a), o in zip(raws, shapes, outs):
                dc, de = acts[a][0], acts[a][1]
                codes = dc.cpu().numpy()[:n_in]
                exps = de.cpu().numpy()[:(n_in + 31) // 32]
                if a < 2:
                    e = exps[exps != 0xFF].astype(int)
                    assert e.max() - e.min() > 23
                want = O.matvec_q8act(t, raw, n, n_in, codes, O.exps_to_scales(exps))
                assert int(o[2][0].item()) == -1
                assert np.array_equal(o[0].cpu().numpy(), want)
    finally:
        lib.apx_plan_destroy(plan)


@pytest.mark.parametrize("t", [Q4_K, Q6_K])
def test_wide_spread_prefill_f32(be, t):
    """The f32 prefill entry (quantize + digit-plane GEMM): tokens whose blocks spread past the
    three-digit route take the wide route, narrow tokens the tensor cores, in one call; every
    column's Q32.32 outputs equal the oracle's, and a second call on the same tensor too."""
    import torch
    lib, ctx = be.lib, be.ctx
    dev = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    n_out, n_in, k = 700, 2048, 40
    raw = synth.payload(t, n_out, n_in, 321)
    ten = be.upload(t, raw, n_out, n_in)
    xs = np.stack([wide_x(n_in, 500 + c, "blocks" if c % 3 == 0 else "super")
                   if c % 2 == 0 else synth.activation_f32(n_in, 500 + c) for c in range(k)])
    dx = torch.from_numpy(np.ascontiguousarray(xs, dtype=np.float32)).to(dev)
    y = torch.zeros(k * n_out, dtype=torch.int64, device=dev)
    ys = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    want = []
    for c in range(k):
        q = quant(xs[c])
        if c % 2 == 0:
            assert spread(q) > 15
        want.append(O.matvec_q8act(t, raw, n_out, n_in, q.codes, q.scales))
    for _ in range(2):
        y.zero_()
        ys.fill_(-1)
        assert lib.apx_matmat_f32_async(ctx, ten.handle, n_out, n_in, k, dx.data_ptr(), n_in,
                                        y.data_ptr(), None, ys.data_ptr(), st) == 0
        torch.cuda.synchronize()
        assert bool((ys[0::2] == -1).all().item())
        got = y.cpu().numpy().reshape(k, n_out)
        for c in range(k):
            assert np.array_equal(got[c], want[c]), c
