"""apx_matvec_f32_noalloc, the allocation-free entry point, against apx_matvec_f32.

Callers that cannot allocate device memory while running (a fixed HBM budget reserved at
start-up, a hard GPU memory quota, a decode loop that cannot absorb an allocation) use the
entry point that stages its quantized activation in a fixed array inside the library.  It
must return exactly what the allocating entry point returns: the f32 path is bit-exact (each
output is the exact Q32.32 projection rounded once to f32), so the tolerance here is zero,
the same as the other f32-path tests.  Two calls in a row with different activations check
that the shared array carries nothing from one call into the next.

Refusals must match too: an activation the quantizer refuses (NaN, Inf, |x| >= 2^31), a row
with a non-finite weight scale, and a call over the first n_out < n rows of the tensor.

This file is collected last (test_zz_*), so a run that stops at the first failure has run
every other test before it; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from apeiron_b200 import _abi, synth
from apeiron_b200.chart import Backend

pytestmark = pytest.mark.gpu


def _decode(be, tensor, status):
    st = _abi.CallStatus(int(status[0].item()) & ((1 << 64) - 1),
                         int(status[1].item()) & ((1 << 64) - 1))
    err = _abi.ApxErr()
    return be.lib.apx_status_decode(be.ctx, tensor.handle, C.byref(st), C.byref(err))


@pytest.mark.parametrize("ggml_type,n_out,n_in", [(12, 1536, 8960), (8, 4864, 896)])
def test_noalloc_matches_the_allocating_entry_point(ggml_type, n_out, n_in):
    import torch

    be = Backend(0)
    try:
        raw = synth.payload(ggml_type, n_out, n_in, 404)
        tensor = be.upload(ggml_type, raw, n_out, n_in)
        dev = torch.device("cuda:0")
        stream = torch.cuda.current_stream(dev).cuda_stream
        for seed in (31, 32):  # two calls in a row, different activations
            x = synth.activation_f32(n_in, seed)
            want = be.matvec_f32(tensor, x)
            dx = torch.from_numpy(x).to(dev)
            dy = torch.full((n_out,), float("nan"), dtype=torch.float32, device=dev)
            status = torch.zeros(2, dtype=torch.int64, device=dev)
            rc = be.lib.apx_matvec_f32_noalloc(be.ctx, tensor.handle, n_out, n_in,
                                               dx.data_ptr(), dy.data_ptr(),
                                               status.data_ptr(), stream)
            assert rc == _abi.APX_OK
            torch.cuda.synchronize(dev)
            assert _decode(be, tensor, status) == _abi.APX_OK
            assert np.array_equal(dy.cpu().numpy(), want)
    finally:
        be.close()


def _both(be, tensor, n_out, n_in, x):
    """(rc, row, y) of apx_matvec_f32 and of apx_matvec_f32_noalloc on the same input."""
    import torch

    err = _abi.ApxErr()
    y = np.full(max(n_out, 1), np.nan, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rc = be.lib.apx_matvec_f32(be.ctx, tensor.handle, n_out, n_in,
                               x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p),
                               C.byref(err))
    want = (rc, err.row if rc else None, y[:n_out] if rc == 0 else None)
    dev = torch.device("cuda:0")
    dx = torch.from_numpy(x).to(dev)
    dy = torch.full((max(n_out, 1),), float("nan"), dtype=torch.float32, device=dev)
    status = torch.zeros(2, dtype=torch.int64, device=dev)
    assert be.lib.apx_matvec_f32_noalloc(be.ctx, tensor.handle, n_out, n_in, dx.data_ptr(),
                                         dy.data_ptr(), status.data_ptr(),
                                         torch.cuda.current_stream(dev).cuda_stream) == 0
    torch.cuda.synchronize(dev)
    st = _abi.CallStatus(int(status[0].item()) & ((1 << 64) - 1),
                         int(status[1].item()) & ((1 << 64) - 1))
    err2 = _abi.ApxErr()
    rc2 = be.lib.apx_status_decode_rows(be.ctx, tensor.handle, n_out, C.byref(st),
                                        C.byref(err2))
    got = (rc2, err2.row if rc2 else None, dy.cpu().numpy()[:n_out] if rc2 == 0 else None)
    return want, got


def _same(want, got):
    assert want[0] == got[0] and want[1] == got[1], (want[:2], got[:2])
    if want[0] == _abi.APX_OK:
        assert np.array_equal(want[2].view(np.uint32), got[2].view(np.uint32))


def test_noalloc_refusals_and_partial_rows_match():
    """A refusing activation (NaN, +Inf, 2^31), a call over the first rows only, and a row whose
    block scale is Inf: the same result or refusal as apx_matvec_f32, twice in a row."""
    be = Backend(0)
    try:
        n_out, n_in = 300, 1024
        raw = synth.payload(8, n_out, n_in, 77)
        tensor = be.upload(8, raw, n_out, n_in)
        x = synth.activation_f32(n_in, 5)
        for bad in (np.nan, np.inf, 2.0 ** 31):
            xb = x.copy()
            xb[700] = bad
            want, got = _both(be, tensor, n_out, n_in, xb)
            assert want[0] == _abi.APX_ERR_QUANT_REFUSED
            _same(want, got)
            _same(*_both(be, tensor, n_out, n_in, x))  # the next call is unaffected
        for rows in (1, 31, 257):
            _same(*_both(be, tensor, rows, n_in, synth.activation_f32(n_in, rows)))
        raw2 = raw.copy()
        raw2[(41 * (n_in // 32) + 3) * 34: (41 * (n_in // 32) + 3) * 34 + 2] = (0x00, 0x7C)
        t2 = be.upload(8, raw2, n_out, n_in)
        want, got = _both(be, t2, n_out, n_in, x)
        assert want[0] == _abi.APX_ERR_NONFINITE_SCALE and want[1] == 41
        _same(want, got)
        _same(*_both(be, t2, 41, n_in, x))  # the rows before it project
    finally:
        be.close()


def test_noalloc_at_its_widest_activation():
    """n_in = APX_NOALLOC_MAX_N_IN: the codes end exactly at the end of the fixed array."""
    be = Backend(0)
    try:
        n_out, n_in = 96, _abi.NOALLOC_MAX_N_IN
        tensor = be.upload(8, synth.payload(8, n_out, n_in, 8), n_out, n_in)
        for seed in (1, 2):
            _same(*_both(be, tensor, n_out, n_in, synth.activation_f32(n_in, seed)))
    finally:
        be.close()


def test_noalloc_rejects_widths_beyond_its_array():
    be = Backend(0)
    try:
        n_in = _abi.NOALLOC_MAX_N_IN + 32
        rc = be.lib.apx_matvec_f32_noalloc(be.ctx, 1, 1, n_in, 1, 1, 1, None)
        assert rc == _abi.APX_ERR_TOO_LARGE
    finally:
        be.close()
