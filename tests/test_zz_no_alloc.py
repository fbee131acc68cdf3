"""apx_matvec_f32_noalloc, the allocation-free entry point, against apx_matvec_f32.

Callers that cannot allocate device memory while running (a fixed HBM budget reserved at
start-up, a hard GPU memory quota, a decode loop that cannot absorb an allocation) use the
entry point that stages its quantized activation in a fixed array inside the library.  It
must return exactly what the allocating entry point returns: the f32 path is bit-exact (each
output is the exact Q32.32 projection rounded once to f32), so the tolerance here is zero,
the same as the other f32-path tests.  Two calls in a row with different activations check
that the shared array carries nothing from one call into the next.

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


def test_noalloc_rejects_widths_beyond_its_array():
    be = Backend(0)
    try:
        n_in = _abi.NOALLOC_MAX_N_IN + 32
        rc = be.lib.apx_matvec_f32_noalloc(be.ctx, 1, 1, n_in, 1, 1, 1, None)
        assert rc == _abi.APX_ERR_TOO_LARGE
    finally:
        be.close()
