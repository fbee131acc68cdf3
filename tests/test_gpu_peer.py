"""Row-sharded projections gathered by peer stores between GPUs (apx_gather_publish_async,
apeiron_b200/shard.py PeerGather): every rank holds the whole, exact output vector of every
projection in both buffer parities; the merged refusal word is the first refusing row of the
whole tensor; a rank that skips a publication makes the others' bounded wait report
APX_ERR_DEVICE_TIMEOUT instead of hanging.  Needs two GPUs (skipped otherwise)."""
import socket

import numpy as np
import pytest

from oracle import oracle as O
from apeiron_b200 import _abi, shard

import peer_worker

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_peer_gather_two_ranks(tmp_path):
    import multiprocessing as mp

    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=peer_worker.run, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = [f.read_text() for f in tmp_path.glob("*.err")]
    assert not errs, errs[0]
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    reps = [np.load(tmp_path / f"rank{r}.npy", allow_pickle=True)[0] for r in range(world)]
    ms = peer_worker.mats()
    from apeiron_b200 import synth
    for j, (t, raw, n_out, n_in) in enumerate(ms):
        x = synth.activation_f32(n_in, 77 + n_in)
        c, e = synth.quant_act_np(synth.f32_to_q32(x))
        out, err = O.matvec_q8act_row(t, raw, n_out, n_in, c, O.exps_to_scales(e))
        for call in range(3):
            for rep in reps:
                got, words = rep[f"call{call}"]
                if err is None:
                    assert words[j] == -1 and np.array_equal(np.array(got[j]), out), (j, call)
                else:
                    nf = shard.first_nonfinite(t, raw, n_out, n_in)
                    assert nf[0] == err.row
                    want = (nf[0] << 24) | (_abi.APX_ERR_NONFINITE_SCALE << 16) | nf[1]
                    assert words[j] == want, (j, call, words[j], want)
    timeout_word = _abi.APX_ERR_DEVICE_TIMEOUT << 16
    assert reps[0]["timeout"] == [timeout_word] * len(ms)


def test_gather_descriptor_ranges_are_checked():
    """A descriptor whose rows, keys, flags or counters reach past the gather buffer's `bytes` is
    refused on the host with APX_ERR_INVALID_ARGUMENT, before anything is launched (one GPU)."""
    import ctypes as C

    import torch
    from apeiron_b200 import synth
    from apeiron_b200.chart import Backend

    be = Backend(0)
    try:
        n_out, n_in = 64, 256
        t = be.upload(8, synth.payload(8, n_out, n_in, 3), n_out, n_in)
        dev = torch.device("cuda:0")
        buf = torch.zeros(4096 // 8, dtype=torch.int64, device=dev)
        st = torch.full((2,), -1, dtype=torch.int64, device=dev)
        ost = torch.full((2,), -1, dtype=torch.int64, device=dev)
        codes = torch.zeros(256, dtype=torch.int8, device=dev)
        exps = torch.full((8,), 255, dtype=torch.uint8, device=dev)
        desc = torch.zeros(8, dtype=torch.int32, device=dev)

        def base():
            d = _abi.GatherDesc()
            d.world, d.rank, d.nproj, d.timeout_us = 1, 0, 1, 1000
            d.peer[0] = buf.data_ptr()
            d.out_off, d.key_off, d.flag_off, d.ctr_off, d.bytes = 0, 1024, 1536, 2048, 4096
            d.rows_off[0], d.rows[0] = 0, n_out
            d.status[0], d.out_status[0] = st.data_ptr(), ost.data_ptr()
            return d

        def gather(d):
            return be.lib.apx_matvec_gather_async(be.ctx, t.handle, n_out, n_in,
                                                  codes.data_ptr(), exps.data_ptr(),
                                                  desc.data_ptr(), C.byref(d), 0, None)

        def publish(d):
            return be.lib.apx_gather_publish_async(be.ctx, C.byref(d), None)

        bad = _abi.APX_ERR_INVALID_ARGUMENT
        for field, value in (("bytes", 511), ("out_off", 4096 - 8 * n_out + 8)):
            d = base()
            setattr(d, field, value)
            assert gather(d) == bad, field
        d = base()
        d.rows_off[0] = (1 << 62)  # 8 · rows_off wraps around
        assert gather(d) == bad
        for field, value in (("key_off", 4096), ("flag_off", 4096), ("ctr_off", 4096 - 8)):
            d = base()
            setattr(d, field, value)
            assert publish(d) == bad, field
        torch.cuda.synchronize(dev)
    finally:
        be.close()
