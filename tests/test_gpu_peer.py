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
