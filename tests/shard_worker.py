"""Rank bodies of the row-sharding tests (gloo on CPU, spawned processes).

Each rank computes its shard with the CPU oracle behind the backend interface `RowShard`
uses, so the tests exercise the sharding logic (row split, payload slices, all-gather
order, first-refusal merge, status reduction) without a GPU.
"""
import os
import traceback

import numpy as np

from oracle import oracle as O
from apeiron_b200 import _abi, chart, shard, synth


class OracleBackend:
    """`upload` / `matvec_q8act` of chart.Backend, computed by the oracle."""

    def upload(self, ggml_type, raw, n_out, n_in):
        return (ggml_type, np.array(raw, dtype=np.uint8, copy=True), n_out, n_in)

    def matvec_q8act(self, ggml_type, tensor, n_out, n_in, q):
        _, raw, _, _ = tensor
        out, err = O.matvec_q8act_row(ggml_type, raw, n_out, n_in, q.codes, q.scales)
        if err is not None:
            e = _abi.ApxErr()
            for f, _ in _abi.ApxErr._fields_:
                if hasattr(err, f):
                    setattr(e, f, getattr(err, f))
            chart._raise(e)
        return out


def cases():
    """(name, ggml_type, raw, n_out, n_in, QuantAct)."""
    out = []
    for name, t, n_out, n_in, seed in (("q4k", 12, 200, 512, 3), ("q8", 8, 97, 96, 4),
                                       ("q6k", 14, 64, 256, 5), ("q4k_ragged", 12, 70, 300, 6)):
        raw = synth.payload(t, n_out, n_in, seed)
        x = synth.activation_f32(n_in, seed + 100)
        c, e = synth.quant_act_np(synth.f32_to_q32(x))
        out.append((name, t, raw, n_out, n_in, chart.QuantAct.from_exps(e, c)))
    # non-finite scales: rows 70 and 80 of a Q8_0 tensor (both on the last rank of 2), and a
    # second tensor with one more at row 10
    t, n_out, n_in = 8, 97, 96
    raw = synth.payload(t, n_out, n_in, 7).copy()
    rb = shard.row_bytes(t, n_in)
    raw[70 * rb + 34: 70 * rb + 36] = (0x00, 0x7C)   # +Inf, block 1 of row 70
    raw[80 * rb: 80 * rb + 2] = (0x01, 0x7E)         # NaN, block 0 of row 80
    x = synth.activation_f32(n_in, 8)
    c, e = synth.quant_act_np(synth.f32_to_q32(x))
    q = chart.QuantAct.from_exps(e, c)
    out.append(("nonfinite_late", t, raw, n_out, n_in, q))
    raw2 = raw.copy()
    raw2[10 * rb + 2 * 34: 10 * rb + 2 * 34 + 2] = (0x00, 0xFC)  # -Inf, block 2 of row 10
    out.append(("nonfinite_early", t, raw2, n_out, n_in, q))
    return out


def run(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        be = OracleBackend()
        report = {}
        for name, t, raw, n_out, n_in, q in cases():
            rs = shard.RowShard(be, t, raw, n_out, n_in, rank, world, dist, "cpu")
            try:
                y = rs.matvec_q8act(q)
                report[name] = ("ok", y.tolist())
            except chart.MatvecError as e:
                report[name] = ("err", type(e).__name__, e.args, e.row)
            # the device path's status reduction, on CPU tensors: every rank's word (a local
            # refusal at its row 3 for odd ranks) folded with the shard's non-finite scale
            w = torch.full((2,), -1, dtype=torch.int64)
            if rank % 2 == 1 and rs.rows > 3:
                w[0] = (3 << 24) | (_abi.APX_ERR_OUTPUT_OVERFLOW << 16)
            rs.reduce_status(w)
            report[name + "/status"] = int(w[0].item())
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.array([report], dtype=object))
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(result_dir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise
