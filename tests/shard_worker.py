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


class Held:
    """An uploaded shard: its bytes and geometry, and a handle for the device-path stand-in."""

    def __init__(self, handle, ggml_type, raw, n_out, n_in):
        self.handle, self.ggml_type, self.raw, self.n_out, self.n_in = \
            handle, ggml_type, raw, n_out, n_in


class OracleBackend:
    """`upload` / `matvec_q8act` of chart.Backend, computed by the oracle."""

    def __init__(self):
        self.held = {}

    def upload(self, ggml_type, raw, n_out, n_in):
        h = Held(len(self.held) + 1, ggml_type, np.array(raw, dtype=np.uint8, copy=True), n_out,
                 n_in)
        self.held[h.handle] = h
        return h

    def matvec_q8act(self, ggml_type, tensor, n_out, n_in, q):
        out, err = O.matvec_q8act_row(ggml_type, tensor.raw, n_out, n_in, q.codes, q.scales)
        if err is not None:
            e = _abi.ApxErr()
            for f, _ in _abi.ApxErr._fields_:
                if hasattr(err, f):
                    setattr(e, f, getattr(err, f))
            chart._raise(e)
        return out


class OracleLib:
    """`apx_matvec_async` over CPU tensors (pointers are host addresses): the shard's Q32.32
    outputs, or its refusal word, computed by the oracle."""

    def __init__(self, backend):
        self.be = backend

    def apx_matvec_async(self, ctx, handle, n_out, n_in, codes, exps, desc, out, f32, status,
                         stream):
        import ctypes as C
        h = self.be.held[handle]
        c = np.ctypeslib.as_array((C.c_int8 * n_in).from_address(codes)).copy()
        nb = (n_in + 31) // 32
        e = np.ctypeslib.as_array((C.c_uint8 * nb).from_address(exps)).copy()
        y, err = O.matvec_q8act_row(h.ggml_type, h.raw, n_out, n_in, c, O.exps_to_scales(e))
        if err is None:
            C.memmove(out, y.ctypes.data, 8 * n_out)
        else:
            word = np.array([(int(err.row) << 24) | (int(err.code) << 16) | (int(err.bits) & 0xFFFF)],
                            dtype=np.uint64).view(np.int64)
            C.memmove(status, word.ctypes.data, 8)
        return 0


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
        # the grouped device path: the first two projections (own activations) and the two
        # non-finite ones through one all-gather per group
        lib = OracleLib(be)
        cs = cases()
        for gname, idx in (("group_ok", [0, 2]), ("group_nf", [4, 5, 1])):
            shards = [shard.RowShard(be, cs[i][1], cs[i][2], cs[i][3], cs[i][4], rank, world,
                                     dist, "cpu") for i in idx]
            acts = []
            for i in idx:
                q = cs[i][5]
                acts.append((torch.from_numpy(q.codes.copy()), torch.from_numpy(q.exps().copy()),
                             torch.zeros(8, dtype=torch.int32)))
            _, _, length = shard.group_layout(shards)
            local = torch.zeros(length, dtype=torch.int64)
            gathered = torch.zeros(world * length, dtype=torch.int64)
            statuses = [torch.full((2,), -1, dtype=torch.int64) for _ in idx]
            shard.matvec_group_async(shards, lib, None, acts, local, gathered, statuses, None)
            g = gathered.numpy()
            report[gname] = [(shard.assemble_group(shards, g, j).tolist(), int(statuses[j][0]))
                             for j in range(len(idx))]
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.array([report], dtype=object))
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(result_dir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise
