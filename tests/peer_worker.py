"""Rank bodies of the peer-store gather GPU test (one process per GPU, gloo for the one-time
exchange of buffer handles; the outputs move by the library's own peer stores)."""
import os
import traceback

import numpy as np

from oracle import oracle as O
from apeiron_b200 import _abi, shard, synth


def mats():
    out = []
    for t, n_out, n_in, seed in ((12, 1000, 512, 1), (8, 4864, 896, 2), (14, 300, 256, 3)):
        raw = synth.payload(t, n_out, n_in, seed).copy()
        if seed == 3:  # a non-finite scale on row 250 (the last rank's rows when world = 2)
            raw[250 * shard.row_bytes(t, n_in) + 208: 250 * shard.row_bytes(t, n_in) + 210] = \
                (0x00, 0x7C)
        out.append((t, raw, n_out, n_in))
    return out


def run(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.cuda.set_device(rank)
        from apeiron_b200.chart import Backend
        be = Backend(rank)
        lib = be.lib
        dev = torch.device(f"cuda:{rank}")
        ms = mats()
        shards = [shard.RowShard(be, t, raw, n_out, n_in, rank, world, dist, "cpu")
                  for t, raw, n_out, n_in in ms]
        acts, qs = [], []
        for t, raw, n_out, n_in in ms:
            x = synth.activation_f32(n_in, 77 + n_in)
            c, e = synth.quant_act_np(synth.f32_to_q32(x))
            pad = lib.apx_act_padded_len(n_in)
            codes = torch.zeros(pad, dtype=torch.int8, device=dev)
            codes[:n_in] = torch.from_numpy(c).to(dev)
            exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
            exps[:e.size] = torch.from_numpy(e).to(dev)
            desc = torch.zeros(8, dtype=torch.int32, device=dev)
            stream = torch.cuda.current_stream().cuda_stream
            assert lib.apx_act_describe_async(be.ctx, codes.data_ptr(), exps.data_ptr(), n_in,
                                              desc.data_ptr(), stream) == 0
            acts.append((codes, exps, desc))
            qs.append((c, e))
        g = shard.PeerGather(lib, be.ctx, shards, timeout_us=300_000)
        st = torch.full((len(ms), 2), -1, dtype=torch.int64, device=dev)
        merged = torch.full((len(ms), 2), -1, dtype=torch.int64, device=dev)
        stream = torch.cuda.current_stream().cuda_stream
        report = {"rows": [(sh.r0, sh.r1) for sh in shards]}
        for call in range(3):  # both parities, and a third publication over the first
            parity = g.run(acts, st, merged, stream)
            torch.cuda.synchronize()
            report[f"call{call}"] = ([g.read(j, parity).tolist() for j in range(len(ms))],
                                     merged[:, 0].cpu().tolist())
        # a rank that skips a publication: the others' bounded wait gives up
        dist.barrier()
        if rank != world - 1:
            g.run(acts, st, merged, stream)
            torch.cuda.synchronize()
            report["timeout"] = merged[:, 0].cpu().tolist()
        dist.barrier()
        torch.cuda.synchronize()
        dist.barrier()
        g.close()
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.array([report], dtype=object))
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(result_dir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise
