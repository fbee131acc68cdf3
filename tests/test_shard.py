"""Row sharding of the projections (apeiron_b200/shard.py) on CPU: the split, the payload
slices, the non-finite scan, and, with gloo ranks (world sizes 2 and 3, spawned processes),
the all-gather order and the first-refusal merge of the host and device interfaces against
the whole-tensor oracle (src/engine/chart/ffn.rs:659-661,705-726)."""
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O
from apeiron_b200 import _abi, chart, shard, synth

import shard_worker


def test_row_split_covers_rows_in_aligned_contiguous_ranges():
    for n_out in (0, 1, 31, 32, 33, 97, 1536, 8192, 28672, 151936):
        for world in (1, 2, 3, 4, 8):
            sp = shard.row_split(n_out, world)
            assert len(sp) == world and sp[0][0] == 0 and sp[-1][1] == n_out
            for (a, b), (c, d) in zip(sp, sp[1:]):
                assert b == c and a <= b
            assert all(a % shard.ROW_ALIGN == 0 for a, _ in sp)
            sizes = [b - a for a, b in sp]
            if n_out % (shard.ROW_ALIGN * world) == 0:
                assert len(set(sizes)) == 1
            assert max(sizes) - min(sizes) <= shard.ROW_ALIGN + n_out % shard.ROW_ALIGN


def test_payload_rows_are_the_rows():
    t, n_out, n_in = 12, 70, 300
    raw = synth.payload(t, n_out, n_in, 1)
    rb = shard.row_bytes(t, n_in)
    assert raw.size == n_out * rb
    assert np.array_equal(shard.payload_rows(t, raw, n_out, n_in, 32, 64), raw[32 * rb: 64 * rb])
    with pytest.raises(chart.ShortPayload):
        shard.check_payload(t, raw.size - 1, n_out, n_in)


@pytest.mark.parametrize("t", [8, 12, 14])
def test_first_nonfinite_in_row_then_dequant_order(t):
    n_out, n_in = 9, 512
    raw = synth.payload(t, n_out, n_in, 2).copy()
    assert shard.first_nonfinite(t, raw, n_out, n_in) is None
    qk, bb = chart.GEOM[t]
    blocks = -(-n_in // qk)
    off = {8: [0], 12: [0, 2], 14: [208]}[t]
    # two bad scales in row 5 (the later one first in memory order of the row's blocks) and
    # one in row 7: row 5's first in dequantization order wins
    rb = blocks * bb
    raw[5 * rb + 1 * bb + off[-1]: 5 * rb + 1 * bb + off[-1] + 2] = (0x00, 0x7C)
    raw[5 * rb + 1 * bb + off[0]: 5 * rb + 1 * bb + off[0] + 2] = (0x12, 0x7E)
    raw[7 * rb + off[0]: 7 * rb + off[0] + 2] = (0x00, 0xFC)
    row, bits = shard.first_nonfinite(t, raw, n_out, n_in)
    assert row == 5 and bits == 0x7E12


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_projections_equal_the_whole_tensor(world, tmp_path):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=shard_worker.run, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    errs = [f.read_text() for f in tmp_path.glob("*.err")]
    assert not errs, errs[0]
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    reports = [np.load(tmp_path / f"rank{r}.npy", allow_pickle=True)[0] for r in range(world)]
    for name, t, raw, n_out, n_in, q in shard_worker.cases():
        out, err = O.matvec_q8act_row(t, raw, n_out, n_in, q.codes, q.scales)
        for rep in reports:  # every rank holds the same answer
            assert rep[name] == reports[0][name]
        got = reports[0][name]
        if err is None:
            assert got[0] == "ok" and np.array_equal(np.array(got[1]), out), name
        else:
            assert got[0] == "err" and got[3] == err.row, (name, got, err.row)
            assert got[1] == "NonFiniteScale" and got[2] == (err.bits,)
        # the device-path reduction: the first of the planted words (odd ranks, local row 3)
        # and the non-finite scales
        splits = shard.row_split(n_out, world)
        cands = []
        for r, (a, b) in enumerate(splits):
            if r % 2 == 1 and b - a > 3:
                cands.append(((a + 3) << 24) | (_abi.APX_ERR_OUTPUT_OVERFLOW << 16))
        nf = shard.first_nonfinite(t, raw, n_out, n_in)
        if nf is not None:
            cands.append((nf[0] << 24) | (_abi.APX_ERR_NONFINITE_SCALE << 16) | nf[1])
        want = min(cands) if cands else -1
        for rep in reports:
            assert rep[name + "/status"] == want, (name, rep[name + "/status"], want)
    # grouped projections, one all-gather per group: outputs where the projection does not
    # refuse, and each projection's own first refusal word
    cs = shard_worker.cases()
    for gname, idx in (("group_ok", [0, 2]), ("group_nf", [4, 5, 1])):
        for rep in reports:
            assert rep[gname] == reports[0][gname]
        for j, i in enumerate(idx):
            name, t, raw, n_out, n_in, q = cs[i]
            got, word = reports[0][gname][j]
            out, err = O.matvec_q8act_row(t, raw, n_out, n_in, q.codes, q.scales)
            if err is None:
                assert word == -1 and np.array_equal(np.array(got), out), (gname, name)
            else:
                nf = shard.first_nonfinite(t, raw, n_out, n_in)
                want = (nf[0] << 24) | (_abi.APX_ERR_NONFINITE_SCALE << 16) | nf[1]
                assert nf[0] == err.row and word == want, (gname, name, word, want)


class _LayoutLib:
    """apx_peer_alloc / apx_peer_open stand-ins that hand out fake addresses and record the
    allocation size (no GPU)."""

    def __init__(self):
        self.size = None

    def apx_peer_alloc(self, ctx, bytes_, ptr, handle, err):
        self.size = bytes_
        ptr._obj.value = 1 << 40
        return 0

    def apx_peer_open(self, ctx, handle, ptr, err):
        ptr._obj.value = 2 << 40
        return 0


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_peer_gather_layout_stays_inside_the_buffer(world):
    """Every region a rank writes (its rows of each projection in both parities, the keys,
    the flags, the epoch counters) lies inside the allocation, 16-byte aligned, with no two
    regions overlapping."""
    shapes = [(12, 28672, 64), (12, 97, 256), (8, 33, 64)]
    be = shard_worker.OracleBackend()
    for nproj in (1, 2, 3):
        for rank in range(world):
            shards = []
            for t, n_out, n_in in shapes[:nproj]:
                raw = np.zeros(n_out * shard.row_bytes(t, n_in), dtype=np.uint8)
                shards.append(shard.RowShard(be, t, raw, n_out, n_in, rank, world, None, "cpu"))
            lib = _LayoutLib()
            g = shard.PeerGather(lib, None, shards)
            d = g.desc
            regions = []
            for parity in (0, 1):
                for j, sh in enumerate(shards):
                    a = g.out_ptr(j, parity) - g.local
                    assert a % 16 == 0 and d.rows_off[j] % 2 == 0
                    regions.append((a, a + 8 * sh.rows))
                    # every rank's rows of projection j (the peers write them here)
                    for a0, b0 in sh.splits:
                        lo = parity * g.stride + 8 * (g.base[j] + a0)
                        assert lo + 8 * (b0 - a0) <= parity * g.stride + g.key_rel
                k = parity * g.stride + g.key_rel
                regions.append((k, k + 8 * world * nproj))
            regions.append((g.flag_off, g.flag_off + 8 * world))
            regions.append((g.ctr_off, g.ctr_off + 16))
            regions.sort()
            for (a, b), (c, e) in zip(regions, regions[1:]):
                assert b <= c or a == b, (regions,)
            assert regions[-1][1] <= lib.size
            assert d.flag_off % 8 == 0 and d.ctr_off % 8 == 0
