"""Row-sharded projections over the GPUs of one node, one process per GPU.

A projection's output rows are independent: the reference splits a row range into
contiguous tasks and concatenates their outputs (src/engine/chart/ffn.rs:705-726), and
`matvec_fixed` computes every row on its own (src/engine/ops/matvec.rs:149-222).  So rank r
of P holds rows [r0, r1) of W, computes those outputs, and one all-gather of the output
slices gives every rank the whole vector.  The activation (a few KB) is replicated; there is
no exchange inside the projection itself.

Refusals keep the reference's order.  Call-level refusals (shape, payload length) are decided
from the whole tensor on every rank before any collective, so all ranks raise alike.  Row
refusals report the first refusing row in row order (ffn.rs:659-661): each rank's refusal is
rebased to its global row and the smallest over the ranks wins.

The collectives run through `torch.distributed` (NCCL over NVLink between GPUs; gloo for the
CPU tests of this logic).
"""
from __future__ import annotations

import pickle
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import _abi, chart

ROW_ALIGN = 32  # a shard boundary on a 32-row tile keeps every shard's units whole

# the refusal word of the asynchronous API: (row << 24) | (kind << 16) | bits, all ones when
# the call did not refuse (apx_call_status in include/apeiron_cuda.h)
_ROW_SHIFT = 24
_NONE = -1                   # all ones, read as int64
_I64_MAX = (1 << 63) - 1


def row_split(n_out: int, world: int, align: int = ROW_ALIGN) -> List[Tuple[int, int]]:
    """Contiguous row ranges [r0, r1) per rank: whole `align`-row tiles, as even as possible
    (the later ranks take the extra tiles), the last range ending at n_out."""
    if world < 1:
        raise ValueError("world must be >= 1")
    tiles = -(-n_out // align) if n_out else 0
    out = []
    for r in range(world):
        t0 = r * tiles // world
        t1 = (r + 1) * tiles // world
        out.append((min(t0 * align, n_out), min(t1 * align, n_out)))
    return out


def row_bytes(ggml_type: int, n_in: int) -> int:
    qk, bb = chart.GEOM[ggml_type]
    return -(-n_in // qk) * bb


def payload_rows(ggml_type: int, raw, n_out: int, n_in: int, r0: int, r1: int) -> np.ndarray:
    """The GGUF bytes of rows [r0, r1) of a row-major payload (rows are contiguous)."""
    buf = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else \
        np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    rb = row_bytes(ggml_type, n_in)
    return buf[r0 * rb: r1 * rb]


def check_payload(ggml_type: int, raw_len: int, n_out: int, n_in: int) -> None:
    """The call-level payload check of the whole tensor, identical on every rank
    (`ShortPayload { need, have }`, src/engine/ops/matvec.rs:119-127)."""
    if ggml_type not in chart.GEOM:
        raise chart.UnsupportedQuant(ggml_type)
    need = n_out * row_bytes(ggml_type, n_in)
    if raw_len < need:
        raise chart.ShortPayload(need, raw_len)


def first_nonfinite(ggml_type: int, rows_raw: np.ndarray, rows: int, n_in: int):
    """(row, bits) of the first Inf/NaN block scale in row order, each row in its
    dequantization order (Q8_0 d per block; Q4_K d then dmin per super-block; Q6_K d;
    src/engine/num/dequant.rs), or None."""
    if rows == 0:
        return None
    qk, bb = chart.GEOM[ggml_type]
    blocks = -(-n_in // qk)
    blk = np.asarray(rows_raw, dtype=np.uint8)[: rows * blocks * bb].reshape(rows, blocks, bb)
    if ggml_type == _abi.Q8_0:
        offs = [0]
    elif ggml_type == _abi.Q4_K:
        offs = [0, 2]
    else:
        offs = [208]
    h = np.stack([blk[:, :, o].astype(np.uint16) | (blk[:, :, o + 1].astype(np.uint16) << 8)
                  for o in offs], axis=2).reshape(rows, -1)
    bad = ((h >> 10) & 0x1F) == 0x1F
    if not bad.any():
        return None
    i = int(np.argmax(bad.reshape(-1)))
    return i // h.shape[1], int(h.reshape(-1)[i])


# refusals a row of W raises (the rest are decided for the whole call)
ROW_REFUSALS = (chart.NonFiniteScale, chart.OutputOverflow, chart.AccumulatorOverflow)


class RowShard:
    """Rank `rank`'s rows of one projection, resident on its device.

    `backend` computes the shard: a `chart.Backend` (the CUDA path) or any object with the same
    `upload` / `matvec_q8act` methods.  `dist` is `torch.distributed` with an initialised
    process group (or None for one rank); `device` is where the collectives' tensors live
    ("cuda:<local>" with NCCL, "cpu" with gloo).
    """

    def __init__(self, backend, ggml_type: int, raw, n_out: int, n_in: int, rank: int = 0,
                 world: int = 1, dist=None, device: str = "cpu", group=None):
        buf = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else \
            np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
        check_payload(ggml_type, buf.size, n_out, n_in)
        self.backend, self.ggml_type = backend, ggml_type
        self.n_out, self.n_in = n_out, n_in
        self.rank, self.world, self.dist, self.device, self.group = rank, world, dist, device, group
        self.splits = row_split(n_out, world)
        self.r0, self.r1 = self.splits[rank]
        self.rows = self.r1 - self.r0
        # every rank's slice padded to the largest, for equal-sized all-gathers
        self.max_rows = max(b - a for a, b in self.splits) if self.splits else 0
        mine = payload_rows(ggml_type, buf, n_out, n_in, self.r0, self.r1)
        self.tensor = backend.upload(ggml_type, mine, self.rows, n_in) if self.rows else None
        # the refusal word of this shard's first non-finite scale (the device kernels see only
        # finite scales; the host folds this one in, as apx_status_decode does)
        nf = first_nonfinite(ggml_type, mine, self.rows, n_in)
        self.nf_word = None if nf is None else (
            ((self.r0 + nf[0]) << _ROW_SHIFT) | (_abi.APX_ERR_NONFINITE_SCALE << 16) | nf[1])

    # -- the host interface: matvec_q8act over the whole tensor --------------------------------
    def matvec_q8act(self, q: chart.QuantAct) -> np.ndarray:
        """`matvec_q8act` (src/engine/chart/mod.rs:1887) of the whole tensor, computed by row
        shards: every rank returns the full Q32.32 vector, or every rank raises the refusal of
        the first refusing row."""
        if len(q) != self.n_in:
            raise chart.ShapeMismatch(len(q), self.n_in)
        local, refusal = None, None
        if self.rows:
            try:
                local = self.backend.matvec_q8act(self.ggml_type, self.tensor, self.rows,
                                                  self.n_in, q)
            except ROW_REFUSALS as e:
                refusal = e  # call-level refusals propagate: decided alike on every rank
        first = self._first_refusal(refusal)
        if first is not None:
            raise first
        return self._gather_rows(local)

    def _first_refusal(self, refusal: Optional[chart.MatvecError]):
        key = (self.r0 + int(refusal.row)) if refusal is not None else None
        mine = (key, pickle.dumps(refusal) if refusal is not None else None)
        if self.world == 1 or self.dist is None:
            allr = [mine]
        else:
            allr = [None] * self.world
            self.dist.all_gather_object(allr, mine, group=self.group)
        hits = [(k, blob) for k, blob in allr if k is not None]
        if not hits:
            return None
        k, blob = min(hits, key=lambda t: t[0])
        err = pickle.loads(blob)
        err.row = k
        return err

    def _gather_rows(self, local: Optional[np.ndarray]) -> np.ndarray:
        if self.world == 1 or self.dist is None:
            return np.asarray(local, dtype=np.int64)[: self.n_out]
        import torch

        mine = torch.zeros(self.max_rows, dtype=torch.int64, device=self.device)
        if self.rows:
            mine[: self.rows] = torch.from_numpy(np.asarray(local, dtype=np.int64)).to(self.device)
        full = torch.empty(self.world * self.max_rows, dtype=torch.int64, device=self.device)
        self.dist.all_gather_into_tensor(full, mine, group=self.group)
        return self.assemble(full.cpu().numpy())

    def assemble(self, gathered: np.ndarray) -> np.ndarray:
        """The whole output from the rank-major, padded all-gather buffer."""
        parts = [gathered[r * self.max_rows: r * self.max_rows + (b - a)]
                 for r, (a, b) in enumerate(self.splits)]
        return np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)

    # -- the device interface ------------------------------------------------------------------
    def matvec_async(self, lib, ctx, codes, exps, desc, local_out, gathered, status, stream):
        """Device path: this rank's rows into `local_out` (int64, max_rows), the all-gather
        into `gathered` (int64, world·max_rows, rank-major; `assemble` or equal splits give the
        vector), and `status` (int64[2], all ones on entry) reduced to the first refusing global
        row over the ranks.  Every pointer argument is a torch tensor on this rank's GPU; the
        work is queued on the current torch stream, which must be `stream`."""
        import torch

        if self.rows:
            rc = lib.apx_matvec_async(ctx, self.tensor.handle, self.rows, self.n_in,
                                      codes.data_ptr(), exps.data_ptr(), desc.data_ptr(),
                                      local_out.data_ptr(), None, status.data_ptr(), stream)
            if rc:
                raise chart.BackendError(f"apx_matvec_async failed with code {rc}")
        if self.world > 1 and self.dist is not None:
            self.dist.all_gather_into_tensor(gathered, local_out, group=self.group)
        elif self.rows:
            gathered[: self.rows].copy_(local_out[: self.rows])
        self.reduce_status(status)

    def _key(self, w):
        """This rank's refusal word (int64 tensor of one) as an order key: rebased to the whole
        tensor's rows, the shard's non-finite scale folded in, "no refusal" the largest."""
        import torch

        keyed = torch.where(w == _NONE, torch.full_like(w, _I64_MAX), w + (self.r0 << _ROW_SHIFT))
        if self.nf_word is not None:
            keyed = torch.minimum(keyed, torch.full_like(w, self.nf_word))
        return keyed

    def reduce_status(self, status) -> None:
        """In place: this rank's refusal word (int64 tensor, first entry; rows of this shard)
        becomes the first refusal over every rank in rows of the whole tensor.  The row is
        rebased, the shard's non-finite scale folded in, "no refusal" (all ones) ordered last,
        and the minimum taken over the ranks."""
        import torch

        w = status[:1]
        keyed = self._key(w)
        if self.world > 1 and self.dist is not None:
            self.dist.all_reduce(keyed, op=self.dist.ReduceOp.MIN, group=self.group)
        status[:1] = torch.where(keyed == _I64_MAX, torch.full_like(w, _NONE), keyed)

    @staticmethod
    def raise_status(word: int) -> None:
        """Raise the refusal a reduced status word of `matvec_async` names (rows of the whole
        tensor), or return when it is all ones."""
        word &= (1 << 64) - 1
        if word == (1 << 64) - 1:
            return
        kind, bits, row = (word >> 16) & 0xFF, word & 0xFFFF, word >> _ROW_SHIFT
        if kind == _abi.APX_ERR_NONFINITE_SCALE:
            raise chart.NonFiniteScale(bits, row=row)
        if kind == _abi.APX_ERR_OUTPUT_OVERFLOW:
            raise chart.OutputOverflow(row=row)
        if kind == _abi.APX_ERR_ACCUMULATOR_OVERFLOW:
            raise chart.AccumulatorOverflow(row=row)
        if kind == _abi.APX_ERR_FIXED_OVERFLOW:
            raise chart.FixedOverflow()
        if kind == _abi.APX_ERR_QUANT_REFUSED:
            raise chart.QuantRefused()
        raise chart.BackendError(f"refusal word {word:#x}")


def group_layout(shards: Sequence[RowShard]) -> Tuple[List[int], int, int]:
    """Offsets of each projection's padded row slice in one rank's group buffer, the offset of
    the refusal keys (one int64 per projection, after the slices) and the buffer length."""
    offs, o = [], 0
    for sh in shards:
        offs.append(o)
        o += sh.max_rows
    return offs, o, o + len(shards)


def matvec_group_async(shards: Sequence[RowShard], lib, ctx, acts, local, gathered, statuses,
                       stream) -> None:
    """Several row-sharded projections with ONE all-gather: each projection's rows into its
    slice of `local` (int64, group_layout length), each refusal word (rebased, non-finite
    folded) as a key after the slices, one all-gather of `local` into `gathered` (world ×
    length, rank-major), and each `statuses[j]` (int64[2], all ones on entry) set to the first
    refusal over the ranks.  `acts[j]` = (codes, exps, desc) device tensors of projection j;
    all tensors on this rank's GPU, queued on the current torch stream (`stream`)."""
    import torch

    offs, k0, length = group_layout(shards)
    for j, sh in enumerate(shards):
        codes, exps, desc = acts[j]
        if sh.rows:
            rc = lib.apx_matvec_async(ctx, sh.tensor.handle, sh.rows, sh.n_in, codes.data_ptr(),
                                      exps.data_ptr(), desc.data_ptr(),
                                      local[offs[j]:].data_ptr(), None,
                                      statuses[j].data_ptr(), stream)
            if rc:
                raise chart.BackendError(f"apx_matvec_async failed with code {rc}")
    keys = torch.stack([sh._key(statuses[j][:1])[0] for j, sh in enumerate(shards)])
    local[k0:k0 + len(shards)] = keys
    sh0 = shards[0]
    if sh0.world > 1 and sh0.dist is not None:
        sh0.dist.all_gather_into_tensor(gathered, local, group=sh0.group)
        first = gathered.view(sh0.world, length)[:, k0:k0 + len(shards)].min(dim=0).values
    else:
        gathered[:length].copy_(local)
        first = keys
    for j in range(len(shards)):
        statuses[j][:1] = torch.where(first[j:j + 1] == _I64_MAX,
                                      torch.full_like(first[j:j + 1], _NONE), first[j:j + 1])


def assemble_group(shards: Sequence[RowShard], gathered: np.ndarray, j: int) -> np.ndarray:
    """Projection j's whole output from a group all-gather buffer."""
    offs, _, length = group_layout(shards)
    sh = shards[j]
    parts = [gathered[r * length + offs[j]: r * length + offs[j] + (b - a)]
             for r, (a, b) in enumerate(sh.splits)]
    return np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)


def _align(n: int, a: int = 256) -> int:
    return -(-n // a) * a


class PeerGather:
    """Row-sharded projections whose outputs move between the ranks' GPUs by peer stores
    (apx_gather_publish_async) instead of a collective library.

    Every rank allocates one gather buffer (apx_peer_alloc) and maps every other rank's
    (CUDA IPC handles exchanged once through `dist`).  Layout, the same on every rank:
      parity p (0, 1) at p·stride: the whole output vectors of the group's projections
      (projection j at element base[j], 32-element aligned), then the refusal keys
      [world][nproj]; after both parities the flags [world] and this rank's epoch counters.
    `run` queues, on `stream`: each projection of this rank's rows, whose kernel stores every
    output row into every rank's buffer, and the publication that posts this rank's refusal
    keys and epoch flag everywhere, waits for everyone's and resets this rank's refusal words.  Nothing else runs between, so the next
    projection streams its weights (programmatic dependent launch) during the publication.  Parities alternate per call; the epoch
    advances on the device, so `run` may be captured in a CUDA graph (an even number of
    calls per graph keeps the parities in step on replay).
    """

    def __init__(self, lib, ctx, shards: Sequence[RowShard], timeout_us: int = 2_000_000):
        import ctypes as C

        sh0 = shards[0]
        if len(shards) > _abi.MAX_GATHER_PROJ or sh0.world > _abi.MAX_PEERS:
            raise ValueError("too many projections or ranks for one gather")
        self.lib, self.ctx, self.shards = lib, ctx, list(shards)
        self.world, self.rank, self.dist, self.group = sh0.world, sh0.rank, sh0.dist, sh0.group
        self.nproj = len(shards)
        self.base, o = [], 0
        for sh in shards:
            self.base.append(o)
            o += _align(max(sh.n_out, 1), 32)
        out_bytes = _align(8 * o)
        key_bytes = _align(8 * self.world * self.nproj)
        self.key_rel = out_bytes
        self.stride = out_bytes + key_bytes
        self.flag_off = 2 * self.stride
        self.ctr_off = self.flag_off + _align(8 * self.world)
        total = self.ctr_off + 256
        ptr, handle = C.c_void_p(), (C.c_ubyte * _abi.PEER_HANDLE_BYTES)()
        err = _abi.ApxErr()
        if lib.apx_peer_alloc(ctx, total, C.byref(ptr), handle, C.byref(err)):
            raise chart.BackendError(f"apx_peer_alloc failed (cuda {err.cuda_error})")
        self.local = ptr.value
        handles = [bytes(handle)] * self.world
        if self.world > 1 and self.dist is not None:
            self.dist.all_gather_object(handles, bytes(handle), group=self.group)
        self.peers, self.opened = [], []
        for r in range(self.world):
            if r == self.rank:
                self.peers.append(self.local)
                continue
            hp, err = C.c_void_p(), _abi.ApxErr()
            hb = (C.c_ubyte * _abi.PEER_HANDLE_BYTES).from_buffer_copy(handles[r])
            if lib.apx_peer_open(ctx, hb, C.byref(hp), C.byref(err)):
                raise chart.BackendError(f"apx_peer_open of rank {r} failed "
                                         f"(cuda {err.cuda_error})")
            self.peers.append(hp.value)
            self.opened.append(hp.value)
        d = _abi.GatherDesc()
        d.world, d.rank, d.nproj, d.timeout_us = self.world, self.rank, self.nproj, timeout_us
        for r, pv in enumerate(self.peers):
            d.peer[r] = pv
        d.flag_off, d.ctr_off, d.bytes = self.flag_off, self.ctr_off, total
        for j, sh in enumerate(shards):
            d.rows_off[j] = self.base[j] + sh.r0
            d.rows[j] = sh.rows
            d.row0[j] = sh.r0
            d.nf_key[j] = sh.nf_word if sh.nf_word is not None else _I64_MAX
        self.desc = d
        self.calls = 0

    def out_ptr(self, j: int, parity: int) -> int:
        """Where this rank's rows of projection j go in the given parity (device address)."""
        return self.local + parity * self.stride + 8 * (self.base[j] + self.shards[j].r0)

    def run(self, acts, statuses, out_statuses, stream, shards=None) -> int:
        """One publication of the group.  `acts[j]` = (codes, exps, desc) device tensors of
        projection j; `statuses` an int64 tensor (nproj, 2) for this rank's refusal words (all
        ones before the first call; each publication resets them after reading them);
        `out_statuses` an int64 tensor (nproj, 2) that receives the first refusal over all
        ranks (whole-tensor rows).  `shards` may name other uploads of the same rows (copies
        of the weights).  Everything is queued on the current torch stream, which must be
        `stream`.  Returns the parity written."""
        import ctypes as C

        parity = (self.calls + 1) % 2
        d = self.desc
        d.out_off = parity * self.stride
        d.key_off = parity * self.stride + self.key_rel
        for j in range(self.nproj):
            d.status[j] = statuses[j].data_ptr()
            d.out_status[j] = out_statuses[j].data_ptr()
        for j, sh in enumerate(shards or self.shards):
            codes, exps, desc = acts[j]
            if sh.rows:  # this rank's rows, stored into every rank's buffer by the kernel
                rc = self.lib.apx_matvec_gather_async(self.ctx, sh.tensor.handle, sh.rows,
                                                      sh.n_in, codes.data_ptr(), exps.data_ptr(),
                                                      desc.data_ptr(), C.byref(d), j, stream)
                if rc:
                    raise chart.BackendError(f"apx_matvec_gather_async failed with code {rc}")
        rc = self.lib.apx_gather_publish_async(self.ctx, C.byref(d), stream)
        if rc:
            raise chart.BackendError(f"apx_gather_publish_async failed with code {rc}")
        self.calls += 1
        return parity

    def read(self, j: int, parity: int) -> np.ndarray:
        """Projection j's whole output vector from this rank's buffer (synchronous)."""
        import ctypes as C

        n = self.shards[j].n_out
        out = np.empty(max(n, 1), dtype=np.int64)
        err = _abi.ApxErr()
        if n and self.lib.apx_device_read(self.ctx, self.local + parity * self.stride +
                                          8 * self.base[j], out.ctypes.data, 8 * n,
                                          C.byref(err)):
            raise chart.BackendError(f"apx_device_read failed (cuda {err.cuda_error})")
        return out[:n]

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank has stopped writing:
        the caller synchronises its stream and the ranks meet at a barrier first)."""
        for pv in self.opened:
            self.lib.apx_peer_close(self.ctx, pv, 1)
        self.opened = []
        if self.local:
            self.lib.apx_peer_close(self.ctx, self.local, 0)
            self.local = 0


class _Ptr:
    """A device address where torch tensors are expected (``.data_ptr()``)."""

    def __init__(self, addr: int):
        self.addr = addr

    def data_ptr(self) -> int:
        return self.addr


class HiddenGather:
    """The quantized hidden activation h of a row-sharded FFN, assembled on every rank.

    Rank r's step plan (apx_plan_*) runs gate and up on its rows with SwiGLU + quant_act in
    their finish (h rows g0..g1, whole 32-row blocks), storing each block's codes and exponent
    byte, and its slice's descriptor, into every rank's buffer here; `publish` then posts the
    gate/up refusal keys and an epoch flag everywhere, waits (bounded) for every rank's, and
    merges the ranks' slice descriptors into the descriptor of the whole h, which the down
    projection reads.  Only the int8 codes and exponent bytes cross NVLink (n_ff + n_ff/32
    bytes per step over all ranks), not the int64 gate and up outputs.

    Layout, the same on every rank, parity p (0, 1) at p·stride: codes [padded n_ff], exponent
    bytes [padded n_ff / 32], slice descriptors [world] × 32 B, the merged descriptor, the keys
    [world][2]; after both parities the flags [world] and this rank's epoch counters.  Parities
    alternate per publication (an even number per CUDA graph keeps them in step on replay).
    """

    def __init__(self, lib, ctx, gate: RowShard, up: RowShard, timeout_us: int = 2_000_000):
        import ctypes as C

        if gate.splits != up.splits or gate.n_out != up.n_out or gate.world > _abi.MAX_PEERS:
            raise ValueError("gate and up must share their row split")
        if any(a % 32 for a, _ in gate.splits):
            raise ValueError("hidden slices must start on 32-row blocks")
        self.lib, self.ctx, self.gate, self.up = lib, ctx, gate, up
        self.world, self.rank, self.dist, self.group = gate.world, gate.rank, gate.dist, gate.group
        self.n = gate.n_out
        pad = int(lib.apx_act_padded_len(self.n))
        self.codes_rel = 0
        self.exps_rel = _align(pad)
        self.desc_rel = self.exps_rel + _align(pad // 32)
        self.merged_rel = self.desc_rel + 32 * self.world
        self.key_rel = _align(self.merged_rel + 32)
        self.stride = _align(self.key_rel + 8 * self.world * 2)
        self.flag_off = 2 * self.stride
        self.ctr_off = self.flag_off + _align(8 * self.world)
        total = self.ctr_off + 256
        ptr, handle = C.c_void_p(), (C.c_ubyte * _abi.PEER_HANDLE_BYTES)()
        err = _abi.ApxErr()
        if lib.apx_peer_alloc(ctx, total, C.byref(ptr), handle, C.byref(err)):
            raise chart.BackendError(f"apx_peer_alloc failed (cuda {err.cuda_error})")
        self.local = ptr.value
        # exponent bytes past n read as zero blocks in both parities
        ff = np.full(pad // 32 - self.n // 32, 0xFF, dtype=np.uint8)
        for par in (0, 1):
            if ff.size and lib.apx_device_write(ctx, self.local + par * self.stride +
                                                self.exps_rel + self.n // 32, ff.ctypes.data,
                                                ff.size, C.byref(err)):
                raise chart.BackendError("apx_device_write failed")
        handles = [bytes(handle)] * self.world
        if self.world > 1 and self.dist is not None:
            self.dist.all_gather_object(handles, bytes(handle), group=self.group)
        self.peers, self.opened = [], []
        for r in range(self.world):
            if r == self.rank:
                self.peers.append(self.local)
                continue
            hp, err = C.c_void_p(), _abi.ApxErr()
            hb = (C.c_ubyte * _abi.PEER_HANDLE_BYTES).from_buffer_copy(handles[r])
            if lib.apx_peer_open(ctx, hb, C.byref(hp), C.byref(err)):
                raise chart.BackendError(f"apx_peer_open of rank {r} failed "
                                         f"(cuda {err.cuda_error})")
            self.peers.append(hp.value)
            self.opened.append(hp.value)
        d = _abi.GatherDesc()
        d.world, d.rank, d.nproj, d.timeout_us = self.world, self.rank, 2, timeout_us
        for r, pv in enumerate(self.peers):
            d.peer[r] = pv
        d.flag_off, d.ctr_off, d.bytes = self.flag_off, self.ctr_off, total
        for j, sh in enumerate((gate, up)):
            d.row0[j] = sh.r0
            d.nf_key[j] = sh.nf_word if sh.nf_word is not None else _I64_MAX
        self.desc = d
        self.calls = 0

    def next_parity(self) -> int:
        return (self.calls + 1) % 2

    def slice_dest(self, parity: int, r: int):
        """(codes, exps, descriptor slot) of this rank's slice in rank r's buffer."""
        base = self.peers[r] + parity * self.stride
        g0 = self.gate.r0
        return (base + self.codes_rel + g0, base + self.exps_rel + g0 // 32,
                base + self.desc_rel + 32 * self.rank)

    def activation(self, parity: int):
        """The whole h in this rank's buffer: (codes, exps, merged descriptor) addresses."""
        base = self.local + parity * self.stride
        return (_Ptr(base + self.codes_rel), _Ptr(base + self.exps_rel),
                _Ptr(base + self.merged_rel))

    def publish(self, statuses, out_statuses, stream) -> int:
        """Queue the publication of the next parity: `statuses` (2, 2) int64, the gate and up
        refusal words the plan wrote (reset by the publication), `out_statuses` (2, 2) the
        first refusal of each over all ranks.  Returns the parity."""
        import ctypes as C

        parity = self.next_parity()
        d = self.desc
        base = parity * self.stride
        d.key_off = base + self.key_rel
        d.desc_off = base + self.desc_rel
        d.merged_off = base + self.merged_rel
        d.out_off = base
        for j in range(2):
            d.status[j] = statuses[j].data_ptr()
            d.out_status[j] = out_statuses[j].data_ptr()
        rc = self.lib.apx_gather_publish_async(self.ctx, C.byref(d), stream)
        if rc:
            raise chart.BackendError(f"apx_gather_publish_async failed with code {rc}")
        self.calls += 1
        return parity

    def read(self, parity: int):
        """(codes, exponent bytes, merged descriptor words) of the whole h (synchronous)."""
        import ctypes as C

        codes = np.empty(self.n, dtype=np.int8)
        exps = np.empty(self.n // 32, dtype=np.uint8)
        desc = np.empty(8, dtype=np.int32)
        err = _abi.ApxErr()
        base = self.local + parity * self.stride
        for addr, arr in ((base + self.codes_rel, codes), (base + self.exps_rel, exps),
                          (base + self.merged_rel, desc)):
            if self.lib.apx_device_read(self.ctx, addr, arr.ctypes.data, arr.nbytes,
                                        C.byref(err)):
                raise chart.BackendError("apx_device_read failed")
        return codes, exps, desc

    def close(self) -> None:
        for pv in self.opened:
            self.lib.apx_peer_close(self.ctx, pv, 1)
        self.opened = []
        if self.local:
            self.lib.apx_peer_close(self.ctx, self.local, 0)
            self.local = 0


def shard_projections(backend, mats: Sequence[Tuple[int, object, int, int]], rank: int,
                      world: int, dist=None, device: str = "cpu", group=None) -> List[RowShard]:
    """Row shards of several projections (ggml_type, raw, n_out, n_in), one per matrix."""
    return [RowShard(backend, t, raw, n_out, n_in, rank, world, dist, device, group)
            for t, raw, n_out, n_in in mats]
