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

    def reduce_status(self, status) -> None:
        """In place: this rank's refusal word (int64 tensor, first entry; rows of this shard)
        becomes the first refusal over every rank in rows of the whole tensor.  The row is
        rebased, the shard's non-finite scale folded in, "no refusal" (all ones) ordered last,
        and the minimum taken over the ranks."""
        import torch

        w = status[:1]
        keyed = torch.where(w == _NONE, torch.full_like(w, _I64_MAX), w + (self.r0 << _ROW_SHIFT))
        if self.nf_word is not None:
            keyed = torch.minimum(keyed, torch.full_like(w, self.nf_word))
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


def shard_projections(backend, mats: Sequence[Tuple[int, object, int, int]], rank: int,
                      world: int, dist=None, device: str = "cpu", group=None) -> List[RowShard]:
    """Row shards of several projections (ggml_type, raw, n_out, n_in), one per matrix."""
    return [RowShard(backend, t, raw, n_out, n_in, rank, world, dist, device, group)
            for t, raw, n_out, n_in in mats]
