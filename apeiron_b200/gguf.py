"""GGUF files and their device residency: the on-disk format on the far side of the projection
path.

`parse_header` restates the reference's reader (src/format/gguf.rs:217-700): little-endian
magic "GGUF", version 2 or 3, tensor and metadata counts (each bounded by the bytes left),
metadata values of scalar types 0-8 and 10-12 and arrays (type 9) nested at most 8 deep, tensor
descriptors (name, at most 4 dims, ggml type, offset), `general.alignment` (default 32) and the
data section at the header's end rounded up to it.  Refusals are the reference's GgufError kinds
and GgufField names.  `tensor_bytes` sizes a tensor as ceil(elements / block) blocks
(quant.rs:129-189) and checks it against the file's end.

`ResidentModel` is the engine's one-time upload (src/engine/loader.rs:937-1020): the file is
mapped once, and every two-dimensional tensor of a served family (Q5_0, Q8_0, Q4_K, Q6_K) is uploaded
and repacked on the device, keyed by tensor index and name.  GGUF dims are (row length, rows):
a projection's n_in is dims[0] and n_out dims[1].
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32
MAX_DIMS = 4
MAX_ARRAY_DEPTH = 8

# quant.rs:21-93: ggml type -> (elements per block, bytes per block)
QK_K = 256
BLOCK_GEOM = {
    0: (1, 4),                     # F32
    1: (1, 2),                     # F16
    30: (1, 2),                    # BF16
    6: (32, 2 + 4 + 16),           # Q5_0
    8: (32, 2 + 32),               # Q8_0
    10: (QK_K, QK_K // 16 + QK_K // 4 + 4),          # Q2_K
    11: (QK_K, QK_K // 8 + QK_K // 4 + 12 + 2),      # Q3_K
    12: (QK_K, 2 + 2 + 12 + QK_K // 2),              # Q4_K
    14: (QK_K, QK_K // 2 + QK_K // 4 + QK_K // 16 + 2),  # Q6_K
    41: (128, 2 + 128 // 8),       # Q1_0
    42: (64, 2 + 64 // 4),         # Q2_0
    142: (128, 2 + 128 // 4),      # PQ2_0
    35: (256, 256 // 4 + 2),       # TQ2_0
    34: (256, (256 - 4 * 256 // 64) // 5 + 256 // 64 + 2),   # TQ1_0
    143: (128, (128 - 4 * 128 // 64) // 5 + 128 // 64 + 2),  # PTQ1_0
}
SERVED = (6, 8, 12, 14)  # the families the device projections take (Q5_0, Q8_0, Q4_K, Q6_K)

# GgufField names (gguf.rs GgufField::name)
F_KV_KEY, F_KV_TYPE, F_KV_VALUE = "kv key", "kv type", "kv value"
F_T_NAME, F_T_NDIMS, F_T_DIMS = "tensor name", "tensor n_dims", "tensor dims"
F_T_TYPE, F_T_OFFSET = "tensor type", "tensor offset"
F_MAGIC, F_VERSION, F_T_COUNT, F_KV_COUNT, F_KVT_COUNT = (
    "magic", "version", "tensor count", "kv count", "kv/tensor count")


class GgufError(Exception):
    """A refusal of the reader (gguf.rs GgufError)."""


class BadMagic(GgufError):
    pass


class UnsupportedVersion(GgufError):
    pass


class Truncated(GgufError):
    def __init__(self, what: str):
        super().__init__(f"truncated: {what}")
        self.what = what


class TooManyDims(GgufError):
    pass


class LengthOverflow(GgufError):
    pass


class UnknownType(GgufError):
    pass


class OutOfBounds(GgufError):
    def __init__(self, at: int, n: int, file_len: int):
        super().__init__(f"tensor [{at}, {at}+{n}) past EOF {file_len}")
        self.at, self.n, self.file_len = at, n, file_len


class MissingTensor(GgufError):
    pass


U64_MAX = (1 << 64) - 1


def block_count(t: int, n_elements: int) -> int:
    geom = BLOCK_GEOM.get(t)
    if geom is None:
        raise UnknownType(f"unknown ggml type {t}")
    return -(-n_elements // geom[0])


def required_bytes(t: int, n_elements: int) -> int:
    n = block_count(t, n_elements) * BLOCK_GEOM[t][1]
    if n > U64_MAX:
        raise LengthOverflow("length overflow")
    return n


@dataclass
class TensorDesc:
    name: bytes
    dims: list
    ggml_type: int
    offset: int
    index: int = 0

    def n_elements(self) -> int:
        acc = 1
        for d in self.dims:
            acc *= d
            if acc > U64_MAX:
                raise LengthOverflow("length overflow")
        return acc

    def n_bytes(self):
        """Storage bytes, or None for a type without a block geometry."""
        if self.ggml_type not in BLOCK_GEOM:
            return None
        return required_bytes(self.ggml_type, self.n_elements())


@dataclass
class GgufHeader:
    version: int
    kv: list = field(default_factory=list)        # [(key bytes, value)]
    tensors: list = field(default_factory=list)   # [TensorDesc]
    alignment: int = DEFAULT_ALIGNMENT
    header_end: int = 0
    data0: int = 0

    def meta(self, key: str):
        kb = key.encode()
        for k, v in self.kv:
            if k == kb:
                return v
        return None

    def meta_i64(self, key: str):
        v = self.meta(key)
        return _as_i64(v)

    def arch(self) -> str:
        v = self.meta("general.architecture")
        return v.decode("utf-8", "replace") if isinstance(v, bytes) else ""

    def tensor(self, name: str):
        nb = name.encode()
        for t in self.tensors:
            if t.name == nb:
                return t
        return None


def _as_i64(v):
    """GVal::as_i64: integers inside i64 and booleans; None otherwise."""
    if isinstance(v, bool):
        return int(v)
    if isinstance(v, int) and -(1 << 63) <= v < (1 << 63):
        return v
    return None


class _Cur:
    def __init__(self, b):
        self.b = b
        self.i = 0

    def take(self, n: int):
        if self.i + n > len(self.b):
            return None
        v = self.b[self.i:self.i + n]
        self.i += n
        return bytes(v)

    def u32(self):
        v = self.take(4)
        return None if v is None else struct.unpack("<I", v)[0]

    def u64(self):
        v = self.take(8)
        return None if v is None else struct.unpack("<Q", v)[0]

    def string(self):
        n = self.u64()
        if n is None or self.i + n > len(self.b):
            return None
        return self.take(n)

    _SCALAR = {0: ("<B", 1), 1: ("<b", 1), 2: ("<H", 2), 3: ("<h", 2), 4: ("<I", 4),
               5: ("<i", 4), 10: ("<Q", 8), 11: ("<q", 8)}

    def scalar(self, t: int):
        if t in self._SCALAR:
            fmt, n = self._SCALAR[t]
            v = self.take(n)
            return None if v is None else struct.unpack(fmt, v)[0]
        if t == 6:                       # f32, kept as its bits
            v = self.u32()
            return None if v is None else ("f32", v)
        if t == 12:                      # f64, kept as its bits
            v = self.u64()
            return None if v is None else ("f64", v)
        if t == 7:
            v = self.take(1)
            return None if v is None else v[0] != 0
        if t == 8:
            return self.string()
        return None

    def array_header(self):
        et = self.u32()
        n = self.u64()
        if et is None or n is None or n > len(self.b) - self.i:
            return None
        return et, n

    def value(self, t: int, depth: int):
        """A metadata value; arrays nest at most `depth` deep (the root counts as one)."""
        if t != 9:
            return self.scalar(t)
        return self._array(depth)

    def _array(self, depth: int):
        if depth == 0:
            return None
        hdr = self.array_header()
        if hdr is None:
            return None
        et, n = hdr
        out = []
        for _ in range(n):
            v = self._array(depth - 1) if et == 9 else self.scalar(et)
            if v is None:
                return None
            out.append(v)
        return ("arr", et, out)


def parse_header(buf, file_len: int | None = None) -> GgufHeader:
    """parse_header (gguf.rs:590-700) over the file's bytes."""
    c = _Cur(buf)
    magic = c.take(4)
    if magic is None:
        raise Truncated(F_MAGIC)
    if magic != GGUF_MAGIC:
        raise BadMagic(f"bad magic {magic!r} — not a GGUF file")
    version = c.u32()
    if version is None:
        raise Truncated(F_VERSION)
    if version not in (2, 3):
        raise UnsupportedVersion(f"unsupported GGUF version {version}")
    n_tensors = c.u64()
    if n_tensors is None:
        raise Truncated(F_T_COUNT)
    n_kv = c.u64()
    if n_kv is None:
        raise Truncated(F_KV_COUNT)
    remaining = len(buf) - c.i
    if n_kv > remaining or n_tensors > remaining:
        raise Truncated(F_KVT_COUNT)
    kv = []
    for _ in range(n_kv):
        key = c.string()
        if key is None:
            raise Truncated(F_KV_KEY)
        t = c.u32()
        if t is None:
            raise Truncated(F_KV_TYPE)
        v = c.value(t, MAX_ARRAY_DEPTH)
        if v is None:
            raise Truncated(F_KV_VALUE)
        kv.append((key, v))
    alignment = DEFAULT_ALIGNMENT
    for k, v in kv:
        if k == b"general.alignment":
            a = _as_i64(v)
            if a is not None and a > 0:
                alignment = a
    tensors = []
    for index in range(n_tensors):
        name = c.string()
        if name is None:
            raise Truncated(F_T_NAME)
        nd = c.u32()
        if nd is None:
            raise Truncated(F_T_NDIMS)
        if nd > MAX_DIMS:
            raise TooManyDims(f"tensor rank {nd} > {MAX_DIMS}")
        dims = []
        for _ in range(nd):
            d = c.u64()
            if d is None:
                raise Truncated(F_T_DIMS)
            dims.append(d)
        t = c.u32()
        if t is None:
            raise Truncated(F_T_TYPE)
        off = c.u64()
        if off is None:
            raise Truncated(F_T_OFFSET)
        tensors.append(TensorDesc(name, dims, t, off, index))
    header_end = c.i
    data0 = -(-header_end // alignment) * alignment
    if data0 > U64_MAX:
        raise LengthOverflow("length overflow")
    return GgufHeader(version, kv, tensors, alignment, header_end, data0)


class Gguf:
    """An opened GGUF file, mapped read-only; tensor payloads are views of the mapping."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self.file_len = os.fstat(self._f.fileno()).st_size
        self._map = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if self.file_len \
            else b""
        with memoryview(self._map) as mv:
            self.header = parse_header(mv, self.file_len)

    def close(self):
        if isinstance(self._map, mmap.mmap):
            try:
                self._map.close()
            except BufferError:
                pass  # payload views are still alive: the mapping goes with the last of them
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def tensor_bytes(self, t: TensorDesc) -> np.ndarray:
        """The tensor's payload (a read-only view), bounds-checked against the file."""
        n = t.n_bytes()
        if n is None:
            raise UnknownType(f"unknown ggml type {t.ggml_type}")
        at = self.header.data0 + t.offset
        if at + n > U64_MAX:
            raise LengthOverflow("length overflow")
        if at + n > self.file_len:
            raise OutOfBounds(at, n, self.file_len)
        return np.frombuffer(self._map, dtype=np.uint8, count=n, offset=at)

    def tensor(self, name: str) -> TensorDesc:
        t = self.header.tensor(name)
        if t is None:
            raise MissingTensor(f"no tensor {name}")
        return t


class ResidentModel:
    """Every served projection of a GGUF file, uploaded once to one device context.

    `projections` maps tensor index -> device Tensor and `by_name` name -> device Tensor; tensors
    of other types or ranks (norms, embeddings in F32/F16, unsupported families) stay on the host
    and are listed in `skipped` with the reason."""

    def __init__(self, backend, gguf: Gguf):
        self.backend = backend
        self.gguf = gguf
        self.projections = {}
        self.by_name = {}
        self.skipped = {}
        for t in gguf.header.tensors:
            name = t.name.decode("utf-8", "replace")
            if len(t.dims) != 2:
                self.skipped[name] = f"rank {len(t.dims)}"
                continue
            if t.ggml_type not in SERVED:
                self.skipped[name] = f"ggml type {t.ggml_type}"
                continue
            n_in, n_out = int(t.dims[0]), int(t.dims[1])
            dev = backend.upload(t.ggml_type, gguf.tensor_bytes(t), n_out, n_in)
            self.projections[t.index] = dev
            self.by_name[name] = dev

    def __getitem__(self, name: str):
        return self.by_name[name]
