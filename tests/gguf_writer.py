"""A GGUF writer for tests (the layout parse_header reads: src/format/gguf.rs:217-700)."""
import struct

SCALAR_FMT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 10: "<Q", 11: "<q"}


def _str(b) -> bytes:
    b = b.encode() if isinstance(b, str) else b
    return struct.pack("<Q", len(b)) + b


def value(t: int, v) -> bytes:
    """The bytes of a metadata value of type t (arrays: v = (element type, [values]))."""
    if t in SCALAR_FMT:
        return struct.pack(SCALAR_FMT[t], v)
    if t == 6:
        return struct.pack("<f", v)
    if t == 12:
        return struct.pack("<d", v)
    if t == 7:
        return struct.pack("<B", 1 if v else 0)
    if t == 8:
        return _str(v)
    if t == 9:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(value(et, x) for x in items)
    raise ValueError(t)


def gguf_bytes(kv, tensors, alignment=None, version=3) -> bytes:
    """kv: [(key, type, value)]; tensors: [(name, dims, ggml_type, payload bytes)].  Tensor
    payloads are laid out in order, each at an offset aligned to the file's alignment."""
    align = alignment or 32
    kv = list(kv)
    if alignment is not None:
        kv.append(("general.alignment", 4, alignment))
    out = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv))
    for k, t, v in kv:
        out += _str(k) + struct.pack("<I", t) + value(t, v)
    offsets, off = [], 0
    for _, _, _, payload in tensors:
        offsets.append(off)
        off = -(-(off + len(payload)) // align) * align
    for (name, dims, gt, _), o in zip(tensors, offsets):
        out += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gt, o)
    out += b"\0" * (-(-len(out) // align) * align - len(out))
    data0 = len(out)
    for (_, _, _, payload), o in zip(tensors, offsets):
        out += b"\0" * (data0 + o - len(out)) + bytes(payload)
    return out
