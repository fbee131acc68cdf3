"""The GGUF reader (apeiron_b200/gguf.py) against the reference's parse_header rules
(src/format/gguf.rs:217-700) on files written here: metadata of every type, nested arrays,
alignment, tensor payload views, and each refusal kind with its field."""
import struct

import numpy as np
import pytest

from apeiron_b200 import gguf as G, synth
from gguf_writer import gguf_bytes


def _kv():
    return [("general.architecture", 8, "qwen2"), ("u8", 0, 200), ("i8", 1, -5),
            ("u16", 2, 60000), ("i16", 3, -300), ("u32", 4, 4_000_000_000), ("i32", 5, -7),
            ("f32", 6, 1.5), ("b", 7, True), ("u64", 10, (1 << 64) - 1), ("i64", 11, -(1 << 62)),
            ("f64", 12, 0.25), ("arr", 9, (9, [(5, [1, 2, 3]), (5, []), (8, ["a", "bc"])])),
            ("qwen2.block_count", 4, 24)]


def _tensors():
    q8 = synth.payload(8, 64, 96, 1)          # Q8_0, 64 rows of 96
    q4 = synth.payload(12, 32, 512, 2)        # Q4_K, 32 rows of 512
    norm = np.arange(96, dtype=np.float32)
    return [("blk.0.ffn_down.weight", [96, 64], 8, q8.tobytes()),
            ("blk.0.ffn_up.weight", [512, 32], 12, q4.tobytes()),
            ("blk.0.attn_norm.weight", [96], 0, norm.tobytes())]


@pytest.mark.parametrize("alignment", [None, 64])
def test_header_metadata_and_payloads(tmp_path, alignment):
    p = tmp_path / "m.gguf"
    tens = _tensors()
    p.write_bytes(gguf_bytes(_kv(), tens, alignment=alignment))
    with G.Gguf(str(p)) as f:
        h = f.header
        assert h.version == 3 and h.alignment == (alignment or 32)
        assert h.data0 % h.alignment == 0 and h.data0 >= h.header_end
        assert h.arch() == "qwen2" and h.meta_i64("qwen2.block_count") == 24
        assert h.meta("u8") == 200 and h.meta("i8") == -5 and h.meta("u16") == 60000
        assert h.meta("i16") == -300 and h.meta("u32") == 4_000_000_000 and h.meta("i32") == -7
        assert h.meta("f32") == ("f32", struct.unpack("<I", struct.pack("<f", 1.5))[0])
        assert h.meta("b") is True and h.meta_i64("b") == 1
        assert h.meta("u64") == (1 << 64) - 1 and h.meta_i64("u64") is None
        assert h.meta("i64") == -(1 << 62)
        assert h.meta("arr") == ("arr", 9, [("arr", 5, [1, 2, 3]), ("arr", 5, []),
                                           ("arr", 8, [b"a", b"bc"])])
        assert [t.name for t in h.tensors] == [t[0].encode() for t in tens]
        for t, (_, dims, gt, payload) in zip(h.tensors, tens):
            assert t.dims == dims and t.ggml_type == gt
            assert f.tensor_bytes(t).tobytes() == payload
        with pytest.raises(G.MissingTensor):
            f.tensor("nope")


def test_refusals(tmp_path):
    good = gguf_bytes(_kv(), _tensors())

    def parse(b):
        return G.parse_header(memoryview(b), len(b))

    with pytest.raises(G.BadMagic):
        parse(b"GGUX" + good[4:])
    for v in (1, 4):
        with pytest.raises(G.UnsupportedVersion):
            parse(good[:4] + struct.pack("<I", v) + good[8:])
    # every truncation point refuses, each with the field it stopped in
    seen = set()
    h = parse(good)
    for cut in range(0, h.header_end):
        with pytest.raises(G.Truncated) as e:
            parse(good[:cut])
        seen.add(e.value.what)
    assert {G.F_MAGIC, G.F_VERSION, G.F_T_COUNT, G.F_KV_COUNT, G.F_KVT_COUNT, G.F_KV_KEY,
            G.F_KV_TYPE, G.F_KV_VALUE, G.F_T_NAME, G.F_T_NDIMS, G.F_T_DIMS, G.F_T_TYPE,
            G.F_T_OFFSET} <= seen
    # rank above 4
    with pytest.raises(G.TooManyDims):
        parse(gguf_bytes([], [("t", [1, 1, 1, 1, 1], 0, b"\0" * 4)]))
    # arrays nest at most 8 deep
    deep = (5, [1])
    for _ in range(7):
        deep = (9, [deep])
    parse(gguf_bytes([("d", 9, deep)], []))
    with pytest.raises(G.Truncated) as e:
        parse(gguf_bytes([("d", 9, (9, [deep]))], []))
    assert e.value.what == G.F_KV_VALUE
    # an unknown scalar type
    with pytest.raises(G.Truncated):
        parse(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 1) + b"k" +
              struct.pack("<I", 13) + b"\0" * 8)


def test_tensor_bounds_and_types(tmp_path):
    p = tmp_path / "t.gguf"
    b = gguf_bytes([], [("w", [96, 64], 8, synth.payload(8, 64, 96, 3).tobytes()),
                        ("x", [32], 77, b"\0" * 16)])
    p.write_bytes(b[:-100])   # the Q8_0 payload runs past the end of the file
    with G.Gguf(str(p)) as f:
        with pytest.raises(G.OutOfBounds):
            f.tensor_bytes(f.tensor("w"))
        with pytest.raises(G.UnknownType):
            f.tensor_bytes(f.tensor("x"))
    assert G.required_bytes(12, 896 * 10) == 35 * 144      # ceil over all elements
    assert G.required_bytes(8, 64) == 2 * 34


@pytest.mark.gpu
def test_resident_model_projections(tmp_path):
    """Every served two-dimensional tensor of a GGUF file is uploaded once and its projections
    equal the oracle's on the file's own bytes; norms and other ranks stay on the host."""
    from apeiron_b200.chart import Backend, QuantAct
    from oracle import oracle as O

    served = [("blk.0.ffn_down.weight", 8, 64, 96), ("blk.0.ffn_up.weight", 12, 32, 512),
              ("output.weight", 14, 48, 256)]
    tens = [(name, [n_in, n_out], t, synth.payload(t, n_out, n_in, 5 + i).tobytes())
            for i, (name, t, n_out, n_in) in enumerate(served)]
    tens.append(("blk.0.attn_norm.weight", [96], 0, np.ones(96, np.float32).tobytes()))
    tens.append(("rope.cache", [4, 4, 2], 0, np.zeros(32, np.float32).tobytes()))
    p = tmp_path / "r.gguf"
    p.write_bytes(gguf_bytes([("general.architecture", 8, "qwen2")], tens))
    be = Backend(0)
    try:
        with G.Gguf(str(p)) as f:
            m = G.ResidentModel(be, f)
            assert set(m.by_name) == {s[0] for s in served}
            assert set(m.skipped) == {"blk.0.attn_norm.weight", "rope.cache"}
            for name, t, n_out, n_in in served:
                c, e = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, 9)))
                q = QuantAct.from_exps(e, c)
                got = be.matvec_q8act(t, m[name], n_out, n_in, q)
                raw = f.tensor_bytes(f.tensor(name))
                want = O.matvec_q8act(t, raw, n_out, n_in, c, O.exps_to_scales(e))
                assert np.array_equal(got, want), name
    finally:
        be.close()
