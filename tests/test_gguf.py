"""GGUF v3 container: the reference's parse KAT (src/gguf/reader.rs:373-500), run
against both the oracle's C reader and the product's reader, plus error cases."""
import struct

import numpy as np
import pytest

import oracle
from talos_b200 import gguf

T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY = 4, 5, 6, 7, 8, 9


def _put(buf, s):
    buf += struct.pack("<Q", len(s)) + s.encode()


def build_kat_gguf() -> bytes:
    """The byte layout of reader.rs:374-454, written independently of GgufWriter."""
    t1 = np.array([1, 2, 3, 4, 5, 6], np.float32)  # dims [3, 2]
    t2 = np.array([-1.5, 0.0, 42.25], np.float32)  # dims [3]
    b = bytearray(b"GGUF")
    b += struct.pack("<IQQ", 3, 2, 5)
    _put(b, "answer.u32"); b += struct.pack("<II", T_UINT32, 42)
    _put(b, "scale.f32"); b += struct.pack("<If", T_FLOAT32, 2.5)
    _put(b, "flag.bool"); b += struct.pack("<I", T_BOOL) + b"\x01"
    _put(b, "names.arr"); b += struct.pack("<IIQ", T_ARRAY, T_STRING, 3)
    for s in ("alpha", "beta", "gamma"):
        _put(b, s)
    _put(b, "types.arr"); b += struct.pack("<IIQ", T_ARRAY, T_INT32, 3) + struct.pack("<3i", -7, 0, 9)
    off2 = (t1.nbytes + 31) // 32 * 32
    _put(b, "tensor.one"); b += struct.pack("<IQQIQ", 2, 3, 2, 0, 0)
    _put(b, "tensor.two"); b += struct.pack("<IQIQ", 1, 3, 0, off2)
    while len(b) % 32:
        b.append(0)
    ds = len(b)
    b += t1.tobytes()
    while len(b) < ds + off2:
        b.append(0)
    b += t2.tobytes()
    return bytes(b)


def test_parse_kat_product_reader():
    g = gguf.GgufFile.from_bytes(build_kat_gguf())
    assert g.get_u32("answer.u32") == 42
    assert g.get_f32("scale.f32") == 2.5
    assert g.get_arr_str("names.arr") == ["alpha", "beta", "gamma"]
    assert g.get_arr_i32("types.arr") == [-7, 0, 9]
    assert g.get_bool("flag.bool") is True
    assert g.get_u32("scale.f32") is None  # wrong-type access
    assert g.get_str("missing") is None
    ts = g.tensors()
    assert [t.name for t in ts] == ["tensor.one", "tensor.two"]
    assert ts[0].dims == [3, 2] and ts[0].dtype == gguf.F32 and ts[0].elem_count() == 6
    assert ts[1].dims == [3]
    assert g.tensor_info("nope") is None
    assert list(g.tensor_f32("tensor.one")) == [1, 2, 3, 4, 5, 6]
    assert list(g.tensor_f32("tensor.two")) == [-1.5, 0.0, 42.25]
    with pytest.raises(gguf.GgufError):
        g.tensor_f32("missing")


def test_parse_kat_oracle_reader(tmp_path):
    p = tmp_path / "kat.gguf"
    p.write_bytes(build_kat_gguf())
    g = oracle.Gguf(path=str(p))
    assert g.get_u32("answer.u32") == 42
    assert g.get_f32("scale.f32") == 2.5
    assert g.get_arr_str("names.arr") == ["alpha", "beta", "gamma"]
    assert g.get_arr_i32("types.arr") == [-7, 0, 9]
    assert g.get_bool("flag.bool") is True
    assert g.get_u32("scale.f32") is None
    assert g.get_str("missing") is None
    ts = g.tensors()
    assert [t[0] for t in ts] == ["tensor.one", "tensor.two"]
    assert ts[0][1] == [3, 2] and ts[0][2] == 0
    assert list(g.tensor_f32("tensor.one")) == [1, 2, 3, 4, 5, 6]
    assert list(g.tensor_f32("tensor.two")) == [-1.5, 0.0, 42.25]
    with pytest.raises(oracle.OracleError):
        g.tensor_f32("missing")


def test_writer_round_trip_both_readers():
    w = gguf.GgufWriter()
    w.add_u32("a", 7)
    w.add_f32("b", -0.25)
    w.add_str("c", "llama")
    w.add_arr_str("d", ["x", "", "yz"])
    w.add_arr_i32("e", [1, -2])
    w.add_bool("f", False)
    q = np.arange(64, dtype=np.uint8).repeat(1)
    raw = oracle.quantize(oracle.Q8_0, np.linspace(-1, 1, 64, dtype=np.float32))
    w.add_tensor("m.weight", [32, 2], gguf.Q8_0, raw.tobytes())
    w.add_tensor("n.weight", [5], gguf.F32, np.arange(5, dtype=np.float32).tobytes())
    data = w.to_bytes()
    g = gguf.GgufFile.from_bytes(data)
    assert (g.get_u32("a"), g.get_f32("b"), g.get_str("c")) == (7, -0.25, "llama")
    assert g.get_arr_str("d") == ["x", "", "yz"] and g.get_arr_i32("e") == [1, -2]
    assert g.get_bool("f") is False
    r, t = g.tensor_raw("m.weight")
    assert t == gguf.Q8_0 and bytes(r) == raw.tobytes()
    og = oracle.Gguf(data=data)
    r2, t2 = og.tensor_raw("m.weight")
    assert t2 == gguf.Q8_0 and r2 == raw.tobytes()
    assert list(og.tensor_f32("n.weight")) == [0, 1, 2, 3, 4]
    assert q.size == 64


@pytest.mark.parametrize("mutate,needle", [
    (lambda b: b"GGUX" + b[4:], "magic"),
    (lambda b: b[:4] + struct.pack("<I", 2) + b[8:], "version"),
    (lambda b: b[:40], "end of file"),
])
def test_errors_both_readers(mutate, needle):
    bad = mutate(build_kat_gguf())
    with pytest.raises(gguf.GgufError, match=needle):
        gguf.GgufFile.from_bytes(bad)
    with pytest.raises(oracle.OracleError, match=needle):
        oracle.Gguf(data=bad)


def test_unsupported_tensor_type_rejected():
    b = bytearray(build_kat_gguf())
    # tensor.one's type tag sits right after its name, n_dims and two dims
    i = b.index(b"tensor.one") + len("tensor.one") + 4 + 16
    b[i:i + 4] = struct.pack("<I", 3)  # Q4_1: not supported (dtype.rs:33-41)
    with pytest.raises(gguf.GgufError, match="unsupported ggml type"):
        gguf.GgufFile.from_bytes(bytes(b))
    with pytest.raises(oracle.OracleError, match="unsupported ggml type"):
        oracle.Gguf(data=bytes(b))


def test_data_past_end():
    b = build_kat_gguf()[:-4]
    g = gguf.GgufFile.from_bytes(b)
    with pytest.raises(gguf.GgufError, match="past end"):
        g.tensor_f32("tensor.two")
    og = oracle.Gguf(data=b)
    with pytest.raises(oracle.OracleError, match="past end"):
        og.tensor_f32("tensor.two")
