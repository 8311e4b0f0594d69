"""The GGUF container, without a GPU: the library's parser (cuq_gguf_*, the one
cuq_model_load_gguf uses) and the Python reader (anedvd_b200.gguf) on the
reference's own fixture tests/golden/gguf/tiny_v3.gguf, with the expectations
of gguf.zig:1648-1715, and on the malformed files of gguf.zig:1717-1769 and
1794-1823 (rebuilt here byte by byte, as the reference's test Builder does)."""
import os
import struct

import numpy as np
import pytest

from anedvd_b200 import gguf
from anedvd_b200 import runtime as rt
from oracle import oracle as orc

TINY = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "gguf", "tiny_v3.gguf")


def _lib_or_skip():
    if not os.path.exists(rt.LIB_PATH):
        from anedvd_b200 import build
        build.build()
    return rt.load()


# ---------------------------------------------------------------- builder --
class Builder:
    """GGUF bytes as gguf.zig's test Builder writes them (header, typed
    metadata entries, tensor infos, padding)."""

    def __init__(self):
        self.b = bytearray()

    def header(self, version, n_tensors, n_kv):
        self.b += struct.pack("<IIQQ", gguf.MAGIC, version, n_tensors, n_kv)

    def _key(self, k, vt):
        self.b += struct.pack("<Q", len(k)) + k.encode() + struct.pack("<I", vt)

    def kv_string(self, k, v):
        self._key(k, gguf.STRING)
        self.b += struct.pack("<Q", len(v)) + v.encode()

    def kv(self, k, vt, fmt, v):
        self._key(k, vt)
        self.b += struct.pack(fmt, v)

    def kv_string_array(self, k, vs):
        self._key(k, gguf.ARRAY)
        self.b += struct.pack("<IQ", gguf.STRING, len(vs))
        for v in vs:
            self.b += struct.pack("<Q", len(v)) + v.encode()

    def tensor_info(self, name, dims, ttype, off):
        self.b += struct.pack("<Q", len(name)) + name.encode() + struct.pack("<I", len(dims))
        self.b += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", ttype, off)

    def pad_to(self, a):
        while len(self.b) % a:
            self.b.append(0)


def tiny_in_memory(alignment=32):
    """gguf.zig:1365-1399 buildTinyGguf: three tensors and eight metadata entries."""
    b = Builder()
    b.header(3, 3, 8)
    b.kv_string("general.architecture", "llama")
    b.kv_string("general.name", "in-memory-fixture")
    b.kv("general.alignment", gguf.U32, "<I", alignment)
    b.kv("llama.block_count", gguf.U32, "<I", 1)
    b.kv("fixture.negative", gguf.I32, "<i", -7)
    b.kv("llama.rope.freq_base", gguf.F32, "<f", 10000.0)
    b.kv("fixture.bool", gguf.BOOL, "<B", 1)
    b.kv_string_array("fixture.strings", ["a", "bb"])
    f32_data = struct.pack("<4f", 1.5, -2.0, 3.25, 0.5)
    f16_data = np.array([1.0, 2.5, -0.75, 4.0, -1.5, 0.25], np.float16).tobytes()
    q4_data = bytes([0x00, 0x38, 0x21]) + bytes(15)
    al = lambda n: (n + alignment - 1) // alignment * alignment
    off1 = al(len(f32_data))
    off2 = al(off1 + len(f16_data))
    b.tensor_info("w.f32", [4], 0, 0)
    b.tensor_info("w.f16", [2, 3], 1, off1)
    b.tensor_info("w.q4_0", [32], 2, off2)
    b.pad_to(alignment)
    b.b += f32_data
    b.pad_to(alignment)
    b.b += f16_data
    b.pad_to(alignment)
    b.b += q4_data
    return bytes(b.b)


# ------------------------------------------------------ the golden fixture --
def test_library_parser_reads_tiny_v3():
    _lib_or_skip()
    g = rt.GgufFile(TINY)
    assert g.version == 3 and g.tensor_count == 4
    assert g.string("general.architecture") == "llama"
    assert g.string("general.name") == "tiny-fixture"
    assert g.u64("fixture.u64") == 1234567890123
    assert g.i64("fixture.i64") & 0xFFFFFFFFFFFFFFFF == 0xFFFFFFFFFFFFFFFF - 1234567890122
    assert g.f64("llama.rope.freq_base") == 10000.0
    assert g.u64("fixture.bool") == 1
    assert g.u64("fixture.u8") == 200 and g.u64("fixture.u16") == 60000
    assert g.array("fixture.u32_array") == [1, 2, 3]
    assert g.array("fixture.empty_array") == []
    s = g.array("fixture.string_array")
    assert len(s) == 3 and s[2] == "ccc"
    assert g.tensor_info("w.f32")[:2] == (0, [4])
    assert g.tensor_info("w.f16")[:2] == (1, [2, 3])
    assert len(g.tensor_bytes("w.f32")) == 16 and len(g.tensor_bytes("w.f16")) == 12
    _check_tiny_values(lambda n: g.tensor_bytes(n))


def test_python_reader_reads_tiny_v3():
    r = gguf.Reader.open(TINY)
    assert r.version == 3 and len(r.tensors) == 4
    assert r.arch() == "llama" and r.kv["general.name"] == "tiny-fixture"
    assert r.kv["fixture.u64"] == 1234567890123
    assert r.kv["fixture.i64"] & 0xFFFFFFFFFFFFFFFF == 0xFFFFFFFFFFFFFFFF - 1234567890122
    assert r.kv["llama.rope.freq_base"] == 10000.0 and r.kv["fixture.bool"] is True
    assert r.kv["fixture.u8"] == 200 and r.kv["fixture.u16"] == 60000
    assert r.kv["fixture.u32_array"] == [1, 2, 3] and r.kv["fixture.empty_array"] == []
    assert r.kv["fixture.string_array"][2] == "ccc"
    assert r.tensors["w.f16"].dims == [2, 3] and r.tensors["w.f32"].ttype == 0
    _check_tiny_values(lambda n: r.tensor_bytes(n).tobytes())


def _check_tiny_values(tensor_bytes):
    # readF32 / readF16 through the oracle's dequantizer (gguf.zig:1690-1714)
    assert list(orc.dequant(0, tensor_bytes("w.f32"))) == [1.5, -2.0, 3.25, 0.5]
    assert list(orc.dequant(1, tensor_bytes("w.f16"))) == [1.0, 2.5, -0.75, 4.0, -1.5, 0.25]
    assert list(orc.read_f16(1, tensor_bytes("w.f16"), 6).view(np.float16)) == [1.0, 2.5, -0.75, 4.0, -1.5, 0.25]
    q4 = orc.dequant(2, tensor_bytes("w.q4_0"))
    assert (q4[0], q4[16], q4[31]) == (-3.5, -3.0, -4.0)
    q8 = orc.dequant(8, tensor_bytes("w.q8_0"))
    assert (q8[0], q8[1], q8[31]) == (-32.0, -31.75, -24.25)
    q4h = orc.read_f16(2, tensor_bytes("w.q4_0"), 32).view(np.float16)
    assert (q4h[0], q4h[16]) == (-3.5, -3.0)


# ------------------------------------------------------------ malformed ---
def _both_reject(data, name):
    _lib_or_skip()
    with pytest.raises(rt.CuqError) as ei:
        rt.GgufFile(data=data)
    assert name in str(ei.value)
    with pytest.raises(gguf.GgufError) as ej:
        gguf.Reader(bytes(data))
    assert name in str(ej.value)


def test_in_memory_fixture_parses():
    _lib_or_skip()
    data = tiny_in_memory()
    g = rt.GgufFile(data=data)
    assert g.i64("fixture.negative") == -7 and g.u64("fixture.negative") is None
    assert g.array("fixture.strings") == ["a", "bb"]
    assert orc.dequant(2, g.tensor_bytes("w.q4_0"))[0] == -3.5


def test_rejects_malformed_files():
    good = bytearray(tiny_in_memory())
    bad = bytearray(good)
    bad[0] = ord("X")
    _both_reject(bytes(bad), "NotGgufFile")
    bad = bytearray(good)
    bad[4] = 4
    _both_reject(bytes(bad), "UnsupportedVersion")
    _both_reject(bytes(good[:len(good) - 400]), "TruncatedFile")
    _both_reject(b"", "TruncatedFile")


def test_tensor_errors():
    _lib_or_skip()
    b = Builder()
    b.header(3, 1, 0)
    b.tensor_info("bad", [32], 16, 0)  # iq2_xxs: a type gguf.zig does not decode
    b.pad_to(32)
    b.b += bytes(200)
    g = rt.GgufFile(data=bytes(b.b))
    with pytest.raises(rt.CuqError) as ei:
        g.tensor_bytes("bad")
    assert ei.value.code == rt.EUNSUPPORTED and "UnsupportedType" in str(ei.value)
    with pytest.raises(gguf.GgufError, match="UnsupportedType"):
        gguf.Reader(bytes(b.b)).tensor_bytes("bad")

    b2 = Builder()
    b2.header(3, 2, 0)
    b2.tensor_info("odd", [48], 2, 0)          # 48 is not a multiple of 32
    b2.tensor_info("past_end", [32], 2, 1 << 20)
    b2.pad_to(32)
    b2.b += bytes(64)
    g2 = rt.GgufFile(data=bytes(b2.b))
    r2 = gguf.Reader(bytes(b2.b))
    for name, err in (("odd", "InvalidTensorShape"), ("past_end", "TensorDataOutOfRange"),
                      ("nope", "TensorNotFound")):
        with pytest.raises(rt.CuqError, match=err):
            g2.tensor_bytes(name)
        with pytest.raises(gguf.GgufError, match=err):
            r2.tensor_bytes(name)


def test_rejects_absurd_entry_counts():
    b = Builder()
    b.header(3, 1 << 30, 0)
    b.b += bytes(64)
    _both_reject(bytes(b.b), "TooManyTensors")
    b = Builder()
    b.header(3, 0, 1 << 30)
    b.b += bytes(64)
    _both_reject(bytes(b.b), "TooManyMetadataEntries")
    # a count the file could hold is not rejected
    b = Builder()
    b.header(3, 0, 0)
    b.pad_to(32)
    assert rt.GgufFile(data=bytes(b.b)).tensor_count == 0
    assert len(gguf.Reader(bytes(b.b)).tensors) == 0
