"""GGUF v2/v3 container: a small reader and writer in numpy.

Mirrors the parts of the reference's ``src/gguf.zig`` that the quantized path
touches: the header and metadata table (``gguf.zig:589-656``), the tensor table
with ggml dim order (``gguf.zig:107-136``; ``dims[0]`` is the row length), the
block geometry (``gguf.zig:49-77``) and tensor byte ranges (``gguf.zig:397-460``).
The C++ engine has its own parser (``csrc/gguf.cpp``); this one generates the
synthetic model files and feeds the CPU oracle in the tests.
"""

import struct

import numpy as np

MAGIC = 0x46554747  # "GGUF"

# ggml type ids (gguf.zig:30-46) -> (elements per block, bytes per block)
LAYOUT = {
    0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
    9: (32, 36), 10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176),
    14: (256, 210), 15: (256, 292), 30: (1, 2),
}
TYPE_NAME = {0: "f32", 1: "f16", 2: "q4_0", 3: "q4_1", 6: "q5_0", 7: "q5_1", 8: "q8_0",
             9: "q8_1", 10: "q2_k", 11: "q3_k", 12: "q4_k", 13: "q5_k", 14: "q6_k",
             15: "q8_k", 30: "bf16"}
TYPE_ID = {v: k for k, v in TYPE_NAME.items()}

# metadata value types (gguf.zig ValueType)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
        BOOL: "<B", U64: "<Q", I64: "<q", F64: "<d"}


class GgufError(ValueError):
    pass


def tensor_nbytes(ttype, n_elems):
    if ttype not in LAYOUT:
        raise GgufError("UnsupportedType: ggml type %d" % ttype)
    epb, bpb = LAYOUT[ttype]
    if n_elems % epb:
        raise GgufError("InvalidTensorShape: %d elements, block of %d" % (n_elems, epb))
    return n_elems // epb * bpb


class Tensor:
    __slots__ = ("name", "dims", "ttype", "offset", "data")

    def __init__(self, name, dims, ttype, offset, data):
        self.name, self.dims, self.ttype, self.offset, self.data = name, dims, ttype, offset, data

    @property
    def n_elems(self):
        n = 1
        for d in self.dims:
            n *= d
        return n


class Reader:
    """Parses a GGUF file held in memory (bytes or a numpy memmap)."""

    def __init__(self, buf):
        self.buf = buf if isinstance(buf, (bytes, bytearray)) else memoryview(buf)
        self.pos = 0
        self.kv = {}
        self.tensors = {}
        self.alignment = 32
        self._parse()

    @classmethod
    def open(cls, path):
        return cls(np.memmap(path, dtype=np.uint8, mode="r"))

    def _take(self, n):
        if self.pos + n > len(self.buf):
            raise GgufError("TruncatedFile")
        b = bytes(self.buf[self.pos:self.pos + n])
        self.pos += n
        return b

    def _u32(self):
        return struct.unpack("<I", self._take(4))[0]

    def _u64(self):
        return struct.unpack("<Q", self._take(8))[0]

    def _str(self):
        n = self._u64()
        if n > len(self.buf) - self.pos:
            raise GgufError("TruncatedFile")
        return self._take(n).decode("utf-8", errors="replace")

    def _value(self, vt):
        if vt == STRING:
            return self._str()
        if vt == ARRAY:
            et = self._u32()
            n = self._u64()
            if n > len(self.buf) - self.pos + 1:
                raise GgufError("TruncatedFile")
            return [self._value(et) for _ in range(n)]
        if vt not in _FMT:
            raise GgufError("InvalidMetadata: value type %d" % vt)
        fmt = _FMT[vt]
        v = struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]
        return bool(v) if vt == BOOL else v

    def _parse(self):
        if len(self.buf) < 24:
            raise GgufError("TruncatedFile")
        if self._u32() != MAGIC:
            raise GgufError("NotGgufFile")
        version = self._u32()
        if version not in (2, 3):
            raise GgufError("UnsupportedVersion")
        self.version = version
        n_tensors, n_kv = self._u64(), self._u64()
        remaining = len(self.buf) - self.pos
        if n_tensors > remaining + 1:
            raise GgufError("TooManyTensors")
        if n_kv > remaining + 1:
            raise GgufError("TooManyMetadataEntries")
        for _ in range(n_kv):
            key = self._str()
            val = self._value(self._u32())
            self.kv.setdefault(key, val)  # duplicate keys: first wins
        al = self.kv.get("general.alignment", 32)
        if not isinstance(al, int) or al == 0 or al > (1 << 24) or al & (al - 1):
            raise GgufError("InvalidMetadata: alignment")
        self.alignment = al
        infos = []
        for _ in range(n_tensors):
            name = self._str()
            nd = self._u32()
            if nd == 0 or nd > 8:
                raise GgufError("InvalidTensorShape")
            dims = [self._u64() for _ in range(nd)]
            ttype, off = self._u32(), self._u64()
            infos.append((name, dims, ttype, off))
        data_off = (self.pos + self.alignment - 1) // self.alignment * self.alignment
        if data_off > len(self.buf):
            raise GgufError("TruncatedFile")
        self.data_offset = data_off
        for name, dims, ttype, off in infos:
            self.tensors.setdefault(name, Tensor(name, dims, ttype, off, None))

    def arch(self):
        return self.kv.get("general.architecture")

    def tensor_bytes(self, name):
        t = self.tensors.get(name)
        if t is None:
            raise GgufError("TensorNotFound: " + name)
        n = tensor_nbytes(t.ttype, t.n_elems)
        start = self.data_offset + t.offset
        if start + n > len(self.buf):
            raise GgufError("TensorDataOutOfRange")
        return np.frombuffer(self.buf[start:start + n], dtype=np.uint8)


def _enc_str(s):
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _enc_value(vt, v):
    if vt == STRING:
        return struct.pack("<I", STRING) + _enc_str(v)
    if vt == ARRAY:
        et, items = v
        out = struct.pack("<IIQ", ARRAY, et, len(items))
        for it in items:
            out += _enc_str(it) if et == STRING else struct.pack(_FMT[et], it)
        return out
    return struct.pack("<I", vt) + struct.pack(_FMT[vt], v)


def write(path, kvs, tensors, alignment=32):
    """kvs: [(key, vtype, value)]; tensors: [(name, dims, ttype, bytes-like)]."""
    header = struct.pack("<IIQQ", MAGIC, 3, len(tensors), len(kvs))
    for key, vt, v in kvs:
        header += _enc_str(key) + _enc_value(vt, v)
    infos = b""
    offsets = []
    off = 0
    for name, dims, ttype, data in tensors:
        off = (off + alignment - 1) // alignment * alignment
        nb = tensor_nbytes(ttype, int(np.prod(dims)))
        if len(data) != nb:
            raise GgufError("%s: %d bytes, expected %d" % (name, len(data), nb))
        offsets.append(off)
        infos += _enc_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", ttype, off)
        off += nb
    head = header + infos
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head + bytes(pad))
        pos = 0
        for (name, dims, ttype, data), o in zip(tensors, offsets):
            if o > pos:
                f.write(bytes(o - pos))
                pos = o
            mv = memoryview(data).cast("B") if not isinstance(data, np.ndarray) else memoryview(
                np.ascontiguousarray(data).view(np.uint8).reshape(-1))
            f.write(mv)
            pos += len(mv)
    return path
