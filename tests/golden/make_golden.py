#!/usr/bin/env python3
"""Regenerate the golden vectors under tests/golden/ from the ANEDVD reference tree.

Run by hand in a checkout that has the reference source next to it:

    python tests/golden/make_golden.py /path/to/ANEDVD

What it writes (all small, all committed; nothing at test time reads the
reference tree):

* ``dequant/<type>.bin`` / ``.f32`` -- the reference's own dequant fixtures
  (``tests/fixtures/dequant/`` in ANEDVD, produced by its
  ``tools/make_fixtures.py`` and pinned bit-for-bit by ``src/gguf.zig:1528-1570``).
  They are copied unchanged, then re-checked against the reference's
  ``tools/ggml_reference.py`` so a corrupted copy cannot pass.
* ``dequant_wide/<type>.bin`` / ``.f32`` -- 64 more blocks per type from a
  seeded generator of this repo (random bytes, finite fp16/f32 scale fields),
  with the expected floats computed by importing the reference's
  ``tools/ggml_reference.py``.  More blocks means every nibble/bit position and
  every 6-bit scale path is exercised, not just the two blocks of the
  reference fixtures.
* ``gguf/tiny_v3.gguf`` -- the reference's hand-written GGUF v3 fixture
  (``tests/fixtures/gguf/tiny_v3.gguf``), for the GGUF parser tests.
"""

import os
import shutil
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

TYPES = {  # ggml id -> fixture name (ANEDVD src/gguf.zig:30-46)
    0: "f32", 1: "f16", 2: "q4_0", 3: "q4_1", 6: "q5_0", 7: "q5_1", 8: "q8_0",
    9: "q8_1", 10: "q2_k", 11: "q3_k", 12: "q4_k", 13: "q5_k", 14: "q6_k",
    15: "q8_k", 30: "bf16",
}

# Byte offsets of fp16 ("h") / f32 ("f") scale fields per block type, so random
# blocks never carry NaN/Inf scales.
SCALE_FIELDS = {
    2: [(0, "h")], 3: [(0, "h"), (2, "h")], 6: [(0, "h")], 7: [(0, "h"), (2, "h")],
    8: [(0, "h")], 9: [(0, "h"), (2, "h")], 10: [(80, "h"), (82, "h")], 11: [(108, "h")],
    12: [(0, "h"), (2, "h")], 13: [(0, "h"), (2, "h")], 14: [(208, "h")], 15: [(0, "f")],
}


class SplitMix64:
    """splitmix64 (Steele, Lea, Flood 2014): small, seedable, reproducible."""

    def __init__(self, seed):
        self.s = seed & 0xFFFFFFFFFFFFFFFF

    def next(self):
        self.s = (self.s + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        z = self.s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        return z ^ (z >> 31)


def finite_half(rng):
    """A finite fp16 scale with random sign, |v| in [2^-10, 2^2)."""
    sign = (rng.next() & 1) << 15
    exp = 5 + rng.next() % 12
    return struct.pack("<H", sign | (exp << 10) | (rng.next() % 1024))


def finite_f32(rng):
    sign = (rng.next() & 1) << 31
    exp = 110 + rng.next() % 20
    return struct.pack("<I", sign | (exp << 23) | (rng.next() % (1 << 23)))


def wide_block_bytes(ttype, rng, nblocks, ref):
    epb, bb = ref.LAYOUT[ttype]
    if ttype == 0:
        return b"".join(finite_f32(rng) for _ in range(nblocks))
    if ttype == 1:
        return b"".join(finite_half(rng) for _ in range(nblocks))
    if ttype == 30:
        return b"".join(finite_f32(rng)[2:4] for _ in range(nblocks))
    out = bytearray()
    for _ in range(nblocks):
        blk = bytearray(rng.next() & 0xFF for _ in range(bb))
        for off, kind in SCALE_FIELDS.get(ttype, []):
            v = finite_half(rng) if kind == "h" else finite_f32(rng)
            blk[off:off + len(v)] = v
        out += blk
    return bytes(out)


def main():
    if len(sys.argv) != 2:
        print(__doc__)
        sys.exit(2)
    ref_root = os.path.abspath(sys.argv[1])
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    import ggml_reference as ref  # the reference's bit-accurate dequantisers

    src_dir = os.path.join(ref_root, "tests", "fixtures", "dequant")
    dq_dir = os.path.join(HERE, "dequant")
    wide_dir = os.path.join(HERE, "dequant_wide")
    os.makedirs(dq_dir, exist_ok=True)
    os.makedirs(wide_dir, exist_ok=True)

    for ttype, name in sorted(TYPES.items()):
        for ext in (".bin", ".f32"):
            shutil.copyfile(os.path.join(src_dir, name + ext), os.path.join(dq_dir, name + ext))
        data = open(os.path.join(dq_dir, name + ".bin"), "rb").read()
        want = open(os.path.join(dq_dir, name + ".f32"), "rb").read()
        got = b"".join(struct.pack("<f", v) for v in ref.dequantize(ttype, data))
        assert got == want, "reference fixture %s does not match ggml_reference" % name

        rng = SplitMix64(0xA11CE000 + ttype)
        epb, _ = ref.LAYOUT[ttype]
        nblocks = 64 if epb > 1 else 512
        wdata = wide_block_bytes(ttype, rng, nblocks, ref)
        wvals = ref.dequantize(ttype, wdata)
        with open(os.path.join(wide_dir, name + ".bin"), "wb") as f:
            f.write(wdata)
        with open(os.path.join(wide_dir, name + ".f32"), "wb") as f:
            f.write(b"".join(struct.pack("<f", v) for v in wvals))
        print("  %-5s fixture %4d B, wide %6d B / %6d values" % (name, len(data), len(wdata), len(wvals)))

    gdir = os.path.join(HERE, "gguf")
    os.makedirs(gdir, exist_ok=True)
    shutil.copyfile(os.path.join(ref_root, "tests", "fixtures", "gguf", "tiny_v3.gguf"),
                    os.path.join(gdir, "tiny_v3.gguf"))
    print("done")


if __name__ == "__main__":
    main()
