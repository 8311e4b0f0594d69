"""The bit and fp16 arithmetic of the Q4_K GEMV decoder (TQ4K in
anedvd_b200/csrc/gemv_impl.cuh), restated on the CPU and checked exhaustively.

* scale_bytes: every lane decodes its two sub-blocks' 6-bit scales and minima
  (get_scale_min_k4, gguf.zig:952-960) side by side in one 32-bit word with
  byte permutes and masks.  Checked for all four lanes against the scales and
  minima the oracle's own Q4_K dequantiser (pinned to the reference's golden
  vectors) reveals for crafted blocks.
* the high-nibble trick: a high nibble read in place is the fp16 value
  1024 + 16 q; one fused multiply-add with the scale / 16 and -64 scale gives
  q * scale exactly, like the low-nibble form 1024 + q with scale and -1024 scale.
"""
import struct

import numpy as np

from oracle import oracle as orc

Q4_K = 12


def byte_perm(x, y, s):
    """PTX prmt (default mode): result byte k is byte (s >> 4k) & 7 of y:x,
    or that byte's sign replicated when bit 3 of the selector nibble is set."""
    src = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for k in range(4):
        nib = (s >> (4 * k)) & 0xF
        b = src[nib & 7]
        if nib & 8:
            b = 0xFF if b & 0x80 else 0x00
        out |= b << (8 * k)
    return out


def scale_bytes(y, z, w, tig):
    """The device decode: [sc(j0), sc(j0+1), m(j0), m(j0+1)] for j0 = 2*tig."""
    lo = tig < 2
    j0, j1 = 2 * tig, 2 * tig + 1
    m32 = 0xFFFFFFFF
    sel_a = (j0 | j1 << 4 | (j0 + 4) << 8 | (j1 + 4) << 12) if lo else \
        ((j0 - 4) | (j1 - 4) << 4 | (j0 - 4) << 8 | (j1 - 4) << 12)
    a = byte_perm(y if lo else w, z if lo else w, sel_a)
    a2 = byte_perm(a, a >> 4, 0x3210 if lo else 0x7610)
    sel_b = (((j0 - 4) & m32) | ((j1 - 4) & m32) << 4 | j0 << 8 | j1 << 12) & m32
    b = byte_perm(y, z, sel_b)
    hb = (b >> 2) & (0 if lo else 0x30303030)
    return (a2 & (0x3F3F3F3F if lo else 0x0F0F0F0F)) | hb


def _block(scales, qbyte):
    return struct.pack("<ee", 1.0, 1.0) + bytes(scales) + bytes([qbyte]) * 128


def _oracle_scales(scales):
    """sc and m of the 8 sub-blocks, read off the oracle's dequant of blocks
    with d = dmin = 1: q = 0 gives -m, q = 1 gives sc - m."""
    y0 = orc.dequant(Q4_K, _block(scales, 0x00))
    y1 = orc.dequant(Q4_K, _block(scales, 0x11))
    m = [int(round(-y0[32 * s])) for s in range(8)]
    sc = [int(round(y1[32 * s])) + m[s] for s in range(8)]
    return sc, m


def test_scale_bytes_matches_get_scale_min_k4():
    rng = np.random.default_rng(7)
    records = [rng.integers(0, 256, 12, dtype=np.uint8) for _ in range(200)]
    records += [np.full(12, v, dtype=np.uint8) for v in (0x00, 0xFF, 0x3F, 0xC0, 0x0F, 0xF0)]
    for rec in records:
        sc, m = _oracle_scales(rec.tolist())
        y, z, w = struct.unpack("<III", rec.tobytes())
        for tig in range(4):
            v = scale_bytes(y, z, w, tig)
            got = [(v >> (8 * k)) & 0xFF for k in range(4)]
            want = [sc[2 * tig], sc[2 * tig + 1], m[2 * tig], m[2 * tig + 1]]
            assert got == want, (rec.tolist(), tig, got, want)


def _fma16(a, b, c):
    """fp16 fused multiply-add: exact in float64 (11-bit operands), rounded once."""
    return np.float16(np.float64(np.float16(a)) * np.float64(np.float16(b)) + np.float64(np.float16(c)))


def test_nibble_forms_give_q_times_scale_exactly():
    for sc in range(64):
        for q in range(16):
            lo = _fma16(1024.0 + q, sc, -1024.0 * sc)            # low nibble: 0x6400 | q
            hi = _fma16(1024.0 + 16 * q, sc / 16.0, -64.0 * sc)  # high nibble in place: 0x6400 | q << 4
            assert float(lo) == q * sc and float(hi) == q * sc, (q, sc, lo, hi)
            # the magic halves themselves are exact fp16 values
            assert float(np.float16(1024.0 + 16 * q)) == 1024.0 + 16 * q
            assert float(np.float16(sc / 16.0)) == sc / 16.0
