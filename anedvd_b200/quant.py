"""Block quantisers for the synthetic models (numpy, vectorised).

The reference never quantises (it only reads GGUF files), so these are this
repo's own, written from the block formats its dequantisers define
(``src/gguf.zig:763-1059``).  Every choice below is documented because parity
is checked on identical bytes, not on how they were produced:

* rounding is ``numpy.rint`` (half to even) everywhere;
* scales are computed in float32 and stored as fp16 (round to nearest even);
* a block whose scale rounds to zero stores all-zero quants.

Input ``w`` is float32 with ``w.size`` a multiple of the block size; the output
is the raw GGUF payload (``uint8``), blocks in order.
"""

import numpy as np


def _f16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16)


def _safe_inv(d):
    d = d.astype(np.float32)
    out = np.zeros_like(d)
    nz = d != 0
    out[nz] = np.float32(1.0) / d[nz]
    return out


def q8_0(w):
    """Q8_0: 34-byte blocks = fp16 d + 32 x int8; d = max|w| / 127, q = rint(w / d)."""
    b = w.reshape(-1, 32).astype(np.float32)
    d16 = _f16(np.abs(b).max(axis=1) / np.float32(127.0))
    inv = _safe_inv(d16.astype(np.float32))[:, None]
    q = np.clip(np.rint(b * inv), -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:34] = q.view(np.uint8)
    return out.reshape(-1)


def _signed_absmax(b):
    idx = np.abs(b).argmax(axis=1)
    return b[np.arange(b.shape[0]), idx]


def q4_0(w):
    """Q4_0: d = m / -8 with m the signed max-|w| value, q = clip(rint(w/d) + 8, 0, 15)."""
    b = w.reshape(-1, 32).astype(np.float32)
    d16 = _f16(_signed_absmax(b) / np.float32(-8.0))
    inv = _safe_inv(d16.astype(np.float32))[:, None]
    q = np.clip(np.rint(b * inv) + 8, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:18] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def q4_1(w):
    """Q4_1: m = min, d = (max - min) / 15, q = clip(rint((w - m) / d), 0, 15)."""
    b = w.reshape(-1, 32).astype(np.float32)
    mn, mx = b.min(axis=1), b.max(axis=1)
    d16, m16 = _f16((mx - mn) / np.float32(15.0)), _f16(mn)
    inv = _safe_inv(d16.astype(np.float32))[:, None]
    q = np.clip(np.rint((b - m16.astype(np.float32)[:, None]) * inv), 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 20), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = m16.view(np.uint8).reshape(-1, 2)
    out[:, 4:20] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def _qh_bits(q5):
    """Bit 4 of each 5-bit value j -> bit j of a little-endian u32 (gguf.zig:808-811)."""
    bits = ((q5 >> 4) & 1).astype(np.uint32)
    return (bits << np.arange(32, dtype=np.uint32)[None, :]).sum(axis=1, dtype=np.uint64).astype(np.uint32)


def q5_0(w):
    """Q5_0: d = m / -16, q = clip(rint(w/d) + 16, 0, 31); low nibbles + qh bits."""
    b = w.reshape(-1, 32).astype(np.float32)
    d16 = _f16(_signed_absmax(b) / np.float32(-16.0))
    inv = _safe_inv(d16.astype(np.float32))[:, None]
    q = np.clip(np.rint(b * inv) + 16, 0, 31).astype(np.uint8)
    out = np.empty((b.shape[0], 22), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:6] = _qh_bits(q).view(np.uint8).reshape(-1, 4)
    out[:, 6:22] = (q[:, :16] & 0xF) | ((q[:, 16:] & 0xF) << 4)
    return out.reshape(-1)


def q5_1(w):
    """Q5_1: m = min, d = (max - min) / 31, q = clip(rint((w - m) / d), 0, 31)."""
    b = w.reshape(-1, 32).astype(np.float32)
    mn, mx = b.min(axis=1), b.max(axis=1)
    d16, m16 = _f16((mx - mn) / np.float32(31.0)), _f16(mn)
    inv = _safe_inv(d16.astype(np.float32))[:, None]
    q = np.clip(np.rint((b - m16.astype(np.float32)[:, None]) * inv), 0, 31).astype(np.uint8)
    out = np.empty((b.shape[0], 24), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = m16.view(np.uint8).reshape(-1, 2)
    out[:, 4:8] = _qh_bits(q).view(np.uint8).reshape(-1, 4)
    out[:, 8:24] = (q[:, :16] & 0xF) | ((q[:, 16:] & 0xF) << 4)
    return out.reshape(-1)


def q4_k(w):
    """Q4_K: 256-weight superblocks of 8 x 32 sub-blocks.

    Per sub-block j: lo = min(0, min w), s_j = (max w - lo) / 15, m_j = -lo.
    Superblock d = max s_j / 63, dmin = max m_j / 63 (fp16); 6-bit sc_j =
    rint(s_j / d), mn_j = rint(m_j / dmin); q = clip(rint((w + m1) / d1), 0, 15)
    with d1 = d*sc_j, m1 = dmin*mn_j -- the decode of gguf.zig:962-996.  The
    6-bit pairs are packed so that getScaleMinK4 (gguf.zig:952-960) reads them.
    """
    sb = w.reshape(-1, 8, 32).astype(np.float32)
    lo = np.minimum(sb.min(axis=2), 0.0).astype(np.float32)
    hi = sb.max(axis=2)
    s = ((hi - lo) / np.float32(15.0)).astype(np.float32)
    m = (-lo).astype(np.float32)
    d16 = _f16(s.max(axis=1) / np.float32(63.0))
    dm16 = _f16(m.max(axis=1) / np.float32(63.0))
    d32, dm32 = d16.astype(np.float32), dm16.astype(np.float32)
    sc = np.clip(np.rint(s * _safe_inv(d32)[:, None]), 0, 63).astype(np.uint8)
    mn = np.clip(np.rint(m * _safe_inv(dm32)[:, None]), 0, 63).astype(np.uint8)
    d1 = (d32[:, None] * sc.astype(np.float32)).astype(np.float32)
    m1 = (dm32[:, None] * mn.astype(np.float32)).astype(np.float32)
    q = np.clip(np.rint((sb + m1[:, :, None]) * _safe_inv(d1)[:, :, None]), 0, 15).astype(np.uint8)
    n = sb.shape[0]
    out = np.empty((n, 144), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(-1, 2)
    scales = np.zeros((n, 12), dtype=np.uint8)
    scales[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    scales[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    scales[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    out[:, 4:16] = scales
    qq = q.reshape(n, 4, 2, 32)           # chunk c: sub-blocks 2c (low) and 2c+1 (high)
    out[:, 16:144] = (qq[:, :, 0, :] | (qq[:, :, 1, :] << 4)).reshape(n, 128)
    return out.reshape(-1)


def q6_k(w):
    """Q6_K: 256-weight superblocks of 16 x 16 sub-blocks, int8 scales, fp16 d.

    s_j = max|w| / 31 (signed by the max-|w| value), d = max|s_j| / 127;
    sc_j = rint(s_j / d) (int8); q = clip(rint(w / (d*sc_j)), -32, 31) + 32,
    laid out as gguf.zig:1036-1059 decodes it (ql low/high nibbles, 2-bit qh).
    """
    sb = w.reshape(-1, 16, 16).astype(np.float32)
    n = sb.shape[0]
    idx = np.abs(sb).argmax(axis=2)
    smax = np.take_along_axis(sb, idx[:, :, None], axis=2)[:, :, 0]
    s = (smax / np.float32(-32.0)).astype(np.float32)
    d16 = _f16(np.abs(s).max(axis=1) / np.float32(127.0))
    d32 = d16.astype(np.float32)
    sc = np.clip(np.rint(s * _safe_inv(d32)[:, None]), -127, 127).astype(np.int8)
    eff = (d32[:, None] * sc.astype(np.float32)).astype(np.float32)
    q = (np.clip(np.rint(sb * _safe_inv(eff)[:, :, None]), -32, 31) + 32).astype(np.uint8)
    q = q.reshape(n, 2, 4, 32)            # [half][t][l]: weight h*128 + 32t + l
    out = np.empty((n, 210), dtype=np.uint8)
    ql = np.empty((n, 2, 64), dtype=np.uint8)
    ql[:, :, 0:32] = (q[:, :, 0] & 0xF) | ((q[:, :, 2] & 0xF) << 4)
    ql[:, :, 32:64] = (q[:, :, 1] & 0xF) | ((q[:, :, 3] & 0xF) << 4)
    qh = ((q[:, :, 0] >> 4) | ((q[:, :, 1] >> 4) << 2) | ((q[:, :, 2] >> 4) << 4) | ((q[:, :, 3] >> 4) << 6))
    out[:, 0:128] = ql.reshape(n, 128)
    out[:, 128:192] = qh.astype(np.uint8).reshape(n, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d16.view(np.uint8).reshape(-1, 2)
    return out.reshape(-1)


def f16(w):
    return np.asarray(w, dtype=np.float32).astype(np.float16).view(np.uint8).reshape(-1)


def bf16(w):
    """Round-to-nearest-even float32 -> bfloat16."""
    u = np.asarray(w, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r.view(np.uint8).reshape(-1)


def f32(w):
    return np.asarray(w, dtype=np.float32).view(np.uint8).reshape(-1)


QUANTIZE = {0: f32, 1: f16, 2: q4_0, 3: q4_1, 6: q5_0, 7: q5_1, 8: q8_0, 12: q4_k, 14: q6_k, 30: bf16}


def quantize(ttype, w):
    if ttype not in QUANTIZE:
        raise ValueError("no quantiser for ggml type %d" % ttype)
    return QUANTIZE[ttype](np.ascontiguousarray(w, dtype=np.float32).reshape(-1))
