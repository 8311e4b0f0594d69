"""The CPU oracle pinned against the reference's own golden vectors and tests.

Each test restates one of the reference's tests (cited) against the oracle,
so the oracle that later checks the CUDA kernels is itself pinned.
"""
import os
import struct

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TYPES = {0: "f32", 1: "f16", 2: "q4_0", 3: "q4_1", 6: "q5_0", 7: "q5_1", 8: "q8_0", 9: "q8_1",
         10: "q2_k", 11: "q3_k", 12: "q4_k", 13: "q5_k", 14: "q6_k", 15: "q8_k", 30: "bf16"}


def _load(sub, name):
    raw = open(os.path.join(GOLD, sub, name + ".bin"), "rb").read()
    want = np.frombuffer(open(os.path.join(GOLD, sub, name + ".f32"), "rb").read(), dtype=np.uint32)
    return raw, want


def test_block_geometry_matches_ggml_table():
    # gguf.zig:1401-1422
    want = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36),
            10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210),
            15: (256, 292), 0: (1, 4), 1: (1, 2), 30: (1, 2)}
    for t, (e, b) in want.items():
        assert (orc.block_elems(t), orc.block_bytes(t)) == (e, b)
    assert orc.block_elems(16) == 0 and orc.block_bytes(16) == 0  # iq2_xxs: unsupported


@pytest.mark.parametrize("ttype", sorted(TYPES))
def test_dequant_bit_exact_reference_fixtures(ttype):
    # gguf.zig:1528-1570 (expectBitEqual on the ggml fixtures)
    raw, want = _load("dequant", TYPES[ttype])
    got = orc.dequant(ttype, raw).view(np.uint32)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("ttype", sorted(TYPES))
def test_dequant_bit_exact_wide_vectors(ttype):
    raw, want = _load("dequant_wide", TYPES[ttype])
    got = orc.dequant(ttype, raw).view(np.uint32)
    if ttype == 2:
        # The reference's q4_0 (gguf.zig:763-776) writes x*d with no "+ m";
        # its Python port adds m = 0.0, which turns -0.0 into +0.0 when d < 0.
        # Both are the same number; compare with the sign of zero folded.
        zero = (want & 0x7FFFFFFF) == 0
        assert np.array_equal(got[zero] & 0x7FFFFFFF, want[zero] & 0x7FFFFFFF)
        got, want = got[~zero], want[~zero]
    assert np.array_equal(got, want)


def _h(v):
    return struct.pack("<e", v)


def test_hand_computed_legacy_blocks():
    # gguf.zig:1424-1488
    q40 = b"\x00\x38" + bytes([0x21]) + bytes(15)
    o = orc.dequant(2, q40)
    assert (o[0], o[16], o[1], o[17], o[31]) == (-3.5, -3.0, -4.0, -4.0, -4.0)
    q41 = b"\x00\x38\x00\x34" + bytes([0x21]) + bytes(15)
    o = orc.dequant(3, q41)
    assert (o[0], o[16], o[1]) == (0.75, 1.25, 0.25)
    q50 = bytes([0x00, 0x34, 0x01, 0x00, 0x01, 0x00, 0x21]) + bytes(15)
    o = orc.dequant(6, q50)
    assert (o[0], o[16], o[1], o[17]) == (0.25, 0.5, -4.0, -4.0)
    q51 = bytes([0x00, 0x38, 0x00, 0x3C, 0x01, 0x00, 0x01, 0x00, 0x21]) + bytes(15)
    o = orc.dequant(7, q51)
    assert (o[0], o[16], o[1]) == (9.5, 10.0, 1.0)
    q80 = bytes([0x00, 0x34, 0x80, 0x7F, 0xFF]) + bytes(29)
    o = orc.dequant(8, q80)
    assert (o[0], o[1], o[2], o[3]) == (-32.0, 31.75, -0.25, 0.0)
    q81 = bytes([0x00, 0x34, 0x00, 0x00, 0x80, 0x7F, 0xFF]) + bytes(29)
    o = orc.dequant(9, q81)
    assert (o[0], o[1], o[2]) == (-32.0, 31.75, -0.25)
    assert list(orc.dequant(1, bytes([0x00, 0x3C, 0x00, 0xC0, 0x00, 0x38]))) == [1.0, -2.0, 0.5]
    bf = orc.dequant(30, bytes([0x80, 0x3F, 0x00, 0xC0, 0x00, 0x80]))
    assert list(bf) == [1.0, -2.0, 0.0] and np.signbit(bf[2])
    f = orc.dequant(0, bytes([0, 0, 0x80, 0x3F, 0, 0, 0, 0xC0, 0, 0, 0x20, 0x40]))
    assert list(f) == [1.0, -2.0, 2.5]


def test_hand_computed_q4_k_block():
    # gguf.zig:1490-1526
    blk = bytearray(144)
    blk[0:2] = b"\x00\x3C"
    blk[2:4] = b"\x00\x38"
    blk[4], blk[5], blk[6], blk[7], blk[8] = 2, 3, 4, 5, 1
    blk[12], blk[13], blk[14], blk[15] = 6, 7, 8, 9
    blk[16] = 0x21
    blk[16 + 32] = 0x0F
    o = orc.dequant(12, bytes(blk))
    assert (o[0], o[1], o[31], o[32], o[33], o[64], o[96], o[128], o[255]) == \
        (1.5, -0.5, -0.5, 6.0, 0.0, 60.0, 0.0, 0.0, 0.0)


def test_dequant_range_block_aligned_chunks():
    # gguf.zig:1771-1792
    raw, want = _load("dequant", "q6_k")
    parts = [orc.dequant(14, raw, n=256, elem_offset=off) for off in range(0, want.size, 256)]
    assert np.array_equal(np.concatenate(parts).view(np.uint32), want)
    with pytest.raises(ValueError):
        orc.dequant(14, raw, n=256, elem_offset=64)  # InvalidTensorShape


def test_dequant_rejects_truncated_and_unsupported():
    with pytest.raises(ValueError):
        orc.dequant(8, bytes(33), n=32)   # one byte short of a q8_0 block
    with pytest.raises(ValueError):
        orc.dequant(16, bytes(64), n=32)  # iq2_xxs: UnsupportedType


def test_f16_rounding_is_round_to_nearest_even():
    # gguf.zig:682-692 relies on @floatCast's RNE conversion; compare to numpy's.
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0,
        rng.standard_normal(2000).astype(np.float32) * 1e-6,     # subnormal fp16 range
        np.array([65504, 65519.99, 65520, 1e6, -1e6, 0.0, -0.0, 2 ** -25, 2 ** -24, 3 * 2 ** -26],
                 dtype=np.float32),
    ])
    assert np.array_equal(orc.f32_to_f16_bits(x), x.astype(np.float16).view(np.uint16))


def test_rmsnorm_unit_rms():
    # cpu.zig:729-737
    out = orc.rmsnorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 0.0)
    assert abs(float(np.sum(out * out)) - 4.0) < 1e-4


def test_rope_preserves_norm():
    # cpu.zig:739-760
    v = np.array([1, 0, 0, 1, 0, 1, 1, 0], np.float32)
    r = orc.rope(v, 2, 4, 7, 100000.0, adjacent=True)
    assert abs(float(np.sum(v * v)) - float(np.sum(r * r))) < 1e-4
    v = np.array([1, 0, 0, 0, 0, 1, 0, 0], np.float32)
    r = orc.rope(v, 2, 4, 3, 10000.0, adjacent=False)
    assert abs(float(np.sum(v * v)) - float(np.sum(r * r))) < 1e-4


def test_exp_approx_accuracy():
    # cpu.zig:762-780
    for x in np.arange(0, -87, -0.37, dtype=np.float64):
        x = float(np.float32(x))
        assert abs(orc.exp_approx(x) - np.exp(np.float32(x))) <= 2e-5 * np.exp(np.float32(x))
    assert abs(orc.exp_approx(0.0) - 1.0) < 1e-6
    for x in (-88.0, -100.0, -200.0):
        assert orc.exp_approx(x) == 0.0


def test_softmax_sums_to_one():
    # cpu.zig:782-796
    s = orc.softmax(np.array([1, 2, 3, 4], np.float32))
    assert abs(float(s.sum()) - 1.0) < 1e-5
    long = (np.sin(np.arange(1000, dtype=np.float32)) * 20.0).astype(np.float32)
    assert abs(float(orc.softmax(long).sum()) - 1.0) < 1e-4


def test_silu_mul_values():
    # cpu.zig:798-803
    out = orc.silu_mul(np.array([0.0, 1.0], np.float32), np.array([1.0, 1.0], np.float32))
    assert abs(out[0]) < 1e-6 and abs(out[1] - 0.7310586) < 1e-5


def _attention_brute(q, k16, v16, n_past, heads, kv_heads, hd):
    """The definition, as in cpu.zig:842-881 (attentionDecodeReference)."""
    k = k16.view(np.float16).astype(np.float32).reshape(-1, kv_heads, hd)
    v = v16.view(np.float16).astype(np.float32).reshape(-1, kv_heads, hd)
    out = np.zeros(heads * hd, np.float64)
    g = heads // kv_heads
    for h in range(heads):
        s = k[:n_past, h // g, :].astype(np.float64) @ q[h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * hd:(h + 1) * hd] = p @ v[:n_past, h // g, :]
    return out


@pytest.mark.parametrize("hd", [64, 128, 8])
def test_attention_decode_matches_brute_force(hd):
    # cpu.zig:883-919
    rng = np.random.default_rng(hd * 7 + 1)
    heads, kv_heads, n_past = 4, 2, 5
    q = (rng.random(heads * hd, dtype=np.float32) * 2 - 1).astype(np.float32)
    k = (rng.random(n_past * kv_heads * hd) * 2 - 1).astype(np.float16).view(np.uint16)
    v = (rng.random(n_past * kv_heads * hd) * 2 - 1).astype(np.float16).view(np.uint16)
    got = orc.attention_decode(q, k, v, n_past, heads, kv_heads, hd)
    want = _attention_brute(q, k, v, n_past, heads, kv_heads, hd)
    assert np.max(np.abs(got - want)) < 1e-3


def test_attention_single_position_returns_v():
    # cpu.zig:1011-1019
    q = np.array([1, 0, 1, 0], np.float32)
    k = np.array([1, 0, 1, 0], np.float16).view(np.uint16)
    v = np.array([0.5, 0.25, 0.125, 0.0625], np.float16).view(np.uint16)
    out = orc.attention_decode(q, k, v, 1, 2, 2, 2)
    assert abs(out[0] - 0.5) < 1e-5 and abs(out[2] - 0.125) < 1e-5


def test_argmax_first_maximum():
    # cpu.zig:477-483 (strict >) and the greedy sampler test cpu.zig:1053-1058
    assert orc.argmax(np.array([0.1, 5.0, 0.2], np.float32)) == 1
    assert orc.argmax(np.array([3.0, 1.0, 3.0, 3.0], np.float32)) == 0


def test_matvec_order_is_thread_independent():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((300, 257)).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(257).astype(np.float32)
    a = orc.matvec_f16(w, x, threads=1)
    b = orc.matvec_f16(w, x, threads=7)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # sequential fp32 accumulation, main.zig:320-326
    wf = w.view(np.float16).astype(np.float32)
    acc = np.zeros(300, np.float32)
    for i in range(257):
        acc = (acc + (wf[:, i] * x[i]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(a.view(np.uint32), acc.view(np.uint32))


def test_attention_prefill_is_per_query_decode():
    """cpu.attentionPrefill (cpu.zig:165-217) runs, for each query, the same dot /
    softmax / fp16 axpy as attentionDecode (cpu.zig:323-395) over the positions
    up to its own: the restatement must agree with the decode one bit for bit,
    threaded or not."""
    rng = np.random.default_rng(5)
    heads, kv_heads, hd, n_past, n_q, pos0 = 6, 2, 64, 70, 20, 50
    q = rng.standard_normal((n_q, heads * hd)).astype(np.float32)
    k = (rng.standard_normal((n_past, kv_heads * hd)) * 0.5).astype(np.float16).view(np.uint16)
    v = rng.standard_normal((n_past, kv_heads * hd)).astype(np.float16).view(np.uint16)
    got1 = orc.attention_prefill(q, k, v, n_past, pos0, heads, kv_heads, hd, threads=1)
    got4 = orc.attention_prefill(q, k, v, n_past, pos0, heads, kv_heads, hd, threads=4)
    assert np.array_equal(got1.view(np.uint32), got4.view(np.uint32))
    for i in range(n_q):
        want = orc.attention_decode(q[i], k, v, min(n_past, pos0 + i + 1), heads, kv_heads, hd)
        assert np.array_equal(got1[i].view(np.uint32), want.view(np.uint32)), i
