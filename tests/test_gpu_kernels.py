"""Per-kernel parity on the GPU: each CUDA entry point against the CPU oracle.

Bars: dequantised weights bit-exact in fp32; per-kernel
outputs within 1e-3 relative error, rel = max|a-b| / max|b| as in the
reference's compareLogits (main.zig:1920-1930).
"""
import ctypes
import os

import numpy as np
import pytest

from anedvd_b200 import quant, synth
from anedvd_b200 import runtime as rt
from oracle import oracle as orc

from .gpu_util import Weight, dev, empty, host, lib, ptr, rel_err

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TYPES = {0: "f32", 1: "f16", 2: "q4_0", 3: "q4_1", 6: "q5_0", 7: "q5_1", 8: "q8_0", 9: "q8_1",
         10: "q2_k", 11: "q3_k", 12: "q4_k", 13: "q5_k", 14: "q6_k", 15: "q8_k", 30: "bf16"}
GEMV_TYPES = [8, 2, 3, 6, 7, 12, 14, 1, 30]
KERNEL_TOL = 1e-3


@pytest.mark.parametrize("sub", ["dequant", "dequant_wide"])
@pytest.mark.parametrize("ttype", sorted(TYPES))
def test_dequant_bit_exact(ttype, sub):
    raw = open(os.path.join(GOLD, sub, TYPES[ttype] + ".bin"), "rb").read()
    want = np.frombuffer(open(os.path.join(GOLD, sub, TYPES[ttype] + ".f32"), "rb").read(), dtype=np.uint32)
    rd = dev(np.frombuffer(raw, dtype=np.uint8))
    out = empty(want.size)
    rt.check(lib().cuq_dequant(ttype, ptr(rd), len(raw), 0, ptr(out), want.size, None))
    got = host(out).view(np.uint32)
    cpu = orc.dequant(ttype, raw).view(np.uint32)
    assert np.array_equal(got, cpu)  # same function as the pinned oracle, bit for bit
    if ttype != 2:                   # q4_0 wide vectors: sign of zero, see test_oracle_golden
        assert np.array_equal(got, want)


def test_dequant_range_offsets_and_errors():
    raw = open(os.path.join(GOLD, "dequant_wide", "q6_k.bin"), "rb").read()
    want = orc.dequant(14, raw)
    rd = dev(np.frombuffer(raw, dtype=np.uint8))
    out = empty(256)
    rt.check(lib().cuq_dequant(14, ptr(rd), len(raw), 512, ptr(out), 256, None))
    assert np.array_equal(host(out).view(np.uint32), want[512:768].view(np.uint32))
    assert lib().cuq_dequant(14, ptr(rd), len(raw), 64, ptr(out), 256, None) == rt.EINVAL
    assert lib().cuq_dequant(16, ptr(rd), len(raw), 0, ptr(out), 256, None) == rt.EUNSUPPORTED
    assert lib().cuq_dequant(14, ptr(rd), 209, 0, ptr(out), 256, None) == rt.EINVAL  # TruncatedFile


def _weights(ttype, rows, cols, seed):
    if ttype in RAW_TYPES and ttype != 0:
        return golden_blocks(ttype, rows * cols, seed)
    w = synth.seeded_normal("test/%d/%d/%d/%d" % (ttype, rows, cols, seed), rows * cols)
    return quant.quantize(ttype, w).tobytes()


# types kept as raw GGUF blocks on the device (no quantiser here: their test
# tensors are drawn from the reference-pinned golden blocks)
RAW_TYPES = [0, 9, 10, 11, 13, 15]


# the block's scale fields (byte offset, fp16 or fp32) and the power of two
# that brings the golden blocks' weights (std 11-550) to a model's scale (~0.02)
SCALE_FIELDS = {9: ([(0, 2)], 12), 10: ([(80, 2), (82, 2)], 9), 11: ([(108, 2)], 11),
                13: ([(0, 2), (2, 2)], 14), 15: ([(0, 4)], 11)}


def golden_blocks(ttype, n, seed, model_scale=False):
    """A payload of n weights whose blocks are drawn (seeded) from the 64 golden
    blocks of the type -- valid blocks the reference's own vectors pin.  With
    model_scale the blocks' d (and dmin) are divided by a power of two so the
    weights have a transformer's magnitude (the golden blocks exercise extreme
    scales, which would overflow a model's fp16 activations)."""
    be, bb = orc.block_elems(ttype), orc.block_bytes(ttype)
    blocks = np.frombuffer(open(os.path.join(GOLD, "dequant_wide", TYPES[ttype] + ".bin"), "rb").read(),
                           dtype=np.uint8).reshape(-1, bb)
    idx = np.random.default_rng(seed).integers(0, blocks.shape[0], size=n // be)
    out = blocks[idx].copy()
    if model_scale and ttype in SCALE_FIELDS:
        fields, shift = SCALE_FIELDS[ttype]
        f = np.float32(2.0 ** -shift)
        for off, size in fields:
            dt = np.float16 if size == 2 else np.float32
            v = (out[:, off:off + size].copy().view(dt).astype(np.float32) * f).astype(dt)
            out[:, off:off + size] = v.view(np.uint8).reshape(-1, size)
    return out.tobytes()


@pytest.mark.parametrize("ttype", GEMV_TYPES)
def test_planes_round_trip_and_f16_dequant(ttype):
    rows, cols = 48, 512
    raw = _weights(ttype, rows, cols, 0)
    W = Weight(ttype, raw, rows, cols)
    assert W.export_raw().tobytes() == raw                       # lossless regrouping
    want16 = orc.read_f16(ttype, raw, rows * cols).reshape(rows, cols)
    assert np.array_equal(W.dequant_f16(), want16)               # Gguf.readF16, bit for bit


def _ref_gemv(ttype, raw, rows, cols, x):
    w16 = orc.read_f16(ttype, raw, rows * cols).reshape(rows, cols)
    return orc.matvec_f16(w16, x, threads=4)


@pytest.mark.parametrize("ttype", GEMV_TYPES)
@pytest.mark.parametrize("shape", [(16, 256), (64, 768), (576, 1536), (4096, 4096), (128, 14336)])
def test_gemv_matches_reference(ttype, shape):
    rows, cols = shape
    raw = _weights(ttype, rows, cols, 1)
    x = synth.seeded_normal("test/x/%d" % cols, cols, std=1.0)
    W = Weight(ttype, raw, rows, cols)
    got = W.gemv(x)
    want = _ref_gemv(ttype, raw, rows, cols, x)
    assert rel_err(got, want) < KERNEL_TOL


@pytest.mark.parametrize("ttype", [8, 2, 3, 6, 7, 1, 30])
def test_gemv_partial_last_iteration(ttype):
    # cols not a multiple of the per-iteration span (64 or 128 columns)
    rows, cols = 32, 96 if ttype not in (1, 30) else 80
    raw = _weights(ttype, rows, cols, 2)
    x = synth.seeded_normal("test/x/odd", cols, std=1.0)
    got = Weight(ttype, raw, rows, cols).gemv(x)
    assert rel_err(got, _ref_gemv(ttype, raw, rows, cols, x)) < KERNEL_TOL


def test_gemv_c1_op_set():
    """The Q8_0 op set of one SmolLM2-135M layer: its eight matrices + the lm_head."""
    for name, rows, cols, raw, x in synth.c1_matrices():
        got = Weight(8, raw, rows, cols).gemv(x)
        e = rel_err(got, _ref_gemv(8, raw, rows, cols, x))
        assert e < KERNEL_TOL, (name, e)


def test_gemm_matches_gemv():
    rows, cols, n = 256, 1024, 5
    raw = _weights(12, rows, cols, 3)
    X = np.stack([synth.seeded_normal("test/X/%d" % i, cols, std=1.0) for i in range(n)])
    W = Weight(12, raw, rows, cols)
    Y = W.gemm(X)
    for i in range(n):
        assert rel_err(Y[i], _ref_gemv(12, raw, rows, cols, X[i])) < KERNEL_TOL


def test_weight_rejects_unknown_types():
    raw = np.zeros(16 * 34, np.uint8)
    L = lib()
    for t in (4, 5, 16, 31):  # ids gguf.zig:30-46 does not define
        assert not L.cuq_weight_create(t, raw.ctypes.data_as(ctypes.c_void_p), raw.size, 16, 32)


@pytest.mark.parametrize("ttype", RAW_TYPES)
@pytest.mark.parametrize("shape", [(16, 256), (48, 1024), (256, 4096)])
def test_gemv_raw_block_types(ttype, shape):
    """The remaining block types (Q8_1, Q2_K, Q3_K, Q5_K, Q8_K, F32;
    gguf.zig:842-949, 998-1034, 1061-1071, 751-761) through the GEMV: every
    weight is the reference's readF16 value."""
    rows, cols = shape
    raw = _weights(ttype, rows, cols, 7)
    x = synth.seeded_normal("test/x/raw/%d" % cols, cols, std=1.0)
    W = Weight(ttype, raw, rows, cols)
    assert W.export_raw().tobytes() == raw
    assert np.array_equal(W.dequant_f16(), orc.read_f16(ttype, raw, rows * cols).reshape(rows, cols))
    assert rel_err(W.gemv(x), _ref_gemv(ttype, raw, rows, cols, x)) < KERNEL_TOL


@pytest.mark.parametrize("ttype", RAW_TYPES)
def test_gemm_raw_block_types(ttype):
    """Their prefill GEMM: the weight expanded to fp16 (readF16 values) in a
    scratch buffer, then the tcgen05 fp16 GEMM."""
    rows, cols, n = 128, 1024, 37
    raw = _weights(ttype, rows, cols, 8)
    X = np.stack([synth.seeded_normal("test/X/raw/%d" % i, cols, std=1.0) for i in range(n)])
    Y = Weight(ttype, raw, rows, cols).gemm(X)
    for i in (0, 17, n - 1):
        assert rel_err(Y[i], _ref_gemv(ttype, raw, rows, cols, X[i])) < KERNEL_TOL


def test_rmsnorm():
    n, rows = 896, 3
    x = np.stack([synth.seeded_normal("t/rms/%d" % i, n, std=3.0) for i in range(rows)])
    w = synth.seeded_normal("t/rmsw", n, std=1.0)
    out = empty(n * rows)
    xd, wd = dev(x), dev(w)  # keep the device buffers alive across the launch
    rt.check(lib().cuq_rmsnorm(ptr(out), ptr(xd), ptr(wd), n, rows, 1e-6, None))
    got = host(out).reshape(rows, n)
    for i in range(rows):
        assert rel_err(got[i], orc.rmsnorm(x[i], w, 1e-6)) < 1e-5


@pytest.mark.parametrize("adjacent", [0, 1])
@pytest.mark.parametrize("hd,pos,theta", [(64, 0, 1e4), (64, 143, 1e4), (128, 2047, 1e6), (128, 4607, 5e5)])
def test_rope(adjacent, hd, pos, theta):
    heads = 5
    v = synth.seeded_normal("t/rope", heads * hd, std=1.0)
    d = dev(v)
    rt.check(lib().cuq_rope(ptr(d), heads, hd, pos, theta, adjacent, None))
    want = orc.rope(v, heads, hd, pos, theta, adjacent=bool(adjacent))
    assert rel_err(host(d), want) < 1e-5


def test_silu_mul():
    n = 4864
    g = synth.seeded_normal("t/g", n, std=2.0)
    u = synth.seeded_normal("t/u", n, std=2.0)
    out = empty(n)
    gd, ud = dev(g), dev(u)
    rt.check(lib().cuq_silu_mul(ptr(out), ptr(gd), ptr(ud), n, None))
    assert rel_err(host(out), orc.silu_mul(g, u)) < 1e-5


@pytest.mark.parametrize("heads,kv_heads,hd,n_past", [(9, 3, 64, 1), (9, 3, 64, 144), (14, 2, 64, 459),
                                                      (12, 2, 128, 2304), (32, 8, 128, 4608), (4, 4, 128, 37)])
def test_attention_decode(heads, kv_heads, hd, n_past):
    stride = n_past + 7
    rng = np.random.default_rng(heads * 1000 + n_past)
    q = rng.standard_normal(heads * hd).astype(np.float32)
    # reference cache layout [pos][kv_heads*hd]; the device wants [kv_head][pos][hd]
    k = (rng.standard_normal((n_past, kv_heads, hd)) * 0.5).astype(np.float16)
    v = rng.standard_normal((n_past, kv_heads, hd)).astype(np.float16)
    kd = np.zeros((kv_heads, stride, hd), np.float16)
    vd = np.zeros((kv_heads, stride, hd), np.float16)
    kd[:, :n_past] = k.transpose(1, 0, 2)
    vd[:, :n_past] = v.transpose(1, 0, 2)
    out = empty(heads * hd)
    qd_, kd_, vd_ = dev(q), dev(kd.view(np.uint16)), dev(vd.view(np.uint16))
    rt.check(lib().cuq_attention_decode(ptr(out), ptr(qd_), ptr(kd_), ptr(vd_), n_past, stride, heads, kv_heads,
                                        hd, None))
    want = orc.attention_decode(q, k.reshape(n_past, -1).view(np.uint16), v.reshape(n_past, -1).view(np.uint16),
                                n_past, heads, kv_heads, hd)
    assert rel_err(host(out), want) < KERNEL_TOL


def test_argmax_first_index():
    v = synth.seeded_normal("t/am", 151936, std=1.0)
    v[7000] = v[90000] = 50.0  # tie: the first index wins (cpu.zig:477-483)
    out = empty(1, np.uint32)
    vd = dev(v)
    rt.check(lib().cuq_argmax(ptr(vd), v.size, ptr(out), None))
    assert int(host(out, np.uint32)[0]) == orc.argmax(v) == 7000
