"""The tensor-core (tcgen05) prefill GEMM through cuq_gemm, against the CPU oracle.

Y[t] = W x[t] for every token t must match the reference's matmulF16 on the
fp16-rounded weights (main.zig:320-326) within the per-kernel 1e-3 bar.  The
weight slice is dequantised to exactly those fp16 values on the device and the
activation is carried as fp16 hi + lo, so the error left is fp32 accumulation.
"""
import numpy as np
import pytest

from anedvd_b200 import quant, synth
from oracle import oracle as orc

from .gpu_util import Weight, rel_err

pytestmark = pytest.mark.gpu
KERNEL_TOL = 1e-3
TYPES = [8, 12, 14, 2, 3, 6, 7, 1, 30]


def _case(ttype, rows, cols, n, seed):
    w = synth.seeded_normal("qg/%d/%d/%d/%d" % (ttype, rows, cols, seed), rows * cols)
    raw = quant.quantize(ttype, w).tobytes()
    X = np.stack([synth.seeded_normal("qg/x/%d/%d/%d" % (cols, i, seed), cols, std=1.0) for i in range(n)])
    W = Weight(ttype, raw, rows, cols)
    Y = W.gemm(X)
    w16 = orc.read_f16(ttype, raw, rows * cols).reshape(rows, cols)
    worst = 0.0
    for i in range(n):
        worst = max(worst, rel_err(Y[i], orc.matvec_f16(w16, X[i], threads=8)))
    return worst


def test_gemm_q8_0_single_tile():
    assert _case(8, 128, 64, 1, 0) < KERNEL_TOL


@pytest.mark.parametrize("ttype", TYPES)
def test_gemm_types(ttype):
    assert _case(ttype, 256, 512, 37, 1) < KERNEL_TOL


@pytest.mark.parametrize("rows,cols,n", [(960, 576, 16), (192, 896, 203), (576, 1536, 130), (2048, 1536, 300)])
def test_gemm_shapes_partial_tiles(rows, cols, n):
    assert _case(8, rows, cols, n, 2) < KERNEL_TOL
    assert _case(12, rows, 1536 if cols % 256 else cols, min(n, 40), 3) < KERNEL_TOL
