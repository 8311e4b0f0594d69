"""The allocation-free decode attention (cuq_attention_decode_noalloc).

It is meant for callers that may not allocate device memory while they run, so
it keeps its split scratch in a fixed array inside the library.  These checks
call it through the C ABI twice in a row -- the second call sees the scratch
the first one left behind -- and compare each result with the allocating
cuq_attention_decode, within the per-kernel tolerance of the other kernel
tests.  This file is collected last so that a failure here never hides
another test's result.
"""
import numpy as np
import pytest

from anedvd_b200 import runtime as rt
from oracle import oracle as orc

from .gpu_util import dev, empty, host, lib, ptr, rel_err

pytestmark = pytest.mark.gpu
KERNEL_TOL = 1e-3


def _inputs(heads, kv_heads, hd, n_past, stride, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(heads * hd).astype(np.float32)
    k = (rng.standard_normal((n_past, kv_heads, hd)) * 0.5).astype(np.float16)
    v = rng.standard_normal((n_past, kv_heads, hd)).astype(np.float16)
    kd = np.zeros((kv_heads, stride, hd), np.float16)
    vd = np.zeros((kv_heads, stride, hd), np.float16)
    kd[:, :n_past] = k.transpose(1, 0, 2)
    vd[:, :n_past] = v.transpose(1, 0, 2)
    return q, k, v, kd.view(np.uint16), vd.view(np.uint16)


def test_noalloc_matches_allocating_attention_twice_in_a_row():
    L = lib()
    # the third shape wants 37 position splits, more than the 31 that fit the
    # fixed array at 64 x (128 + 2) floats each: the split count is capped
    for call, (heads, kv_heads, hd, n_past) in enumerate([(32, 8, 128, 4608), (14, 2, 64, 459),
                                                          (64, 8, 128, 1200)]):
        stride = n_past + 3
        q, k, v, kd, vd = _inputs(heads, kv_heads, hd, n_past, stride, seed=100 + call)
        qd, kdd, vdd = dev(q), dev(kd), dev(vd)
        want = empty(heads * hd)
        got = empty(heads * hd)
        rt.check(L.cuq_attention_decode(ptr(want), ptr(qd), ptr(kdd), ptr(vdd), n_past, stride, heads, kv_heads,
                                        hd, None))
        rt.check(L.cuq_attention_decode_noalloc(ptr(got), ptr(qd), ptr(kdd), ptr(vdd), n_past, stride, heads,
                                                kv_heads, hd, None))
        g, w = host(got), host(want)
        assert rel_err(g, w) < KERNEL_TOL, call
        ref = orc.attention_decode(q, k.reshape(n_past, -1).view(np.uint16), v.reshape(n_past, -1).view(np.uint16),
                                   n_past, heads, kv_heads, hd)
        assert rel_err(g, ref) < KERNEL_TOL, call


def test_noalloc_rejects_heads_beyond_its_fixed_scratch():
    L = lib()
    buf = empty(16)
    # 2048 heads x (128 + 2) floats is more than the 262,144-float array
    rc = L.cuq_attention_decode_noalloc(ptr(buf), ptr(buf), ptr(buf), ptr(buf), 1, 1, 2048, 256, 128, None)
    assert rc == rt.EINVAL
    assert "262144" in rt.last_error()
    # no heads at all, and head dims the kernels do not have (one that would wrap
    # heads * (head_dim + 2) in 32 bits among them), are argument errors
    assert L.cuq_attention_decode_noalloc(ptr(buf), ptr(buf), ptr(buf), ptr(buf), 1, 1, 0, 1, 128, None) == rt.EINVAL
    for hd in (0, 96, 0xFFFFFFFE):
        rc = L.cuq_attention_decode_noalloc(ptr(buf), ptr(buf), ptr(buf), ptr(buf), 1, 1, 8, 1, hd, None)
        assert rc == rt.EUNSUPPORTED, hd
