"""Helpers for the GPU parity tests: device buffers through torch, the C ABI
through ctypes, and the reference's comparison metric."""
import ctypes

import numpy as np

from anedvd_b200 import runtime as rt


def rel_err(got, want):
    """compareLogits / reportKernel (main.zig:1920-1930, engine.zig:1494-1514): max|a-b| / max|b|."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def dev(a):
    """numpy -> CUDA torch tensor (same bytes)."""
    import torch
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.uint8).copy()).cuda().view(_torch_dtype(a.dtype)).reshape(a.shape)


def _torch_dtype(dt):
    import torch
    return {np.dtype(np.float32): torch.float32, np.dtype(np.uint8): torch.uint8,
            np.dtype(np.uint16): torch.int16, np.dtype(np.uint32): torch.int32,
            np.dtype(np.int32): torch.int32}[np.dtype(dt)]


def empty(n, dtype=np.float32):
    import torch
    return torch.empty(n, dtype=_torch_dtype(dtype), device="cuda")


def host(t, dtype=np.float32):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy().view(dtype)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def lib():
    L = rt.load()
    rt.init(0)
    return L


class Weight:
    """A cuq_weight handle owning its device planes."""

    def __init__(self, ttype, raw, rows, cols):
        raw = np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8))
        self.h = lib().cuq_weight_create(ttype, raw.ctypes.data_as(ctypes.c_void_p), raw.size, rows, cols)
        if not self.h:
            raise rt.CuqError(rt.EINVAL, rt.last_error())
        self.rows, self.cols, self.nbytes = rows, cols, raw.size

    def gemv(self, x):
        xd = dev(np.asarray(x, dtype=np.float32))
        y = empty(self.rows)
        rt.check(lib().cuq_gemv(self.h, ptr(xd), ptr(y), None))
        return host(y)

    def gemm(self, X):
        X = np.ascontiguousarray(X, dtype=np.float32)
        xd = dev(X)
        y = empty(X.shape[0] * self.rows)
        rt.check(lib().cuq_gemm(self.h, ptr(xd), X.shape[0], ptr(y), None))
        return host(y).reshape(X.shape[0], self.rows)

    def export_raw(self):
        out = np.empty(self.nbytes, dtype=np.uint8)
        rt.check(lib().cuq_weight_export_raw(self.h, out.ctypes.data_as(ctypes.c_void_p), out.size))
        return out

    def dequant_f16(self):
        out = empty(self.rows * self.cols, np.uint16)
        rt.check(lib().cuq_weight_dequant_f16(self.h, ptr(out), None))
        return host(out, np.uint16).reshape(self.rows, self.cols)

    def __del__(self):
        if getattr(self, "h", None):
            rt.load().cuq_weight_free(self.h)
            self.h = None
