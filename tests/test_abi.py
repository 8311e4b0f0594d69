"""The C-ABI library: builds, loads without a GPU, exports every symbol cuq.h declares."""
import ctypes
import os
import re

import pytest

from anedvd_b200 import runtime as rt

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "cuq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cuq_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    if not os.path.exists(rt.LIB_PATH):
        from anedvd_b200 import build
        build.build()
    lib = ctypes.CDLL(rt.LIB_PATH)
    missing = [f for f in header_functions() if not hasattr(lib, f)]
    assert not missing, missing


def test_binding_covers_the_header():
    bound = {name for name, _, _ in rt.SIGNATURES}
    assert set(header_functions()) == bound


def test_block_geometry_without_gpu():
    L = rt.load()
    assert (L.cuq_block_elems(8), L.cuq_block_bytes(8)) == (32, 34)
    assert (L.cuq_block_elems(12), L.cuq_block_bytes(12)) == (256, 144)
    assert (L.cuq_block_elems(14), L.cuq_block_bytes(14)) == (256, 210)
    assert L.cuq_block_elems(16) == 0  # iq2_xxs: UnsupportedType


def test_init_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = rt.load()
    rc = L.cuq_init(0)
    assert rc != rt.OK
    assert "device" in rt.last_error()


def test_missing_library_is_an_error(tmp_path):
    rt_mod = rt
    saved = rt_mod._lib
    rt_mod._lib = None
    try:
        with pytest.raises(FileNotFoundError):
            rt_mod.load(str(tmp_path / "libcuq.so"))
    finally:
        rt_mod._lib = saved
