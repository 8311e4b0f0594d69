"""HuggingFace model directories without a GPU: the library's safetensors
reader against the rules and error names of safetensors.zig:104-233, and its
config.json reader against hf.zig's defaults."""
import json
import os
import struct

import numpy as np
import pytest

from anedvd_b200 import runtime as rt

from .hf_util import safetensors_bytes


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(rt.LIB_PATH):
        from anedvd_b200 import build
        build.build()
    return rt.load()


def test_reads_tensors_in_header_order(L):
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    b = np.array([1.0, -2.5], np.float16)
    data = safetensors_bytes([("a", "F32", [2, 3], a.tobytes()), ("b", "F16", [2], b.tobytes()),
                              ("s", "BF16", [], b"\x80\x3f")], metadata={"format": "pt"})
    f = rt.SafetensorsFile(data=data)
    assert f.names() == ["a", "b", "s"]  # __metadata__ is not a tensor
    dt, shape, raw = f.tensor("a")
    assert (dt, shape) == ("F32", [2, 3]) and np.array_equal(np.frombuffer(raw, np.float32).reshape(2, 3), a)
    assert f.tensor("b")[0] == "F16" and f.tensor("s") == ("BF16", [], b"\x80\x3f")  # a scalar: one element
    with pytest.raises(rt.CuqError, match="TensorNotFound"):
        f.tensor("nope")


def _rejects(data, name):
    with pytest.raises(rt.CuqError) as ei:
        rt.SafetensorsFile(data=data)
    assert name in str(ei.value), str(ei.value)


def _raw_header(h, payload=b""):
    h = h.encode() if isinstance(h, str) else h
    return struct.pack("<Q", len(h)) + h + payload


def test_rejects_malformed_files(L):
    _rejects(b"\x01\x02", "HeaderTooSmall")
    _rejects(struct.pack("<Q", 1000) + b"{}", "InvalidHeaderLength")
    _rejects(_raw_header("{not json"), "InvalidHeader")
    _rejects(_raw_header("[1, 2]"), "InvalidHeader")
    _rejects(_raw_header('{"t": 5}'), "InvalidTensorEntry")
    _rejects(_raw_header('{"t": {"shape": [1], "data_offsets": [0, 4]}}', bytes(4)), "InvalidTensorEntry")
    _rejects(_raw_header('{"t": {"dtype": "F8_E4M3", "shape": [1], "data_offsets": [0, 1]}}', bytes(1)),
             "UnsupportedDtype")
    _rejects(_raw_header('{"t": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}', bytes(4)),
             "InvalidTensorEntry")
    _rejects(_raw_header('{"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}', bytes(4)),
             "DataSizeMismatch")  # 2 x 4 bytes declared, 4 present
    _rejects(_raw_header('{"t": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}', bytes(4)),
             "DataSizeMismatch")  # reversed
    _rejects(_raw_header('{"t": {"dtype": "F32", "shape": [1], "data_offsets": [0, 8]}}', bytes(4)),
             "DataSizeMismatch")  # past the payload


def test_config_json_defaults(L, tmp_path):
    d = str(tmp_path)
    json.dump({"hidden_size": 512, "num_hidden_layers": 3, "num_attention_heads": 8, "intermediate_size": 1024,
               "vocab_size": 4096, "rope_parameters": {"rope_theta": 500000.0}}, open(os.path.join(d, "config.json"), "w"))
    c = rt.hf_config(d)
    assert (c.hidden, c.layers, c.heads, c.inter, c.vocab) == (512, 3, 8, 1024, 4096)
    assert c.kv_heads == 8 and c.head_dim == 64      # num_key_value_heads = heads, head_dim = hidden / heads
    assert abs(c.eps - 1e-6) < 1e-12                  # rms_norm_eps default
    assert c.rope_theta == 500000.0                   # rope_parameters.rope_theta
    assert c.rope_adjacent == 0 and c.tie_embeddings == 0
    json.dump({"hidden_size": 512}, open(os.path.join(d, "config.json"), "w"))
    with pytest.raises(rt.CuqError, match="MissingField"):
        rt.hf_config(d)
