"""ctypes binding of libcuq.so, the C ABI in include/cuq.h.

This is the same binding a Zig maintainer writes as `extern fn`
declarations; Python uses it for the tests and the benchmark.  Loading fails
loudly when the library is missing: there is no CPU fallback.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcuq.so")

OK, EINVAL, ENOMEM, ECUDA, ECONTEXT, EUNSUPPORTED, ETIMEOUT, EFORMAT, ENOTREADY = 0, -1, -2, -3, -4, -5, -6, -7, -8
TP_HANDLE_BYTES = 64

ROLE = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "attn_norm": 7, "ffn_norm": 8,
        "q_bias": 9, "k_bias": 10, "v_bias": 11, "o_bias": 12, "embed": 13, "output": 14, "final_norm": 15}

P, U32, U64, I32, SZ, F32 = (ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_size_t,
                             ctypes.c_float)

# (name, restype, argtypes) for every symbol include/cuq.h declares
SIGNATURES = [
    ("cuq_init", I32, [I32]),
    ("cuq_ready", I32, []),
    ("cuq_last_error", ctypes.c_char_p, []),
    ("cuq_version", ctypes.c_char_p, []),
    ("cuq_block_elems", I32, [I32]),
    ("cuq_block_bytes", I32, [I32]),
    ("cuq_dequant", I32, [I32, P, SZ, U64, P, SZ, P]),
    ("cuq_weight_create", P, [I32, P, SZ, U32, U32]),
    ("cuq_weight_export_raw", I32, [P, P, SZ]),
    ("cuq_weight_nbytes", SZ, [P]),
    ("cuq_weight_free", None, [P]),
    ("cuq_gemv", I32, [P, P, P, P]),
    ("cuq_xq_halves", SZ, [U32]),
    ("cuq_prepare_x", I32, [P, U32, P, P]),
    ("cuq_gemv_prepared", I32, [P, P, P, P]),
    ("cuq_gemm", I32, [P, P, U32, P, P]),
    ("cuq_weight_dequant_f16", I32, [P, P, P]),
    ("cuq_rmsnorm", I32, [P, P, P, U32, U32, F32, P]),
    ("cuq_rope", I32, [P, U32, U32, U32, F32, I32, P]),
    ("cuq_silu_mul", I32, [P, P, P, U32, P]),
    ("cuq_attention_decode", I32, [P, P, P, P, U32, U32, U32, U32, U32, P]),
    ("cuq_attention_decode_noalloc", I32, [P, P, P, P, U32, U32, U32, U32, U32, P]),
    ("cuq_attention_prefill", I32, [P, P, P, P, U32, U32, U32, U32, U32, U32, P]),
    ("cuq_argmax", I32, [P, U32, P, P]),
    ("cuq_sample", I32, [P, U32, P, P, U32, P, P, P]),
    ("cuq_model_create", P, [P, P]),
    ("cuq_upload_tensor", I32, [P, I32, I32, I32, P, SZ, U32, U32]),
    ("cuq_upload_f32", I32, [P, I32, I32, P, SZ]),
    ("cuq_model_finalize", I32, [P]),
    ("cuq_model_load_gguf", P, [ctypes.c_char_p, P]),
    ("cuq_model_get_config", I32, [P, P]),
    ("cuq_gguf_open", P, [ctypes.c_char_p]),
    ("cuq_gguf_open_bytes", P, [P, SZ]),
    ("cuq_gguf_close", None, [P]),
    ("cuq_gguf_version", U32, [P]),
    ("cuq_gguf_tensor_count", U64, [P]),
    ("cuq_gguf_kv_type", I32, [P, ctypes.c_char_p]),
    ("cuq_gguf_get_u64", I32, [P, ctypes.c_char_p, ctypes.POINTER(U64)]),
    ("cuq_gguf_get_i64", I32, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]),
    ("cuq_gguf_get_f64", I32, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    ("cuq_gguf_get_string", ctypes.c_char_p, [P, ctypes.c_char_p]),
    ("cuq_gguf_array_info", I32, [P, ctypes.c_char_p, ctypes.POINTER(U64), ctypes.POINTER(I32)]),
    ("cuq_gguf_array_u64", I32, [P, ctypes.c_char_p, U64, ctypes.POINTER(U64)]),
    ("cuq_gguf_array_string", ctypes.c_char_p, [P, ctypes.c_char_p, U64]),
    ("cuq_gguf_tensor_info", I32, [P, ctypes.c_char_p, ctypes.POINTER(I32), ctypes.POINTER(U32),
                                   ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    ("cuq_gguf_tensor_bytes", I32, [P, ctypes.c_char_p, ctypes.POINTER(P), ctypes.POINTER(SZ)]),
    ("cuq_safetensors_open", P, [ctypes.c_char_p]),
    ("cuq_safetensors_open_bytes", P, [P, SZ]),
    ("cuq_safetensors_close", None, [P]),
    ("cuq_safetensors_count", U64, [P]),
    ("cuq_safetensors_name", ctypes.c_char_p, [P, U64]),
    ("cuq_safetensors_tensor", I32, [P, ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(U32),
                                     ctypes.POINTER(U64), ctypes.POINTER(P), ctypes.POINTER(SZ)]),
    ("cuq_hf_read_config", I32, [ctypes.c_char_p, P]),
    ("cuq_model_load_hf", P, [ctypes.c_char_p, P]),
    ("cuq_tp_comm_handle", I32, [P, P]),
    ("cuq_tp_connect", I32, [P, P]),
    ("cuq_shard_rows", I32, [I32, U32, U32, U32, U32, P, P]),
    ("cuq_shard_cols", I32, [I32, U32, U32, U32, U32, P, P]),
    ("cuq_forward", I32, [P, U32, U32, P, P]),
    ("cuq_prefill", I32, [P, P, U32, U32, P, P]),
    ("cuq_generate", I32, [P, P, U32, U32, P]),
    ("cuq_generate_sampled", I32, [P, P, U32, U32, U32, P, U32, U32, P]),
    ("cuq_decode_greedy", I32, [P, U32, U32, U32, P]),
    ("cuq_kv_write", I32, [P, U32, U32, U32, P, P]),
    ("cuq_kv_read", I32, [P, U32, U32, U32, P, P]),
    ("cuq_reset", I32, [P]),
    ("cuq_model_stats", I32, [P, P]),
    ("cuq_profile_decode", I32, [P, U32, U32, U32, P]),
    ("cuq_model_stream", P, [P]),
    ("cuq_model_free", None, [P]),
]


class CuqConfig(ctypes.Structure):
    _fields_ = [("hidden", U32), ("layers", U32), ("heads", U32), ("kv_heads", U32), ("head_dim", U32),
                ("inter", U32), ("vocab", U32), ("eps", F32), ("rope_theta", F32),
                ("rope_adjacent", ctypes.c_int32), ("tie_embeddings", ctypes.c_int32)]


class CuqOptions(ctypes.Structure):
    _fields_ = [("max_seq", U32), ("max_chunk", U32), ("use_graphs", ctypes.c_int32),
                ("tp_rank", ctypes.c_int32), ("tp_size", ctypes.c_int32),
                ("decode_kernel", ctypes.c_int32), ("persistent_ctas", ctypes.c_int32), ("wait_limit_ms", U32)]


DECODE_AUTO, DECODE_PER_OP, DECODE_PERSISTENT = 0, 1, 2

SAMPLE_MAX_VOCAB, SAMPLE_MAX_WINDOW = 327680, 8192


class CuqSamplerParams(ctypes.Structure):
    """cuq_sampler_params = cpu.SamplerParams (cpu.zig:502-518); defaults are the reference's."""
    _fields_ = [("temperature", F32), ("top_k", U32), ("top_p", F32), ("repetition_penalty", F32),
                ("presence_penalty", F32), ("frequency_penalty", F32), ("min_keep_delta", F32)]

    def __init__(self, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, presence_penalty=0.0,
                 frequency_penalty=0.0, min_keep_delta=20.0):
        super().__init__(temperature, top_k, top_p, repetition_penalty, presence_penalty, frequency_penalty,
                         min_keep_delta)


class CuqStats(ctypes.Structure):
    _fields_ = [("tokens", U64), ("prefill_tokens", U64), ("decode_ms", ctypes.c_double),
                ("prefill_ms", ctypes.c_double), ("weight_bytes", U64), ("kv_bytes", U64),
                ("graph_replays", U64), ("kernels_per_step", U64),
                ("kernel_launches", U64), ("persistent_ctas", U64)]


NODE_NAMES = ["embed", "qkv", "attention", "o", "gate_up", "down", "lm_head", "norm"]


class CuqNodeTime(ctypes.Structure):
    _fields_ = [("launches", U64), ("ms", ctypes.c_double), ("bytes", ctypes.c_double)]


class CuqError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__("cuq error %d: %s" % (code, msg))
        self.code = code


_lib = None


def load(path=LIB_PATH):
    """Load libcuq.so (built by anedvd_b200.build); raises if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise FileNotFoundError("%s is missing: run `python -m anedvd_b200.build` (no CPU fallback exists)"
                                    % path)
        L = ctypes.CDLL(path)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error():
    return load().cuq_last_error().decode(errors="replace")


def check(rc):
    if rc != OK:
        raise CuqError(rc, last_error())
    return rc


def init(device=0):
    return check(load().cuq_init(device))


class GgufFile:
    """The library's GGUF parser (cuq_gguf_*), as gguf.zig's Gguf: metadata
    getters with the reference's conversions, the tensor table and raw bytes.
    Host only; raises CuqError with the parser's error name."""

    def __init__(self, path=None, data=None):
        L = load()
        if data is not None:
            self._buf = ctypes.create_string_buffer(bytes(data), len(data))
            self._h = L.cuq_gguf_open_bytes(self._buf, len(data))
        else:
            self._h = L.cuq_gguf_open(path.encode())
        if not self._h:
            raise CuqError(EFORMAT, last_error())

    def close(self):
        if getattr(self, "_h", None):
            load().cuq_gguf_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def version(self):
        return load().cuq_gguf_version(self._h)

    @property
    def tensor_count(self):
        return load().cuq_gguf_tensor_count(self._h)

    def kv_type(self, key):
        return load().cuq_gguf_kv_type(self._h, key.encode())

    def _get(self, fn, ctype, key):
        v = ctype()
        return v.value if fn(self._h, key.encode(), ctypes.byref(v)) == OK else None

    def u64(self, key):
        return self._get(load().cuq_gguf_get_u64, U64, key)

    def i64(self, key):
        return self._get(load().cuq_gguf_get_i64, ctypes.c_int64, key)

    def f64(self, key):
        return self._get(load().cuq_gguf_get_f64, ctypes.c_double, key)

    def string(self, key):
        s = load().cuq_gguf_get_string(self._h, key.encode())
        return None if s is None else s.decode()

    def array(self, key):
        L = load()
        n, et = U64(), I32()
        if L.cuq_gguf_array_info(self._h, key.encode(), ctypes.byref(n), ctypes.byref(et)) != OK:
            return None
        out = []
        for i in range(n.value):
            if et.value == 8:
                out.append(L.cuq_gguf_array_string(self._h, key.encode(), i).decode())
            else:
                v = U64()
                check(L.cuq_gguf_array_u64(self._h, key.encode(), i, ctypes.byref(v)))
                out.append(v.value)
        return out

    def tensor_info(self, name):
        t, nd, dims, off = I32(), U32(), (U64 * 8)(), U64()
        check(load().cuq_gguf_tensor_info(self._h, name.encode(), ctypes.byref(t), ctypes.byref(nd), dims,
                                          ctypes.byref(off)))
        return t.value, list(dims[:nd.value]), off.value

    def tensor_bytes(self, name):
        p, n = P(), SZ()
        check(load().cuq_gguf_tensor_bytes(self._h, name.encode(), ctypes.byref(p), ctypes.byref(n)))
        return ctypes.string_at(p, n.value)


class SafetensorsFile:
    """The library's safetensors reader (cuq_safetensors_*), host only."""

    def __init__(self, path=None, data=None):
        L = load()
        if data is not None:
            self._buf = ctypes.create_string_buffer(bytes(data), len(data))
            self._h = L.cuq_safetensors_open_bytes(self._buf, len(data))
        else:
            self._h = L.cuq_safetensors_open(path.encode())
        if not self._h:
            raise CuqError(EFORMAT, last_error())

    def close(self):
        if getattr(self, "_h", None):
            load().cuq_safetensors_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def names(self):
        L = load()
        return [L.cuq_safetensors_name(self._h, i).decode() for i in range(L.cuq_safetensors_count(self._h))]

    def tensor(self, name):
        """(dtype, shape, bytes)"""
        dt = ctypes.create_string_buffer(8)
        rank, shape, p, n = U32(), (U64 * 8)(), P(), SZ()
        check(load().cuq_safetensors_tensor(self._h, name.encode(), dt, ctypes.byref(rank), shape, ctypes.byref(p),
                                            ctypes.byref(n)))
        return dt.value.decode(), list(shape[:rank.value]), ctypes.string_at(p, n.value)


def hf_config(path):
    """config.json of a HuggingFace model directory as a CuqConfig (cuq_hf_read_config)."""
    c = CuqConfig()
    check(load().cuq_hf_read_config(path.encode(), ctypes.byref(c)))
    return c
