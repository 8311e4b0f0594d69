"""ctypes binding of libcuq.so, the C ABI in include/cuq.h.

This is the same binding a Zig maintainer writes as `extern fn` declarations
(INTEGRATION.md); Python uses it for the tests and the benchmark.  Loading
fails loudly when the library is missing: there is no CPU fallback.
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
    ("cuq_model_create", P, [P, P]),
    ("cuq_upload_tensor", I32, [P, I32, I32, I32, P, SZ, U32, U32]),
    ("cuq_upload_f32", I32, [P, I32, I32, P, SZ]),
    ("cuq_model_finalize", I32, [P]),
    ("cuq_model_load_gguf", P, [ctypes.c_char_p, P]),
    ("cuq_model_get_config", I32, [P, P]),
    ("cuq_tp_comm_handle", I32, [P, P]),
    ("cuq_tp_connect", I32, [P, P]),
    ("cuq_shard_rows", I32, [I32, U32, U32, U32, U32, P, P]),
    ("cuq_shard_cols", I32, [I32, U32, U32, U32, U32, P, P]),
    ("cuq_forward", I32, [P, U32, U32, P, P]),
    ("cuq_prefill", I32, [P, P, U32, U32, P, P]),
    ("cuq_generate", I32, [P, P, U32, U32, P]),
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
                ("decode_kernel", ctypes.c_int32), ("persistent_ctas", ctypes.c_int32)]


DECODE_AUTO, DECODE_PER_OP, DECODE_PERSISTENT = 0, 1, 2


class CuqStats(ctypes.Structure):
    _fields_ = [("tokens", U64), ("prefill_tokens", U64), ("decode_ms", ctypes.c_double),
                ("prefill_ms", ctypes.c_double), ("weight_bytes", U64), ("kv_bytes", U64),
                ("graph_replays", U64), ("kernels_per_step", U64),
                ("kernel_launches", U64), ("persistent_ctas", U64)]


NODE_NAMES = ["embed", "qkv", "attention", "o", "gate_up", "down", "lm_head"]


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
