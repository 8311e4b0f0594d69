"""ctypes binding of the C oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker -- never by the anedvd_b200
product path.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

ROLE = {
    "q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6,
    "attn_norm": 7, "ffn_norm": 8, "q_bias": 9, "k_bias": 10, "v_bias": 11,
    "o_bias": 12, "embed": 13, "output": 14, "final_norm": 15,
}


def build(force=False):
    """Compile liboracle.so with the committed Makefile (gcc, no GPU needed)."""
    src = os.path.join(HERE, "oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class OrcConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_uint32), ("layers", ctypes.c_uint32), ("heads", ctypes.c_uint32),
        ("kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32), ("inter", ctypes.c_uint32),
        ("vocab", ctypes.c_uint32), ("max_seq", ctypes.c_uint32), ("eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float), ("rope_adjacent", ctypes.c_int),
        ("tie_embeddings", ctypes.c_int), ("threads", ctypes.c_int),
    ]


class SamplerParams(ctypes.Structure):
    """cpu.SamplerParams (cpu.zig:502-518); the defaults are the reference's."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_uint32), ("top_p", ctypes.c_float),
                ("repetition_penalty", ctypes.c_float), ("presence_penalty", ctypes.c_float),
                ("frequency_penalty", ctypes.c_float), ("min_keep_delta", ctypes.c_float)]

    def __init__(self, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, presence_penalty=0.0,
                 frequency_penalty=0.0, min_keep_delta=20.0):
        super().__init__(temperature, top_k, top_p, repetition_penalty, presence_penalty, frequency_penalty,
                         min_keep_delta)


class SamplerInfo(ctypes.Structure):
    _fields_ = [("candidates", ctypes.c_uint32), ("kept", ctypes.c_uint32), ("sorted_for_top_p", ctypes.c_int32),
                ("path", ctypes.c_int32), ("max_logit", ctypes.c_float), ("sum", ctypes.c_float),
                ("target", ctypes.c_float), ("draw_margin", ctypes.c_float), ("top_p_margin", ctypes.c_float),
                ("topk_gap", ctypes.c_float)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        L.orc_block_elems.argtypes = [ctypes.c_int]
        L.orc_block_bytes.argtypes = [ctypes.c_int]
        L.orc_dequant_range.argtypes = [ctypes.c_int, P, ctypes.c_size_t, ctypes.c_uint64, P, ctypes.c_size_t]
        L.orc_read_f16.argtypes = [ctypes.c_int, P, ctypes.c_size_t, P, ctypes.c_size_t]
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f32_to_f16_n.argtypes = [P, P, ctypes.c_size_t]
        L.orc_matvec_f16.argtypes = [P, P, P, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int]
        L.orc_rmsnorm.argtypes = [P, P, P, ctypes.c_size_t, ctypes.c_float]
        L.orc_rope.argtypes = [P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_float]
        L.orc_rope_adjacent.argtypes = L.orc_rope.argtypes
        L.orc_silu_mul.argtypes = [P, P, P, ctypes.c_size_t]
        L.orc_exp_approx.argtypes = [ctypes.c_float]
        L.orc_exp_approx.restype = ctypes.c_float
        L.orc_softmax.argtypes = [P, ctypes.c_size_t]
        L.orc_attention_decode.argtypes = [P, P, P, P, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32,
                                           ctypes.c_uint32]
        L.orc_argmax.argtypes = [P, ctypes.c_size_t]
        L.orc_argmax.restype = ctypes.c_uint32
        L.orc_apply_penalties.argtypes = [P, ctypes.c_size_t, ctypes.POINTER(SamplerParams), P, ctypes.c_size_t]
        L.orc_sample.argtypes = [P, ctypes.c_size_t, ctypes.POINTER(SamplerParams), P, ctypes.c_size_t,
                                 ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(SamplerInfo)]
        L.orc_sample.restype = ctypes.c_uint32
        L.orc_model_create.argtypes = [ctypes.POINTER(OrcConfig)]
        L.orc_model_create.restype = P
        L.orc_model_free.argtypes = [P]
        L.orc_model_set_linear.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, ctypes.c_size_t,
                                           ctypes.c_uint32, ctypes.c_uint32]
        L.orc_model_set_f32.argtypes = [P, ctypes.c_int, ctypes.c_int, P, ctypes.c_size_t]
        L.orc_model_forward.argtypes = [P, ctypes.c_uint32, ctypes.c_uint32, P]
        L.orc_model_last_hidden.argtypes = [P]
        L.orc_model_last_hidden.restype = ctypes.POINTER(ctypes.c_float)
        L.orc_model_kv_row.argtypes = [P, ctypes.c_uint32, ctypes.c_uint32, P, P]
        L.orc_model_set_kv.argtypes = [P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, P, P]
        L.orc_attention_prefill.argtypes = [P, P, ctypes.c_size_t, ctypes.c_size_t, P, P, ctypes.c_size_t,
                                            ctypes.c_size_t, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32,
                                            ctypes.c_uint32, ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def block_elems(t):
    return lib().orc_block_elems(t)


def block_bytes(t):
    return lib().orc_block_bytes(t)


def dequant(ttype, raw, n=None, elem_offset=0):
    """dequantizeRange: raw GGUF blocks -> float32 (bit-exact reference values)."""
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw,
                               dtype=np.uint8)
    if n is None:
        n = raw.size // block_bytes(ttype) * block_elems(ttype) - elem_offset
    out = np.empty(n, dtype=np.float32)
    rc = lib().orc_dequant_range(ttype, _ptr(raw), raw.size, elem_offset, _ptr(out), n)
    if rc:
        raise ValueError("orc_dequant_range failed: %d" % rc)
    return out


def read_f16(ttype, raw, n):
    """Gguf.readF16: dequantise and round each weight to fp16 (returns uint16 bits)."""
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw,
                               dtype=np.uint8)
    out = np.empty(n, dtype=np.uint16)
    rc = lib().orc_read_f16(ttype, _ptr(raw), raw.size, _ptr(out), n)
    if rc:
        raise ValueError("orc_read_f16 failed: %d" % rc)
    return out


def f32_to_f16_bits(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_n(_ptr(x), _ptr(out), x.size)
    return out


def matvec_f16(w16_bits, x, threads=1):
    """main.zig:320-326 scalar-order matvec; w16_bits is uint16 [rows][cols]."""
    w = np.ascontiguousarray(w16_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = w.shape
    out = np.empty(rows, dtype=np.float32)
    lib().orc_matvec_f16(_ptr(out), _ptr(w), _ptr(x), rows, cols, threads)
    return out


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_ptr(out), _ptr(x), _ptr(w), x.size, eps)
    return out


def rope(v, heads, hd, pos, theta, adjacent):
    v = np.array(v, dtype=np.float32, copy=True)
    fn = lib().orc_rope_adjacent if adjacent else lib().orc_rope
    fn(_ptr(v), heads, hd, pos, theta)
    return v


def silu_mul(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    lib().orc_silu_mul(_ptr(out), _ptr(g), _ptr(u), g.size)
    return out


def softmax(s):
    s = np.array(s, dtype=np.float32, copy=True)
    lib().orc_softmax(_ptr(s), s.size)
    return s


def exp_approx(x):
    return lib().orc_exp_approx(x)


def attention_decode(q, k_cache16, v_cache16, n_past, heads, kv_heads, hd):
    """cpu.attentionDecode over fp16 caches laid out [pos][kv_heads*hd] (uint16 bits)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k_cache16, dtype=np.uint16)
    v = np.ascontiguousarray(v_cache16, dtype=np.uint16)
    out = np.empty(heads * hd, dtype=np.float32)
    lib().orc_attention_decode(_ptr(out), _ptr(q), _ptr(k), _ptr(v), n_past, heads, kv_heads, hd)
    return out


def attention_prefill(q, k_cache16, v_cache16, n_past, q_pos0, heads, kv_heads, hd, threads=8):
    """cpu.attentionPrefill on position-major q [n_q][heads*hd] (float32) and fp16
    caches [pos][kv_heads*hd] (uint16 bits); returns [n_q][heads*hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    n_q = q.shape[0]
    k = np.ascontiguousarray(k_cache16, dtype=np.uint16)
    v = np.ascontiguousarray(v_cache16, dtype=np.uint16)
    out = np.empty((n_q, heads * hd), dtype=np.float32)
    lib().orc_attention_prefill(_ptr(out), _ptr(q), 1, heads * hd, _ptr(k), _ptr(v), n_past, n_q, q_pos0, heads,
                                kv_heads, hd, threads)
    return out


def argmax(v):
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().orc_argmax(_ptr(v), v.size))


def apply_penalties(logits, params, recent):
    """cpu.applyPenalties on a copy of `logits`."""
    v = np.array(logits, dtype=np.float32, copy=True)
    r = np.ascontiguousarray(recent, dtype=np.uint32)
    lib().orc_apply_penalties(_ptr(v), v.size, ctypes.byref(params), _ptr(r) if r.size else None, r.size)
    return v


def sample(logits, params, recent, rng):
    """cpu.sampleProfiled on a copy of `logits`: (token, rng after, SamplerInfo,
    the penalised logits)."""
    v = np.array(logits, dtype=np.float32, copy=True)
    r = np.ascontiguousarray(recent, dtype=np.uint32)
    st = ctypes.c_uint32(rng)
    info = SamplerInfo()
    tok = lib().orc_sample(_ptr(v), v.size, ctypes.byref(params), _ptr(r) if r.size else None, r.size,
                           ctypes.byref(st), ctypes.byref(info))
    return int(tok), int(st.value), info, v


class Model:
    """The reference's pure-CPU forward (refForward + the engine's dense MLP)."""

    def __init__(self, cfg, threads=1, max_seq=None):
        c = OrcConfig()
        c.hidden, c.layers, c.heads = cfg.hidden, cfg.layers, cfg.heads
        c.kv_heads, c.head_dim, c.inter, c.vocab = cfg.kv_heads, cfg.head_dim, cfg.inter, cfg.vocab
        c.max_seq = max_seq or cfg.max_seq
        c.eps, c.rope_theta = cfg.eps, cfg.rope_theta
        c.rope_adjacent, c.tie_embeddings, c.threads = int(cfg.rope_adjacent), int(cfg.tie_embeddings), threads
        self.cfg = cfg
        self._h = lib().orc_model_create(ctypes.byref(c))
        if not self._h:
            raise ValueError("orc_model_create rejected the config")

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_model_free(self._h)
            self._h = None

    def set_linear(self, layer, role, ttype, raw, rows, cols):
        raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw,
                                   dtype=np.uint8)
        rc = lib().orc_model_set_linear(self._h, layer, ROLE[role], ttype, _ptr(raw), raw.size, rows, cols)
        if rc:
            raise ValueError("set_linear(%s, layer %d) failed: %d" % (role, layer, rc))

    def set_f32(self, layer, role, v):
        v = np.ascontiguousarray(v, dtype=np.float32)
        rc = lib().orc_model_set_f32(self._h, layer, ROLE[role], _ptr(v), v.size)
        if rc:
            raise ValueError("set_f32(%s, layer %d) failed: %d" % (role, layer, rc))

    def load(self, model):
        """Load every tensor of an anedvd_b200.gguf-style model description."""
        for t in model.tensors():
            if t.role in ("attn_norm", "ffn_norm", "final_norm", "q_bias", "k_bias", "v_bias", "o_bias"):
                self.set_f32(t.layer, t.role, np.frombuffer(t.data, dtype=np.float32))
            else:
                self.set_linear(t.layer, t.role, t.ggml_type, t.data, t.rows, t.cols)

    def forward(self, token, pos, want_logits=True):
        """One refForward step; without want_logits the lm_head is skipped
        (returns None) and only the KV cache and hidden state advance."""
        logits = np.empty(self.cfg.vocab, dtype=np.float32) if want_logits else None
        rc = lib().orc_model_forward(self._h, token, pos, _ptr(logits) if want_logits else None)
        if rc:
            raise ValueError("orc_model_forward failed: %d" % rc)
        return logits

    def last_hidden(self):
        p = lib().orc_model_last_hidden(self._h)
        return np.ctypeslib.as_array(p, shape=(self.cfg.hidden,)).copy()

    def set_kv(self, layer, pos0, k16, v16):
        """Overwrite cache rows [pos0, pos0 + n) with fp16 bits [n][kv_dim]."""
        k = np.ascontiguousarray(k16, dtype=np.uint16)
        v = np.ascontiguousarray(v16, dtype=np.uint16)
        n = k.size // (self.cfg.kv_heads * self.cfg.head_dim)
        rc = lib().orc_model_set_kv(self._h, layer, pos0, n, _ptr(k), _ptr(v))
        if rc:
            raise ValueError("set_kv failed: %d" % rc)

    def kv_row(self, layer, pos):
        kvd = self.cfg.kv_heads * self.cfg.head_dim
        k = np.empty(kvd, dtype=np.uint16)
        v = np.empty(kvd, dtype=np.uint16)
        rc = lib().orc_model_kv_row(self._h, layer, pos, _ptr(k), _ptr(v))
        if rc:
            raise ValueError("kv_row failed")
        return k, v
