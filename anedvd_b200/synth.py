"""Seeded synthetic models with the architectures of the benchmark configs.

The reference runs trained checkpoints; none exist here (no network), so every
config is a random-init model of the same architecture.  Weights are float32
N(0, 0.02) from ``numpy.random.default_rng(seed)``, seed = crc32 of
"<config>/<tensor name>", quantised by ``quant.py``; norm weights are 1.0 and
qwen2 q/k/v biases are N(0, 0.02) float32.  Throughput does not depend on
weight values, so tok/s is comparable to a trained model of the same shape.

Tensor names and dims follow GGUF's llama/qwen2 conventions, which is what the
reference's loader reads (``src/load_gguf.zig:423-567``): linear tensors have
``dims = [in, out]`` (ggml order) and a row-major ``[out][in]`` payload.
"""

import dataclasses
import os
import zlib

import numpy as np

from . import gguf, quant

Q8_0, Q4_K, Q6_K, F32 = 8, 12, 14, 0


@dataclasses.dataclass
class Config:
    name: str
    arch: str            # "llama" (adjacent-pair RoPE) or "qwen2" (half-split RoPE)
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    eps: float
    rope_theta: float
    tie_embeddings: bool
    qkv_bias: bool
    quant_mix: str       # "q8_0" or "q4_k_m"
    prompt: int
    decode: int
    max_seq: int = 0

    def __post_init__(self):
        if not self.max_seq:
            self.max_seq = self.prompt + self.decode

    @property
    def rope_adjacent(self):
        # load_gguf.zig:81-90: qwen2 is a NeoX (half-split) architecture, llama is not.
        return self.arch != "qwen2"

    @property
    def q_dim(self):
        return self.heads * self.head_dim

    @property
    def kv_dim(self):
        return self.kv_heads * self.head_dim


CONFIGS = {
    # c2: SmolLM2-135M architecture, Q8_0
    "smollm2-135m": Config("smollm2-135m", "llama", 30, 576, 9, 3, 64, 1536, 49152, 1e-5, 10000.0,
                           True, False, "q8_0", 16, 128),
    # c3: Qwen2.5-0.5B architecture, Q8_0
    "qwen2.5-0.5b": Config("qwen2.5-0.5b", "qwen2", 24, 896, 14, 2, 64, 4864, 151936, 1e-6, 1e6,
                           True, True, "q8_0", 203, 256),
    # c4: Qwen2.5-1.5B architecture, Q4_K_M mix
    "qwen2.5-1.5b": Config("qwen2.5-1.5b", "qwen2", 28, 1536, 12, 2, 128, 8960, 151936, 1e-6, 1e6,
                           True, True, "q4_k_m", 2048, 256),
    # c5: Llama-3-8B architecture, Q4_K_M mix, untied
    "llama3-8b": Config("llama3-8b", "llama", 32, 4096, 32, 8, 128, 14336, 128256, 1e-5, 5e5,
                        False, False, "q4_k_m", 4096, 512),
}

# c1: the Q8_0 op set of one SmolLM2-135M layer, (name, out, in)
C1_MATRICES = [("q", 576, 576), ("k", 192, 576), ("v", 192, 576), ("o", 576, 576),
               ("gate", 1536, 576), ("up", 1536, 576), ("down", 576, 1536), ("lm_head", 49152, 576)]


def shrink(cfg, layers=None, vocab=None, name_suffix="-small", **kw):
    """Same architecture with fewer layers / a smaller vocabulary (for fast parity tests)."""
    c = dataclasses.replace(cfg, name=cfg.name + name_suffix, **kw)
    if layers is not None:
        c.layers = layers
    if vocab is not None:
        c.vocab = vocab
    return c


def seeded_normal(key, n, std=0.02):
    rng = np.random.default_rng(zlib.crc32(key.encode()))
    return (rng.standard_normal(n, dtype=np.float32) * np.float32(std)).astype(np.float32)


def tensor_type(cfg, role, layer):
    """The Q4_K_M mix of the Qwen2.5-1.5B and Llama-3-8B benchmark models: Q6_K for attn_v, ffn_down of even
    layers and the output matrix (token_embd when tied); Q4_K elsewhere."""
    if role in ("attn_norm", "ffn_norm", "final_norm", "q_bias", "k_bias", "v_bias"):
        return F32
    if cfg.quant_mix == "q8_0":
        return Q8_0
    if role == "v" or (role == "down" and layer % 2 == 0) or role == "output":
        return Q6_K
    if role == "embed":
        return Q6_K if cfg.tie_embeddings else Q4_K
    return Q4_K


@dataclasses.dataclass
class SynthTensor:
    name: str        # GGUF tensor name
    role: str        # q k v o gate up down attn_norm ffn_norm q_bias k_bias v_bias embed output final_norm
    layer: int       # -1 for model-level tensors
    ggml_type: int
    rows: int        # out features (1 for vectors)
    cols: int        # in features / length
    data: bytes      # raw GGUF payload

    @property
    def dims(self):
        return [self.cols] if self.rows == 1 else [self.cols, self.rows]


TILE_SAMPLE = 1 << 16  # weights quantised per tensor in "tiled" payloads


def tiled_blocks(ttype, key, n):
    """Raw payload of n weights built from real quantised blocks: TILE_SAMPLE
    N(0, 0.02) weights are quantised, then each block of the tensor is one of
    those blocks picked by a seeded generator.  Every block is a valid block of
    the type with the scale/min statistics quantisation of N(0, 0.02) gives;
    generating an 8B model this way takes seconds instead of quantising 8e9
    weights in numpy.  Throughput does not depend on the values."""
    be, bb = gguf.LAYOUT[ttype]
    m = min(n, TILE_SAMPLE)
    sample = quant.quantize(ttype, seeded_normal(key + "/sample", m)).reshape(-1, bb)
    if m == n:
        return sample.tobytes()
    rng = np.random.default_rng(zlib.crc32((key + "/tile").encode()))
    idx = rng.integers(0, sample.shape[0], size=n // be)
    return sample[idx].tobytes()


class SynthModel:
    """A synthetic model: config + raw GGUF tensors, generated lazily and cached.

    payload "quantized": every weight drawn and quantised (the parity models);
    "tiled": blocks drawn from a quantised sample (``tiled_blocks``), for the
    multi-GB benchmark models."""

    def __init__(self, cfg, payload="quantized", cache=True):
        assert payload in ("quantized", "tiled")
        self.cfg = cfg
        self.payload = payload
        self.cache = cache
        self._cache = {}

    def _make(self, name, role, layer, rows, cols):
        key = (name,)
        if key in self._cache:
            return self._cache[key]
        t = tensor_type(self.cfg, role, layer)
        n = rows * cols
        if role in ("attn_norm", "ffn_norm", "final_norm"):
            data = quant.quantize(t, np.ones(n, dtype=np.float32)).tobytes()
        elif self.payload == "tiled" and t != F32:
            data = tiled_blocks(t, self.cfg.name + "/" + name, n)
        else:
            data = quant.quantize(t, seeded_normal(self.cfg.name + "/" + name, n)).tobytes()
        st = SynthTensor(name, role, layer, t, rows, cols, data)
        if self.cache:
            self._cache[key] = st
        return st

    def tensor_list(self):
        c = self.cfg
        out = [("token_embd.weight", "embed", -1, c.vocab, c.hidden)]
        for l in range(c.layers):
            p = "blk.%d." % l
            out += [(p + "attn_norm.weight", "attn_norm", l, 1, c.hidden),
                    (p + "attn_q.weight", "q", l, c.q_dim, c.hidden),
                    (p + "attn_k.weight", "k", l, c.kv_dim, c.hidden),
                    (p + "attn_v.weight", "v", l, c.kv_dim, c.hidden)]
            if c.qkv_bias:
                out += [(p + "attn_q.bias", "q_bias", l, 1, c.q_dim),
                        (p + "attn_k.bias", "k_bias", l, 1, c.kv_dim),
                        (p + "attn_v.bias", "v_bias", l, 1, c.kv_dim)]
            out += [(p + "attn_output.weight", "o", l, c.hidden, c.q_dim),
                    (p + "ffn_norm.weight", "ffn_norm", l, 1, c.hidden),
                    (p + "ffn_gate.weight", "gate", l, c.inter, c.hidden),
                    (p + "ffn_up.weight", "up", l, c.inter, c.hidden),
                    (p + "ffn_down.weight", "down", l, c.hidden, c.inter)]
        out.append(("output_norm.weight", "final_norm", -1, 1, c.hidden))
        if not c.tie_embeddings:
            out.append(("output.weight", "output", -1, c.vocab, c.hidden))
        return out

    def tensors(self):
        for name, role, layer, rows, cols in self.tensor_list():
            yield self._make(name, role, layer, rows, cols)

    def tensor(self, name):
        for n, role, layer, rows, cols in self.tensor_list():
            if n == name:
                return self._make(n, role, layer, rows, cols)
        raise KeyError(name)

    def weight_bytes_per_token(self):
        """Algorithmic weight bytes one decode step streams (every projection + lm_head)."""
        total = 0
        for name, role, layer, rows, cols in self.tensor_list():
            if role in ("q", "k", "v", "o", "gate", "up", "down", "output") or \
                    (role == "embed" and self.cfg.tie_embeddings):
                t = tensor_type(self.cfg, role, layer)
                total += gguf.tensor_nbytes(t, rows * cols)
        return total

    def metadata(self):
        c = self.cfg
        a = c.arch
        return [
            ("general.architecture", gguf.STRING, a),
            ("general.name", gguf.STRING, c.name),
            ("general.alignment", gguf.U32, 32),
            (a + ".block_count", gguf.U32, c.layers),
            (a + ".embedding_length", gguf.U32, c.hidden),
            (a + ".feed_forward_length", gguf.U32, c.inter),
            (a + ".attention.head_count", gguf.U32, c.heads),
            (a + ".attention.head_count_kv", gguf.U32, c.kv_heads),
            (a + ".attention.key_length", gguf.U32, c.head_dim),
            (a + ".attention.layer_norm_rms_epsilon", gguf.F32, c.eps),
            (a + ".rope.freq_base", gguf.F32, c.rope_theta),
            (a + ".vocab_size", gguf.U32, c.vocab),
        ]

    def write_gguf(self, path):
        ts = [(t.name, t.dims, t.ggml_type, t.data) for t in self.tensors()]
        return gguf.write(path, self.metadata(), ts)


def model(name_or_cfg, payload="quantized", cache=True, **shrink_kw):
    cfg = CONFIGS[name_or_cfg] if isinstance(name_or_cfg, str) else name_or_cfg
    if shrink_kw:
        cfg = shrink(cfg, **shrink_kw)
    return SynthModel(cfg, payload=payload, cache=cache)


def cached_gguf(m, directory=None):
    """Write the model's GGUF once under `directory` (default: $TMPDIR) and return the path."""
    directory = directory or os.environ.get("TMPDIR", "/tmp")
    path = os.path.join(directory, "anedvd_%s_L%d_V%d.gguf" % (m.cfg.name, m.cfg.layers, m.cfg.vocab))
    if not os.path.exists(path):
        tmp = path + ".part%d" % os.getpid()
        m.write_gguf(tmp)
        os.replace(tmp, path)
    return path


def c1_matrices():
    """The SmolLM2-135M layer op set: the eight Q8_0 matrices and their fp32 N(0,1) inputs."""
    out = []
    for name, rows, cols in C1_MATRICES:
        w = seeded_normal("c1/" + name, rows * cols)
        x = seeded_normal("c1/x/" + name, cols, std=1.0)
        out.append((name, rows, cols, quant.q8_0(w).tobytes(), x))
    return out
