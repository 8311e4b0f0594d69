"""Test helpers: safetensors files and HuggingFace model directories written
from synthetic models (the library reads them; nothing here is on the product
path)."""
import json
import os
import struct

import numpy as np

from anedvd_b200 import quant

DTYPE_BYTES = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "I16": 2, "I8": 1, "U8": 1, "BOOL": 1}


def safetensors_bytes(tensors, metadata=None):
    """tensors: list of (name, dtype string, shape, raw bytes) -> file bytes."""
    header, off = {}, 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dt, shape, data in tensors:
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        off += len(data)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    return struct.pack("<Q", len(h)) + h + b"".join(t[3] for t in tensors)


# GGUF role of a synth tensor -> HF name (load_hf.zig:143-230 naming)
def hf_name(role, layer):
    p = "model.layers.%d." % layer
    return {"embed": "model.embed_tokens.weight", "final_norm": "model.norm.weight", "output": "lm_head.weight",
            "attn_norm": p + "input_layernorm.weight", "ffn_norm": p + "post_attention_layernorm.weight",
            "q": p + "self_attn.q_proj.weight", "k": p + "self_attn.k_proj.weight",
            "v": p + "self_attn.v_proj.weight", "o": p + "self_attn.o_proj.weight",
            "q_bias": p + "self_attn.q_proj.bias", "k_bias": p + "self_attn.k_proj.bias",
            "v_bias": p + "self_attn.v_proj.bias", "gate": p + "mlp.gate_proj.weight",
            "up": p + "mlp.up_proj.weight", "down": p + "mlp.down_proj.weight"}[role]


def to_hf_types(model, linear_type=1):
    """Give every linear tensor of a synth model F16 (1) or BF16 (30) data drawn
    from the model's seeded normal weights; norms and biases stay F32."""
    from anedvd_b200 import synth
    for t in model.tensors():
        if t.ggml_type != 0:
            w = synth.seeded_normal(model.cfg.name + "/hf/" + t.name, t.rows * t.cols)
            t.ggml_type = linear_type
            t.data = quant.quantize(linear_type, w).tobytes()
    return model


def write_hf_dir(model, path, shards=2):
    """config.json + model-0000k-of-0000n.safetensors + model.safetensors.index.json."""
    os.makedirs(path, exist_ok=True)
    c = model.cfg
    cfg = {"architectures": ["Qwen2ForCausalLM" if c.arch == "qwen2" else "LlamaForCausalLM"],
           "hidden_size": c.hidden, "num_hidden_layers": c.layers, "num_attention_heads": c.heads,
           "num_key_value_heads": c.kv_heads, "head_dim": c.head_dim, "intermediate_size": c.inter,
           "vocab_size": c.vocab, "rms_norm_eps": c.eps, "rope_theta": c.rope_theta,
           "tie_word_embeddings": bool(c.tie_embeddings)}
    json.dump(cfg, open(os.path.join(path, "config.json"), "w"))
    names = {0: "F32", 1: "F16", 30: "BF16"}
    items = []
    for t in model.tensors():
        shape = [t.cols] if t.rows == 1 else [t.rows, t.cols]
        items.append((hf_name(t.role, t.layer), names[t.ggml_type], shape, bytes(t.data)))
    per = (len(items) + shards - 1) // shards
    weight_map = {}
    for k in range(shards):
        fn = "model-%05d-of-%05d.safetensors" % (k + 1, shards)
        part = items[k * per:(k + 1) * per]
        open(os.path.join(path, fn), "wb").write(safetensors_bytes(part, {"format": "pt"}))
        for it in part:
            weight_map[it[0]] = fn
    json.dump({"metadata": {}, "weight_map": weight_map}, open(os.path.join(path, "model.safetensors.index.json"), "w"))
    return path
