// gguf.cpp -- GGUF v2/v3 parsing (src/gguf.zig:328-656) and the loader
// (src/load_gguf.zig loadConfig :96-302, loadLayer :650-713, loadRuntime
// :578-647), uploading every tensor's raw blocks instead of an fp16 copy.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <cstdint>

#include "../../include/cuq.h"

namespace cuq {
void set_error(const char *fmt, ...);
}

namespace {

struct Value {
    uint32_t type = 0;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    uint64_t arr_len = 0;
    uint32_t arr_type = 0;
    std::vector<Value> arr;  // array elements
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
};

struct Gguf {
    const uint8_t *data = nullptr;
    size_t size = 0, pos = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_off = 0;
    std::map<std::string, Value> kv;
    std::map<std::string, TensorInfo> tensors;
    std::string err;

    bool need(size_t n) {
        if (size - pos < n) {
            err = "TruncatedFile";
            return false;
        }
        return true;
    }
    bool u32(uint32_t &v) {
        if (!need(4)) return false;
        memcpy(&v, data + pos, 4);
        pos += 4;
        return true;
    }
    bool u64(uint64_t &v) {
        if (!need(8)) return false;
        memcpy(&v, data + pos, 8);
        pos += 8;
        return true;
    }
    bool str(std::string &s) {
        uint64_t n;
        if (!u64(n) || !need(n)) return false;
        s.assign((const char *)data + pos, n);
        pos += n;
        return true;
    }
    bool scalar(uint32_t t, Value &v) {
        static const int sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t > 12 || t == 8 || t == 9) {
            err = "InvalidMetadata";
            return false;
        }
        int n = sz[t];
        if (!need(n)) return false;
        uint64_t raw = 0;
        memcpy(&raw, data + pos, n);
        pos += n;
        v.type = t;
        switch (t) {
        case 0: case 2: case 4: case 10: case 7: v.u = raw; v.i = (int64_t)raw; v.f = (double)raw; break;
        case 1: v.i = (int8_t)raw; v.u = (uint64_t)v.i; v.f = (double)v.i; break;
        case 3: v.i = (int16_t)raw; v.u = (uint64_t)v.i; v.f = (double)v.i; break;
        case 5: v.i = (int32_t)raw; v.u = (uint64_t)v.i; v.f = (double)v.i; break;
        case 11: v.i = (int64_t)raw; v.u = raw; v.f = (double)v.i; break;
        case 6: { float f; memcpy(&f, &raw, 4); v.f = f; v.u = (uint64_t)f; break; }
        case 12: { double d; memcpy(&d, &raw, 8); v.f = d; v.u = (uint64_t)d; break; }
        }
        return true;
    }
    bool value(uint32_t t, Value &v) {
        if (t == 8) {
            v.type = 8;
            return str(v.s);
        }
        if (t == 9) {
            v.type = 9;
            if (!u32(v.arr_type) || !u64(v.arr_len)) return false;
            if (v.arr_len > size - pos + 1) {
                err = "TruncatedFile";
                return false;
            }
            v.arr.reserve((size_t)v.arr_len);
            for (uint64_t k = 0; k < v.arr_len; k++) {
                Value e;
                if (!value(v.arr_type, e)) return false;
                v.arr.push_back(std::move(e));
            }
            return true;
        }
        return scalar(t, v);
    }
    bool parse() {
        uint32_t magic;
        if (!u32(magic)) return false;  // empty input: TruncatedFile
        if (magic != 0x46554747u) {
            err = "NotGgufFile";
            return false;
        }
        if (!u32(version)) return false;
        if (version < 2 || version > 3) {
            err = "UnsupportedVersion";
            return false;
        }
        uint64_t nt, nkv;
        if (!u64(nt) || !u64(nkv)) return false;
        if (nt > size - pos + 1) {
            err = "TooManyTensors";
            return false;
        }
        if (nkv > size - pos + 1) {
            err = "TooManyMetadataEntries";
            return false;
        }
        for (uint64_t k = 0; k < nkv; k++) {
            std::string key;
            uint32_t t;
            Value v;
            if (!str(key) || !u32(t) || !value(t, v)) return false;
            kv.emplace(key, v);  // duplicate keys: first wins
        }
        auto al = kv.find("general.alignment");
        if (al != kv.end()) {
            uint64_t a = al->second.u;
            if (a == 0 || a > (1u << 24) || (a & (a - 1))) {
                err = "InvalidMetadata";
                return false;
            }
            alignment = a;
        }
        for (uint64_t k = 0; k < nt; k++) {
            TensorInfo ti;
            uint32_t nd;
            if (!str(ti.name) || !u32(nd)) return false;
            if (nd == 0 || nd > 8) {
                err = "InvalidTensorShape";
                return false;
            }
            ti.dims.resize(nd);
            for (auto &d : ti.dims)
                if (!u64(d)) return false;
            if (!u32(ti.type) || !u64(ti.offset)) return false;
            tensors.emplace(ti.name, ti);
        }
        data_off = (pos + alignment - 1) / alignment * alignment;
        if (data_off > size) {
            err = "TruncatedFile";
            return false;
        }
        return true;
    }
    const Value *get(const std::string &k) const {
        auto it = kv.find(k);
        return it == kv.end() ? nullptr : &it->second;
    }
};

// load_gguf.zig:81-90: architectures whose HF code uses rotate_half (NeoX RoPE).
bool rope_is_adjacent(const std::string &arch) {
    static const char *neox[] = {"qwen2", "qwen2moe", "qwen2vl", "qwen3", "qwen3moe", "phi3", "gptneox",
                                 "stablelm", "gemma", "gemma2", "gemma3", "gemma4", "olmo", "olmo2"};
    for (auto *a : neox)
        if (arch == a) return false;
    return true;
}

}  // namespace

extern "C" cuq_model *cuq_model_load_gguf(const char *path, const cuq_options *opts) {
    using cuq::set_error;
    if (!path) {
        set_error("cuq_model_load_gguf: null path");
        return nullptr;
    }
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        set_error("cuq_model_load_gguf: cannot open %s", path);
        return nullptr;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        set_error("TruncatedFile: %s", path);
        return nullptr;
    }
    size_t size = (size_t)st.st_size;
    void *map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) {
        set_error("cuq_model_load_gguf: mmap failed");
        return nullptr;
    }
    Gguf g;
    g.data = (const uint8_t *)map;
    g.size = size;
    cuq_model *m = nullptr;
    do {
        if (!g.parse()) {
            set_error("%s: %s", g.err.c_str(), path);
            break;
        }
        const Value *av = g.get("general.architecture");
        std::string arch = av && av->type == 8 ? av->s : "llama";
        auto u = [&](const char *suffix, uint64_t dflt, bool required, bool &ok) -> uint64_t {
            const Value *v = g.get(arch + "." + suffix);
            if (!v) {
                if (required) {
                    set_error("gguf: no %s.%s in this file (arch \"%s\")", arch.c_str(), suffix, arch.c_str());
                    ok = false;
                }
                return dflt;
            }
            return v->u;
        };
        auto f = [&](const char *suffix, double dflt) -> double {
            const Value *v = g.get(arch + "." + suffix);
            return v ? v->f : dflt;
        };
        bool ok = true;
        cuq_config c{};
        c.hidden = (uint32_t)u("embedding_length", 0, true, ok);
        c.layers = (uint32_t)u("block_count", 0, true, ok);
        c.heads = (uint32_t)u("attention.head_count", 0, true, ok);
        if (!ok) break;
        c.kv_heads = (uint32_t)u("attention.head_count_kv", c.heads, false, ok);
        c.inter = (uint32_t)u("feed_forward_length", 0, true, ok);
        if (!ok) break;
        c.head_dim = (uint32_t)u("attention.key_length", c.heads ? c.hidden / c.heads : 0, false, ok);
        c.eps = (float)f("attention.layer_norm_rms_epsilon", 1e-5);
        c.rope_theta = (float)f("rope.freq_base", 10000.0);
        const Value *vs = g.get(arch + ".vocab_size");
        if (vs)
            c.vocab = (uint32_t)vs->u;
        else {
            const Value *toks = g.get("tokenizer.ggml.tokens");
            if (!toks) {
                set_error("gguf: no %s.vocab_size and no tokenizer.ggml.tokens to fall back on", arch.c_str());
                break;
            }
            c.vocab = (uint32_t)toks->arr_len;
        }
        c.tie_embeddings = g.tensors.count("output.weight") ? 0 : 1;
        c.rope_adjacent = rope_is_adjacent(arch) ? 1 : 0;
        m = cuq_model_create(&c, opts);
        if (!m) break;
        auto tensor_bytes = [&](const TensorInfo &t, size_t &nb) -> const uint8_t * {
            int epb = cuq_block_elems((int)t.type), bpb = cuq_block_bytes((int)t.type);
            if (!epb) {
                set_error("UnsupportedType: %s has ggml type %u", t.name.c_str(), t.type);
                return nullptr;
            }
            uint64_t n = 1;
            for (auto d : t.dims) n *= d;
            if (n % epb) {
                set_error("InvalidTensorShape: %s", t.name.c_str());
                return nullptr;
            }
            nb = n / epb * bpb;
            uint64_t start = g.data_off + t.offset;
            if (start + nb > g.size) {
                set_error("TensorDataOutOfRange: %s", t.name.c_str());
                return nullptr;
            }
            return g.data + start;
        };
        auto linear = [&](const std::string &name, int layer, int role, uint32_t in, uint32_t out) -> bool {
            auto it = g.tensors.find(name);
            if (it == g.tensors.end()) {
                set_error("MissingTensor: %s", name.c_str());
                return false;
            }
            const TensorInfo &t = it->second;
            if (t.dims.size() < 2 || t.dims[0] != in || t.dims[1] != out) {
                // The reference transposes a [out][in] file defensively (load_gguf.zig:378-384);
                // blocks run along the row, so a quantized transpose is not a byte shuffle.
                set_error("DimensionMismatch: %s is not [%u, %u] in ggml order", name.c_str(), in, out);
                return false;
            }
            size_t nb;
            const uint8_t *p = tensor_bytes(t, nb);
            if (!p) return false;
            return cuq_upload_tensor(m, layer, role, (int)t.type, p, nb, out, in) == CUQ_OK;
        };
        auto vec = [&](const std::string &name, int layer, int role, uint32_t n, bool required) -> bool {
            auto it = g.tensors.find(name);
            if (it == g.tensors.end()) {
                if (required) set_error("MissingTensor: %s", name.c_str());
                return !required;
            }
            const TensorInfo &t = it->second;
            size_t nb;
            const uint8_t *p = tensor_bytes(t, nb);
            if (!p) return false;
            if (t.type != 0 || nb != (size_t)n * 4) {
                set_error("DimensionMismatch: %s must be %u f32 values", name.c_str(), n);
                return false;
            }
            std::vector<float> v(n);
            memcpy(v.data(), p, nb);
            return cuq_upload_f32(m, layer, role, v.data(), n) == CUQ_OK;
        };
        uint32_t qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
        bool good = linear("token_embd.weight", -1, CUQ_ROLE_EMBED, c.hidden, c.vocab) &&
                    vec("output_norm.weight", -1, CUQ_ROLE_FINAL_NORM, c.hidden, true);
        if (good && !c.tie_embeddings) good = linear("output.weight", -1, CUQ_ROLE_OUTPUT, c.hidden, c.vocab);
        for (uint32_t l = 0; good && l < c.layers; l++) {
            std::string p = "blk." + std::to_string(l) + ".";
            good = vec(p + "attn_norm.weight", l, CUQ_ROLE_ATTN_NORM, c.hidden, true) &&
                   vec(p + "ffn_norm.weight", l, CUQ_ROLE_FFN_NORM, c.hidden, true) &&
                   linear(p + "attn_q.weight", l, CUQ_ROLE_Q, c.hidden, qd) &&
                   linear(p + "attn_k.weight", l, CUQ_ROLE_K, c.hidden, kvd) &&
                   linear(p + "attn_v.weight", l, CUQ_ROLE_V, c.hidden, kvd) &&
                   linear(p + "attn_output.weight", l, CUQ_ROLE_O, qd, c.hidden) &&
                   linear(p + "ffn_gate.weight", l, CUQ_ROLE_GATE, c.hidden, c.inter) &&
                   linear(p + "ffn_up.weight", l, CUQ_ROLE_UP, c.hidden, c.inter) &&
                   linear(p + "ffn_down.weight", l, CUQ_ROLE_DOWN, c.inter, c.hidden);
            // qwen2 biases (load_gguf.zig:533-549): all three or none
            if (good && g.tensors.count(p + "attn_q.bias"))
                good = vec(p + "attn_q.bias", l, CUQ_ROLE_Q_BIAS, qd, true) &&
                       vec(p + "attn_k.bias", l, CUQ_ROLE_K_BIAS, kvd, true) &&
                       vec(p + "attn_v.bias", l, CUQ_ROLE_V_BIAS, kvd, true);
            if (good && g.tensors.count(p + "attn_output.bias"))
                good = vec(p + "attn_output.bias", l, CUQ_ROLE_O_BIAS, c.hidden, true);
        }
        // a tensor-parallel model is finalized by the caller after cuq_tp_connect
        const bool tp = opts && opts->tp_size > 1;
        if (!good || (!tp && cuq_model_finalize(m) != CUQ_OK)) {
            cuq_model_free(m);
            m = nullptr;
        }
    } while (0);
    munmap(map, size);
    return m;
}

// ------------------------------------------------------- inspection API ---
// The container as Gguf (gguf.zig:328-656) exposes it: header, metadata with
// the reference's value conversions (gguf.zig:198-291), the tensor table and
// each tensor's byte range (tensorBytes, gguf.zig:448-460).  Host only.

struct cuq_gguf {
    Gguf g;
    std::vector<uint8_t> copy;  // cuq_gguf_open_bytes: the bytes parsed
    void *map = nullptr;        // cuq_gguf_open: the mapping
    size_t map_size = 0;
};

namespace {

// Value as u64 / i64 / f64 / bool (asU64, asI64, asF32, asBool): false when the
// type does not convert (strings, arrays, floats for the integer forms) or a
// negative signed value is asked for as unsigned.
bool value_u64(const Value &v, uint64_t &out) {
    switch (v.type) {
    case 0: case 2: case 4: case 10: case 7: out = v.u; return true;
    case 1: case 3: case 5: case 11:
        if (v.i < 0) return false;
        out = (uint64_t)v.i;
        return true;
    default: return false;
    }
}
bool value_i64(const Value &v, int64_t &out) {
    switch (v.type) {
    case 0: case 2: case 4: case 7: out = (int64_t)v.u; return true;
    case 10:
        if (v.u > (uint64_t)INT64_MAX) return false;
        out = (int64_t)v.u;
        return true;
    case 1: case 3: case 5: case 11: out = v.i; return true;
    default: return false;
    }
}
bool value_f64(const Value &v, double &out) {
    switch (v.type) {
    case 6: case 12: out = v.f; return true;
    case 0: case 2: case 4: case 10: case 7: out = (double)v.u; return true;
    case 1: case 3: case 5: case 11: out = (double)v.i; return true;
    default: return false;
    }
}

const Value *find_kv(const cuq_gguf *h, const char *key) {
    if (!h || !key) return nullptr;
    return h->g.get(key);
}

cuq_gguf *finish_open(cuq_gguf *h) {
    if (!h->g.parse()) {
        cuq::set_error("%s", h->g.err.c_str());
        cuq_gguf_close(h);
        return nullptr;
    }
    return h;
}

}  // namespace

extern "C" {

cuq_gguf *cuq_gguf_open(const char *path) {
    if (!path) {
        cuq::set_error("cuq_gguf_open: null path");
        return nullptr;
    }
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        cuq::set_error("FileNotFound: %s", path);
        return nullptr;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        cuq::set_error("cuq_gguf_open: cannot stat %s", path);
        return nullptr;
    }
    cuq_gguf *h = new cuq_gguf();
    if (st.st_size > 0) {
        void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (map == MAP_FAILED) {
            close(fd);
            delete h;
            cuq::set_error("cuq_gguf_open: mmap failed");
            return nullptr;
        }
        h->map = map;
        h->map_size = (size_t)st.st_size;
        h->g.data = (const uint8_t *)map;
        h->g.size = (size_t)st.st_size;
    }
    close(fd);
    return finish_open(h);
}

cuq_gguf *cuq_gguf_open_bytes(const void *data, size_t n) {
    if (!data && n) {
        cuq::set_error("cuq_gguf_open_bytes: null data");
        return nullptr;
    }
    cuq_gguf *h = new cuq_gguf();
    if (n) h->copy.assign((const uint8_t *)data, (const uint8_t *)data + n);
    h->g.data = h->copy.data();
    h->g.size = n;
    return finish_open(h);
}

void cuq_gguf_close(cuq_gguf *h) {
    if (!h) return;
    if (h->map) munmap(h->map, h->map_size);
    delete h;
}

uint32_t cuq_gguf_version(const cuq_gguf *h) { return h ? h->g.version : 0; }
uint64_t cuq_gguf_tensor_count(const cuq_gguf *h) { return h ? (uint64_t)h->g.tensors.size() : 0; }

int cuq_gguf_kv_type(const cuq_gguf *h, const char *key) {
    const Value *v = find_kv(h, key);
    return v ? (int)v->type : -1;
}

int cuq_gguf_get_u64(const cuq_gguf *h, const char *key, uint64_t *out) {
    const Value *v = find_kv(h, key);
    uint64_t x;
    if (!v || !out || !value_u64(*v, x)) return CUQ_EINVAL;
    *out = x;
    return CUQ_OK;
}

int cuq_gguf_get_i64(const cuq_gguf *h, const char *key, int64_t *out) {
    const Value *v = find_kv(h, key);
    int64_t x;
    if (!v || !out || !value_i64(*v, x)) return CUQ_EINVAL;
    *out = x;
    return CUQ_OK;
}

int cuq_gguf_get_f64(const cuq_gguf *h, const char *key, double *out) {
    const Value *v = find_kv(h, key);
    double x;
    if (!v || !out || !value_f64(*v, x)) return CUQ_EINVAL;
    *out = x;
    return CUQ_OK;
}

const char *cuq_gguf_get_string(const cuq_gguf *h, const char *key) {
    const Value *v = find_kv(h, key);
    return v && v->type == 8 ? v->s.c_str() : nullptr;
}

int cuq_gguf_array_info(const cuq_gguf *h, const char *key, uint64_t *len, int *elem_type) {
    const Value *v = find_kv(h, key);
    if (!v || v->type != 9) return CUQ_EINVAL;
    if (len) *len = v->arr_len;
    if (elem_type) *elem_type = (int)v->arr_type;
    return CUQ_OK;
}

int cuq_gguf_array_u64(const cuq_gguf *h, const char *key, uint64_t i, uint64_t *out) {
    const Value *v = find_kv(h, key);
    uint64_t x;
    if (!v || v->type != 9 || i >= v->arr.size() || !out || !value_u64(v->arr[i], x)) return CUQ_EINVAL;
    *out = x;
    return CUQ_OK;
}

const char *cuq_gguf_array_string(const cuq_gguf *h, const char *key, uint64_t i) {
    const Value *v = find_kv(h, key);
    if (!v || v->type != 9 || i >= v->arr.size() || v->arr[i].type != 8) return nullptr;
    return v->arr[i].s.c_str();
}

int cuq_gguf_tensor_info(const cuq_gguf *h, const char *name, int *ggml_type, uint32_t *n_dims, uint64_t *dims,
                         uint64_t *offset) {
    if (!h || !name) return CUQ_EINVAL;
    auto it = h->g.tensors.find(name);
    if (it == h->g.tensors.end()) {
        cuq::set_error("TensorNotFound: %s", name);
        return CUQ_EINVAL;
    }
    const TensorInfo &t = it->second;
    if (ggml_type) *ggml_type = (int)t.type;
    if (n_dims) *n_dims = (uint32_t)t.dims.size();
    if (dims)
        for (size_t k = 0; k < t.dims.size(); k++) dims[k] = t.dims[k];
    if (offset) *offset = t.offset;
    return CUQ_OK;
}

int cuq_gguf_tensor_bytes(const cuq_gguf *h, const char *name, const void **data, size_t *nbytes) {
    if (!h || !name || !data || !nbytes) return CUQ_EINVAL;
    auto it = h->g.tensors.find(name);
    if (it == h->g.tensors.end()) {
        cuq::set_error("TensorNotFound: %s", name);
        return CUQ_EINVAL;
    }
    const TensorInfo &t = it->second;
    const int epb = cuq_block_elems((int)t.type), bpb = cuq_block_bytes((int)t.type);
    if (!epb || !bpb) {
        cuq::set_error("UnsupportedType: %s has ggml type %u", name, t.type);
        return CUQ_EUNSUPPORTED;
    }
    uint64_t n = 1;
    for (auto d : t.dims) {
        if (d && n > UINT64_MAX / d) {
            cuq::set_error("TensorDataOutOfRange: %s", name);
            return CUQ_EFORMAT;
        }
        n *= d;
    }
    if (n % (uint64_t)epb) {
        cuq::set_error("InvalidTensorShape: %s (%llu elements, block of %d)", name, (unsigned long long)n, epb);
        return CUQ_EINVAL;
    }
    const uint64_t nb = n / epb * bpb;
    const uint64_t start = h->g.data_off + t.offset;
    if (t.offset > UINT64_MAX - h->g.data_off || nb > UINT64_MAX - start || start + nb > h->g.size) {
        cuq::set_error("TensorDataOutOfRange: %s", name);
        return CUQ_EFORMAT;
    }
    *data = h->g.data + start;
    *nbytes = (size_t)nb;
    return CUQ_OK;
}

}  // extern "C"
