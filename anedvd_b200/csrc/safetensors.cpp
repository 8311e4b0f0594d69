// safetensors.cpp -- the HuggingFace side of the loader: safetensors shards
// (src/safetensors.zig) and config.json (src/hf.zig) of a model directory,
// uploaded raw (load_hf.zig:143-230 minus the fp16 expansion of `linear`):
// F16 and BF16 weights go to the device as they are on disk and the GEMV /
// GEMM round them like readF16 does; F32 weights are kept as raw blocks.
// Norms and biases are read as f32 (load_hf.zig `norm`, readF32).  RoPE is the
// half-split convention, as the reference uses for every HF directory.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "../../include/cuq.h"

namespace cuq {
void set_error(const char *fmt, ...);
}

namespace {

// ------------------------------------------------------------------ JSON ---
// Enough of JSON for safetensors headers and config.json: objects, arrays,
// strings (escapes kept as their code units), numbers, true / false / null.
struct Json {
    enum Kind { NUL, BOOL, INT, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    long long i = 0;   // INT (integral literal without fraction or exponent)
    double d = 0;      // INT and NUM
    std::string s;
    std::vector<Json> a;
    std::vector<std::pair<std::string, Json>> o;  // in file order
    const Json *get(const char *k) const {
        for (auto &kv : o)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JsonParser {
    const char *p, *e;
    int depth = 0;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool lit(const char *w) {
        size_t n = strlen(w);
        if ((size_t)(e - p) < n || memcmp(p, w, n) != 0) return false;
        p += n;
        return true;
    }
    bool str(std::string &out) {
        if (p >= e || *p != '"') return false;
        p++;
        while (p < e && *p != '"') {
            if (*p == '\\') {
                if (++p >= e) return false;
                switch (*p) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    if (e - p < 5) return false;
                    unsigned v = 0;
                    for (int k = 1; k <= 4; k++) {
                        char c = p[k];
                        v = v * 16 + (unsigned)(c >= '0' && c <= '9' ? c - '0'
                                               : c >= 'a' && c <= 'f' ? c - 'a' + 10
                                               : c >= 'A' && c <= 'F' ? c - 'A' + 10
                                                                      : 99);
                        if ((c < '0' || c > '9') && (c < 'a' || c > 'f') && (c < 'A' || c > 'F')) return false;
                    }
                    p += 4;
                    if (v < 0x80) out += (char)v;
                    else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 63)); }
                    else { out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 63)); out += (char)(0x80 | (v & 63)); }
                    break;
                }
                default: return false;
                }
                p++;
            } else {
                if ((unsigned char)*p < 0x20) return false;
                out += *p++;
            }
        }
        if (p >= e) return false;
        p++;
        return true;
    }
    bool num(Json &v) {
        const char *s = p;
        if (p < e && *p == '-') p++;
        if (p >= e || *p < '0' || *p > '9') return false;
        while (p < e && *p >= '0' && *p <= '9') p++;
        bool integral = true;
        if (p < e && *p == '.') {
            integral = false;
            p++;
            while (p < e && *p >= '0' && *p <= '9') p++;
        }
        if (p < e && (*p == 'e' || *p == 'E')) {
            integral = false;
            p++;
            if (p < e && (*p == '+' || *p == '-')) p++;
            while (p < e && *p >= '0' && *p <= '9') p++;
        }
        std::string t(s, p);
        v.d = strtod(t.c_str(), nullptr);
        if (integral) {
            errno = 0;
            long long x = strtoll(t.c_str(), nullptr, 10);
            if (errno) return false;  // out of range for an integer
            v.kind = Json::INT;
            v.i = x;
        } else {
            v.kind = Json::NUM;
        }
        return true;
    }
    bool value(Json &v) {
        if (++depth > 64) return false;
        ws();
        bool ok = false;
        if (p >= e) ok = false;
        else if (*p == '{') {
            v.kind = Json::OBJ;
            p++;
            ws();
            if (p < e && *p == '}') { p++; ok = true; }
            else {
                while (true) {
                    ws();
                    std::string k;
                    if (!str(k)) break;
                    ws();
                    if (p >= e || *p != ':') break;
                    p++;
                    Json x;
                    if (!value(x)) break;
                    v.o.emplace_back(std::move(k), std::move(x));
                    ws();
                    if (p < e && *p == ',') { p++; continue; }
                    if (p < e && *p == '}') { p++; ok = true; }
                    break;
                }
            }
        } else if (*p == '[') {
            v.kind = Json::ARR;
            p++;
            ws();
            if (p < e && *p == ']') { p++; ok = true; }
            else {
                while (true) {
                    Json x;
                    if (!value(x)) break;
                    v.a.push_back(std::move(x));
                    ws();
                    if (p < e && *p == ',') { p++; continue; }
                    if (p < e && *p == ']') { p++; ok = true; }
                    break;
                }
            }
        } else if (*p == '"') {
            v.kind = Json::STR;
            ok = str(v.s);
        } else if (lit("true")) { v.kind = Json::BOOL; v.b = true; ok = true; }
        else if (lit("false")) { v.kind = Json::BOOL; v.b = false; ok = true; }
        else if (lit("null")) { v.kind = Json::NUL; ok = true; }
        else ok = num(v);
        depth--;
        return ok;
    }
};

bool parse_json(const char *data, size_t n, Json &out) {
    JsonParser ps{data, data + n};
    if (!ps.value(out)) return false;
    ps.ws();
    return ps.p == ps.e;
}

// ---------------------------------------------------------- safetensors ---
struct StTensor {
    std::string dtype;
    std::vector<uint64_t> shape;
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
};

int dtype_size(const std::string &d) {
    if (d == "F64" || d == "I64") return 8;
    if (d == "F32" || d == "I32") return 4;
    if (d == "F16" || d == "BF16" || d == "I16") return 2;
    if (d == "I8" || d == "U8" || d == "BOOL") return 1;
    return 0;
}

}  // namespace

struct cuq_safetensors {
    std::vector<uint8_t> copy;
    void *map = nullptr;
    size_t size = 0;
    const uint8_t *bytes = nullptr;
    std::vector<std::string> order;  // header order
    std::map<std::string, StTensor> tensors;
    std::string err;

    // Safetensors.initOwned / parseHeader (safetensors.zig:152-233), same checks
    // and error names.
    bool parse() {
        if (size < 8) return fail("HeaderTooSmall");
        uint64_t hl;
        memcpy(&hl, bytes, 8);
        if (hl > size - 8) return fail("InvalidHeaderLength");
        const uint8_t *payload = bytes + 8 + hl;
        const size_t plen = size - 8 - hl;
        Json root;
        if (!parse_json((const char *)bytes + 8, (size_t)hl, root) || root.kind != Json::OBJ)
            return fail("InvalidHeader");
        for (auto &kv : root.o) {
            if (kv.first == "__metadata__") continue;
            const Json &ent = kv.second;
            if (ent.kind != Json::OBJ) return fail("InvalidTensorEntry");
            const Json *dt = ent.get("dtype");
            if (!dt || dt->kind != Json::STR) return fail("InvalidTensorEntry");
            const int esz = dtype_size(dt->s);
            if (!esz) return fail("UnsupportedDtype");
            const Json *sh = ent.get("shape");
            if (!sh || sh->kind != Json::ARR) return fail("InvalidTensorEntry");
            StTensor t;
            t.dtype = dt->s;
            unsigned __int128 numel = 1;
            for (auto &d : sh->a) {
                if (d.kind != Json::INT || d.i < 0) return fail("InvalidTensorEntry");
                t.shape.push_back((uint64_t)d.i);
                numel *= (uint64_t)d.i;
                if (numel > ((unsigned __int128)1 << 62)) return fail("DataSizeMismatch");
            }
            const Json *off = ent.get("data_offsets");
            if (!off || off->kind != Json::ARR || off->a.size() != 2) return fail("InvalidTensorEntry");
            if (off->a[0].kind != Json::INT || off->a[1].kind != Json::INT) return fail("InvalidTensorEntry");
            if (off->a[0].i < 0 || off->a[1].i < 0) return fail("DataSizeMismatch");
            const uint64_t b = (uint64_t)off->a[0].i, en = (uint64_t)off->a[1].i;
            if (b > en || en > plen) return fail("DataSizeMismatch");
            if ((unsigned __int128)(en - b) != numel * (unsigned)esz) return fail("DataSizeMismatch");
            t.data = payload + b;
            t.nbytes = (size_t)(en - b);
            if (!tensors.count(kv.first)) order.push_back(kv.first);
            tensors[kv.first] = t;
        }
        return true;
    }
    bool fail(const char *e) {
        err = e;
        return false;
    }
};

namespace {

cuq_safetensors *st_finish(cuq_safetensors *h, const char *what) {
    if (!h->parse()) {
        cuq::set_error("%s: %s", h->err.c_str(), what);
        cuq_safetensors_close(h);
        return nullptr;
    }
    return h;
}

bool read_file(const std::string &path, std::string &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
    fclose(f);
    return true;
}

// hf.zig Config fields this path uses (defaults as there: num_key_value_heads =
// heads, head_dim = hidden / heads, rms_norm_eps 1e-6, rope_theta 10000 or
// rope_parameters / rope_scaling.rope_theta).
int hf_config(const std::string &dir, cuq_config &c) {
    std::string text;
    const std::string path = dir + "/config.json";
    if (!read_file(path, text)) {
        cuq::set_error("FileNotFound: %s", path.c_str());
        return CUQ_EFORMAT;
    }
    Json root;
    if (!parse_json(text.data(), text.size(), root) || root.kind != Json::OBJ) {
        cuq::set_error("InvalidConfig: %s is not a JSON object", path.c_str());
        return CUQ_EFORMAT;
    }
    auto u32 = [&](const char *k, bool required, uint32_t dflt, bool &ok) -> uint32_t {
        const Json *v = root.get(k);
        if (!v || v->kind != Json::INT || v->i < 0 || v->i > 0xFFFFFFFFll) {
            if (required) {
                cuq::set_error("MissingField: %s in %s", k, path.c_str());
                ok = false;
            }
            return dflt;
        }
        return (uint32_t)v->i;
    };
    auto f32 = [&](const Json *o, const char *k, double dflt, bool &found) -> double {
        const Json *v = o ? o->get(k) : nullptr;
        if (!v || (v->kind != Json::INT && v->kind != Json::NUM)) return dflt;
        found = true;
        return v->d;
    };
    bool ok = true;
    memset(&c, 0, sizeof c);
    c.hidden = u32("hidden_size", true, 0, ok);
    c.layers = u32("num_hidden_layers", true, 0, ok);
    c.heads = u32("num_attention_heads", true, 0, ok);
    c.inter = u32("intermediate_size", true, 0, ok);
    c.vocab = u32("vocab_size", true, 0, ok);
    if (!ok) return CUQ_EFORMAT;
    if (!c.hidden || !c.layers || !c.heads || !c.inter) {
        cuq::set_error("UnsupportedArchitecture: %s", path.c_str());
        return CUQ_EFORMAT;
    }
    c.kv_heads = u32("num_key_value_heads", false, c.heads, ok);
    c.head_dim = u32("head_dim", false, c.hidden / c.heads, ok);
    bool found = false;
    c.eps = (float)f32(&root, "rms_norm_eps", 1e-6, found);
    found = false;
    double th = f32(&root, "rope_theta", 0, found);
    if (!found) th = f32(root.get("rope_parameters"), "rope_theta", 0, found);
    if (!found) th = f32(root.get("rope_scaling"), "rope_theta", 0, found);
    c.rope_theta = (float)(found ? th : 10000.0);
    const Json *tie = root.get("tie_word_embeddings");
    c.tie_embeddings = tie && tie->kind == Json::BOOL && tie->b ? 1 : 0;
    c.rope_adjacent = 0;  // HF keeps the rotate_half (half-split) layout (load_hf.zig:96)
    return CUQ_OK;
}

// hf.findShards: the files of model.safetensors.index.json's weight_map, or
// every *.safetensors file of the directory, sorted by name.
int find_shards(const std::string &dir, std::vector<std::string> &out) {
    std::string text;
    if (read_file(dir + "/model.safetensors.index.json", text)) {
        Json root;
        const Json *wm = nullptr;
        if (!parse_json(text.data(), text.size(), root) || !(wm = root.get("weight_map")) || wm->kind != Json::OBJ) {
            cuq::set_error("InvalidIndex: %s/model.safetensors.index.json", dir.c_str());
            return CUQ_EFORMAT;
        }
        std::set<std::string> files;
        for (auto &kv : wm->o)
            if (kv.second.kind == Json::STR) files.insert(kv.second.s);
        for (auto &f : files) out.push_back(dir + "/" + f);
        return CUQ_OK;
    }
    DIR *d = opendir(dir.c_str());
    if (!d) {
        cuq::set_error("FileNotFound: %s", dir.c_str());
        return CUQ_EFORMAT;
    }
    while (dirent *e = readdir(d)) {
        std::string n = e->d_name;
        if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) out.push_back(dir + "/" + n);
    }
    closedir(d);
    std::sort(out.begin(), out.end());
    if (out.empty()) {
        cuq::set_error("NoShardsFound: %s", dir.c_str());
        return CUQ_EFORMAT;
    }
    return CUQ_OK;
}

float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t u;
    if (e == 0) {
        if (m == 0) u = s;
        else {  // subnormal: normalise
            int k = 0;
            uint32_t mm = m;
            while (!(mm & 1024)) { mm <<= 1; k++; }
            u = s | ((uint32_t)(127 - 15 - k + 1) << 23) | ((mm & 1023) << 13);
        }
    } else if (e == 31) u = s | 0x7F800000u | (m << 13);
    else u = s | ((e - 15 + 127) << 23) | (m << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// readF32 of a float tensor (convertTo, safetensors.zig:297-330) for norms and biases.
bool to_f32(const StTensor &t, std::vector<float> &v) {
    const size_t n = t.nbytes / (size_t)dtype_size(t.dtype);
    v.resize(n);
    for (size_t k = 0; k < n; k++) {
        if (t.dtype == "F32") memcpy(&v[k], t.data + 4 * k, 4);
        else if (t.dtype == "F16") { uint16_t h; memcpy(&h, t.data + 2 * k, 2); v[k] = f16_to_f32(h); }
        else if (t.dtype == "BF16") { uint16_t h; memcpy(&h, t.data + 2 * k, 2); v[k] = bf16_to_f32(h); }
        else if (t.dtype == "F64") { double d; memcpy(&d, t.data + 8 * k, 8); v[k] = (float)d; }
        else return false;
    }
    return true;
}

}  // namespace

extern "C" {

cuq_safetensors *cuq_safetensors_open(const char *path) {
    if (!path) {
        cuq::set_error("cuq_safetensors_open: null path");
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
        cuq::set_error("cuq_safetensors_open: cannot stat %s", path);
        return nullptr;
    }
    cuq_safetensors *h = new cuq_safetensors();
    if (st.st_size > 0) {
        void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (map == MAP_FAILED) {
            close(fd);
            delete h;
            cuq::set_error("cuq_safetensors_open: mmap failed");
            return nullptr;
        }
        h->map = map;
        h->bytes = (const uint8_t *)map;
        h->size = (size_t)st.st_size;
    }
    close(fd);
    return st_finish(h, path);
}

cuq_safetensors *cuq_safetensors_open_bytes(const void *data, size_t n) {
    if (!data && n) {
        cuq::set_error("cuq_safetensors_open_bytes: null data");
        return nullptr;
    }
    cuq_safetensors *h = new cuq_safetensors();
    if (n) h->copy.assign((const uint8_t *)data, (const uint8_t *)data + n);
    h->bytes = h->copy.data();
    h->size = n;
    return st_finish(h, "in-memory file");
}

void cuq_safetensors_close(cuq_safetensors *h) {
    if (!h) return;
    if (h->map) munmap(h->map, h->size);
    delete h;
}

uint64_t cuq_safetensors_count(const cuq_safetensors *h) { return h ? (uint64_t)h->order.size() : 0; }

const char *cuq_safetensors_name(const cuq_safetensors *h, uint64_t i) {
    return h && i < h->order.size() ? h->order[(size_t)i].c_str() : nullptr;
}

int cuq_safetensors_tensor(const cuq_safetensors *h, const char *name, char *dtype_out, uint32_t *rank,
                           uint64_t *shape, const void **data, size_t *nbytes) {
    if (!h || !name) return CUQ_EINVAL;
    auto it = h->tensors.find(name);
    if (it == h->tensors.end()) {
        cuq::set_error("TensorNotFound: %s", name);
        return CUQ_EINVAL;
    }
    const StTensor &t = it->second;
    if (dtype_out) {
        memset(dtype_out, 0, 8);
        memcpy(dtype_out, t.dtype.c_str(), std::min<size_t>(7, t.dtype.size()));
    }
    if (rank) *rank = (uint32_t)t.shape.size();
    if (shape)
        for (size_t k = 0; k < t.shape.size() && k < 8; k++) shape[k] = t.shape[k];
    if (data) *data = t.data;
    if (nbytes) *nbytes = t.nbytes;
    return CUQ_OK;
}

int cuq_hf_read_config(const char *dir, cuq_config *out) {
    if (!dir || !out) {
        cuq::set_error("cuq_hf_read_config: null argument");
        return CUQ_EINVAL;
    }
    return hf_config(dir, *out);
}

cuq_model *cuq_model_load_hf(const char *dir_c, const cuq_options *opts) {
    if (!dir_c) {
        cuq::set_error("cuq_model_load_hf: null directory");
        return nullptr;
    }
    const std::string dir = dir_c;
    cuq_config c;
    if (hf_config(dir, c) != CUQ_OK) return nullptr;
    std::vector<std::string> paths;
    if (find_shards(dir, paths) != CUQ_OK) return nullptr;
    std::vector<std::unique_ptr<cuq_safetensors, void (*)(cuq_safetensors *)>> shards;
    for (auto &p : paths) {
        cuq_safetensors *s = cuq_safetensors_open(p.c_str());
        if (!s) return nullptr;
        shards.emplace_back(s, cuq_safetensors_close);
    }
    auto find = [&](const std::string &name) -> const StTensor * {
        for (auto &s : shards) {
            auto it = s->tensors.find(name);
            if (it != s->tensors.end()) return &it->second;
        }
        return nullptr;
    };
    // the head is tied when the directory has no lm_head (load_hf.zig:227-229)
    c.tie_embeddings = find("lm_head.weight") ? 0 : 1;
    cuq_model *m = cuq_model_create(&c, opts);
    if (!m) return nullptr;
    auto linear = [&](const std::string &name, int layer, int role, uint32_t in, uint32_t out) -> bool {
        const StTensor *t = find(name);
        if (!t) {
            cuq::set_error("MissingTensor: %s", name.c_str());
            return false;
        }
        // load_hf.zig:172-177: PyTorch [out][in], no transpose
        if (t->shape.size() != 2 || t->shape[0] != out || t->shape[1] != in) {
            cuq::set_error("DimensionMismatch: %s is not [%u, %u]", name.c_str(), out, in);
            return false;
        }
        int type;
        if (t->dtype == "F16") type = CUQ_F16;
        else if (t->dtype == "BF16") type = CUQ_BF16;
        else if (t->dtype == "F32") type = CUQ_F32;
        else {
            cuq::set_error("UnsupportedDtype: %s is %s", name.c_str(), t->dtype.c_str());
            return false;
        }
        return cuq_upload_tensor(m, layer, role, type, t->data, t->nbytes, out, in) == CUQ_OK;
    };
    auto vec = [&](const std::string &name, int layer, int role, uint32_t n) -> bool {
        const StTensor *t = find(name);
        if (!t) {
            cuq::set_error("MissingTensor: %s", name.c_str());
            return false;
        }
        std::vector<float> v;
        if (!to_f32(*t, v) || v.size() != n) {
            cuq::set_error("DimensionMismatch: %s must be %u float values", name.c_str(), n);
            return false;
        }
        return cuq_upload_f32(m, layer, role, v.data(), n) == CUQ_OK;
    };
    const uint32_t qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
    bool good = linear("model.embed_tokens.weight", -1, CUQ_ROLE_EMBED, c.hidden, c.vocab) &&
                vec("model.norm.weight", -1, CUQ_ROLE_FINAL_NORM, c.hidden);
    if (good && !c.tie_embeddings) good = linear("lm_head.weight", -1, CUQ_ROLE_OUTPUT, c.hidden, c.vocab);
    for (uint32_t l = 0; good && l < c.layers; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        good = vec(p + "input_layernorm.weight", l, CUQ_ROLE_ATTN_NORM, c.hidden) &&
               vec(p + "post_attention_layernorm.weight", l, CUQ_ROLE_FFN_NORM, c.hidden) &&
               linear(p + "self_attn.q_proj.weight", l, CUQ_ROLE_Q, c.hidden, qd) &&
               linear(p + "self_attn.k_proj.weight", l, CUQ_ROLE_K, c.hidden, kvd) &&
               linear(p + "self_attn.v_proj.weight", l, CUQ_ROLE_V, c.hidden, kvd) &&
               linear(p + "self_attn.o_proj.weight", l, CUQ_ROLE_O, qd, c.hidden) &&
               linear(p + "mlp.gate_proj.weight", l, CUQ_ROLE_GATE, c.hidden, c.inter) &&
               linear(p + "mlp.up_proj.weight", l, CUQ_ROLE_UP, c.hidden, c.inter) &&
               linear(p + "mlp.down_proj.weight", l, CUQ_ROLE_DOWN, c.inter, c.hidden);
        // qwen2 attention biases (load_hf.zig:167-181): all three or none
        if (good && find(p + "self_attn.q_proj.bias"))
            good = vec(p + "self_attn.q_proj.bias", l, CUQ_ROLE_Q_BIAS, qd) &&
                   vec(p + "self_attn.k_proj.bias", l, CUQ_ROLE_K_BIAS, kvd) &&
                   vec(p + "self_attn.v_proj.bias", l, CUQ_ROLE_V_BIAS, kvd);
    }
    const bool tp = opts && opts->tp_size > 1;  // finalized by the caller after cuq_tp_connect
    if (!good || (!tp && cuq_model_finalize(m) != CUQ_OK)) {
        cuq_model_free(m);
        return nullptr;
    }
    return m;
}

}  // extern "C"
