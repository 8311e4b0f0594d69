// capi.cu -- the extern "C" boundary (include/cuq.h): lifecycle, last error,
// dequantisation, weight handles and the standalone op entry points.
#include <cmath>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "ops.cuh"

namespace cuq {

static thread_local char g_err[1024] = "";
static thread_local int g_ready_device = -1;

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}
const char *get_error() { return g_err; }

int sm_count_current() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

void build_rope_table(float *out, uint32_t max_seq, uint32_t hd, float theta) {
    uint32_t half = hd / 2;
    for (uint32_t i = 0; i < half; i++) {
        // cpu.zig:26-31: freq = 1 / pow(theta, 2i/hd); angle = f32(pos) * freq (all f32)
        float freq = 1.0f / powf(theta, (float)(2 * i) / (float)hd);
        for (uint32_t pos = 0; pos < max_seq; pos++) {
            float angle = (float)pos * freq;
            out[(size_t)pos * hd + i] = cosf(angle);
            out[(size_t)pos * hd + half + i] = sinf(angle);
        }
    }
}

}  // namespace cuq

using namespace cuq;

struct cuq_weight {
    Planes p;
    float *ws = nullptr;
    unsigned int *counters = nullptr;
    int ksplit = 1;
    __half *xq = nullptr;     // scratch activation for cuq_gemv
    size_t xq_cap = 0;        // halves
    size_t raw_nbytes = 0;
};

extern "C" {

int cuq_init(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        set_error("cuq_init: no CUDA device (%s)", e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
        return CUQ_ECUDA;
    }
    if (device < 0 || device >= n) {
        set_error("cuq_init: device %d out of range (have %d)", device, n);
        return CUQ_EINVAL;
    }
    CUQ_CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop;
    CUQ_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) {
        set_error("cuq_init: device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
                  prop.minor);
        return CUQ_EUNSUPPORTED;
    }
    CUQ_CUDA_TRY(cudaFree(nullptr));  // create the context now
    g_ready_device = device;
    return CUQ_OK;
}

int cuq_ready(void) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    return g_ready_device >= 0 && dev == g_ready_device;
}

const char *cuq_last_error(void) { return get_error(); }

#define CUQ_XSTR(x) #x
#define CUQ_STR(x) CUQ_XSTR(x)
const char *cuq_version(void) {
    return "cuq 0.1 (sm_100a; nvcc " CUQ_STR(__CUDACC_VER_MAJOR__) "." CUQ_STR(__CUDACC_VER_MINOR__) ")";
}

int cuq_block_elems(int t) { return block_elems(t); }
int cuq_block_bytes(int t) { return block_bytes(t); }

int cuq_dequant(int ggml_type, const void *raw_dev, size_t raw_bytes, uint64_t elem_offset, float *out_dev,
                size_t out_n, void *stream) {
    if (!raw_dev || (!out_dev && out_n)) {
        set_error("cuq_dequant: null pointer");
        return CUQ_EINVAL;
    }
    return launch_dequant_raw(ggml_type, (const uint8_t *)raw_dev, raw_bytes, elem_offset, out_dev, out_n,
                              (cudaStream_t)stream);
}

cuq_weight *cuq_weight_create(int ggml_type, const void *raw_host, size_t nbytes, uint32_t rows, uint32_t cols) {
    int epb = block_elems(ggml_type), bpb = block_bytes(ggml_type);
    if (!epb) {
        set_error("UnsupportedType: ggml type %d", ggml_type);
        return nullptr;
    }
    if (!raw_host || rows == 0 || cols == 0 || cols % epb) {
        set_error("InvalidTensorShape: %u x %u for a block of %d", rows, cols, epb);
        return nullptr;
    }
    size_t need = (size_t)rows * (cols / epb) * bpb;
    if (nbytes != need) {
        set_error("cuq_weight_create: %zu bytes, %u x %u %s needs %zu", nbytes, rows, cols, "ggml", need);
        return nullptr;
    }
    cuq_weight *w = new cuq_weight();
    w->p.type = ggml_type;
    w->p.rows = rows;
    w->p.cols = cols;
    w->raw_nbytes = nbytes;
    uint8_t *staging = nullptr;
    bool ok = false;
    do {
        if (!plan_planes(w->p)) {
            // not a GEMV type: keep the raw blocks as they are (dequantiser input)
            w->p.raw = true;
            w->p.nbytes = nbytes;
            if (cudaMalloc(&w->p.base, nbytes) != cudaSuccess) break;
            if (cudaMemcpy(w->p.base, raw_host, nbytes, cudaMemcpyHostToDevice) != cudaSuccess) break;
            ok = true;
            break;
        }
        if (cudaMalloc(&w->p.base, w->p.nbytes) != cudaSuccess) break;
        if (cudaMalloc(&staging, nbytes) != cudaSuccess) break;
        if (cudaMemcpy(staging, raw_host, nbytes, cudaMemcpyHostToDevice) != cudaSuccess) break;
        if (launch_repack(staging, w->p, 0) != CUQ_OK) break;
        if (cudaDeviceSynchronize() != cudaSuccess) break;
        w->ksplit = gemv_pick_ksplit(w->p, sm_count_current());
        if (w->ksplit > 1) {
            if (cudaMalloc(&w->ws, sizeof(float) * (size_t)w->ksplit * rows * 2) != cudaSuccess) break;
            if (cudaMalloc(&w->counters, sizeof(unsigned) * (rows / 16 + 1)) != cudaSuccess) break;
            if (cudaMemset(w->counters, 0, sizeof(unsigned) * (rows / 16 + 1)) != cudaSuccess) break;
        }
        ok = true;
    } while (0);
    if (staging) cudaFree(staging);
    if (!ok) {
        set_error("cuq_weight_create: %s", cudaGetErrorString(cudaGetLastError()));
        cuq_weight_free(w);
        return nullptr;
    }
    return w;
}

size_t cuq_weight_nbytes(const cuq_weight *w) { return w ? w->raw_nbytes : 0; }

int cuq_weight_export_raw(const cuq_weight *w, void *raw_host, size_t nbytes) {
    CUQ_CHECK_ARG(w && raw_host && nbytes == w->raw_nbytes, "cuq_weight_export_raw: need %zu bytes",
                  w ? w->raw_nbytes : (size_t)0);
    if (w->p.raw) {
        CUQ_CUDA_TRY(cudaMemcpy(raw_host, w->p.base, nbytes, cudaMemcpyDeviceToHost));
        return CUQ_OK;
    }
    uint8_t *tmp = nullptr;
    CUQ_CUDA_TRY(cudaMalloc(&tmp, nbytes));
    int rc = launch_unpack(w->p, tmp, 0);
    if (rc == CUQ_OK) {
        cudaError_t e = cudaMemcpy(raw_host, tmp, nbytes, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            set_error("export: %s", cudaGetErrorString(e));
            rc = CUQ_ECUDA;
        }
    }
    cudaFree(tmp);
    return rc;
}

void cuq_weight_free(cuq_weight *w) {
    if (!w) return;
    if (w->p.base) cudaFree(w->p.base);
    if (w->ws) cudaFree(w->ws);
    if (w->counters) cudaFree(w->counters);
    if (w->xq) cudaFree(w->xq);
    delete w;
}

}  // extern "C"

namespace cuq {
const Planes *weight_planes(const cuq_weight *w, float **ws, unsigned int **counters, int *ksplit) {
    if (!w) return nullptr;
    *ws = w->ws;
    *counters = w->counters;
    *ksplit = w->ksplit;
    return &w->p;
}
}  // namespace cuq

extern "C" {

static int ensure_xq(cuq_weight *w, size_t halves) {
    if (w->xq_cap >= halves) return CUQ_OK;
    if (w->xq) cudaFree(w->xq);
    w->xq = nullptr;
    w->xq_cap = 0;
    CUQ_CUDA_TRY(cudaMalloc(&w->xq, halves * sizeof(__half)));
    w->xq_cap = halves;
    return CUQ_OK;
}

int cuq_gemv(const cuq_weight *wc, const float *x_dev, float *y_dev, void *stream) {
    CUQ_CHECK_ARG(wc && x_dev && y_dev, "cuq_gemv: null argument");
    cuq_weight *w = const_cast<cuq_weight *>(wc);
    cudaStream_t s = (cudaStream_t)stream;
    int rc = ensure_xq(w, xq_halves(w->p.cols));
    if (rc) return rc;
    rc = launch_to_xq(x_dev, w->p.cols, 1, w->p.cols, w->xq, s);
    if (rc) return rc;
    GemvArgs a;
    a.w = &w->p;
    a.xq = w->xq;
    a.y = y_dev;
    a.ws = w->ws;
    a.counters = w->counters;
    a.ksplit = w->ksplit;
    return launch_gemv(a, EPI_STORE, s);
}

size_t cuq_xq_halves(uint32_t n) { return xq_halves(n); }

int cuq_prepare_x(const float *x_dev, uint32_t n, uint16_t *xq_dev, void *stream) {
    CUQ_CHECK_ARG(x_dev && xq_dev && n > 0, "cuq_prepare_x: bad argument");
    return launch_to_xq(x_dev, n, 1, n, (__half *)xq_dev, (cudaStream_t)stream);
}

int cuq_gemv_prepared(const cuq_weight *w, const uint16_t *xq_dev, float *y_dev, void *stream) {
    CUQ_CHECK_ARG(w && xq_dev && y_dev, "cuq_gemv_prepared: null argument");
    GemvArgs a;
    a.w = &w->p;
    a.xq = (const __half *)xq_dev;
    a.y = y_dev;
    a.ws = w->ws;
    a.counters = w->counters;
    a.ksplit = w->ksplit;
    return launch_gemv(a, EPI_STORE, (cudaStream_t)stream);
}

int cuq_weight_dequant_f16(const cuq_weight *w, uint16_t *out_dev, void *stream) {
    CUQ_CHECK_ARG(w && out_dev, "cuq_weight_dequant_f16: null argument");
    return launch_dequant_planes_f16(w->p, (__half *)out_dev, (cudaStream_t)stream);
}

int cuq_rmsnorm(float *out_dev, const float *x_dev, const float *w_dev, uint32_t n, uint32_t n_rows, float eps,
                void *stream) {
    CUQ_CHECK_ARG(out_dev && x_dev && w_dev && n > 0, "cuq_rmsnorm: bad argument");
    return launch_rmsnorm(out_dev, x_dev, w_dev, n, n_rows, eps, (cudaStream_t)stream);
}

int cuq_rope(float *v_dev, uint32_t heads, uint32_t hd, uint32_t pos, float theta, int adjacent, void *stream) {
    CUQ_CHECK_ARG(v_dev && hd >= 2 && hd % 2 == 0 && hd <= 256, "cuq_rope: bad argument (head_dim %u)", hd);
    // one row of the table for this position, computed with the reference formula
    // (cpu.zig:26-31) and handed to the kernel by value: nothing to copy or wait for
    RopeRow row;
    uint32_t half = hd / 2;
    for (uint32_t i = 0; i < half; i++) {
        float freq = 1.0f / powf(theta, (float)(2 * i) / (float)hd);
        float angle = (float)pos * freq;
        row.v[i] = cosf(angle);
        row.v[half + i] = sinf(angle);
    }
    return launch_rope(v_dev, heads, hd, row, adjacent, (cudaStream_t)stream);
}

int cuq_silu_mul(float *out_dev, const float *g_dev, const float *u_dev, uint32_t n, void *stream) {
    CUQ_CHECK_ARG(out_dev && g_dev && u_dev, "cuq_silu_mul: null argument");
    return launch_silu_mul(out_dev, g_dev, u_dev, n, (cudaStream_t)stream);
}

int cuq_attention_decode(float *out_dev, const float *q_dev, const uint16_t *k_dev, const uint16_t *v_dev,
                         uint32_t n_past, uint32_t cache_stride, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                         void *stream) {
    CUQ_CHECK_ARG(out_dev && q_dev && k_dev && v_dev && n_past >= 1 && n_past <= cache_stride,
                  "cuq_attention_decode: bad argument (n_past %u, stride %u)", n_past, cache_stride);
    CUQ_CHECK_ARG(heads > 0 && kv_heads > 0 && heads % kv_heads == 0,
                  "cuq_attention_decode: heads (%u) must be a positive multiple of kv_heads (%u)", heads, kv_heads);
    if (hd != 64 && hd != 128) {
        set_error("cuq_attention_decode: unsupported head_dim %u (64 or 128)", hd);
        return CUQ_EUNSUPPORTED;
    }
    cudaStream_t s = (cudaStream_t)stream;
    int nsplit = attn_pick_nsplit(kv_heads, n_past, sm_count_current());
    float *part = nullptr;
    CUQ_CUDA_TRY(cudaMallocAsync(&part, sizeof(float) * (size_t)nsplit * heads * ((size_t)hd + 2), s));
    int rc = launch_attention_decode(q_dev, (const __half *)k_dev, (const __half *)v_dev, cache_stride, nullptr,
                                     n_past, heads, kv_heads, hd, part, nsplit, out_dev, nullptr, s);
    cudaFreeAsync(part, s);
    return rc;
}

int cuq_attention_prefill(float *out_dev, const float *q_dev, const uint16_t *k_dev, const uint16_t *v_dev,
                          uint32_t n, uint32_t pos0, uint32_t cache_stride, uint32_t heads, uint32_t kv_heads,
                          uint32_t hd, void *stream) {
    CUQ_CHECK_ARG(out_dev && q_dev && k_dev && v_dev && n >= 1 && (uint64_t)pos0 + n <= cache_stride,
                  "cuq_attention_prefill: bad argument (n %u, pos0 %u, stride %u)", n, pos0, cache_stride);
    CUQ_CHECK_ARG(heads > 0 && kv_heads > 0 && heads % kv_heads == 0,
                  "cuq_attention_prefill: heads (%u) must be a positive multiple of kv_heads (%u)", heads, kv_heads);
    if (hd != 64 && hd != 128) {
        set_error("cuq_attention_prefill: unsupported head_dim %u (64 or 128)", hd);
        return CUQ_EUNSUPPORTED;
    }
    cudaStream_t s = (cudaStream_t)stream;
    const size_t count = (size_t)n * heads * hd;
    __half *hl = nullptr;  // the kernel's output: fp16 hi and lo planes (the o GEMM's input)
    CUQ_CUDA_TRY(cudaMallocAsync(&hl, sizeof(__half) * 2 * count, s));
    int rc = launch_attention_prefill(q_dev, (const __half *)k_dev, (const __half *)v_dev, cache_stride, pos0, n,
                                      heads, kv_heads, hd, hl, hl + count, s);
    if (rc == CUQ_OK) rc = launch_hilo_sum(hl, hl + count, count, out_dev, s);
    cudaFreeAsync(hl, s);
    return rc;
}

int cuq_argmax(const float *v_dev, uint32_t n, uint32_t *out_dev, void *stream) {
    CUQ_CHECK_ARG(v_dev && out_dev && n > 0, "cuq_argmax: bad argument");
    return launch_argmax(v_dev, n, out_dev, (cudaStream_t)stream);
}

}  // extern "C"

// cuq_gemm: prefill projection.  Defined in gemm.cu.
