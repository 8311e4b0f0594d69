// ops.cu -- RMSNorm, RoPE + KV-cache write, decode attention, SiLU, argmax, embedding.
//
// Each kernel restates one reference CPU op (src/cpu.zig) and names it.  The
// KV cache is fp16 like the reference's (engine.zig:447-458, 952-970) but laid
// out [kv_head][position][head_dim] so one head's keys are contiguous.
#include "attn_impl.cuh"
#include "common.cuh"
#include "ops.cuh"

namespace cuq {

namespace {

// -------------------------------------------------------------- RMSNorm ---
// cpu.rmsnorm (cpu.zig:11-18): one CTA per row.
__global__ void rmsnorm_kernel(float *out, const float *__restrict__ x, const float *__restrict__ w, uint32_t n,
                               float eps) {
    const float *xr = x + (size_t)blockIdx.x * n;
    float *o = out + (size_t)blockIdx.x * n;
    __shared__ float part[32];
    float acc = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) acc += xr[i] * xr[i];
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
        if (threadIdx.x == 0) part[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(part[0] / (float)n + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// ----------------------------------------------------------------- RoPE ---
// cpu.rope (pairs i, i+hd/2) / cpu.ropeAdjacent (pairs 2j, 2j+1), cpu.zig:22-62,
// with cos/sin of f32(pos)*freq taken from a host-built table [pos][hd/2].
__device__ __forceinline__ void rope_pair(float &a, float &b, float c, float s) {
    float na = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    float nb = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    a = na;
    b = nb;
}

__global__ void rope_kernel(float *v, uint32_t heads, uint32_t hd, const RopeRow cs_row, int adjacent) {
    const uint32_t half = hd / 2;
    for (uint32_t t = threadIdx.x + blockIdx.x * blockDim.x; t < heads * half; t += blockDim.x * gridDim.x) {
        uint32_t h = t / half, i = t % half;
        float c = cs_row.v[i], s = cs_row.v[half + i];
        float *base = v + (size_t)h * hd;
        if (adjacent)
            rope_pair(base[2 * i], base[2 * i + 1], c, s);
        else
            rope_pair(base[i], base[i + half], c, s);
    }
}

// Engine.ropeAndCache (engine.zig:952-970) for `n_tok` consecutive positions:
// rotate q in place (into q_out) and k, round k and v to fp16 into the cache.
// qkv rows are [q | k | v] (the q||k||v concatenation of load_gguf.zig:677-682).
__global__ void rope_cache_kernel(const float *__restrict__ qkv, uint32_t qkv_stride, float *q_out,
                                  __half *k_cache, __half *v_cache, uint32_t cache_stride, const float *__restrict__ cs,
                                  const int *pos_ptr, uint32_t pos_val, uint32_t heads, uint32_t kv_heads,
                                  uint32_t hd, int adjacent) {
    const uint32_t tok = blockIdx.y;
    const uint32_t pos = (pos_ptr ? (uint32_t)*pos_ptr : pos_val) + tok;
    const float *row = qkv + (size_t)tok * qkv_stride;
    float *qo = q_out + (size_t)tok * heads * hd;
    const uint32_t half = hd / 2, qd = heads * hd, kvd = kv_heads * hd;
    const float *csr = cs + (size_t)pos * hd;  // [pos][cos(half) | sin(half)]
    const uint32_t npairs = (heads + kv_heads) * half;
    for (uint32_t t = threadIdx.x + blockIdx.x * blockDim.x; t < npairs + kvd; t += blockDim.x * gridDim.x) {
        if (t < npairs) {
            uint32_t h = t / half, i = t % half;
            float c = csr[i], s = csr[half + i];
            bool is_q = h < heads;
            const float *src = is_q ? row + (size_t)h * hd : row + qd + (size_t)(h - heads) * hd;
            uint32_t ia = adjacent ? 2 * i : i, ib = adjacent ? 2 * i + 1 : i + half;
            float a = src[ia], b = src[ib];
            rope_pair(a, b, c, s);
            if (is_q) {
                qo[(size_t)h * hd + ia] = a;
                qo[(size_t)h * hd + ib] = b;
            } else {
                uint32_t kh = h - heads;
                __half *kc = k_cache + ((size_t)kh * cache_stride + pos) * hd;
                kc[ia] = __float2half_rn(a);
                kc[ib] = __float2half_rn(b);
            }
        } else {
            uint32_t e = t - npairs, kh = e / hd, d = e % hd;
            v_cache[((size_t)kh * cache_stride + pos) * hd + d] = __float2half_rn(row[qd + kvd + e]);
        }
    }
}

template <int HD, int G>
__global__ void __launch_bounds__(128) attn_decode_kernel(const float *__restrict__ q, const __half *__restrict__ kc,
                                                           const __half *__restrict__ vc, uint32_t cache_stride,
                                                           const int *pos_ptr, uint32_t n_val, uint32_t heads,
                                                           float *part, int nsplit) {
    constexpr int E = 8, LPP = HD / E;
    const uint32_t kvh = blockIdx.x, split = blockIdx.y;
    const uint32_t n = pos_ptr ? (uint32_t)(*pos_ptr) + 1u : n_val;
    const SplitRange r = split_range(n, nsplit, split);
    if (split >= r.nact) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lp = lane % LPP, pg = lane / LPP;
    float qr[G][E];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < E; e++) qr[g][e] = q[(size_t)(kvh * G + g) * HD + lp * E + e];
    float m[G], l[G], o[G][E];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < E; e++) o[g][e] = 0.f;
    }
    attn_walk<HD, G>(qr, kc + (size_t)kvh * cache_stride * HD, vc + (size_t)kvh * cache_stride * HD, r.p0, r.p1,
                     warp, lp, pg, m, l, o);
    __shared__ float scr[attn_store_floats(HD, G)];
    attn_store_split<HD, G>(m, l, o, warp, lp, pg, part, split, nsplit, heads, kvh, scr);
}

// Merge for the standalone decode attention: CTA per query head.
template <int HD>
__global__ void __launch_bounds__(128) attn_combine_kernel(const float *__restrict__ part, int nsplit,
                                                            const int *pos_ptr, uint32_t n_val, uint32_t heads,
                                                            float *out, __half *xq, uint32_t kpad) {
    __shared__ float res[HD];
    __shared__ float scr[attn_merge_floats(1)];
    const uint32_t n = pos_ptr ? (uint32_t)(*pos_ptr) + 1u : n_val;
    const SplitRange r = split_range(n, nsplit, 0);
    attn_merge<HD, 1>(part, nsplit, r.nact, heads, blockIdx.x, res, scr);
    attn_emit(res, HD, blockIdx.x * HD, out, xq, kpad);
}

template <int HD, int G>
__global__ void __launch_bounds__(128) attn_step_kernel(const AttnStepArgs p) {
    griddep_wait();
    griddep_launch();
    __shared__ __align__(16) float scr[attn_step_floats(HD, G)];
    attn_step_body<HD, G, true>(p, blockIdx.x, blockIdx.y, (uint32_t)p.state->pos, scr);
}

// ------------------------------------------------------ prefill helpers --

// cpu.rmsnorm (cpu.zig:11-18) over n_rows rows, written as fp16 hi + lo
// (x = hi + lo) for the tensor-core GEMM.  One CTA per row.
__global__ void rmsnorm_hilo_kernel(const float *__restrict__ x, const float *__restrict__ w, uint32_t n, float eps,
                                    __half *__restrict__ hi, __half *__restrict__ lo) {
    const float *xr = x + (size_t)blockIdx.x * n;
    __shared__ float part[32];
    float acc = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) acc += xr[i] * xr[i];
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
        if (threadIdx.x == 0) part[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(part[0] / (float)n + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        float f = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
        __half h = __float2half_rn(f);
        hi[(size_t)blockIdx.x * n + i] = h;
        lo[(size_t)blockIdx.x * n + i] = __float2half_rn(f - __half2float(h));
    }
}


// siluMul (cpu.zig:65-70) of separate gate / up GEMM outputs, as hi + lo.
__global__ void silu_hilo_kernel(const float *__restrict__ g, const float *__restrict__ u, size_t count,
                                 __half *__restrict__ hi, __half *__restrict__ lo) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        float gv = g[i];
        float s = 1.0f / (1.0f + expf(-gv));
        float a = (gv * s) * u[i];
        __half h = __float2half_rn(a);
        hi[i] = h;
        lo[i] = __float2half_rn(a - __half2float(h));
    }
}

// --------------------------------------------------------------- others ---

__global__ void silu_mul_kernel(float *out, const float *g, const float *u, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float gv = g[i];
        float s = 1.0f / (1.0f + expf(-gv));
        out[i] = (gv * s) * u[i];
    }
}

__device__ __forceinline__ unsigned long long pack_argmax(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v);
    uint32_t key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

// cpu.argmax (cpu.zig:477-483), one CTA.
__global__ void argmax_kernel(const float *v, uint32_t n, uint32_t *out) {
    unsigned long long best = 0ull;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        unsigned long long k = pack_argmax(v[i], i);
        best = k > best ? k : best;
    }
    __shared__ unsigned long long sb[32];
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        unsigned long long o = __shfl_xor_sync(0xffffffffu, best, s);
        best = o > best ? o : best;
    }
    if ((threadIdx.x & 31) == 0) sb[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = sb[w] > best ? sb[w] : best;
        best = sb[0] > best ? sb[0] : best;
        *out = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull);
    }
}

}  // namespace

int launch_rmsnorm(float *out, const float *x, const float *w, uint32_t n, uint32_t n_rows, float eps,
                   cudaStream_t s) {
    rmsnorm_kernel<<<n_rows, 256, 0, s>>>(out, x, w, n, eps);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

__global__ void hilo_sum_kernel(const __half *__restrict__ hi, const __half *__restrict__ lo, size_t count,
                                float *__restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __half2float(hi[i]) + __half2float(lo[i]);
}

int launch_hilo_sum(const __half *hi, const __half *lo, size_t count, float *out, cudaStream_t s) {
    const size_t blocks = (count + 255) / 256;
    hilo_sum_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(hi, lo, count, out);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_rope(float *v, uint32_t heads, uint32_t hd, const RopeRow &cs_row, int adjacent, cudaStream_t s) {
    rope_kernel<<<1, 256, 0, s>>>(v, heads, hd, cs_row, adjacent);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_rope_cache(const float *qkv, uint32_t qkv_stride, float *q_out, __half *k_cache, __half *v_cache,
                      uint32_t cache_stride, const float *cs, const int *pos_ptr, uint32_t pos_val, uint32_t n_tok,
                      uint32_t heads, uint32_t kv_heads, uint32_t hd, int adjacent, cudaStream_t s) {
    dim3 grid(1, n_tok);
    rope_cache_kernel<<<grid, 256, 0, s>>>(qkv, qkv_stride, q_out, k_cache, v_cache, cache_stride, cs, pos_ptr,
                                           pos_val, heads, kv_heads, hd, adjacent);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int attn_pick_nsplit(uint32_t kv_heads, uint32_t max_seq, int sm_count) {
    // CTAs per SM the splits aim at (128 threads, 168 registers: at most 3 fit)
    int per_sm = 2;
    if (const char *e = getenv("CUQ_ATTN_CTAS_PER_SM")) per_sm = atoi(e) > 0 ? atoi(e) : 2;
    int want = (per_sm * sm_count + (int)kv_heads - 1) / (int)kv_heads;
    int maxs = (int)((max_seq + ATT_MIN_CHUNK - 1) / ATT_MIN_CHUNK);
    if (want > maxs) want = maxs;
    if (want > ATT_MAX_SPLIT) want = ATT_MAX_SPLIT;
    if (want < 1) want = 1;
    return want;
}

template <int HD, int G>
static void attn_launch(const float *q, const __half *kc, const __half *vc, uint32_t cs, const int *pp, uint32_t nv,
                        uint32_t heads, uint32_t kvh, float *part, int nsplit, cudaStream_t s) {
    attn_decode_kernel<HD, G><<<dim3(kvh, nsplit), 128, 0, s>>>(q, kc, vc, cs, pp, nv, heads, part, nsplit);
}

int launch_attention_decode(const float *q, const __half *k_cache, const __half *v_cache, uint32_t cache_stride,
                            const int *pos_ptr, uint32_t n_val, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                            float *part, int nsplit, float *out, __half *xq, cudaStream_t s) {
    if (kv_heads == 0 || heads % kv_heads) {
        set_error("attention: heads (%u) must be a multiple of kv_heads (%u)", heads, kv_heads);
        return CUQ_EINVAL;
    }
    if (nsplit < 1 || nsplit > ATT_MAX_SPLIT) {
        set_error("attention: nsplit %d outside 1..%d", nsplit, ATT_MAX_SPLIT);
        return CUQ_EINVAL;
    }
    uint32_t G = heads / kv_heads;
#define CUQ_ATT(HDV, GV)                                                                           \
    if (hd == HDV && G == GV) {                                                                    \
        attn_launch<HDV, GV>(q, k_cache, v_cache, cache_stride, pos_ptr, n_val, heads, kv_heads, part, \
                             nsplit, s);                                                           \
    } else
    CUQ_ATT(64, 1) CUQ_ATT(64, 2) CUQ_ATT(64, 3) CUQ_ATT(64, 4) CUQ_ATT(64, 6) CUQ_ATT(64, 7) CUQ_ATT(64, 8)
    CUQ_ATT(128, 1) CUQ_ATT(128, 2) CUQ_ATT(128, 3) CUQ_ATT(128, 4) CUQ_ATT(128, 6) CUQ_ATT(128, 7)
    CUQ_ATT(128, 8) {
        set_error("attention: unsupported head_dim %u / group %u (head_dim 64 or 128, group 1-8)", hd, G);
        return CUQ_EUNSUPPORTED;
    }
#undef CUQ_ATT
    CUQ_CUDA_TRY(cudaGetLastError());
    if (hd == 64)
        attn_combine_kernel<64><<<heads, 128, 0, s>>>(part, nsplit, pos_ptr, n_val, heads, out, xq,
                                                       xq ? xq_pad(heads * hd) : 0);
    else
        attn_combine_kernel<128><<<heads, 128, 0, s>>>(part, nsplit, pos_ptr, n_val, heads, out, xq,
                                                        xq ? xq_pad(heads * hd) : 0);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_attention_step(const float *qkv, const float *cs, const StepState *state, __half *k_cache,
                          __half *v_cache, uint32_t cache_stride, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                          int adjacent, float *part, int nsplit, unsigned int *tickets, __half *xq, bool pdl,
                          cudaStream_t s) {
    if (kv_heads == 0 || heads % kv_heads) {
        set_error("attention: heads (%u) must be a multiple of kv_heads (%u)", heads, kv_heads);
        return CUQ_EINVAL;
    }
    AttnStepArgs a{qkv, cs, state, k_cache, v_cache, cache_stride, heads, kv_heads, adjacent, nsplit, part, tickets,
                   xq};
    uint32_t G = heads / kv_heads;
    dim3 grid(kv_heads, nsplit);
    cudaError_t e = cudaErrorInvalidValue;
#define CUQ_ATS(HDV, GV) \
    if (hd == HDV && G == GV) e = launch_maybe_pdl(attn_step_kernel<HDV, GV>, grid, dim3(128), 0, s, pdl, a); else
    CUQ_ATS(64, 1) CUQ_ATS(64, 2) CUQ_ATS(64, 3) CUQ_ATS(64, 4) CUQ_ATS(64, 6) CUQ_ATS(64, 7) CUQ_ATS(64, 8)
    CUQ_ATS(128, 1) CUQ_ATS(128, 2) CUQ_ATS(128, 3) CUQ_ATS(128, 4) CUQ_ATS(128, 6) CUQ_ATS(128, 7)
    CUQ_ATS(128, 8) {
        set_error("attention: unsupported head_dim %u / group %u (head_dim 64 or 128, group 1-8)", hd, G);
        return CUQ_EUNSUPPORTED;
    }
#undef CUQ_ATS
    if (e != cudaSuccess) {
        set_error("attention launch: %s", cudaGetErrorString(e));
        return CUQ_ECUDA;
    }
    return CUQ_OK;
}

int launch_rmsnorm_hilo(const float *x, const float *w, uint32_t n, uint32_t n_rows, float eps, __half *hi,
                        __half *lo, cudaStream_t s) {
    if (n_rows == 0) return CUQ_OK;
    rmsnorm_hilo_kernel<<<n_rows, 256, 0, s>>>(x, w, n, eps, hi, lo);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}


int launch_silu_hilo(const float *g, const float *u, size_t count, __half *hi, __half *lo, cudaStream_t s) {
    size_t grid = (count + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    silu_hilo_kernel<<<(unsigned)(grid ? grid : 1), 256, 0, s>>>(g, u, count, hi, lo);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_silu_mul(float *out, const float *g, const float *u, uint32_t n, cudaStream_t s) {
    silu_mul_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, g, u, n);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_argmax(const float *v, uint32_t n, uint32_t *out, cudaStream_t s) {
    argmax_kernel<<<1, 1024, 0, s>>>(v, n, out);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

}  // namespace cuq
