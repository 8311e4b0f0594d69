// ops.cu -- RMSNorm, RoPE + KV-cache write, decode attention, SiLU, argmax, embedding.
//
// Each kernel restates one reference CPU op (src/cpu.zig) and names it.  The
// KV cache is fp16 like the reference's (engine.zig:447-458, 952-970) but laid
// out [kv_head][position][head_dim] so one head's keys are contiguous.
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

__global__ void rope_kernel(float *v, uint32_t heads, uint32_t hd, const float *__restrict__ cs_row, int adjacent) {
    const uint32_t half = hd / 2;
    for (uint32_t t = threadIdx.x + blockIdx.x * blockDim.x; t < heads * half; t += blockDim.x * gridDim.x) {
        uint32_t h = t / half, i = t % half;
        float c = cs_row[i], s = cs_row[half + i];
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

// ------------------------------------------------------------ attention ---
// cpu.attentionDecode (cpu.zig:323-395) as split-position flash decoding.  CTA
// (kv head, split) covers a contiguous range of cache positions for every query
// head of that KV group (GQA: query head h reads KV head h / (heads / kv_heads)).
// hd/8 lanes share one position (8 dims each: one 16-byte K and V load); a warp
// walks U * 32/(hd/8) positions per iteration with all their loads issued before
// the math, and keeps an online softmax (m, l, o).  Scores are dot(q, k) *
// (1 / sqrt(hd)) in fp32.  Splits write partial (o, m, l) to `part`:
//   part[s][h][hd] (unnormalised o), then at part + nsplit*heads*hd: [s][h][2] (m, l).
// Splits cover at least ATT_MIN_CHUNK positions, so a short context uses few
// splits and the merge reads few partials.
constexpr uint32_t ATT_MIN_CHUNK = 32;
constexpr int ATT_MAX_SPLIT = 64;

struct SplitRange {
    uint32_t p0, p1, nact;
};

__device__ __forceinline__ SplitRange split_range(uint32_t n, int nsplit, uint32_t split) {
    uint32_t chunk = (n + (uint32_t)nsplit - 1) / (uint32_t)nsplit;
    chunk = (chunk + 15u) & ~15u;
    if (chunk < ATT_MIN_CHUNK) chunk = ATT_MIN_CHUNK;
    SplitRange r;
    r.nact = (n + chunk - 1) / chunk;
    r.p0 = split * chunk;
    r.p1 = min(n, r.p0 + chunk);
    return r;
}

// Walk positions [p0, p1) of one KV head with this CTA's 4 warps.  Warp-uniform
// loop bound: every lane reaches every shuffle; lanes past the end load zeros
// and score -inf.
template <int HD, int G>
__device__ __forceinline__ void attn_walk(const float (&qr)[G][8], const __half *kh, const __half *vh, uint32_t p0,
                                          uint32_t p1, int warp, int lp, int pg, float (&m)[G], float (&l)[G],
                                          float (&o)[G][8]) {
    constexpr int E = 8, LPP = HD / E, PPW = 32 / LPP, U = G <= 4 ? 4 : 2;
    const float scale = 1.0f / sqrtf((float)HD);
    for (uint32_t pb = p0 + (uint32_t)warp * PPW * U; pb < p1; pb += 4u * PPW * U) {
        uint4 ku[U], vu[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const uint32_t p = pb + u * PPW + pg;
            ku[u] = make_uint4(0u, 0u, 0u, 0u);
            vu[u] = ku[u];
            if (p < p1) {
                ku[u] = *reinterpret_cast<const uint4 *>(kh + (size_t)p * HD + lp * E);
                vu[u] = *reinterpret_cast<const uint4 *>(vh + (size_t)p * HD + lp * E);
            }
        }
        float s[U][G];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const __half2 *k2 = reinterpret_cast<const __half2 *>(&ku[u]);
            float kf[E];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float2 kk = __half22float2(k2[j]);
                kf[2 * j] = kk.x;
                kf[2 * j + 1] = kk.y;
            }
            const bool valid = pb + u * PPW + pg < p1;
#pragma unroll
            for (int g = 0; g < G; g++) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < E; e++) d = fmaf(qr[g][e], kf[e], d);
#pragma unroll
                for (int sh = 1; sh < LPP; sh <<= 1) d += __shfl_xor_sync(0xffffffffu, d, sh);
                s[u][g] = valid ? d * scale : -INFINITY;
            }
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            float mx = s[0][g];
#pragma unroll
            for (int u = 1; u < U; u++) mx = fmaxf(mx, s[u][g]);
            const float mn = fmaxf(m[g], mx);
            if (mn == -INFINITY) continue;  // nothing valid yet (no shuffles below)
            const float corr = expf(m[g] - mn);
            l[g] *= corr;
#pragma unroll
            for (int e = 0; e < E; e++) o[g][e] *= corr;
#pragma unroll
            for (int u = 0; u < U; u++) {
                const float pe = expf(s[u][g] - mn);  // 0 for an invalid lane
                const __half2 *v2 = reinterpret_cast<const __half2 *>(&vu[u]);
                l[g] += pe;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float2 vv = __half22float2(v2[j]);
                    o[g][2 * j] = fmaf(pe, vv.x, o[g][2 * j]);
                    o[g][2 * j + 1] = fmaf(pe, vv.y, o[g][2 * j + 1]);
                }
            }
            m[g] = mn;
        }
    }
}

// Merge the lanes of each warp and the CTA's 4 warps; write the split's partial
// (o, m, l) for query heads kvh*G .. kvh*G+G-1.
template <int HD, int G>
__device__ __forceinline__ void attn_store_split(float (&m)[G], float (&l)[G], float (&o)[G][8], int warp, int lp,
                                                 int pg, float *part, uint32_t split, int nsplit, uint32_t heads,
                                                 uint32_t kvh) {
    constexpr int E = 8, LPP = HD / E;
#pragma unroll
    for (int g = 0; g < G; g++) {
#pragma unroll
        for (int sh = LPP; sh < 32; sh <<= 1) {
            float mo = __shfl_xor_sync(0xffffffffu, m[g], sh);
            float lo = __shfl_xor_sync(0xffffffffu, l[g], sh);
            float mn = fmaxf(m[g], mo);
            float ca = mn == -INFINITY ? 0.f : expf(m[g] - mn);
            float cb = mn == -INFINITY ? 0.f : expf(mo - mn);
            l[g] = l[g] * ca + lo * cb;
#pragma unroll
            for (int e = 0; e < E; e++) {
                float oo = __shfl_xor_sync(0xffffffffu, o[g][e], sh);
                o[g][e] = o[g][e] * ca + oo * cb;
            }
            m[g] = mn;
        }
    }
    __shared__ float sm_m[4][G], sm_l[4][G], sm_o[4][G][HD];
    if (pg == 0) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            if (lp == 0) {
                sm_m[warp][g] = m[g];
                sm_l[warp][g] = l[g];
            }
#pragma unroll
            for (int e = 0; e < E; e++) sm_o[warp][g][lp * E + e] = o[g][e];
        }
    }
    __syncthreads();
    float *po = part + ((size_t)split * heads + kvh * G) * HD;
    float *pml = part + (size_t)nsplit * heads * HD + ((size_t)split * heads + kvh * G) * 2;
    for (int t = threadIdx.x; t < G * HD; t += blockDim.x) {
        const int g = t / HD, dd = t % HD;
        const float mm = fmaxf(fmaxf(sm_m[0][g], sm_m[1][g]), fmaxf(sm_m[2][g], sm_m[3][g]));
        float acc = 0.f, ll = 0.f;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const float c = mm == -INFINITY ? 0.f : expf(sm_m[w][g] - mm);
            acc += sm_o[w][g][dd] * c;
            ll += sm_l[w][g] * c;
        }
        po[t] = acc;
        if (dd == 0) {
            pml[2 * g] = mm;
            pml[2 * g + 1] = ll;
        }
    }
}

// Merge the nact splits of query heads h0 .. h0+NH-1 (one CTA, any size):
// out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s.  Every split's weight is
// computed once into shared memory, then each thread sums float4 columns with
// independent loads.  `res` receives the NH*HD results.
template <int HD, int NH>
__device__ __forceinline__ void attn_merge(const float *part, int nsplit, uint32_t nact, uint32_t heads, uint32_t h0,
                                           float *res) {
    __shared__ float cw[ATT_MAX_SPLIT][NH];
    __shared__ float inv_l[NH];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float *pml = part + (size_t)nsplit * heads * HD;
    for (int g = warp; g < NH; g += nw) {
        const uint32_t h = h0 + g;
        float ms[2], ls[2];
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const uint32_t s = lane + 32 * j;
            ms[j] = s < nact ? __ldcg(pml + ((size_t)s * heads + h) * 2) : -INFINITY;
            ls[j] = s < nact ? __ldcg(pml + ((size_t)s * heads + h) * 2 + 1) : 0.f;
            M = fmaxf(M, ms[j]);
        }
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
        float L = 0.f;
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const uint32_t s = lane + 32 * j;
            const float c = ms[j] == -INFINITY ? 0.f : expf(ms[j] - M);
            if (s < nact) cw[s][g] = c;
            L += ls[j] * c;
        }
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sh);
        if (lane == 0) inv_l[g] = 1.0f / L;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < NH * HD / 4; t += blockDim.x) {
        const int g = t / (HD / 4), d4 = t % (HD / 4);
        const float4 *src = reinterpret_cast<const float4 *>(part + (size_t)(h0 + g) * HD) + d4;
        const size_t sstride = (size_t)heads * HD / 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (uint32_t s = 0; s < nact; s++) {
            const float4 v = __ldcg(src + s * sstride);
            const float c = cw[s][g];
            acc.x = fmaf(v.x, c, acc.x);
            acc.y = fmaf(v.y, c, acc.y);
            acc.z = fmaf(v.z, c, acc.z);
            acc.w = fmaf(v.w, c, acc.w);
        }
        const float il = inv_l[g];
        res[4 * t] = acc.x * il;
        res[4 * t + 1] = acc.y * il;
        res[4 * t + 2] = acc.z * il;
        res[4 * t + 3] = acc.w * il;
    }
    __syncthreads();
}

// Write merged head outputs as the o projection's xq input (hi/lo + per-16 sums)
// and/or fp32.  `res` holds NH*HD values for columns c0 .. c0+NH*HD-1.
__device__ __forceinline__ void attn_emit(const float *res, uint32_t count, uint32_t c0, float *out, __half *xq,
                                          uint32_t kpad) {
    for (uint32_t t = threadIdx.x; t < count; t += blockDim.x) {
        const float r = res[t];
        const uint32_t i = c0 + t;
        if (out) out[i] = r;
        if (xq) {
            const __half hi = __float2half_rn(r);
            xq[xq_pos(i)] = hi;
            xq[kpad + xq_pos(i)] = __float2half_rn(r - __half2float(hi));
        }
    }
    if (xq) {  // c0 and count are multiples of 16
        for (uint32_t u = threadIdx.x; u < count / 16; u += blockDim.x) {
            float a = 0.f;
            for (int j = 0; j < 16; j++) a += res[16 * u + j];
            xq_sums(xq, kpad)[c0 / 16 + u] = a;
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
    attn_store_split<HD, G>(m, l, o, warp, lp, pg, part, split, nsplit, heads, kvh);
}

// Merge for the standalone decode attention: CTA per query head.
template <int HD>
__global__ void __launch_bounds__(128) attn_combine_kernel(const float *__restrict__ part, int nsplit,
                                                            const int *pos_ptr, uint32_t n_val, uint32_t heads,
                                                            float *out, __half *xq, uint32_t kpad) {
    __shared__ float res[HD];
    const uint32_t n = pos_ptr ? (uint32_t)(*pos_ptr) + 1u : n_val;
    const SplitRange r = split_range(n, nsplit, 0);
    attn_merge<HD, 1>(part, nsplit, r.nact, heads, blockIdx.x, res);
    attn_emit(res, HD, blockIdx.x * HD, out, xq, kpad);
}

// ---------------------------------------------------- fused decode attention
// One decode step's attention for one layer, in one launch (engine.zig:595-612
// + ropeAndCache 952-970 + cpu.attentionDecode 323-395):
//   * every CTA rotates its KV group's queries from the qkv vector itself
//     (RoPE from the host-built cos|sin table, cpu.zig:22-62);
//   * the CTA whose split holds the step's position rotates k, rounds k and v
//     to fp16 and writes them into the cache before it reads that position;
//   * splits run attn_walk as attn_decode_kernel does;
//   * the last split CTA of each KV group to finish (atomic ticket) merges the
//     group's splits and writes the o projection's xq input directly.
struct AttnStepArgs {
    const float *qkv;            // [q | k | v] after bias
    const float *cs;             // [max_seq][hd] cos | sin
    const StepState *state;      // pos
    __half *k_cache, *v_cache;   // [kv_heads][cache_stride][hd]
    uint32_t cache_stride, heads, kv_heads;
    int adjacent, nsplit;
    float *part;                 // nsplit * heads * (hd + 2) floats
    unsigned int *tickets;       // [kv_heads], self-resetting
    __half *xq;                  // o-projection input (heads*hd columns)
};

template <int HD>
__device__ __forceinline__ float rope_elem(const float *v, uint32_t d, const float *csr, int adjacent) {
    // rotated element d of one head vector `v` (cpu.zig:33-36 / 57-60)
    constexpr uint32_t half = HD / 2;
    if (adjacent) {
        uint32_t j = d >> 1;
        float a = v[2 * j], b = v[2 * j + 1], c = csr[j], s = csr[half + j];
        return (d & 1) ? __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c)) : __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    }
    uint32_t i = d < half ? d : d - half;
    float a = v[i], b = v[i + half], c = csr[i], s = csr[half + i];
    return d < half ? __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)) : __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

template <int HD, int G>
__global__ void __launch_bounds__(128) attn_step_kernel(const AttnStepArgs p) {
    constexpr int E = 8, LPP = HD / E;
    griddep_wait();
    griddep_launch();
    const uint32_t kvh = blockIdx.x, split = blockIdx.y;
    const uint32_t pos = (uint32_t)p.state->pos, n = pos + 1u;
    const SplitRange r = split_range(n, p.nsplit, split);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lp = lane % LPP, pg = lane / LPP;
    const uint32_t qd = p.heads * HD, kvd = p.kv_heads * HD;
    const float *csr = p.cs + (size_t)pos * HD;
    __half *kh = p.k_cache + (size_t)kvh * p.cache_stride * HD;
    __half *vh = p.v_cache + (size_t)kvh * p.cache_stride * HD;

    if (split < r.nact) {
        if (pos >= r.p0 && pos < r.p1) {  // this CTA owns the new position: write its K/V row
            const float *kin = p.qkv + qd + (size_t)kvh * HD;
            const float *vin = p.qkv + qd + kvd + (size_t)kvh * HD;
            for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x) {
                kh[(size_t)pos * HD + d] = __float2half_rn(rope_elem<HD>(kin, d, csr, p.adjacent));
                vh[(size_t)pos * HD + d] = __float2half_rn(vin[d]);
            }
        }
        float qr[G][E];
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float *qh = p.qkv + (size_t)(kvh * G + g) * HD;
#pragma unroll
            for (int e = 0; e < E; e++) qr[g][e] = rope_elem<HD>(qh, lp * E + e, csr, p.adjacent);
        }
        __syncthreads();  // the K/V row written above is read below
        float m[G], l[G], o[G][E];
#pragma unroll
        for (int g = 0; g < G; g++) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int e = 0; e < E; e++) o[g][e] = 0.f;
        }
        attn_walk<HD, G>(qr, kh, vh, r.p0, r.p1, warp, lp, pg, m, l, o);
        attn_store_split<HD, G>(m, l, o, warp, lp, pg, p.part, split, p.nsplit, p.heads, kvh);
    }
    // the last CTA of this KV group (active or not) merges the group's heads
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(&p.tickets[kvh], 1u) == (unsigned)p.nsplit - 1u;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    __shared__ float res[G * HD];
    attn_merge<HD, G>(p.part, p.nsplit, r.nact, p.heads, kvh * G, res);
    attn_emit(res, G * HD, kvh * G * HD, nullptr, p.xq, xq_pad(qd));
    if (threadIdx.x == 0) p.tickets[kvh] = 0u;
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

int launch_rope(float *v, uint32_t heads, uint32_t hd, const float *cs_row, int adjacent, cudaStream_t s) {
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
    int want = (2 * sm_count + (int)kv_heads - 1) / (int)kv_heads;
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
