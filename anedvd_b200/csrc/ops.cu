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
// cpu.attentionDecode (cpu.zig:323-395) as split-position flash decoding: CTA
// (kv head, split) covers a contiguous position range for all query heads of
// that KV group (GQA: query head h reads KV head h / (heads / kv_heads)).
// hd/8 lanes share one position (8 dims each, one 16-byte K and V load); a warp
// walks 32/(hd/8) positions at a time with an online softmax; partial (m, l, o)
// go to `part` and the combine kernel merges the splits.  Scores are dot(q, k) * (1 / sqrt(hd)) in fp32.
template <int HD, int G>
__global__ void __launch_bounds__(128) attn_decode_kernel(const float *__restrict__ q, const __half *__restrict__ kc,
                                                           const __half *__restrict__ vc, uint32_t cache_stride,
                                                           const int *pos_ptr, uint32_t n_val, uint32_t heads,
                                                           uint32_t kv_heads, float *part, int nsplit) {
    constexpr int E = 8;            // dims per lane: one 16-byte load of K and of V
    constexpr int LPP = HD / E;     // lanes per position (8 at hd 64, 16 at hd 128)
    constexpr int PPW = 32 / LPP;   // positions a warp walks at once
    const uint32_t kvh = blockIdx.x, split = blockIdx.y;
    const uint32_t n = pos_ptr ? (uint32_t)(*pos_ptr) + 1u : n_val;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lp = lane % LPP, pg = lane / LPP;
    uint32_t chunk = (n + nsplit - 1) / nsplit;
    chunk = (chunk + 15u) & ~15u;
    const uint32_t p0 = split * chunk, p1 = min(n, p0 + chunk);
    const float scale = 1.0f / sqrtf((float)HD);

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
    const __half *kh = kc + (size_t)kvh * cache_stride * HD;
    const __half *vh = vc + (size_t)kvh * cache_stride * HD;
    // The loop bound depends only on the warp, so every lane reaches every
    // shuffle below; lanes whose position is past the end compute on zeros and
    // skip the softmax update.
    for (uint32_t pb = p0 + warp * PPW; pb < p1; pb += 4 * PPW) {
        const uint32_t p = pb + pg;
        const bool valid = p < p1;
        float kf[E], vf[E];
        uint4 ku = make_uint4(0u, 0u, 0u, 0u), vu = make_uint4(0u, 0u, 0u, 0u);
        if (valid) {
            ku = *reinterpret_cast<const uint4 *>(kh + (size_t)p * HD + lp * E);
            vu = *reinterpret_cast<const uint4 *>(vh + (size_t)p * HD + lp * E);
        }
        const __half2 *k2 = reinterpret_cast<const __half2 *>(&ku);
        const __half2 *v2 = reinterpret_cast<const __half2 *>(&vu);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float2 kk = __half22float2(k2[j]), vv = __half22float2(v2[j]);
            kf[2 * j] = kk.x;
            kf[2 * j + 1] = kk.y;
            vf[2 * j] = vv.x;
            vf[2 * j + 1] = vv.y;
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < E; e++) d = fmaf(qr[g][e], kf[e], d);
#pragma unroll
            for (int sh = 1; sh < LPP; sh <<= 1) d += __shfl_xor_sync(0xffffffffu, d, sh);
            if (valid) {  // no shuffles inside: divergence here is harmless
                float s = d * scale;
                float mn = fmaxf(m[g], s);
                float corr = expf(m[g] - mn);  // exp(-inf) = 0 on the first position
                float pe = expf(s - mn);
                l[g] = l[g] * corr + pe;
#pragma unroll
                for (int e = 0; e < E; e++) o[g][e] = o[g][e] * corr + pe * vf[e];
                m[g] = mn;
            }
        }
    }
    // merge the position groups of the warp (lanes lp, lp + LPP, ...)
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
    // merge the 4 warps through shared memory
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
    const size_t stride = HD + 2;
    for (int t = threadIdx.x; t < G * HD; t += blockDim.x) {
        int g = t / HD, dd = t % HD;
        float mm = fmaxf(fmaxf(sm_m[0][g], sm_m[1][g]), fmaxf(sm_m[2][g], sm_m[3][g]));
        float acc = 0.f, ll = 0.f;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            float c = mm == -INFINITY ? 0.f : expf(sm_m[w][g] - mm);
            acc += sm_o[w][g][dd] * c;
            ll += sm_l[w][g] * c;
        }
        float *pp = part + ((size_t)split * heads + kvh * G + g) * stride;
        pp[dd] = acc;
        if (dd == 0) {
            pp[HD] = mm;
            pp[HD + 1] = ll;
        }
    }
}

// Merge the splits: out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s.
__global__ void attn_combine_kernel(const float *__restrict__ part, int nsplit, uint32_t heads, uint32_t hd,
                                    float *out, __half *xq, uint32_t kpad) {
    const uint32_t h = blockIdx.x;
    const size_t stride = hd + 2;
    __shared__ float res[128];  // hd <= 128
    float M = -INFINITY;
    for (int s = 0; s < nsplit; s++) M = fmaxf(M, part[((size_t)s * heads + h) * stride + hd]);
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.f, L = 0.f;
        for (int s = 0; s < nsplit; s++) {
            const float *pp = part + ((size_t)s * heads + h) * stride;
            float c = pp[hd] == -INFINITY ? 0.f : expf(pp[hd] - M);
            acc += pp[d] * c;
            L += pp[hd + 1] * c;
        }
        float r = acc / L;
        uint32_t i = h * hd + d;
        if (out) out[i] = r;
        if (xq) {
            __half hi = __float2half_rn(r);
            __half lo = __float2half_rn(r - __half2float(hi));
            xq[xq_pos(i)] = hi;
            xq[kpad + xq_pos(i)] = lo;
        }
        if (d < 128) res[d] = r;
    }
    if (xq) {  // per-16 sums of this head's outputs (hd is a multiple of 16)
        __syncthreads();
        for (uint32_t u = threadIdx.x; u < hd / 16; u += blockDim.x) {
            float acc = 0.f;
            for (int j = 0; j < 16; j++) acc += res[16 * u + j];
            xq_sums(xq, kpad)[(h * hd) / 16 + u] = acc;
        }
    }
}

// ---------------------------------------------------- fused decode attention
// One decode step's attention for one layer, in one launch (engine.zig:595-612
// + ropeAndCache 952-970 + cpu.attentionDecode 323-395):
//   * every CTA rotates its KV group's queries from the qkv vector itself
//     (RoPE from the host-built cos|sin table, cpu.zig:22-62);
//   * the CTA whose split holds the step's position rotates k, rounds k and v
//     to fp16 and writes them into the cache before it reads that position;
//   * splits run the online softmax as attn_decode_kernel does;
//   * the last split CTA of each KV group to finish (atomic ticket) merges the
//     group's splits and writes the o projection's xq input directly.
struct AttnStepArgs {
    const float *qkv;            // [q | k | v] after bias
    const float *cs;             // [max_seq][hd] cos | sin
    const StepState *state;      // pos
    __half *k_cache, *v_cache;   // [kv_heads][cache_stride][hd]
    uint32_t cache_stride, heads, kv_heads;
    int adjacent, nsplit;
    float *part;                 // [nsplit][heads][hd + 2]
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
    constexpr int E = 8, LPP = HD / E, PPW = 32 / LPP;
    griddep_wait();
    griddep_launch();
    const uint32_t kvh = blockIdx.x, split = blockIdx.y;
    const uint32_t pos = (uint32_t)p.state->pos, n = pos + 1u;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lp = lane % LPP, pg = lane / LPP;
    uint32_t chunk = (n + p.nsplit - 1) / p.nsplit;
    chunk = (chunk + 15u) & ~15u;
    const uint32_t p0 = split * chunk, p1 = min(n, p0 + chunk);
    const float scale = 1.0f / sqrtf((float)HD);
    const uint32_t qd = p.heads * HD, kvd = p.kv_heads * HD;
    const float *csr = p.cs + (size_t)pos * HD;
    __half *kh = p.k_cache + (size_t)kvh * p.cache_stride * HD;
    __half *vh = p.v_cache + (size_t)kvh * p.cache_stride * HD;

    if (pos >= p0 && pos < p1) {  // this CTA owns the new position: write its K/V row
        const float *kin = p.qkv + qd + (size_t)kvh * HD;
        const float *vin = p.qkv + qd + kvd + (size_t)kvh * HD;
        for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x) {
            kh[(size_t)pos * HD + d] = __float2half_rn(rope_elem<HD>(kin, d, csr, p.adjacent));
            vh[(size_t)pos * HD + d] = __float2half_rn(vin[d]);
        }
        __threadfence_block();
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
    for (uint32_t pb = p0 + warp * PPW; pb < p1; pb += 4 * PPW) {  // warp-uniform bound
        const uint32_t pp = pb + pg;
        const bool valid = pp < p1;
        float kf[E], vf[E];
        uint4 ku = make_uint4(0u, 0u, 0u, 0u), vu = make_uint4(0u, 0u, 0u, 0u);
        if (valid) {
            ku = *reinterpret_cast<const uint4 *>(kh + (size_t)pp * HD + lp * E);
            vu = *reinterpret_cast<const uint4 *>(vh + (size_t)pp * HD + lp * E);
        }
        const __half2 *k2 = reinterpret_cast<const __half2 *>(&ku);
        const __half2 *v2 = reinterpret_cast<const __half2 *>(&vu);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float2 kk = __half22float2(k2[j]), vv = __half22float2(v2[j]);
            kf[2 * j] = kk.x;
            kf[2 * j + 1] = kk.y;
            vf[2 * j] = vv.x;
            vf[2 * j + 1] = vv.y;
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < E; e++) d = fmaf(qr[g][e], kf[e], d);
#pragma unroll
            for (int sh = 1; sh < LPP; sh <<= 1) d += __shfl_xor_sync(0xffffffffu, d, sh);
            if (valid) {
                float s = d * scale;
                float mn = fmaxf(m[g], s);
                float corr = expf(m[g] - mn);
                float pe = expf(s - mn);
                l[g] = l[g] * corr + pe;
#pragma unroll
                for (int e = 0; e < E; e++) o[g][e] = o[g][e] * corr + pe * vf[e];
                m[g] = mn;
            }
        }
    }
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
    const size_t stride = HD + 2;
    for (int t = threadIdx.x; t < G * HD; t += blockDim.x) {
        int g = t / HD, dd = t % HD;
        float mm = fmaxf(fmaxf(sm_m[0][g], sm_m[1][g]), fmaxf(sm_m[2][g], sm_m[3][g]));
        float acc = 0.f, ll = 0.f;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            float c = mm == -INFINITY ? 0.f : expf(sm_m[w][g] - mm);
            acc += sm_o[w][g][dd] * c;
            ll += sm_l[w][g] * c;
        }
        float *pp = p.part + ((size_t)split * p.heads + kvh * G + g) * stride;
        pp[dd] = acc;
        if (dd == 0) {
            pp[HD] = mm;
            pp[HD + 1] = ll;
        }
    }
    // the last split of this KV group merges the group's heads
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(&p.tickets[kvh], 1u) == (unsigned)p.nsplit - 1u;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const uint32_t kpad = xq_pad(qd);
    __shared__ float res[G * HD];
    for (int t = threadIdx.x; t < G * HD; t += blockDim.x) {
        int g = t / HD, dd = t % HD;
        uint32_t h = kvh * G + g;
        float M = -INFINITY;
        for (int s = 0; s < p.nsplit; s++) M = fmaxf(M, __ldcg(p.part + ((size_t)s * p.heads + h) * stride + HD));
        float acc = 0.f, L = 0.f;
        for (int s = 0; s < p.nsplit; s++) {
            const float *pp = p.part + ((size_t)s * p.heads + h) * stride;
            float ms = __ldcg(pp + HD);
            float c = ms == -INFINITY ? 0.f : expf(ms - M);
            acc += __ldcg(pp + dd) * c;
            L += __ldcg(pp + HD + 1) * c;
        }
        float r = acc / L;
        uint32_t i = h * HD + dd;
        __half hi = __float2half_rn(r);
        __half lo = __float2half_rn(r - __half2float(hi));
        p.xq[xq_pos(i)] = hi;
        p.xq[kpad + xq_pos(i)] = lo;
        res[t] = r;
    }
    __syncthreads();
    for (int u = threadIdx.x; u < G * HD / 16; u += blockDim.x) {  // per-16 sums (HD % 16 == 0)
        float a = 0.f;
        for (int j = 0; j < 16; j++) a += res[16 * u + j];
        xq_sums(p.xq, kpad)[(kvh * G * HD) / 16 + u] = a;
    }
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

// Causal attention for a chunk of prompt positions (cpu.attentionPrefill,
// cpu.zig:165-217, semantically attentionDecode per position): CTA (kv head,
// query) walks cache positions [0, pos] with the online softmax of
// attn_decode_kernel and writes the normalised result as fp16 hi + lo.
template <int HD, int G>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const float *__restrict__ q, const __half *__restrict__ kc,
                                                            const __half *__restrict__ vc, uint32_t cache_stride,
                                                            uint32_t pos0, uint32_t heads, __half *__restrict__ oh,
                                                            __half *__restrict__ ol) {
    constexpr int E = 8, LPP = HD / E, PPW = 32 / LPP;
    const uint32_t kvh = blockIdx.x, qi = blockIdx.y;
    const uint32_t n = pos0 + qi + 1;  // positions this query sees
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lp = lane % LPP, pg = lane / LPP;
    const float scale = 1.0f / sqrtf((float)HD);
    const uint32_t qd = heads * HD;
    float qr[G][E];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < E; e++) qr[g][e] = q[(size_t)qi * qd + (size_t)(kvh * G + g) * HD + lp * E + e];
    float m[G], l[G], o[G][E];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < E; e++) o[g][e] = 0.f;
    }
    const __half *kh = kc + (size_t)kvh * cache_stride * HD;
    const __half *vh = vc + (size_t)kvh * cache_stride * HD;
    for (uint32_t pb = warp * PPW; pb < n; pb += 4 * PPW) {  // warp-uniform bound
        const uint32_t pp = pb + pg;
        const bool valid = pp < n;
        float kf[E], vf[E];
        uint4 ku = make_uint4(0u, 0u, 0u, 0u), vu = make_uint4(0u, 0u, 0u, 0u);
        if (valid) {
            ku = *reinterpret_cast<const uint4 *>(kh + (size_t)pp * HD + lp * E);
            vu = *reinterpret_cast<const uint4 *>(vh + (size_t)pp * HD + lp * E);
        }
        const __half2 *k2 = reinterpret_cast<const __half2 *>(&ku);
        const __half2 *v2 = reinterpret_cast<const __half2 *>(&vu);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float2 kk = __half22float2(k2[j]), vv = __half22float2(v2[j]);
            kf[2 * j] = kk.x;
            kf[2 * j + 1] = kk.y;
            vf[2 * j] = vv.x;
            vf[2 * j + 1] = vv.y;
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < E; e++) d = fmaf(qr[g][e], kf[e], d);
#pragma unroll
            for (int sh = 1; sh < LPP; sh <<= 1) d += __shfl_xor_sync(0xffffffffu, d, sh);
            if (valid) {
                float s = d * scale;
                float mn = fmaxf(m[g], s);
                float corr = expf(m[g] - mn);
                float pe = expf(s - mn);
                l[g] = l[g] * corr + pe;
#pragma unroll
                for (int e = 0; e < E; e++) o[g][e] = o[g][e] * corr + pe * vf[e];
                m[g] = mn;
            }
        }
    }
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
    for (int t = threadIdx.x; t < G * HD; t += blockDim.x) {
        int g = t / HD, dd = t % HD;
        float mm = fmaxf(fmaxf(sm_m[0][g], sm_m[1][g]), fmaxf(sm_m[2][g], sm_m[3][g]));
        float acc = 0.f, ll = 0.f;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            float c = mm == -INFINITY ? 0.f : expf(sm_m[w][g] - mm);
            acc += sm_o[w][g][dd] * c;
            ll += sm_l[w][g] * c;
        }
        float r = acc / ll;
        size_t i = (size_t)qi * qd + (size_t)(kvh * G + g) * HD + dd;
        __half h = __float2half_rn(r);
        oh[i] = h;
        ol[i] = __float2half_rn(r - __half2float(h));
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
    int maxs = (int)((max_seq + 15) / 16);
    if (want > maxs) want = maxs;
    if (want < 1) want = 1;
    return want;
}

template <int HD, int G>
static void attn_launch(const float *q, const __half *kc, const __half *vc, uint32_t cs, const int *pp, uint32_t nv,
                        uint32_t heads, uint32_t kvh, float *part, int nsplit, cudaStream_t s) {
    attn_decode_kernel<HD, G><<<dim3(kvh, nsplit), 128, 0, s>>>(q, kc, vc, cs, pp, nv, heads, kvh, part, nsplit);
}

int launch_attention_decode(const float *q, const __half *k_cache, const __half *v_cache, uint32_t cache_stride,
                            const int *pos_ptr, uint32_t n_val, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                            float *part, int nsplit, float *out, __half *xq, cudaStream_t s) {
    if (kv_heads == 0 || heads % kv_heads) {
        set_error("attention: heads (%u) must be a multiple of kv_heads (%u)", heads, kv_heads);
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
    attn_combine_kernel<<<heads, hd, 0, s>>>(part, nsplit, heads, hd, out, xq, xq ? xq_pad(heads * hd) : 0);
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

int launch_attention_prefill(const float *q, const __half *k_cache, const __half *v_cache, uint32_t cache_stride,
                             uint32_t pos0, uint32_t n_q, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                             __half *oh, __half *ol, cudaStream_t s) {
    if (kv_heads == 0 || heads % kv_heads) {
        set_error("attention: heads (%u) must be a multiple of kv_heads (%u)", heads, kv_heads);
        return CUQ_EINVAL;
    }
    if (n_q == 0) return CUQ_OK;
    uint32_t G = heads / kv_heads;
    dim3 grid(kv_heads, n_q);
#define CUQ_ATP(HDV, GV) \
    if (hd == HDV && G == GV) attn_prefill_kernel<HDV, GV><<<grid, 128, 0, s>>>(q, k_cache, v_cache, cache_stride, pos0, heads, oh, ol); else
    CUQ_ATP(64, 1) CUQ_ATP(64, 2) CUQ_ATP(64, 3) CUQ_ATP(64, 4) CUQ_ATP(64, 6) CUQ_ATP(64, 7) CUQ_ATP(64, 8)
    CUQ_ATP(128, 1) CUQ_ATP(128, 2) CUQ_ATP(128, 3) CUQ_ATP(128, 4) CUQ_ATP(128, 6) CUQ_ATP(128, 7)
    CUQ_ATP(128, 8) {
        set_error("attention: unsupported head_dim %u / group %u (head_dim 64 or 128, group 1-8)", hd, G);
        return CUQ_EUNSUPPORTED;
    }
#undef CUQ_ATP
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
