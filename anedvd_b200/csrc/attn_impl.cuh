// attn_impl.cuh -- device code of the decode attention (split flash decoding
// with an in-kernel merge), shared by ops.cu and the persistent decode kernel.
#pragma once

#include "common.cuh"

namespace cuq {

namespace {

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
constexpr int ATT_MAX_SPLIT = 128;
// Contexts up to this many positions are walked by one CTA per KV group, which
// then writes the result directly (no partials, no merge).
constexpr uint32_t ATT_DIRECT_MAX = 128;

struct SplitRange {
    uint32_t p0, p1, nact;
};

__device__ __forceinline__ SplitRange split_range(uint32_t n, int nsplit, uint32_t split) {
    uint32_t chunk = (n + (uint32_t)nsplit - 1) / (uint32_t)nsplit;
    chunk = (chunk + 15u) & ~15u;
    if (chunk < ATT_MIN_CHUNK) chunk = ATT_MIN_CHUNK;
    if (n <= ATT_DIRECT_MAX) chunk = n;  // one split
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
    constexpr uint32_t STEP = 4u * PPW * U;  // positions per iteration of the CTA's 4 warps
    const float scale = 1.0f / sqrtf((float)HD);
    // K/V of this warp's positions pb + u*PPW + pg; the next iteration's are
    // loaded before this one computes, so the walk keeps one round trip in flight
    auto fetch = [&](uint32_t pb, uint4 (&kx)[U], uint4 (&vx)[U]) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const uint32_t p = pb + u * PPW + pg;
            kx[u] = make_uint4(0u, 0u, 0u, 0u);
            vx[u] = kx[u];
            if (p < p1) {
                kx[u] = *reinterpret_cast<const uint4 *>(kh + (size_t)p * HD + lp * E);
                vx[u] = *reinterpret_cast<const uint4 *>(vh + (size_t)p * HD + lp * E);
            }
        }
    };
    uint4 kn[U], vn[U];
    const uint32_t pb0 = p0 + (uint32_t)warp * PPW * U;
    if (pb0 < p1) fetch(pb0, kn, vn);
    for (uint32_t pb = pb0; pb < p1; pb += STEP) {
        uint4 ku[U], vu[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            ku[u] = kn[u];
            vu[u] = vn[u];
        }
        if (pb + STEP < p1) fetch(pb + STEP, kn, vn);
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

// Shared-memory scratch (floats) of the split store, the merge and the fused
// step body for a group of G query heads of dimension HD.  The kernels own it
// (a static array, or a slice of the persistent kernel's dynamic shared memory
// that other phases reuse), so instantiations do not each add static memory.
constexpr int attn_store_floats(int HD, int G) { return 8 * G + 4 * G * HD; }
constexpr int attn_merge_floats(int NH) { return (ATT_MAX_SPLIT + 4) * NH; }  // cw, inv_l (16-byte aligned end)
constexpr int attn_step_floats(int HD, int G) {
    // the direct path keeps its result after the store scratch; the merge path after the merge scratch
    return attn_store_floats(HD, G) > attn_merge_floats(G) ? attn_store_floats(HD, G) + G * HD
                                                           : attn_merge_floats(G) + G * HD;
}

template <int HD, int G>
__device__ __forceinline__ void attn_store_cta(float *part, uint32_t split, int nsplit, uint32_t heads, uint32_t kvh,
                                               float *scr, float *direct);

// Merge the lanes of each warp and the CTA's 4 warps; write the split's partial
// (o, m, l) for query heads kvh*G .. kvh*G+G-1, or, when `direct` is set (the
// split is the whole context), the final o / l into direct[0 .. G*HD).
// scr: attn_store_floats(HD, G).
template <int HD, int G>
__device__ __forceinline__ void attn_store_split(float (&m)[G], float (&l)[G], float (&o)[G][8], int warp, int lp,
                                                 int pg, float *part, uint32_t split, int nsplit, uint32_t heads,
                                                 uint32_t kvh, float *scr, float *direct = nullptr) {
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
    float(*sm_m)[G] = reinterpret_cast<float(*)[G]>(scr);
    float(*sm_l)[G] = reinterpret_cast<float(*)[G]>(scr + 4 * G);
    float(*sm_o)[G][HD] = reinterpret_cast<float(*)[G][HD]>(scr + 8 * G);
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
    attn_store_cta<HD, G>(part, split, nsplit, heads, kvh, scr, direct);
}

// Combine the 4 warps' (m, l, o) of each head from shared memory (scr: per warp
// m[G], then l[G], then o[G][HD]) into the split's partial, or, with `direct`,
// the final result.
template <int HD, int G>
__device__ __forceinline__ void attn_store_cta(float *part, uint32_t split, int nsplit, uint32_t heads, uint32_t kvh,
                                               float *scr, float *direct) {
    float(*sm_m)[G] = reinterpret_cast<float(*)[G]>(scr);
    float(*sm_l)[G] = reinterpret_cast<float(*)[G]>(scr + 4 * G);
    float(*sm_o)[G][HD] = reinterpret_cast<float(*)[G][HD]>(scr + 8 * G);
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
        if (direct) {
            direct[t] = acc * (1.0f / ll);  // as attn_merge does for a single split
            continue;
        }
        po[t] = acc;
        if (dd == 0) {
            pml[2 * g] = mm;
            pml[2 * g + 1] = ll;
        }
    }
}

// ------------------------------------------------ tensor-core decode walk ---
// The online softmax of attn_walk with both contractions on mma.sync m16n8k16
// (fp16 operands, fp32 accumulation), 16 positions per warp at a time.
//   Scores: S (16 rows x 8 positions, two tiles) = Q . K^T.  Row g < G holds
//   query head g's fp32 q rounded to fp16 (hi), row 8 + g the remainder q - hi
//   (lo), so S[g] + S[8 + g] is the fp32 dot product to about 2^-22 |q||k| (K is
//   fp16 in the cache; the tensor core multiplies fp16 exactly and adds in fp32).
//   Output: O (16 rows x HD) += P . V with P split the same way (row g: fp16(p),
//   row 8 + g: p - fp16(p)); the head's result is O[g] + O[8 + g].
// A lane loads 16 contiguous bytes of each K row it needs: the dims of one
// k-step are permuted accordingly (the dot product does not depend on their
// order), k-step 2b + h taking dims 32b + 8*q4 + 4h + {0,1} (A cols 2*q4 +
// {0,1}) and + {2,3} (cols 2*q4 + 8 + {0,1}).  For V it loads 16 bytes of four
// position rows and packs the two positions of each dim with byte_perm; column
// n of output tile T is dim 64*(T/8) + 8n + T%8.
__device__ __forceinline__ void attn_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16 hi / lo halves of two floats, packed (first value in the low half)
__device__ __forceinline__ void attn_split2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 r = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&r);
}

__host__ __device__ constexpr int attn_tc_dim(int T, int n) { return 64 * (T / 8) + 8 * n + (T % 8); }

// Walk positions [p0, p1) of one KV head: warp `warp` of the CTA's 4 takes the
// 16-position tiles p0 + 16*(warp + 4i).  qs: the G rotated query heads (fp32,
// G * HD in shared memory).  Returns the lane's row max m (shared by the 4
// lanes of a row), its partial row sum l and the O fragments.
template <int HD, int G>
__device__ __forceinline__ void attn_walk_tc(const float *qs, const __half *kh, const __half *vh, uint32_t p0,
                                             uint32_t p1, int warp, float &m, float &l, float (&o)[HD / 8][4]) {
    static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
    static_assert(G >= 1 && G <= 8, "1 to 8 query heads per KV head");
    constexpr int NKB = HD / 32, NT = HD / 8, NH = HD / 64;
    const int lane = threadIdx.x & 31, g4 = lane >> 2, q4 = lane & 3;
    const float scale = 1.0f / sqrtf((float)HD);
    uint32_t qa[NKB][2][4];  // A fragments of Q, constant over the walk
#pragma unroll
    for (int b = 0; b < NKB; b++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (g4 < G) {
#pragma unroll
                for (int e = 0; e < 4; e++) v[e] = qs[g4 * HD + 32 * b + 8 * q4 + 4 * h + e];
            }
            attn_split2(v[0], v[1], qa[b][h][0], qa[b][h][1]);
            attn_split2(v[2], v[3], qa[b][h][2], qa[b][h][3]);
        }
    }
    m = -INFINITY;
    l = 0.f;
#pragma unroll
    for (int t = 0; t < NT; t++) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    // K rows t0 + 8j + g4 (dims 32b + 8*q4 ..); V rows t0 + 8*(r/2) + 2*q4 + r%2
    // (dims 64h + 8*g4 ..).  The next tile's rows are requested before this
    // tile's math, so a warp keeps one tile in flight while it computes.
    uint4 kn[2][NKB], vn[4][NH];
    auto fetch = [&](uint32_t t0) {
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const uint32_t p = t0 + 8u * j + g4;
#pragma unroll
            for (int b = 0; b < NKB; b++)
                kn[j][b] = p < p1 ? *reinterpret_cast<const uint4 *>(kh + (size_t)p * HD + 32 * b + 8 * q4) : z;
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const uint32_t p = t0 + 8u * (r >> 1) + 2u * q4 + (r & 1);
#pragma unroll
            for (int h = 0; h < NH; h++)
                vn[r][h] = p < p1 ? *reinterpret_cast<const uint4 *>(vh + (size_t)p * HD + 64 * h + 8 * g4) : z;
        }
    };
    if (p0 + 16u * (uint32_t)warp < p1) fetch(p0 + 16u * (uint32_t)warp);
    for (uint32_t t0 = p0 + 16u * (uint32_t)warp; t0 < p1; t0 += 64u) {
        uint4 kx[2][NKB], vx[4][NH];
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int b = 0; b < NKB; b++) kx[j][b] = kn[j][b];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int h = 0; h < NH; h++) vx[r][h] = vn[r][h];
        if (t0 + 64u < p1) fetch(t0 + 64u);
        float s[2][4];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
            for (int b = 0; b < NKB; b++) {
                const uint32_t *kw = reinterpret_cast<const uint32_t *>(&kx[j][b]);
                attn_mma(s[j], qa[b][0], kw[0], kw[1]);
                attn_mma(s[j], qa[b][1], kw[2], kw[3]);
            }
        }
        // the lane's positions: t0 + 2*q4 + {0,1} (tile 0) and t0 + 8 + 2*q4 + {0,1} (tile 1)
        float sc[4];
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int e = 0; e < 2; e++)
                sc[2 * j + e] = t0 + 8u * j + 2u * q4 + e < p1 ? (s[j][e] + s[j][2 + e]) * scale : -INFINITY;
        float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);  // finite: position t0 is valid
        const float corr = expf(m - mn);
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; i++) pr[i] = expf(sc[i] - mn);
        l = l * corr + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
        m = mn;
        uint32_t pa[4];
        attn_split2(pr[0], pr[1], pa[0], pa[1]);
        attn_split2(pr[2], pr[3], pa[2], pa[3]);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const int h = t / 8, e = t % 8;
            const uint32_t sel = (e & 1) ? 0x7632u : 0x5410u;
            const uint32_t b0 = __byte_perm(reinterpret_cast<const uint32_t *>(&vx[0][h])[e >> 1],
                                            reinterpret_cast<const uint32_t *>(&vx[1][h])[e >> 1], sel);
            const uint32_t b1 = __byte_perm(reinterpret_cast<const uint32_t *>(&vx[2][h])[e >> 1],
                                            reinterpret_cast<const uint32_t *>(&vx[3][h])[e >> 1], sel);
#pragma unroll
            for (int i = 0; i < 4; i++) o[t][i] *= corr;
            attn_mma(o[t], pa, b0, b1);
        }
    }
}

// The walk's state into the shared-memory layout of attn_store_split (per warp
// m, l and o of each of the G heads), then the CTA's combine.
template <int HD, int G>
__device__ __forceinline__ void attn_store_split_tc(float m, float l, const float (&o)[HD / 8][4], int warp,
                                                    float *part, uint32_t split, int nsplit, uint32_t heads,
                                                    uint32_t kvh, float *scr, float *direct = nullptr) {
    const int lane = threadIdx.x & 31, g4 = lane >> 2, q4 = lane & 3;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    float(*sm_m)[G] = reinterpret_cast<float(*)[G]>(scr);
    float(*sm_l)[G] = reinterpret_cast<float(*)[G]>(scr + 4 * G);
    float(*sm_o)[G][HD] = reinterpret_cast<float(*)[G][HD]>(scr + 8 * G);
    if (g4 < G) {
        if (q4 == 0) {
            sm_m[warp][g4] = m;
            sm_l[warp][g4] = l;
        }
#pragma unroll
        for (int t = 0; t < HD / 8; t++)
#pragma unroll
            for (int e = 0; e < 2; e++) sm_o[warp][g4][attn_tc_dim(t, 2 * q4 + e)] = o[t][e] + o[t][2 + e];
    }
    attn_store_cta<HD, G>(part, split, nsplit, heads, kvh, scr, direct);
}

// Merge the nact splits of query heads h0 .. h0+NH-1 (one CTA, any size):
// out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s.  Every split's weight is
// computed once into shared memory, then each thread sums float4 columns in
// split order, MB splits' loads in flight at a time; the first MB of its first
// column are requested before the weights are computed.  `res` receives the
// NH*HD results; scr: attn_merge_floats(NH), not overlapping res.
template <int HD, int NH, int MB = 8>
__device__ __forceinline__ void attn_merge(const float *part, int nsplit, uint32_t nact, uint32_t heads, uint32_t h0,
                                           float *res, float *scr) {
    float(*cw)[NH] = reinterpret_cast<float(*)[NH]>(scr);
    float *inv_l = scr + ATT_MAX_SPLIT * NH;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float *pml = part + (size_t)nsplit * heads * HD;
    const int ncol = NH * HD / 4;
    const size_t sstride = (size_t)heads * HD / 4;
    auto column = [&](int t) { return reinterpret_cast<const float4 *>(part + (size_t)(h0 + t / (HD / 4)) * HD) + t % (HD / 4); };
    float4 v[MB];
    auto load = [&](const float4 *src, uint32_t s0) {
#pragma unroll
        for (int j = 0; j < MB; j++)
            v[j] = s0 + j < nact ? __ldcg(src + (s0 + j) * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    if ((int)threadIdx.x < ncol) load(column(threadIdx.x), 0);
    for (int g = warp; g < NH; g += nw) {
        const uint32_t h = h0 + g;
        constexpr int J = ATT_MAX_SPLIT / 32;
        float ms[J], ls[J];
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < J; j++) {
            const uint32_t s = lane + 32 * j;
            ms[j] = s < nact ? __ldcg(pml + ((size_t)s * heads + h) * 2) : -INFINITY;
            ls[j] = s < nact ? __ldcg(pml + ((size_t)s * heads + h) * 2 + 1) : 0.f;
            M = fmaxf(M, ms[j]);
        }
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
        float L = 0.f;
#pragma unroll
        for (int j = 0; j < J; j++) {
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
    for (int t = threadIdx.x; t < ncol; t += blockDim.x) {
        const int g = t / (HD / 4);
        const float4 *src = column(t);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t s0 = 0; s0 < nact; s0 += MB) {
            if (t != (int)threadIdx.x || s0 != 0) load(src, s0);
#pragma unroll
            for (int j = 0; j < MB; j++) {
                if (s0 + j >= nact) break;
                const float c = cw[s0 + j][g];
                acc.x = fmaf(v[j].x, c, acc.x);
                acc.y = fmaf(v[j].y, c, acc.y);
                acc.z = fmaf(v[j].z, c, acc.z);
                acc.w = fmaf(v[j].w, c, acc.w);
            }
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

// KV group kvh, position split `split` of the step at position pos; scr:
// attn_step_floats(HD, G) floats of shared memory.  TC: the tensor-core walk
// (about 250 registers per thread), else the FMA walk (fits the persistent
// kernel's 128).
template <int HD, int G, bool TC = false>
__device__ __forceinline__ void attn_step_body(const AttnStepArgs &p, uint32_t kvh, uint32_t split, uint32_t pos,
                                               float *scr) {
    constexpr int E = 8, LPP = HD / E;
    const uint32_t n = pos + 1u;
    const SplitRange r = split_range(n, p.nsplit, split);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lp = lane % LPP, pg = lane / LPP;
    const uint32_t qd = p.heads * HD, kvd = p.kv_heads * HD;
    const float *csr = p.cs + (size_t)pos * HD;
    __half *kh = p.k_cache + (size_t)kvh * p.cache_stride * HD;
    __half *vh = p.v_cache + (size_t)kvh * p.cache_stride * HD;

    const bool direct = r.nact == 1;  // one CTA per KV group: it writes the output itself
    if (direct && split != 0) return;
    if (split < r.nact) {
        if (pos >= r.p0 && pos < r.p1) {  // this CTA owns the new position: write its K/V row
            const float *kin = p.qkv + qd + (size_t)kvh * HD;
            const float *vin = p.qkv + qd + kvd + (size_t)kvh * HD;
            for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x) {
                kh[(size_t)pos * HD + d] = __float2half_rn(rope_elem<HD>(kin, d, csr, p.adjacent));
                vh[(size_t)pos * HD + d] = __float2half_rn(vin[d]);
            }
        }
        if constexpr (TC) {
            // the G rotated query heads in shared memory, after the store scratch
            // (the direct result later takes the same place, after the store's barrier)
            float *qs = scr + attn_store_floats(HD, G);
            for (uint32_t i = threadIdx.x; i < (uint32_t)(G * HD); i += blockDim.x)
                qs[i] = rope_elem<HD>(p.qkv + (size_t)(kvh * G) * HD + (i / HD) * HD, i % HD, csr, p.adjacent);
            __syncthreads();  // qs, and the K/V row written above, are read below
            float m, l, o[HD / 8][4];
            attn_walk_tc<HD, G>(qs, kh, vh, r.p0, r.p1, warp, m, l, o);
            if (direct) {
                float *res = scr + attn_store_floats(HD, G);
                attn_store_split_tc<HD, G>(m, l, o, warp, p.part, split, p.nsplit, p.heads, kvh, scr, res);
                __syncthreads();
                attn_emit(res, G * HD, kvh * G * HD, nullptr, p.xq, xq_pad(qd));
                return;
            }
            attn_store_split_tc<HD, G>(m, l, o, warp, p.part, split, p.nsplit, p.heads, kvh, scr);
        } else {
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
        if (direct) {
            float *res = scr + attn_store_floats(HD, G);
            attn_store_split<HD, G>(m, l, o, warp, lp, pg, p.part, split, p.nsplit, p.heads, kvh, scr, res);
            __syncthreads();
            attn_emit(res, G * HD, kvh * G * HD, nullptr, p.xq, xq_pad(qd));
            return;
        }
        attn_store_split<HD, G>(m, l, o, warp, lp, pg, p.part, split, p.nsplit, p.heads, kvh, scr);
        }
    }
    // the last CTA of this KV group (active or not) merges the group's heads.
    // The barrier orders every thread's partial stores before thread 0's fence
    // (cumulative), which publishes them before the ticket counts this CTA.
    __shared__ int is_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        is_last = atomicAdd(&p.tickets[kvh], 1u) == (unsigned)p.nsplit - 1u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float *res = scr + attn_merge_floats(G);
    attn_merge<HD, G, TC ? 40 : 8>(p.part, p.nsplit, r.nact, p.heads, kvh * G, res, scr);
    attn_emit(res, G * HD, kvh * G * HD, nullptr, p.xq, xq_pad(qd));
    if (threadIdx.x == 0) p.tickets[kvh] = 0u;
}

}  // namespace

}  // namespace cuq
