// attn_prefill.cu -- causal attention over a prefill chunk on the tensor cores
// (flash-attention style), cpu.attentionPrefill (cpu.zig:165-217): query at
// position p attends to cache positions [0, p] of its KV head (GQA: query head h
// reads KV head h / (heads / kv_heads)).
//
// CTA = one KV head x 16 consecutive queries; warp w = query head kvh*G + w, so
// the G heads sharing a KV head share every K/V tile.  Per 64-key block:
//   * K and V rows are staged in shared memory by cp.async (double-buffered,
//     padded rows: conflict-free ldmatrix);
//   * S = Q K^T with mma.sync m16n8k16, fp32 accumulate; q is carried as fp16
//     hi + lo (two MMAs), so scores keep ~22 bits of q like the reference's fp32;
//   * scores are scaled by 1/sqrt(hd) (the reference's order: dot, then scale),
//     masked causally, and folded into an online softmax (running max m, sum l);
//   * O += P V with each probability rounded once to fp16 (a value in [0, 1]:
//     relative error <= 2^-11) and l summing those same rounded values, so O is
//     an exactly normalised mean over slightly perturbed weights.
// The normalised O is written as fp16 hi + lo, the o projection GEMM's input.
#include "common.cuh"
#include "ops.cuh"

namespace cuq {

namespace {

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// 16 bytes global -> shared; src_bytes 0 writes zeros without reading.
__device__ __forceinline__ void cp_async16z(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// fp32 pair -> (hi, lo) fp16 pairs with x = hi + lo
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    hi = h2u(h);
    lo = h2u(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}

constexpr int FA_KB = 64;  // keys per block

template <int HD>
constexpr int fa_row_bytes() { return HD * 2 + 16; }
template <int HD>
constexpr int fa_smem() { return 2 * 2 * FA_KB * fa_row_bytes<HD>(); }

template <int HD, int G>
__global__ void __launch_bounds__(32 * G) fa_prefill_kernel(const float *__restrict__ q, const __half *__restrict__ kc,
                                                            const __half *__restrict__ vc, uint32_t cache_stride,
                                                            uint32_t pos0, uint32_t n_q, uint32_t heads,
                                                            __half *__restrict__ oh, __half *__restrict__ ol) {
    constexpr int KS = HD / 16;           // k-steps of S over the head dimension
    constexpr int NT = HD / 8;            // n-tiles of O over the head dimension
    constexpr int ROW = fa_row_bytes<HD>();
    constexpr int TILE = FA_KB * ROW;     // one K or V tile
    constexpr int NTHR = 32 * G;
    extern __shared__ __align__(16) uint8_t fa_sm[];
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(fa_sm);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const uint32_t kvh = blockIdx.x, qi0 = blockIdx.y * 16;
    const uint32_t head = kvh * G + warp, qd = heads * HD;
    const uint32_t last_q = min(n_q, qi0 + 16) - 1;
    const uint32_t nkeys = pos0 + last_q + 1;
    const uint32_t nkb = (nkeys + FA_KB - 1) / FA_KB;
    const float scale = 1.0f / sqrtf((float)HD);
    const __half *kh = kc + (size_t)kvh * cache_stride * HD;
    const __half *vh = vc + (size_t)kvh * cache_stride * HD;

    // K/V tile kb -> buffer b: 2 * 64 rows of HD*2 bytes, 16-byte chunks spread over the CTA
    auto load_tile = [&](uint32_t kb, int b) {
        constexpr int CPR = HD * 2 / 16;  // chunks per row
        for (int c = threadIdx.x; c < 2 * FA_KB * CPR; c += NTHR) {
            const int isv = c / (FA_KB * CPR), rem = c % (FA_KB * CPR), r = rem / CPR, ch = rem % CPR;
            const uint32_t key = kb * FA_KB + r;
            const bool ok = key < nkeys;
            const __half *src = (isv ? vh : kh) + (size_t)(ok ? key : 0) * HD + ch * 8;
            const uint32_t dst = sbase + (uint32_t)(((b * 2 + isv) * TILE) + r * ROW + ch * 16);
            cp_async16z(dst, src, ok ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // this warp's 16 queries (rows g and g+8) as A fragments, hi and lo
    uint32_t qa_hi[KS][4], qa_lo[KS][4];
    {
        const uint32_t r0 = qi0 + g, r1 = qi0 + g + 8;
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
#pragma unroll
            for (int half = 0; half < 2; half++) {  // k columns 2tig (+8 for half 1)
                const uint32_t d = 16 * ks + 2 * tig + 8 * half;
                float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
                if (r0 < n_q) a = *reinterpret_cast<const float2 *>(q + (size_t)r0 * qd + (size_t)head * HD + d);
                if (r1 < n_q) b = *reinterpret_cast<const float2 *>(q + (size_t)r1 * qd + (size_t)head * HD + d);
                split2(a.x, a.y, qa_hi[ks][2 * half], qa_lo[ks][2 * half]);
                split2(b.x, b.y, qa_hi[ks][2 * half + 1], qa_lo[ks][2 * half + 1]);
            }
        }
    }
    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    const uint32_t qpos[2] = {pos0 + qi0 + g, pos0 + qi0 + g + 8};
    const bool qok[2] = {qi0 + g < n_q, qi0 + g + 8 < n_q};

    load_tile(0, 0);
    for (uint32_t kb = 0; kb < nkb; kb++) {
        const int b = kb & 1;
        if (kb + 1 < nkb) {
            load_tile(kb + 1, b ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const uint32_t ktile = sbase + (uint32_t)((b * 2) * TILE), vtile = ktile + TILE;

        // ---- S = Q K^T (16 queries x 64 keys per warp)
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ks += 2) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint32_t kb4[4];  // b0, b1 of k-step ks, then of ks + 1
                ldsm_x4(ktile + (uint32_t)((8 * j + (lane & 7)) * ROW + (16 * ks + 8 * (lane >> 3)) * 2), kb4);
                mma16816(s[j], qa_hi[ks], kb4[0], kb4[1]);
                mma16816(s[j], qa_lo[ks], kb4[0], kb4[1]);
                mma16816(s[j], qa_hi[ks + 1], kb4[2], kb4[3]);
                mma16816(s[j], qa_lo[ks + 1], kb4[2], kb4[3]);
            }
        }
        // ---- scale, causal mask, online softmax
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 8; j++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int ri = e >> 1;
                const uint32_t key = kb * FA_KB + 8 * j + 2 * tig + (e & 1);
                const float v = (qok[ri] && key <= qpos[ri]) ? s[j][e] * scale : -INFINITY;
                s[j][e] = v;
                mx[ri] = fmaxf(mx[ri], v);
            }
        }
        float corr[2];
#pragma unroll
        for (int ri = 0; ri < 2; ri++) {
            mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
            mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
            const float mn = fmaxf(m[ri], mx[ri]);
            corr[ri] = m[ri] == -INFINITY ? 0.f : expf(m[ri] - mn);
            m[ri] = mn;
            l[ri] *= corr[ri];
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            o[nt][0] *= corr[0];
            o[nt][1] *= corr[0];
            o[nt][2] *= corr[1];
            o[nt][3] *= corr[1];
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int ri = e >> 1;
                // p rounded to fp16 once: the PV MMA reads it exactly and l sums
                // the same values, so O is a weighted mean with exact weights
                const float p = s[j][e] == -INFINITY ? 0.f : __half2float(__float2half_rn(expf(s[j][e] - m[ri])));
                s[j][e] = p;
                l[ri] += p;
            }
        }
        // ---- O += P V
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {  // 16 keys per k-step
            uint32_t pa[4];  // exact: p is already an fp16 value
            pa[0] = h2u(__floats2half2_rn(s[2 * kk][0], s[2 * kk][1]));
            pa[1] = h2u(__floats2half2_rn(s[2 * kk][2], s[2 * kk][3]));
            pa[2] = h2u(__floats2half2_rn(s[2 * kk + 1][0], s[2 * kk + 1][1]));
            pa[3] = h2u(__floats2half2_rn(s[2 * kk + 1][2], s[2 * kk + 1][3]));
#pragma unroll
            for (int nt = 0; nt < NT; nt += 2) {
                uint32_t vb[4];  // b0, b1 of n-tile nt, then of nt + 1
                const int mi = lane >> 3;
                ldsm_x4_t(vtile + (uint32_t)((16 * kk + (lane & 7) + 8 * (mi & 1)) * ROW + (8 * (nt + (mi >> 1))) * 2),
                          vb);
                mma16816(o[nt], pa, vb[0], vb[1]);
                mma16816(o[nt + 1], pa, vb[2], vb[3]);
            }
        }
        __syncthreads();  // buffer b is refilled two blocks from now
    }
    // ---- normalise and write hi + lo
#pragma unroll
    for (int ri = 0; ri < 2; ri++) {
        l[ri] += __shfl_xor_sync(0xffffffffu, l[ri], 1);
        l[ri] += __shfl_xor_sync(0xffffffffu, l[ri], 2);
    }
#pragma unroll
    for (int ri = 0; ri < 2; ri++) {
        const uint32_t qi = qi0 + g + 8 * ri;
        if (qi >= n_q) continue;
        const float inv = 1.0f / l[ri];
        const size_t base = (size_t)qi * qd + (size_t)head * HD + 2 * tig;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            uint32_t hi, lo;
            split2(o[nt][2 * ri] * inv, o[nt][2 * ri + 1] * inv, hi, lo);
            *reinterpret_cast<uint32_t *>(oh + base + 8 * nt) = hi;
            *reinterpret_cast<uint32_t *>(ol + base + 8 * nt) = lo;
        }
    }
}

template <int HD, int G>
int fa_launch(const float *q, const __half *kc, const __half *vc, uint32_t cs, uint32_t pos0, uint32_t n_q,
              uint32_t heads, uint32_t kv_heads, __half *oh, __half *ol, cudaStream_t s) {
    auto kern = fa_prefill_kernel<HD, G>;
    static bool attr = false;  // per instantiation
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem<HD>());
        if (e != cudaSuccess) {
            set_error("prefill attention: shared memory opt-in failed: %s", cudaGetErrorString(e));
            return CUQ_ECUDA;
        }
        attr = true;
    }
    dim3 grid(kv_heads, (n_q + 15) / 16);
    kern<<<grid, 32 * G, fa_smem<HD>(), s>>>(q, kc, vc, cs, pos0, n_q, heads, oh, ol);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

}  // namespace

int launch_attention_prefill(const float *q, const __half *k_cache, const __half *v_cache, uint32_t cache_stride,
                             uint32_t pos0, uint32_t n_q, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                             __half *oh, __half *ol, cudaStream_t s) {
    if (kv_heads == 0 || heads % kv_heads) {
        set_error("attention: heads (%u) must be a multiple of kv_heads (%u)", heads, kv_heads);
        return CUQ_EINVAL;
    }
    if (n_q == 0) return CUQ_OK;
    const uint32_t G = heads / kv_heads;
#define CUQ_FA(HDV, GV) \
    if (hd == HDV && G == GV) return fa_launch<HDV, GV>(q, k_cache, v_cache, cache_stride, pos0, n_q, heads, kv_heads, oh, ol, s);
    CUQ_FA(64, 1) CUQ_FA(64, 2) CUQ_FA(64, 3) CUQ_FA(64, 4) CUQ_FA(64, 6) CUQ_FA(64, 7) CUQ_FA(64, 8)
    CUQ_FA(128, 1) CUQ_FA(128, 2) CUQ_FA(128, 3) CUQ_FA(128, 4) CUQ_FA(128, 6) CUQ_FA(128, 7) CUQ_FA(128, 8)
#undef CUQ_FA
    set_error("attention: unsupported head_dim %u / group %u (head_dim 64 or 128, group 1-8)", hd, G);
    return CUQ_EUNSUPPORTED;
}

}  // namespace cuq
