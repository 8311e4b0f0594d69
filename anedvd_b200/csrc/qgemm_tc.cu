// qgemm_tc.cu -- the prefill projection on the 5th-generation tensor cores:
// Y[n][rows] = X[n][cols] W^T with W in its quantized planes (engine.zig:975-1329).
//
// One CTA computes a 128-row x 128-token tile.  Per 64-column K step:
//   * 4 producer warps dequantise the 128 x 64 weight slice to the reference's
//     fp16 values (RN16 of the fp32 dequant, gguf.zig:751-1071 / load_gguf.zig:371)
//     straight into shared memory in the UMMA K-major 128-byte-swizzled layout,
//     and copy the activation slice: x is carried as fp16 hi + lo (x = hi + lo
//     to ~22 bits), stacked as 256 "tokens" (128 hi, then 128 lo);
//   * one thread issues 4 x tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256,
//     K=16) accumulating fp32 in tensor memory (128 lanes x 256 columns);
//   * tcgen05.commit releases the stage back to the producers (mbarriers, 4 stages).
// The epilogue warps read TMEM with tcgen05.ld and write hi + lo (+ bias, or
// += into the residual, or SiLU*mul for a gate|up pair) to global memory.
// Every mbarrier wait is bounded: on timeout the CTA records an error, stops
// issuing, releases its tensor memory and returns.
#include "common.cuh"
#include "qgemm.cuh"

namespace cuq {

namespace {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;        // 16 KB
constexpr int B_BYTES = 2 * BN * BK * 2;    // 32 KB (hi + lo)
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /* align */ + 256 /* barriers */;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t WAIT_LIMIT = 1u << 24;   // try_wait polls before giving up (seconds)

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok;
}
// Bounded wait for the phase with `parity`; false on timeout or when another
// thread of the CTA has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    for (uint32_t i = 0; i < WAIT_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte swizzle, 8-row atoms of 1024 B stacked along M/N.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);   // start address (16 B units)
    d |= (uint64_t)1u << 16;                   // leading byte offset (unused by swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;         // stride byte offset: next 8-row group
    d |= (uint64_t)1u << 46;                   // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                   // SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, M=128, N=256.
constexpr uint32_t IDESC = (1u << 4) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accum)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 columns of fp32 from TMEM (lane = this warp's quarter + lane id).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// ----------------------------------------------------- weight dequant ----
// 64 consecutive weights of one row, as the reference's fp16 values
// (RN16 of the fp32 dequant, gguf.zig:751-1071).  Arithmetic rounds where the
// reference rounds (explicit _rn intrinsics: no FMA contraction).

struct WPlanes {
    const uint8_t *q, *q2, *s, *s2;
    uint32_t rows, cols;
};

__device__ __forceinline__ float f16bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *q, int &d, int &m) {
    if (j < 4) {
        d = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

template <int T>
__device__ void dequant64(const WPlanes &w, uint32_t row, uint32_t kb, __half (&o)[64]) {
    const uint32_t k0 = kb * 64;
    if (T == CUQ_Q8_0) {  // gguf.zig:827-840: d * q
        const int8_t *qs = reinterpret_cast<const int8_t *>(w.q) + (size_t)row * w.cols + k0;
        const __half *dp = reinterpret_cast<const __half *>(w.s);
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = reinterpret_cast<const uint4 *>(qs)[i];
        const int8_t *b = reinterpret_cast<const int8_t *>(v);
#pragma unroll
        for (int blk = 0; blk < 2; blk++) {
            float d = __half2float(dp[(size_t)(k0 / 32 + blk) * w.rows + row]);
#pragma unroll
            for (int j = 0; j < 32; j++) o[blk * 32 + j] = __float2half_rn(__fmul_rn(d, (float)b[blk * 32 + j]));
        }
    } else if (T == CUQ_Q4_0 || T == CUQ_Q4_1 || T == CUQ_Q5_0 || T == CUQ_Q5_1) {
        const uint8_t *qs = w.q + (size_t)row * (w.cols / 2) + k0 / 2;
        uint4 v[2];
        v[0] = reinterpret_cast<const uint4 *>(qs)[0];
        v[1] = reinterpret_cast<const uint4 *>(qs)[1];
        const uint8_t *b = reinterpret_cast<const uint8_t *>(v);
#pragma unroll
        for (int blk = 0; blk < 2; blk++) {
            const size_t bi = (size_t)(k0 / 32 + blk) * w.rows + row;
            float d, m = 0.f;
            if (T == CUQ_Q4_0 || T == CUQ_Q5_0) {
                d = __half2float(reinterpret_cast<const __half *>(w.s)[bi]);
            } else {
                __half2 dm = reinterpret_cast<const __half2 *>(w.s)[bi];
                d = __low2float(dm);
                m = __high2float(dm);
            }
            uint32_t qh = (T == CUQ_Q5_0 || T == CUQ_Q5_1) ? reinterpret_cast<const uint32_t *>(w.q2)[bi] : 0u;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                int byte = b[blk * 16 + (j & 15)];
                int nib = j < 16 ? (byte & 0xF) : (byte >> 4);
                float val;
                if (T == CUQ_Q4_0) {
                    val = __fmul_rn((float)(nib - 8), d);  // gguf.zig:763-776
                } else if (T == CUQ_Q4_1) {
                    val = __fadd_rn(__fmul_rn((float)nib, d), m);  // gguf.zig:778-792
                } else {
                    int hb = j < 16 ? (int)(((qh >> j) << 4) & 0x10u) : (int)((qh >> (j - 16 + 12)) & 0x10u);
                    float x = (float)((nib | hb) - (T == CUQ_Q5_0 ? 16 : 0));
                    val = __fadd_rn(__fmul_rn(x, d), m);  // gguf.zig:795-825
                }
                o[blk * 32 + j] = __float2half_rn(val);
            }
        }
    } else if (T == CUQ_Q4_K) {  // gguf.zig:962-996: (d*sc)*q - dmin*m
        const uint32_t sb = kb / 4, c = kb % 4;
        const uint8_t *qs = w.q + (size_t)row * (w.cols / 2) + (size_t)sb * 128 + 32 * c;
        uint4 v[2];
        v[0] = reinterpret_cast<const uint4 *>(qs)[0];
        v[1] = reinterpret_cast<const uint4 *>(qs)[1];
        uint4 meta = *reinterpret_cast<const uint4 *>(w.s + ((size_t)sb * w.rows + row) * 16);
        const uint8_t *mb = reinterpret_cast<const uint8_t *>(&meta);
        const uint8_t *b = reinterpret_cast<const uint8_t *>(v);
        float d = f16bits((uint16_t)(meta.x & 0xFFFF)), dmin = f16bits((uint16_t)(meta.x >> 16));
#pragma unroll
        for (int part = 0; part < 2; part++) {
            int sc, mm;
            scale_min_k4(2 * c + part, mb + 4, sc, mm);
            float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mm);
#pragma unroll
            for (int l = 0; l < 32; l++) {
                float q = (float)(part ? (b[l] >> 4) : (b[l] & 0xF));
                o[part * 32 + l] = __float2half_rn(__fsub_rn(__fmul_rn(d1, q), m1));
            }
        }
    } else if (T == CUQ_Q6_K) {  // gguf.zig:1036-1059: (d*sc)*(q-32)
        const uint32_t sb = kb / 4, qtr = kb % 4, h = qtr / 2, t0 = 2 * (qtr % 2);
        const uint8_t *ql = w.q + (size_t)row * (w.cols / 2) + (size_t)sb * 128 + 64 * h;
        const uint8_t *qh = w.q2 + (size_t)row * (w.cols / 4) + (size_t)sb * 64 + 32 * h;
        uint4 scv = *reinterpret_cast<const uint4 *>(w.s + ((size_t)sb * w.rows + row) * 16);
        const int8_t *sc = reinterpret_cast<const int8_t *>(&scv);
        float d = __half2float(reinterpret_cast<const __half *>(w.s2)[(size_t)sb * w.rows + row]);
        uint4 lv[4], hv[2];
#pragma unroll
        for (int i = 0; i < 4; i++) lv[i] = reinterpret_cast<const uint4 *>(ql)[i];
        hv[0] = reinterpret_cast<const uint4 *>(qh)[0];
        hv[1] = reinterpret_cast<const uint4 *>(qh)[1];
        const uint8_t *L = reinterpret_cast<const uint8_t *>(lv), *H = reinterpret_cast<const uint8_t *>(hv);
#pragma unroll
        for (int tt = 0; tt < 2; tt++) {
            const int t = t0 + tt;
#pragma unroll
            for (int l = 0; l < 32; l++) {
                int lo = (t & 1) ? L[32 + l] : L[l];
                int q = ((t >= 2) ? (lo >> 4) : (lo & 0xF)) | (((H[l] >> (2 * t)) & 3) << 4);
                float s = __fmul_rn(d, (float)sc[8 * h + 2 * t + (l >> 4)]);
                o[tt * 32 + l] = __float2half_rn(__fmul_rn(s, (float)(q - 32)));
            }
        }
    } else if (T == CUQ_F16) {
        const uint4 *src = reinterpret_cast<const uint4 *>(w.q + ((size_t)row * w.cols + k0) * 2);
#pragma unroll
        for (int i = 0; i < 8; i++) reinterpret_cast<uint4 *>(o)[i] = src[i];
    } else if (T == CUQ_BF16) {  // Gguf.readF16 of a bf16 tensor: RN16(f32(bf16))
        const uint16_t *src = reinterpret_cast<const uint16_t *>(w.q + ((size_t)row * w.cols + k0) * 2);
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = reinterpret_cast<const uint4 *>(src)[i];
        const uint16_t *bb = reinterpret_cast<const uint16_t *>(v);
#pragma unroll
        for (int j = 0; j < 64; j++) o[j] = __float2half_rn(__uint_as_float((uint32_t)bb[j] << 16));
    }
}

// ------------------------------------------------------------- kernel ----

struct QgArgs {
    WPlanes w, w2;             // w2: the up matrix of a gate|up pair
    const __half *xh, *xl;     // [n][cols] activation hi / lo
    uint32_t n;
    float *y;                  // [n][ldy] fp32 output (STORE / ADD)
    uint32_t ldy;
    const float *bias;
    __half *oh, *ol;           // SILU: act hi / lo, [n][rows]
    int *err;                  // set to 1 when a wait timed out
};

template <int T, int EPI>
__global__ void __launch_bounds__(160, 1) qgemm_tc_kernel(const QgArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *done = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    __shared__ float xchg[64][33];  // SILU: up values handed to the gate rows

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr bool DUAL = (EPI == EPI_SILU_XQ);
    const uint32_t rows = p.w.rows, cols = p.w.cols;
    const uint32_t nkb = cols / BK;
    // DUAL: the tile is 64 gate rows followed by the same 64 up rows
    const uint32_t row0 = blockIdx.x * (DUAL ? BM / 2 : BM);
    const uint32_t tok0 = blockIdx.y * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 128);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {  // tensor memory for the 128 x 256 fp32 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ---------------------------------------------------- producers
        const uint32_t t = threadIdx.x;  // A row within the tile
        for (uint32_t kb = 0; kb < nkb; kb++) {
            const int s = kb % STAGES;
            if (kb >= (uint32_t)STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, abort_flag)) break;
            uint8_t *A = smem + s * STAGE_BYTES, *B = A + A_BYTES;
            // A: one weight row per thread, 64 fp16 = 8 chunks of 16 B, swizzled
            {
                __half vals[64];
                uint32_t r;
                const WPlanes *wp = &p.w;
                if (DUAL) {
                    r = row0 + (t & 63);
                    wp = t < 64 ? &p.w : &p.w2;
                } else {
                    r = row0 + t;
                }
                if (r < rows)
                    dequant64<T>(*wp, r, kb, vals);
                else
#pragma unroll
                    for (int j = 0; j < 64; j++) vals[j] = __float2half_rn(0.f);
#pragma unroll
                for (int c = 0; c < 8; c++)
                    *reinterpret_cast<uint4 *>(A + t * 128 + ((c ^ (t & 7)) * 16)) = reinterpret_cast<uint4 *>(vals)[c];
            }
            // B: 256 rows (128 hi tokens, 128 lo tokens) x 8 chunks, 16 per thread
#pragma unroll 4
            for (int j = 0; j < 16; j++) {
                const uint32_t q = t + 128 * j, b = q >> 3, c = q & 7;
                const uint32_t tok = tok0 + (b & 127);
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (tok < p.n) {
                    const __half *src = (b < 128 ? p.xh : p.xl) + (size_t)tok * cols + kb * BK + c * 8;
                    v = *reinterpret_cast<const uint4 *>(src);
                }
                *reinterpret_cast<uint4 *>(B + b * 128 + ((c ^ (b & 7)) * 16)) = v;
            }
            fence_async_smem();
            mbar_arrive(&full[s]);
        }
        // ---------------------------------------------------- epilogue
        mbar_wait(done, 0, abort_flag);
        asm volatile("bar.sync 1, 128;" ::: "memory");  // all producers past the wait: abort_flag is final
        const bool ok = *abort_flag == 0;
        tc_fence_after();
        if (ok) {
            const uint32_t lane_base = (uint32_t)warp * 32;
#pragma unroll 1
            for (int ch = 0; ch < BN / 32; ch++) {
                float hi[32], lo[32];
                tmem_ld32(tmem + (lane_base << 16) + ch * 32, hi);
                tmem_ld32(tmem + (lane_base << 16) + BN + ch * 32, lo);
                const uint32_t trow = lane_base + lane;  // row within the tile
                if (DUAL) {
                    // rows 64..127 hold "up": hand them to the gate threads
                    if (trow >= 64)
#pragma unroll
                        for (int i = 0; i < 32; i++) xchg[trow - 64][i] = hi[i] + lo[i];
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (trow < 64) {
                        const uint32_t r = row0 + trow;
#pragma unroll 4
                        for (int i = 0; i < 32; i++) {
                            const uint32_t tok = tok0 + ch * 32 + i;
                            if (tok >= p.n || r >= rows) continue;
                            float g = hi[i] + lo[i], u = xchg[trow][i];
                            float sg = 1.0f / (1.0f + expf(-g));  // cpu.siluMul (cpu.zig:65-70)
                            float act = (g * sg) * u;
                            __half ah = __float2half_rn(act);
                            p.oh[(size_t)tok * rows + r] = ah;
                            p.ol[(size_t)tok * rows + r] = __float2half_rn(act - __half2float(ah));
                        }
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                } else {
                    const uint32_t r = row0 + trow;
                    if (r < rows) {
                        const float b = p.bias ? p.bias[r] : 0.f;
#pragma unroll 4
                        for (int i = 0; i < 32; i++) {
                            const uint32_t tok = tok0 + ch * 32 + i;
                            if (tok >= p.n) break;
                            float v = hi[i] + lo[i];
                            if (p.bias) v = v + b;
                            float *dst = p.y + (size_t)tok * p.ldy + r;
                            if (EPI == EPI_ADD)
                                *dst = *dst + v;
                            else
                                *dst = v;
                        }
                    }
                }
            }
        }
    } else if (lane == 0) {
        // ---------------------------------------------------- MMA issuer
        bool ok = true;
        for (uint32_t kb = 0; kb < nkb; kb++) {
            const int s = kb % STAGES;
            if (!mbar_wait(&full[s], (kb / STAGES) & 1, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a = smem_u32(smem + s * STAGE_BYTES), b = a + A_BYTES;
#pragma unroll
            for (int k = 0; k < BK / 16; k++)
                umma_f16(tmem, sdesc_sw128(a + 32 * k), sdesc_sw128(b + 32 * k), (kb | k) ? 1u : 0u);
            umma_commit(&empty[s]);  // frees the stage when these MMAs complete
        }
        if (ok) umma_commit(done);
        else mbar_arrive(done);      // let the epilogue stop waiting
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 0) *p.err = 1;
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

template <int T, int EPI>
int launch_tq(const QgArgs &a, uint32_t rows, uint32_t n, cudaStream_t s) {
    auto kern = qgemm_tc_kernel<T, EPI>;
    static bool attr_set = false;  // per instantiation
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) {
            set_error("qgemm: shared memory opt-in failed: %s", cudaGetErrorString(e));
            return CUQ_ECUDA;
        }
        attr_set = true;
    }
    const uint32_t rows_per_cta = EPI == EPI_SILU_XQ ? BM / 2 : BM;
    dim3 grid((rows + rows_per_cta - 1) / rows_per_cta, (n + BN - 1) / BN);
    kern<<<grid, 160, SMEM_BYTES, s>>>(a);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

template <int EPI>
int dispatch(int type, const QgArgs &a, uint32_t rows, uint32_t n, cudaStream_t s) {
    switch (type) {
    case CUQ_Q8_0: return launch_tq<CUQ_Q8_0, EPI>(a, rows, n, s);
    case CUQ_Q4_0: return launch_tq<CUQ_Q4_0, EPI>(a, rows, n, s);
    case CUQ_Q4_1: return launch_tq<CUQ_Q4_1, EPI>(a, rows, n, s);
    case CUQ_Q5_0: return launch_tq<CUQ_Q5_0, EPI>(a, rows, n, s);
    case CUQ_Q5_1: return launch_tq<CUQ_Q5_1, EPI>(a, rows, n, s);
    case CUQ_Q4_K: return launch_tq<CUQ_Q4_K, EPI>(a, rows, n, s);
    case CUQ_Q6_K: return launch_tq<CUQ_Q6_K, EPI>(a, rows, n, s);
    case CUQ_F16: return launch_tq<CUQ_F16, EPI>(a, rows, n, s);
    case CUQ_BF16: return launch_tq<CUQ_BF16, EPI>(a, rows, n, s);
    }
    set_error("UnsupportedType: no tensor-core GEMM for ggml type %d", type);
    return CUQ_EUNSUPPORTED;
}

WPlanes wplanes(const Planes &p) {
    WPlanes w;
    w.q = p.base + p.off_q;
    w.q2 = p.off_q2 == SIZE_MAX ? nullptr : p.base + p.off_q2;
    w.s = p.off_s == SIZE_MAX ? nullptr : p.base + p.off_s;
    w.s2 = p.off_s2 == SIZE_MAX ? nullptr : p.base + p.off_s2;
    w.rows = p.rows;
    w.cols = p.cols;
    return w;
}

}  // namespace

int launch_qgemm(const QgemmArgs &g, int epi, cudaStream_t s) {
    const Planes &w = *g.w;
    if (!gemv_supported(w.type)) {
        set_error("UnsupportedType: no tensor-core GEMM for ggml type %d", w.type);
        return CUQ_EUNSUPPORTED;
    }
    if (w.cols % BK) {
        set_error("qgemm: cols (%u) must be a multiple of %d", w.cols, BK);
        return CUQ_EINVAL;
    }
    if (epi == EPI_SILU_XQ && (!g.w2 || g.w2->type != w.type || g.w2->rows != w.rows || g.w2->cols != w.cols)) {
        set_error("qgemm: gate/up must share type and shape");
        return CUQ_EINVAL;
    }
    if (g.n == 0) return CUQ_OK;
    QgArgs a;
    a.w = wplanes(w);
    if (g.w2) a.w2 = wplanes(*g.w2);
    a.xh = g.xh;
    a.xl = g.xl;
    a.n = g.n;
    a.y = g.y;
    a.ldy = g.ldy ? g.ldy : w.rows;
    a.bias = g.bias;
    a.oh = g.oh;
    a.ol = g.ol;
    a.err = g.err;
    switch (epi) {
    case EPI_STORE: return dispatch<EPI_STORE>(w.type, a, w.rows, g.n, s);
    case EPI_ADD: return dispatch<EPI_ADD>(w.type, a, w.rows, g.n, s);
    case EPI_SILU_XQ: return dispatch<EPI_SILU_XQ>(w.type, a, w.rows, g.n, s);
    }
    set_error("qgemm: bad epilogue %d", epi);
    return CUQ_EINVAL;
}

// x fp32 [n][cols] -> hi, lo fp16 [n][cols] (x = hi + lo).
__global__ void split_hilo_kernel(const float *__restrict__ x, size_t count, __half *__restrict__ hi,
                                  __half *__restrict__ lo) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        float f = x[i];
        __half h = __float2half_rn(f);
        hi[i] = h;
        lo[i] = __float2half_rn(f - __half2float(h));
    }
}

int launch_split_hilo(const float *x, size_t count, __half *hi, __half *lo, cudaStream_t s) {
    size_t g = (count + 255) / 256;
    if (g > 148 * 32) g = 148 * 32;
    split_hilo_kernel<<<(unsigned)(g ? g : 1), 256, 0, s>>>(x, count, hi, lo);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

}  // namespace cuq
