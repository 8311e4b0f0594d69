// qgemm_tc.cu -- the prefill projection on the 5th-generation tensor cores:
// Y[n][rows] = X[n][cols] W^T with W in its quantized planes (engine.zig:975-1329).
//
// Persistent CTAs (one per SM, 448 threads) walk 128-row x 256-token tiles.
//   * warps 0-7 copy each tile's raw quant bytes and scales with cp.async into a
//     small ring (two threads per weight row) and dequantise them to the
//     reference's fp16 values (RN16 of the fp32 dequant, gguf.zig:751-1071 /
//     load_gguf.zig:371) straight into the A stage, UMMA K-major with a 64-byte
//     swizzle, 32 columns per stage;
//   * warp 9 loads the activation tiles by TMA: x as fp16 hi and lo (x = hi + lo
//     to ~22 bits), 256 tokens x 32 columns each;
//   * one lane of warp 8 issues tcgen05.mma.cta_group::1.kind::f16 (M=128,
//     N=256, K=16) for hi and then lo into the same fp32 TMEM accumulator, and
//     tcgen05.commit releases each stage (mbarriers, 4 stages); two accumulators
//     alternate between tiles;
//   * warps 10-13 read the finished accumulator with tcgen05.ld and write the
//     output (+ bias, += into the residual, or SiLU*mul for an interleaved
//     gate|up tile) while the next tile's MMAs run.
// Every mbarrier wait is bounded: on timeout the CTA records an error, stops
// issuing, releases its tensor memory and returns.
#include <cuda.h>

#include "common.cuh"
#include "qgemm.cuh"

namespace cuq {

int sm_count_current();

namespace {

// Tile: 128 weight rows x 256 tokens.  Weights are dequantised 64 columns at a
// time (RAW_K, one "raw step"), and fed to the MMA in stages of 32 columns
// (BK): A = 128 x 32 fp16 and B = 256 x 32 x (hi, lo) fp16 in the 64-byte
// swizzled K-major layout.  hi and lo accumulate into the same TMEM columns.
constexpr int BM = 128, BN = 256, BK = 32, RAW_K = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;        // 8 KB
constexpr int B_BYTES = 2 * BN * BK * 2;    // 32 KB (hi + lo)
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t TMEM_COLS = 256;         // one accumulator: 256 token columns
constexpr unsigned long long WAIT_NS = 2000000000ull;  // a stage wait gives up after 2 s
constexpr uint32_t SUSPEND_NS = 20000;                   // try_wait sleeps up to 20 us per poll

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes (or the hint expires) instead of spinning, so waiting warps take
// no issue slots from the producers sharing their SM sub-partition.
__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(SUSPEND_NS)
        : "memory");
    return ok;
}
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long v;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(v));
    return v;
}
// Bounded wait for the phase with `parity`; false on timeout (WAIT_NS) or when
// another thread of the CTA has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (now_ns() - t0 > WAIT_NS) break;
    }
    *abort_flag = 1;
    return false;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 64-byte swizzle: 8-row atoms of 512 B (rows of 64 B, 16-byte chunk c
// of row r at chunk c ^ ((r >> 1) & 3)) stacked along M/N.
__device__ __forceinline__ uint64_t sdesc_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);   // start address (16 B units)
    d |= (uint64_t)1u << 16;                   // leading byte offset (unused by swizzled K-major)
    d |= (uint64_t)(512u >> 4) << 32;          // stride byte offset: next 8-row group
    d |= (uint64_t)1u << 46;                   // descriptor version (sm_100)
    d |= (uint64_t)4u << 61;                   // SWIZZLE_64B
    return d;
}
__device__ __forceinline__ int sw64_chunk(int r, int c) { return c ^ ((r >> 1) & 3); }

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

// ----------------------------------------------------- weight planes ----

struct WPlanes {
    const uint8_t *q, *q2, *s, *s2;
    uint32_t rows, cols;
};

// Raw bytes of one 64-column K step, staged per weight row in shared memory by
// cp.async (prefetched RAWD-1 steps ahead), then dequantised from there.
//   RAW_ROW: quant bytes per row (padded to a power of two for the swizzle);
//   SIDE:    per-step side data (scales, 5th bits) for the tile's 128 rows.
template <int T>
struct RawGeom;
template <> struct RawGeom<CUQ_Q8_0> { static constexpr int RAW_ROW = 64, SIDE = 2 * 256; };
template <> struct RawGeom<CUQ_Q4_0> { static constexpr int RAW_ROW = 32, SIDE = 2 * 256; };
template <> struct RawGeom<CUQ_Q4_1> { static constexpr int RAW_ROW = 32, SIDE = 2 * 512; };
template <> struct RawGeom<CUQ_Q5_0> { static constexpr int RAW_ROW = 32, SIDE = 2 * 256 + 2 * 512; };
template <> struct RawGeom<CUQ_Q5_1> { static constexpr int RAW_ROW = 32, SIDE = 2 * 512 + 2 * 512; };
template <> struct RawGeom<CUQ_Q4_K> { static constexpr int RAW_ROW = 32, SIDE = 128 * 16; };
template <> struct RawGeom<CUQ_Q6_K> { static constexpr int RAW_ROW = 96, SIDE = 128 * 16 + 256; };
template <> struct RawGeom<CUQ_F16> { static constexpr int RAW_ROW = 128, SIDE = 0; };
template <> struct RawGeom<CUQ_BF16> { static constexpr int RAW_ROW = 128, SIDE = 0; };

template <int T>
struct Geo {
    static constexpr int RAW_ROW = RawGeom<T>::RAW_ROW, SIDE = RawGeom<T>::SIDE;
    static constexpr int CH = RAW_ROW / 16;                        // 16-byte chunks per row
    static constexpr int SLOT = BM * RAW_ROW + SIDE;               // bytes per raw slot
    static constexpr int RAWD = SLOT > 12288 ? 2 : 3;              // raw ring depth (fits 227 KB)
    static constexpr int SMEM = STAGES * STAGE_BYTES + RAWD * SLOT + 1024 + 256;  // + barriers
};

// physical 16-byte chunk of logical chunk c in row r (conflict-free 16-byte reads
// by consecutive rows: 8 consecutive rows cover the 8 bank groups)
template <int CH>
__device__ __forceinline__ int raw_chunk(int r, int c) {
    if (CH & (CH - 1)) return c;  // not a power of two (Q6_K, 6 chunks): plain rows, 2-way conflicts
    return CH >= 8 ? (c ^ (r & 7)) : c ^ ((r / (8 / CH)) & (CH - 1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Issue the copies of K step kb into `slot` for the 16 A rows of producer warp
// pw (lane = 2 * row + half): every warp loads, and later reads, only its own
// rows' bytes, so the 8 producer warps never wait for one another.
// A row ar of a dual tile interleaves gate and up: matrix ar & 1, row ar >> 1.
// Side records (scales, 5th bits) are indexed by side row sr: ar for a plain
// tile, (ar & 1) * 64 + (ar >> 1) for a dual one, so 8 or 16 consecutive
// matrix rows stay contiguous and copy as 16-byte chunks.
template <int T>
__device__ __forceinline__ void raw_issue(const WPlanes &w, const WPlanes &w2, bool dual, uint32_t row0, uint32_t kb,
                                          uint8_t *slot, int pw, int lane) {
    using G = Geo<T>;
    const uint32_t sb = kb / 4;
    const int ar = 16 * pw + (lane >> 1), half = lane & 1;
    const WPlanes &wq = (dual && (ar & 1)) ? w2 : w;
    const uint32_t rq = dual ? row0 + (ar >> 1) : row0 + ar;
    const uint32_t rr = rq < wq.rows ? rq : wq.rows - 1;  // rows past the end: any valid row (results unused)
    const uint8_t *src;
    if (T == CUQ_Q8_0)
        src = wq.q + (size_t)rr * wq.cols + kb * 64;
    else if (T == CUQ_F16 || T == CUQ_BF16)
        src = wq.q + ((size_t)rr * wq.cols + kb * 64) * 2;
    else if (T == CUQ_Q6_K)
        src = wq.q + (size_t)rr * (wq.cols / 2) + (size_t)sb * 128 + 64 * ((kb % 4) / 2);
    else
        src = wq.q + (size_t)rr * (wq.cols / 2) + (size_t)kb * 32;
    const uint32_t base = smem_u32(slot) + ar * G::RAW_ROW;
    if (T == CUQ_Q6_K) {  // ql 64 B = chunks 0-3, qh 32 B = chunks 4-5; three per thread
        const uint8_t *qh = wq.q2 + (size_t)rr * (wq.cols / 4) + (size_t)sb * 64 + 32 * ((kb % 4) / 2);
#pragma unroll
        for (int i = 0; i < 3; i++) {
            const int c = 3 * half + i;
            cp_async16(base + raw_chunk<G::CH>(ar, c) * 16, c < 4 ? src + 16 * c : qh + 16 * (c - 4));
        }
    } else {
#pragma unroll
        for (int i = 0; i < G::CH / 2; i++) {
            const int c = half * (G::CH / 2) + i;
            cp_async16(base + raw_chunk<G::CH>(ar, c) * 16, src + 16 * c);
        }
    }
    const uint32_t sside = smem_u32(slot + BM * G::RAW_ROW);
    // the warp's side rows: one run of 16 (plain) or two runs of 8 (dual: gate, up)
    const int nrun = dual ? 2 : 1, run_rows = dual ? 8 : 16;
    if (T == CUQ_Q4_K || T == CUQ_Q6_K) {
        // 16 bytes of scales per row of superblock sb: one chunk per side row
        if (half == 0) {
            const int sr = dual ? (ar & 1) * 64 + (ar >> 1) : ar;
            const WPlanes &a = (dual && sr >= 64) ? w2 : w;
            const uint32_t ra = row0 + (dual ? (sr & 63) : sr);
            if (ra < a.rows) cp_async16(sside + 16 * sr, a.s + ((size_t)sb * a.rows + ra) * 16);
        }
        if (T == CUQ_Q6_K && lane < nrun * run_rows * 2 / 16) {  // d: fp16 per row, 8 rows per chunk
            const int run = dual ? lane : 0, cir = dual ? 0 : lane;
            const WPlanes &a = run ? w2 : w;
            const int sr0 = dual ? run * 64 + 8 * pw : 16 * pw;
            const uint32_t first = row0 + (dual ? 8 * pw : 16 * pw) + 8 * cir;
            if (first < a.rows)
                cp_async16(sside + 2048 + 2 * (sr0 + 8 * cir), a.s2 + ((size_t)sb * a.rows + first) * 2);
        }
    } else if (T != CUQ_F16 && T != CUQ_BF16) {
        // two 32-blocks per step; per block: d (2 B) or d|m (4 B) per row; Q5: qh 4 B per row
        constexpr int SE = (T == CUQ_Q4_1 || T == CUQ_Q5_1) ? 4 : 2;
        constexpr int SB = 128 * SE;  // side bytes per block
        constexpr bool Q5 = (T == CUQ_Q5_0 || T == CUQ_Q5_1);
        const int cpr = run_rows * SE / 16;      // chunks per run of scale records
        const int cq5 = run_rows * 4 / 16;       // chunks per run of qh words
        const int per_blk = nrun * (cpr + (Q5 ? cq5 : 0));
        for (int c = lane; c < 2 * per_blk; c += 32) {
            const int blk = c / per_blk, rem = c % per_blk;
            const bool isq = rem >= nrun * cpr;
            const int r2 = isq ? rem - nrun * cpr : rem;
            const int per = isq ? cq5 : cpr, esz = isq ? 4 : SE;
            const int run = r2 / per, cc = r2 % per;
            const WPlanes &a = run ? w2 : w;
            const int sr0 = (dual ? run * 64 + 8 * pw : 16 * pw) + cc * (16 / esz);
            const uint32_t first = row0 + (dual ? 8 * pw : 16 * pw) + cc * (16 / esz);
            if (first < a.rows) {
                if (isq)
                    cp_async16(sside + 2 * SB + blk * 512 + 4 * sr0, a.q2 + ((size_t)(kb * 2 + blk) * a.rows + first) * 4);
                else
                    cp_async16(sside + blk * SB + esz * sr0, a.s + ((size_t)(kb * 2 + blk) * a.rows + first) * esz);
            }
        }
    }
}

// -------------------------------------------------------- packed helpers --
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }
typedef unsigned long long u64;
__device__ __forceinline__ u64 f2pack(float a, float b) {
    return (u64)__float_as_uint(a) | ((u64)__float_as_uint(b) << 32);
}
__device__ __forceinline__ u64 ffma2(u64 a, u64 b, u64 c) {
    u64 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ u64 fmul2(u64 a, u64 b) {
    u64 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ u64 fsub2(u64 a, u64 b) {
    u64 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// RN16 of both fp32 lanes -> half2 (lane 0 low)
__device__ __forceinline__ uint32_t cvt_h2(u64 v) {
    return h2u(__floats2half2_rn(__uint_as_float((uint32_t)v), __uint_as_float((uint32_t)(v >> 32))));
}
// bytes b0, b1 of w (small unsigned ints) as exact floats 2^23 + b (magic), packed
__device__ __forceinline__ u64 bytes01_magic(uint32_t w, uint32_t sel0, uint32_t sel1) {
    return (u64)__byte_perm(w, 0x4B000000u, sel0) | ((u64)__byte_perm(w, 0x4B000000u, sel1) << 32);
}
#define MAGIC23 8388608.0f

// ------------------------------------------------- dequant from shared ----
// Half `half` (32 weights) of A row ar's 64 weights of step kb, as the
// reference's fp16 values (RN16 of the fp32 dequant, gguf.zig:751-1071 /
// load_gguf.zig:371), in natural k order: out[i] = weights 32 half + 8i .. +7.
// Arithmetic rounds where the reference rounds.
template <int T>
__device__ __forceinline__ void dequant_half(const uint8_t *slot, int ar, int half, uint32_t kb, bool dual,
                                             uint4 (&out)[4]) {
    using G = Geo<T>;
    const uint8_t *row = slot + ar * G::RAW_ROW;
    const uint8_t *side = slot + BM * G::RAW_ROW;
    auto chunk = [&](int c) { return *reinterpret_cast<const uint4 *>(row + raw_chunk<G::CH>(ar, c) * 16); };
    const int srow = dual ? (ar & 1) * 64 + (ar >> 1) : ar;  // side index of this row
    if (T == CUQ_Q8_0) {  // gguf.zig:827-840: RN16(d * q), the product is exact
        const __half2 off = __float2half2_rn(1152.f);
        const __half2 d = __half2half2(reinterpret_cast<const __half *>(side)[half * 128 + srow]);
#pragma unroll
        for (int c2 = 0; c2 < 2; c2++) {
            const uint4 v = chunk(2 * half + c2);
            const uint32_t wv[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
            uint32_t o[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                o[2 * i] = h2u(__hmul2(__hsub2(u2h(__byte_perm(wv[i], 0x64646464u, 0x4140u)), off), d));
                o[2 * i + 1] = h2u(__hmul2(__hsub2(u2h(__byte_perm(wv[i], 0x64646464u, 0x4342u)), off), d));
            }
            out[2 * c2] = make_uint4(o[0], o[1], o[2], o[3]);
            out[2 * c2 + 1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
    } else if (T == CUQ_Q4_K) {  // gguf.zig:962-996: fp32 (d*sc)*q - dmin*m, then RN16
        const uint32_t c = kb % 4;
        const uint4 meta = reinterpret_cast<const uint4 *>(side)[srow];
        const float d = __half2float(__ushort_as_half((uint16_t)(meta.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((uint16_t)(meta.x >> 16)));
        // sub-block 2c (low nibbles, half 0) or 2c+1 (high nibbles, half 1)
        const int j = 2 * c + half, sh = 8 * (j & 3);
        const uint32_t b0 = (meta.y >> sh) & 0xFFu, b1 = (meta.z >> sh) & 0xFFu, b2 = (meta.w >> sh) & 0xFFu;
        const int sc = j < 4 ? (int)(b0 & 63u) : (int)((b2 & 0xFu) | ((b0 >> 6) << 4));
        const int mm = j < 4 ? (int)(b1 & 63u) : (int)((b2 >> 4) | ((b1 >> 6) << 4));
        const float a = __fmul_rn(d, (float)sc), m = __fmul_rn(dmin, (float)mm);
        const u64 d1 = f2pack(a, a), nm1 = f2pack(-m, -m), mg = f2pack(MAGIC23, MAGIC23);
        const uint4 q0 = chunk(0), q1 = chunk(1);
        const uint32_t wv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {  // 4 weights (one word) per i
            const uint32_t nib = half ? ((wv[i] >> 4) & 0x0F0F0F0Fu) : (wv[i] & 0x0F0F0F0Fu);
            const u64 a01 = fsub2(bytes01_magic(nib, 0x7440u, 0x7441u), mg);
            const u64 a23 = fsub2(bytes01_magic(nib, 0x7442u, 0x7443u), mg);
            uint32_t *o = reinterpret_cast<uint32_t *>(&out[i / 2]);
            o[(i & 1) * 2] = cvt_h2(ffma2(d1, a01, nm1));
            o[(i & 1) * 2 + 1] = cvt_h2(ffma2(d1, a23, nm1));
        }
    } else if (T == CUQ_Q6_K) {  // gguf.zig:1036-1059: fp32 (d*sc) * (q-32), then RN16
        const uint32_t qtr = kb % 4, h = qtr / 2, tq = 2 * (qtr % 2) + half;
        const uint4 scv = reinterpret_cast<const uint4 *>(side)[srow];
        const float d = __half2float(reinterpret_cast<const __half *>(side + 2048)[srow]);
        const uint4 La = chunk((tq & 1) ? 2 : 0), Lb = chunk((tq & 1) ? 3 : 1), H0 = chunk(4), H1 = chunk(5);
        const uint32_t Lw[8] = {La.x, La.y, La.z, La.w, Lb.x, Lb.y, Lb.z, Lb.w};
        const uint32_t Hw[8] = {H0.x, H0.y, H0.z, H0.w, H1.x, H1.y, H1.z, H1.w};
        const u64 mg = f2pack(MAGIC23 + 32.f, MAGIC23 + 32.f);
#pragma unroll
        for (int sub = 0; sub < 2; sub++) {  // l in [16 sub, 16 sub + 16): one int8 scale
            const int si = 8 * h + 2 * tq + sub;
            const uint32_t sw = si < 4 ? scv.x : si < 8 ? scv.y : si < 12 ? scv.z : scv.w;
            const float scale = __fmul_rn(d, (float)(int)(int8_t)((sw >> (8 * (si & 3))) & 0xFFu));
            const u64 s2 = f2pack(scale, scale);
#pragma unroll
            for (int i = 0; i < 4; i++) {  // 4 words of 4 weights
                const int l4 = sub * 4 + i;
                const uint32_t L = Lw[l4];
                const uint32_t lo = (tq >= 2) ? ((L >> 4) & 0x0F0F0F0Fu) : (L & 0x0F0F0F0Fu);
                const uint32_t q = lo | (((Hw[l4] >> (2 * tq)) & 0x03030303u) << 4);
                const u64 a01 = fsub2(bytes01_magic(q, 0x7440u, 0x7441u), mg);
                const u64 a23 = fsub2(bytes01_magic(q, 0x7442u, 0x7443u), mg);
                uint32_t *o = reinterpret_cast<uint32_t *>(&out[l4 / 2]);
                o[(l4 & 1) * 2] = cvt_h2(fmul2(s2, a01));
                o[(l4 & 1) * 2 + 1] = cvt_h2(fmul2(s2, a23));
            }
        }
    } else if (T == CUQ_F16) {
#pragma unroll
        for (int c = 0; c < 4; c++) out[c] = chunk(4 * half + c);
    } else if (T == CUQ_BF16) {  // Gguf.readF16 of a bf16 tensor: RN16(f32(bf16))
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 v = chunk(4 * half + c);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                o[i] = h2u(__floats2half2_rn(__uint_as_float(wv[i] << 16), __uint_as_float(wv[i] & 0xFFFF0000u)));
            out[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    } else {  // legacy 32-blocks (gguf.zig:763-825), scalar fp32 as the reference; block = half
        constexpr int SE = (T == CUQ_Q4_1 || T == CUQ_Q5_1) ? 4 : 2;
        const uint4 qv = chunk(half);
        const uint8_t *bb = reinterpret_cast<const uint8_t *>(&qv);
        float dd, m = 0.f;
        if (SE == 2) {
            dd = __half2float(reinterpret_cast<const __half *>(side)[half * 128 + srow]);
        } else {
            const __half2 dm = reinterpret_cast<const __half2 *>(side)[half * 128 + srow];
            dd = __low2float(dm);
            m = __high2float(dm);
        }
        const uint32_t qh = (T == CUQ_Q5_0 || T == CUQ_Q5_1)
                                ? reinterpret_cast<const uint32_t *>(side + 2 * 128 * SE + half * 512)[srow]
                                : 0u;
        __half vals[32];
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int byte = bb[j & 15];
            const int nib = j < 16 ? (byte & 0xF) : (byte >> 4);
            float val;
            if (T == CUQ_Q4_0) {
                val = __fmul_rn((float)(nib - 8), dd);
            } else if (T == CUQ_Q4_1) {
                val = __fadd_rn(__fmul_rn((float)nib, dd), m);
            } else {
                const int hb = j < 16 ? (int)(((qh >> j) << 4) & 0x10u) : (int)((qh >> (j - 16 + 12)) & 0x10u);
                const float x = (float)((nib | hb) - (T == CUQ_Q5_0 ? 16 : 0));
                val = __fadd_rn(__fmul_rn(x, dd), m);
            }
            vals[j] = __float2half_rn(val);
        }
#pragma unroll
        for (int c = 0; c < 4; c++) out[c] = reinterpret_cast<const uint4 *>(vals)[c];
    }
}

// ---------------------------------------------------------------- TMA ----
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------- kernel ----

struct __align__(64) QgArgs {
    CUtensorMap mh, ml;        // x hi / lo [n][cols] fp16, box 32 x 256, 64-byte swizzle
    WPlanes w, w2;             // w2: the up matrix of a gate|up pair
    uint32_t n;
    float *y;                  // [n][ldy] fp32 output (STORE / ADD)
    uint32_t ldy;
    const float *bias;
    __half *oh, *ol;           // SILU: act hi / lo, [n][rows]
    int *err;                  // set to 1 when a wait timed out
};

// Persistent CTAs (one per SM), tiles (128 weight rows x 128 tokens) taken
// round-robin, row tiles fastest so neighbouring CTAs share the x tile in L2.
// Warps 0-7: weight producers (raw prefetch + dequant into the A stage; each
// warp owns 16 A rows, two threads per row); warp 8: TMEM allocation and the MMA
// issuer (lane 0); warp 9 lane 0: TMA loads of the x hi / lo tiles into the B
// stage; warps 10-13: epilogue.  Two TMEM
// accumulators (2 x 256 columns) let the epilogue of one tile overlap the
// main loop of the next.  The stage and raw rings run continuously across tiles.
constexpr int NTHREADS = 448;  // 8 producer warps, MMA, TMA, 4 epilogue warps

template <int T, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) qgemm_tc_kernel(const __grid_constant__ QgArgs p) {
    using G = Geo<T>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *raw = smem + STAGES * STAGE_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(raw + G::RAWD * G::SLOT);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;    // [2] MMA -> epilogue
    uint64_t *acc_empty = acc_full + 2;     // [2] epilogue -> MMA
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *stop = abort_flag + 1;  // [2] producers' per-step snapshot of abort_flag

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr bool DUAL = (EPI == EPI_SILU_XQ);
    const uint32_t rows = p.w.rows, cols = p.w.cols;
    const uint32_t nkb = cols / RAW_K;  // raw steps per tile; 2 MMA stages each
    const uint32_t rows_per_tile = DUAL ? BM / 2 : BM;
    const uint32_t mtiles = (rows + rows_per_tile - 1) / rows_per_tile, ntiles = (p.n + BN - 1) / BN;
    const uint32_t ntile_total = mtiles * ntiles;
    const uint32_t my_tiles = blockIdx.x < ntile_total ? (ntile_total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    auto tile_of = [&](uint32_t j, uint32_t &row0, uint32_t &tok0) {
        const uint32_t i = blockIdx.x + j * gridDim.x;
        row0 = (i % mtiles) * rows_per_tile;
        tok0 = (i / mtiles) * BN;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 129);  // 128 producer arrivals (one half each) + the TMA thread's expect_tx
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 128);
        }
        *abort_flag = 0;
        stop[0] = stop[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 8) {  // tensor memory: two 128 x 256 fp32 accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t total = my_tiles * nkb;  // steps this CTA runs

    if (warp < 8) {
        // ---------------------------------------------------- producers
        const int pw = warp, ar = 16 * pw + (lane >> 1), half = lane & 1;
        auto issue = [&](uint32_t gi) {
            uint32_t row0, tok0;
            tile_of(gi / nkb, row0, tok0);
            raw_issue<T>(p.w, p.w2, DUAL, row0, gi % nkb, raw + (gi % G::RAWD) * G::SLOT, pw, lane);
        };
        for (uint32_t i = 0; i + 1 < (uint32_t)G::RAWD; i++) {
            if (i < total) issue(i);
            cp_async_commit();
        }
        for (uint32_t gs = 0; gs < total; gs++) {
            // raw step gs feeds MMA stages 2gs (columns 0-31, half 0) and 2gs+1 (half 1)
            const uint32_t sg = 2 * gs + half;
            const int s = sg % STAGES;
            int stopw = 0;
            if (lane < 2) {  // lane 0 waits for the half-0 stage, lane 1 for the half-1 stage
                if (sg >= (uint32_t)STAGES) mbar_wait(&empty[s], ((sg / STAGES) - 1) & 1, abort_flag);
                stopw = *abort_flag;
            }
            stopw = __shfl_sync(0xffffffffu, stopw, 0) | __shfl_sync(0xffffffffu, stopw, 1);
            cp_async_wait<G::RAWD - 2>();
            __syncwarp();  // the warp's raw step gs landed; its slot of gs-1 is free
            if (stopw) break;
            if (gs + G::RAWD - 1 < total) issue(gs + G::RAWD - 1);
            cp_async_commit();
            uint4 vals[4];
            dequant_half<T>(raw + (gs % G::RAWD) * G::SLOT, ar, half, gs % nkb, DUAL, vals);
            uint8_t *A = smem + s * STAGE_BYTES;
#pragma unroll
            for (int c = 0; c < 4; c++) *reinterpret_cast<uint4 *>(A + ar * 64 + sw64_chunk(ar, c) * 16) = vals[c];
            fence_async_smem();
            mbar_arrive(&full[s]);
        }
        cp_async_wait<0>();
    } else if (warp == 8) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            uint32_t gs = 0;
            bool ok = true;
            for (uint32_t j = 0; j < my_tiles && ok; j++) {
                const uint32_t ab = j & 1;
                if (j >= 2 && !mbar_wait(&acc_empty[ab], ((j >> 1) - 1) & 1, abort_flag)) break;
                tc_fence_after();
                const uint32_t acc = tmem + ab * TMEM_COLS;
                for (uint32_t ks = 0; ks < 2 * nkb; ks++, gs++) {
                    const int s = gs % STAGES;
                    if (!mbar_wait(&full[s], (gs / STAGES) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(smem + s * STAGE_BYTES), b = a + A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 16; k++) {
                        const uint64_t ad = sdesc_sw64(a + 32 * k);
                        umma_f16(acc, ad, sdesc_sw64(b + 32 * k), (ks | k) ? 1u : 0u);        // A x_hi
                        umma_f16(acc, ad, sdesc_sw64(b + B_BYTES / 2 + 32 * k), 1u);          // + A x_lo
                    }
                    umma_commit(&empty[s]);  // frees the stage when these MMAs complete
                }
                if (ok) umma_commit(&acc_full[ab]);
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            // ------------------------------------------------ TMA: x hi / lo
            uint32_t gs = 0;
            for (uint32_t j = 0; j < my_tiles; j++) {
                uint32_t row0, tok0;
                tile_of(j, row0, tok0);
                bool ok = true;
                for (uint32_t ks = 0; ks < 2 * nkb; ks++, gs++) {
                    const int s = gs % STAGES;
                    if (gs >= (uint32_t)STAGES && !mbar_wait(&empty[s], ((gs / STAGES) - 1) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t b = smem_u32(smem + s * STAGE_BYTES + A_BYTES);
                    mbar_expect_tx(&full[s], B_BYTES);
                    tma_load_2d(b, &p.mh, (int)(ks * BK), (int)tok0, &full[s]);
                    tma_load_2d(b + B_BYTES / 2, &p.ml, (int)(ks * BK), (int)tok0, &full[s]);
                }
                if (!ok) break;
            }
        }
    } else {
        // ---------------------------------------------------- epilogue (warps 10-13)
        const uint32_t quarter = (uint32_t)(warp & 3);  // TMEM lanes this warp may read
        const uint32_t trow = quarter * 32 + lane;      // row of the tile = TMEM lane
        for (uint32_t j = 0; j < my_tiles; j++) {
            const uint32_t ab = j & 1;
            if (!mbar_wait(&acc_full[ab], (j >> 1) & 1, abort_flag)) break;
            tc_fence_after();
            uint32_t row0, tok0;
            tile_of(j, row0, tok0);
            const uint32_t acc = tmem + ab * TMEM_COLS + ((quarter * 32) << 16);
#pragma unroll 1
            for (int ch = 0; ch < BN / 32; ch++) {
                float hi[32];
                tmem_ld32(acc + ch * 32, hi);
                if (DUAL) {
                    // even lanes hold gate row row0 + trow/2, odd lanes the same row of up
                    const uint32_t r = row0 + (trow >> 1);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float mine = hi[i];
                        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
                        const uint32_t tok = tok0 + ch * 32 + i;
                        if ((trow & 1) || tok >= p.n || r >= rows) continue;
                        const float g = mine, u = other;
                        const float sg = 1.0f / (1.0f + expf(-g));  // cpu.siluMul (cpu.zig:65-70)
                        const float act = (g * sg) * u;
                        const __half ah = __float2half_rn(act);
                        p.oh[(size_t)tok * rows + r] = ah;
                        p.ol[(size_t)tok * rows + r] = __float2half_rn(act - __half2float(ah));
                    }
                } else {
                    const uint32_t r = row0 + trow;
                    if (r < rows) {
                        const float b = p.bias ? p.bias[r] : 0.f;
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            const uint32_t tok = tok0 + ch * 32 + i;
                            if (tok >= p.n) continue;
                            float v = hi[i];
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
            tc_fence_before();
            mbar_arrive(&acc_empty[ab]);  // this accumulator may be overwritten
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 0) *p.err = 1;
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TMEM_COLS)
                     : "memory");
    }
}

template <int T, int EPI>
int launch_tq(const QgArgs &a, uint32_t rows, uint32_t n, cudaStream_t s) {
    auto kern = qgemm_tc_kernel<T, EPI>;
    static bool attr_set = false;  // per instantiation
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<T>::SMEM);
        if (e != cudaSuccess) {
            set_error("qgemm: shared memory opt-in failed: %s", cudaGetErrorString(e));
            return CUQ_ECUDA;
        }
        attr_set = true;
    }
    const uint32_t rows_per_tile = EPI == EPI_SILU_XQ ? BM / 2 : BM;
    const uint32_t tiles = ((rows + rows_per_tile - 1) / rows_per_tile) * ((n + BN - 1) / BN);
    const uint32_t ctas = tiles < (uint32_t)sm_count_current() ? tiles : (uint32_t)sm_count_current();
    kern<<<ctas, NTHREADS, Geo<T>::SMEM, s>>>(a);
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

// Tensor map of an x part [n][cols] fp16 (row stride cols*2 bytes): boxes of
// 32 columns x 256 tokens in the 64-byte swizzle the MMA descriptors expect;
// tokens past n read as zero.
int make_x_map(CUtensorMap *m, const __half *base, uint32_t n, uint32_t cols) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16) {
        set_error("qgemm: activation must be 16-byte aligned with 16-byte rows");
        return CUQ_EINVAL;
    }
    cuuint64_t dims[2] = {cols, n};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {BK, BN};  // 32 columns (64 bytes) x 256 tokens
    cuuint32_t estr[2] = {1, 1};
    // the driver's encoder, looked up through the runtime (the library does not
    // link libcuda, so it loads on machines without a GPU driver)
    typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            set_error("qgemm: cuTensorMapEncodeTiled is not available from the driver");
            return CUQ_ECUDA;
        }
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(base), dims,
                                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("qgemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return CUQ_ECUDA;
    }
    return CUQ_OK;
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

size_t qgemm_scratch_halves(const Planes &w, bool dual) {
    return w.raw ? (size_t)w.rows * w.cols * (dual ? 2 : 1) : 0;
}

int launch_qgemm(const QgemmArgs &g, int epi, cudaStream_t s) {
    const Planes &w = *g.w;
    if (w.raw) {
        // expand to fp16 (the reference's own weight values) and run the fp16 GEMM
        if (!g.f16_scratch) {
            set_error("qgemm: ggml type %d needs an fp16 scratch buffer", w.type);
            return CUQ_EINVAL;
        }
        const bool dual = epi == EPI_SILU_XQ;
        const size_t n1 = (size_t)w.rows * w.cols;
        Planes f[2];
        for (int i = 0; i < (dual ? 2 : 1); i++) {
            const Planes &src = i ? *g.w2 : w;
            if (!src.raw || src.rows != w.rows || src.cols != w.cols) {
                set_error("qgemm: gate/up must share type and shape");
                return CUQ_EINVAL;
            }
            int rc = launch_dequant_planes_f16(src, g.f16_scratch + i * n1, s);
            if (rc) return rc;
            f[i].type = CUQ_F16;
            f[i].rows = w.rows;
            f[i].cols = w.cols;
            f[i].base = reinterpret_cast<uint8_t *>(g.f16_scratch + i * n1);
            f[i].nbytes = n1 * 2;
            f[i].off_q = 0;
        }
        QgemmArgs g2 = g;
        g2.w = &f[0];
        g2.w2 = dual ? &f[1] : nullptr;
        g2.f16_scratch = nullptr;
        return launch_qgemm(g2, epi, s);
    }
    if (!planes_fast_type(w.type)) {
        set_error("UnsupportedType: no tensor-core GEMM for ggml type %d", w.type);
        return CUQ_EUNSUPPORTED;
    }
    if (w.cols % RAW_K) {
        set_error("qgemm: cols (%u) must be a multiple of %d", w.cols, RAW_K);
        return CUQ_EINVAL;
    }
    if (epi == EPI_SILU_XQ && (!g.w2 || g.w2->type != w.type || g.w2->rows != w.rows || g.w2->cols != w.cols)) {
        set_error("qgemm: gate/up must share type and shape");
        return CUQ_EINVAL;
    }
    if (g.n == 0) return CUQ_OK;
    QgArgs a;
    int rc = make_x_map(&a.mh, g.xh, g.n, w.cols);
    if (rc == CUQ_OK) rc = make_x_map(&a.ml, g.xl, g.n, w.cols);
    if (rc) return rc;
    a.w = wplanes(w);
    if (g.w2) a.w2 = wplanes(*g.w2);
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
