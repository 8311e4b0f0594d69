// gemv_tma.cu -- the batch-1 quantized GEMV with its weights streamed by the
// Tensor Memory Accelerator: the decode projection (engine.zig:547-819) for the
// block types of the benchmark configs (Q4_K, Q6_K, Q8_0).
//
// A decode GEMV reads every weight byte once and does little arithmetic per
// byte, so what bounds it is how many bytes are in flight to HBM.  Register
// prefetch (the other GEMV kernel) keeps a few KB per warp in flight; here one
// thread of each CTA requests the CTA's whole K range for its 16-row tile at
// launch, as TMA tensor copies into shared memory (up to ~48 KB per CTA, four
// CTAs per SM), before it even waits for the activation, so the weights of a
// whole matrix are requested within a few microseconds of the launch.  Each
// stage of ST iterations lands on its own mbarrier; the eight warps decode from
// shared memory as the stages land, with the same register decoders and
// tensor-core fragments as the other kernel (gemv_impl.cuh), and the same
// epilogues, split-K reduction and post-ops.
//
// Shared-memory layout of one stage (per matrix; a gate|up CTA holds both):
//   Q4_K: q   [ST][16 rows][128 B]  (3-D box, 128-byte swizzle: 16-byte chunk c
//                                    of row r at c ^ (r & 7))
//         meta[ST][16 rows][16 B]   (d, dmin, scales: the planes' block-major record)
//   Q6_K: ql  [ST][16][128 B] swizzled, qh [ST][16][64 B], sc [ST][16][16 B], d [ST][16] fp16
//   Q8_0: q   [ST/2 lines][16][128 B] swizzled (a line = 128 columns = 2 iterations),
//         d   [ST*2 blocks][16] fp16
// The tensor maps address the planes (common.cuh) directly, so the weight
// layout in HBM is the one the GEMM and the other kernels read.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "gemv_impl.cuh"
#include "tp.cuh"

namespace cuq {

namespace {

constexpr int TMA_MAX_STAGES = 24;
constexpr size_t TMA_CTA_BYTES = 49152;  // weight bytes one CTA stages at most
constexpr unsigned long long TMA_WAIT_NS = 2000000000ull;  // a stage wait gives up after 2 s

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void tbar_init(uint64_t *bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool tbar_try(uint64_t *bar) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0, 10000;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar))
        : "memory");
    return ok != 0;
}
// Bounded wait for a stage (each barrier completes one phase, parity 0).
// False when it did not land within TMA_WAIT_NS or another warp gave up.
__device__ __forceinline__ bool tbar_wait(uint64_t *bar, volatile int *abort_flag) {
    if (tbar_try(bar)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (!tbar_try(bar)) {
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > TMA_WAIT_NS) {
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ uint4 lds16(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

// ------------------------------------------------------ per-type geometry --
// ST iterations per stage; plane offsets and sizes inside one matrix's slice of
// a stage (swizzled planes first, at 1024-byte aligned offsets); TX = bytes the
// stage's copies deliver per matrix; SLICE = the slice's size in shared memory.
template <class TT> struct TmaGeo;

template <> struct TmaGeo<TQ4K> {
    static constexpr int ST = 4;
    static constexpr uint32_t Q = 0, META = 8192, TX = 9216, SLICE = 9216;
    __device__ static void issue(uint32_t dst, const CUtensorMap *m, uint32_t tile, int it, uint64_t *bar) {
        tma_3d(dst + Q, &m[0], 0, (int)tile * 16, it, bar);
        tma_2d(dst + META, &m[1], (int)tile * 256, it, bar);
    }
    // this lane's Raw of slot j: rows g and g + 8, 32-byte group tig
    __device__ static void load(TQ4K::Raw &R, const uint8_t *sb, int j, int g, int tig) {
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const int row = g + 8 * rr;
            const uint8_t *line = sb + Q + (j * 16 + row) * 128;
            R.q[rr][0] = lds16(line + (((2 * tig) ^ (row & 7)) << 4));
            R.q[rr][1] = lds16(line + (((2 * tig + 1) ^ (row & 7)) << 4));
            R.meta[rr] = lds16(sb + META + j * 256 + row * 16);
        }
    }
};

template <> struct TmaGeo<TQ6K> {
    static constexpr int ST = 4;
    static constexpr uint32_t QL = 0, QH = 8192, SC = 12288, D = 13312, TX = 13440, SLICE = 14336;
    __device__ static void issue(uint32_t dst, const CUtensorMap *m, uint32_t tile, int it, uint64_t *bar) {
        tma_3d(dst + QL, &m[0], 0, (int)tile * 16, it, bar);
        tma_3d(dst + QH, &m[1], 0, (int)tile * 16, it, bar);
        tma_2d(dst + SC, &m[2], (int)tile * 256, it, bar);
        tma_2d(dst + D, &m[3], (int)tile * 32, it, bar);
    }
    // the ql chunks a lane needs are a = 4h + (tig & 1) and a + 2 (h = tig / 2);
    // lanes with odd tig load them in the other order, which keeps each load's
    // eight lanes of a phase (rows g, g + 1) on distinct swizzled chunks
    __device__ static void load(TQ6K::Raw &R, const uint8_t *sb, int j, int g, int tig) {
        const int hh = tig >> 1, odd = tig & 1;
        const int ca = hh * 4 + odd, cb = ca + 2;
        const int c1 = odd ? cb : ca, c2 = odd ? ca : cb;
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const int row = g + 8 * rr;
            const uint8_t *line = sb + QL + (j * 16 + row) * 128;
            const uint4 v1 = lds16(line + ((c1 ^ (row & 7)) << 4));
            const uint4 v2 = lds16(line + ((c2 ^ (row & 7)) << 4));
            R.a[rr] = odd ? v2 : v1;
            R.b[rr] = odd ? v1 : v2;
            R.h[rr] = lds16(sb + QH + (j * 16 + row) * 64 + (hh * 2 + odd) * 16);
            R.scv[rr] = lds16(sb + SC + j * 256 + row * 16);
            R.d[rr] = *reinterpret_cast<const __half *>(sb + D + j * 32 + row * 2);
        }
    }
};

template <> struct TmaGeo<TQ8_0> {
    static constexpr int ST = 8;  // 8 iterations of 64 columns: 4 lines of 128
    static constexpr uint32_t Q = 0, DS = 8192, TX = 8704, SLICE = 9216;
    __device__ static void issue(uint32_t dst, const CUtensorMap *m, uint32_t tile, int it, uint64_t *bar) {
#pragma unroll
        for (int l = 0; l < 4; l++) tma_2d(dst + Q + l * 2048, &m[0], it * 64 + l * 128, (int)tile * 16, bar);
        tma_2d(dst + DS, &m[1], (int)tile * 32, it * 2, bar);
    }
    __device__ static void load(TQ8_0::Raw &R, const uint8_t *sb, int j, int g, int tig) {
        const int chunk = (j & 1) * 4 + tig, blk = j * 2 + (tig >> 1);
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const int row = g + 8 * rr;
            R.q[rr] = lds16(sb + Q + (j >> 1) * 2048 + row * 128 + ((chunk ^ (row & 7)) << 4));
            R.d[rr] = __half2half2(*reinterpret_cast<const __half *>(sb + DS + blk * 32 + row * 2));
        }
    }
};

struct __align__(64) TmaGemvArgs {
    CUtensorMap map[2][4];  // [matrix][plane] (matrix 1: the up weight of a gate|up pair)
    KArgs k;
    int ni;                 // iterations over the whole K
    int per;                // iterations per K part (gridDim.y parts)
    int *err;               // set when a stage wait gave up (may be null)
    uint32_t xs_off;        // k.ss_in: byte offset of the CTA's staged input in dynamic shared memory
};

// One CTA: 16-row tile blockIdx.x (of both matrices for gate|up), K part
// blockIdx.y.  Thread 0 requests every stage of the part, then all threads wait
// for the activation (programmatic dependent launch) and the eight warps walk
// the iterations (warp w takes iterations w, w + 8, ...; gate|up: warps 0-3 the
// gate rows and 4-7 the up rows, four each).  Eight warps rather than four: the
// decoders are issue-bound and shared memory limits the CTAs per SM; measured,
// a persistent variant (a producer warp feeding a ring across tiles) was slower.
constexpr int TMA_WARPS = 8;  // warps per CTA

template <class TT, int EPI>
__global__ void __launch_bounds__(32 * TMA_WARPS, 4) gemv_tma_kernel(const __grid_constant__ TmaGemvArgs P) {
    using G = TmaGeo<TT>;
    constexpr bool DUAL = (EPI == EPI_SILU_XQ);
    constexpr int NMAT = DUAL ? 2 : 1, KWE = DUAL ? TMA_WARPS / 2 : TMA_WARPS;
    extern __shared__ __align__(1024) uint8_t tma_dyn_raw[];
    // the 128-byte swizzle needs 1024-byte aligned boxes: align the base by hand
    // (the launch adds 1024 bytes of slack)
    uint8_t *tma_dyn = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tma_dyn_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ GemvShared sh;
    __shared__ __align__(8) uint64_t bars[TMA_MAX_STAGES];
    __shared__ int abort_flag;
    const KArgs &p = P.k;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const uint32_t tile = blockIdx.x, by = blockIdx.y;
    const int it0 = (int)by * P.per, it1 = min(P.ni, it0 + P.per);
    const int nst = it1 > it0 ? (it1 - it0 + G::ST - 1) / G::ST : 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; s++) tbar_init(&bars[s]);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // the weights do not depend on the previous kernel: request them all now
        const uint32_t base = smem_addr(tma_dyn);
        for (int s = 0; s < nst; s++) {
            tbar_expect_tx(&bars[s], NMAT * G::TX);
#pragma unroll
            for (int m = 0; m < NMAT; m++)
                G::issue(base + (uint32_t)(s * NMAT + m) * G::SLICE, P.map[m], tile, it0 + s * G::ST, &bars[s]);
        }
    }
    griddep_wait();
    griddep_launch();

    // The input from the residual (k.ss_in): this CTA's K range [kc0, kc0 +
    // klen) of xq = split((x * inv) * w) (cpu.rmsnorm, cpu.zig:11-18), with
    // mean(x^2) from the producer's per-tile sums of squares (summed in a
    // fixed order), staged in shared memory: hi halves, then lo halves.
    const uint32_t kc0 = (uint32_t)it0 * TT::SPAN, klen = (uint32_t)P.per * TT::SPAN;
    __half *xs = reinterpret_cast<__half *>(tma_dyn + P.xs_off);
    if (p.ss_in) {
        // each thread: 8 consecutive columns per pass, all loads issued before
        // the mean square is known (one L2 round trip per pass)
        constexpr int XP = 1;  // passes held in registers (more run below, loads then math)
        float4 xv[XP][2], wv[XP][2];
#pragma unroll
        for (int ps = 0; ps < XP; ps++) {
            const uint32_t i = (ps * blockDim.x + threadIdx.x) * 8u, c = kc0 + i;
            const bool in = i < klen && c < p.pre_n;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                xv[ps][h] = in ? __ldcg(reinterpret_cast<const float4 *>(p.pre_x + c) + h) : make_float4(0, 0, 0, 0);
                wv[ps][h] = in ? __ldg(reinterpret_cast<const float4 *>(p.pre_w + c) + h) : make_float4(0, 0, 0, 0);
            }
        }
        __shared__ float s_inv;
        if (warp == 0) {
            float s = 0.f;
            for (uint32_t i = lane; i < p.pre_n / 16; i += 32) s += __ldcg(p.ss_in + i);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) s_inv = 1.0f / sqrtf(s / (float)p.pre_n + p.pre_eps);
        }
        __syncthreads();
        const float inv = s_inv;
        // (x * inv) * w for 8 columns at i, then hi / lo halves in the
        // fragment order (0, 2, 1, 3) of each group of 4
        auto emit = [&](uint32_t i, const float4 &x0, const float4 &x1, const float4 &w0, const float4 &w1) {
            const float f[8] = {(x0.x * inv) * w0.x, (x0.y * inv) * w0.y, (x0.z * inv) * w0.z, (x0.w * inv) * w0.w,
                                (x1.x * inv) * w1.x, (x1.y * inv) * w1.y, (x1.z * inv) * w1.z, (x1.w * inv) * w1.w};
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int a = (q >> 1) * 4 + (q & 1), b = a + 2;  // pairs (0,2) (1,3) (4,6) (5,7)
                const __half ha = __float2half_rn(f[a]), hb = __float2half_rn(f[b]);
                hw[q] = h2u(__halves2half2(ha, hb));
                lw[q] = h2u(__halves2half2(__float2half_rn(f[a] - __half2float(ha)),
                                           __float2half_rn(f[b] - __half2float(hb))));
            }
            *reinterpret_cast<uint4 *>(xs + i) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(xs + klen + i) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        };
#pragma unroll
        for (int ps = 0; ps < XP; ps++) {
            const uint32_t i = (ps * blockDim.x + threadIdx.x) * 8u;
            if (i < klen) emit(i, xv[ps][0], xv[ps][1], wv[ps][0], wv[ps][1]);
        }
        for (uint32_t i = (XP * blockDim.x + threadIdx.x) * 8u; i < klen; i += blockDim.x * 8u) {
            const uint32_t c = kc0 + i;
            const bool in = c < p.pre_n;
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 *xp = reinterpret_cast<const float4 *>(p.pre_x + c);
            const float4 *wp = reinterpret_cast<const float4 *>(p.pre_w + c);
            emit(i, in ? __ldcg(xp) : z, in ? __ldcg(xp + 1) : z, in ? __ldg(wp) : z, in ? __ldg(wp + 1) : z);
        }
        __syncthreads();
    }
    // (when the producer wrote xq, the k-steps read it from global memory through
    // L1: copying the K range to shared memory first measured slower)

    const int m = DUAL ? warp / KWE : 0, kw = DUAL ? warp % KWE : warp;
    const __half *xb = p.ss_in ? xs + (g == 1 ? klen : 0u) - kc0 : p.xq + (g == 1 ? p.kpad : 0);
    const bool bl = g < 2;
    // two accumulators (even and odd k-steps) halve the MMA dependency chain
    float c[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int it = it0 + kw; it < it1; it += KWE) {
        const int j = it - it0, s = j / G::ST;
        if (!tbar_wait(&bars[s], &abort_flag)) {
            ok = false;
            break;
        }
        const uint8_t *sb = tma_dyn + (size_t)(s * NMAT + m) * G::SLICE;
        typename TT::Raw R;
        G::load(R, sb, j % G::ST, g, tig);
        typename TT::Prep Pp;
        TT::prep(R, tig, Pp);
#pragma unroll
        for (int k = 0; k < TT::KSTEPS; k++) {
            uint2 b = make_uint2(0u, 0u);
            if (bl) b = *reinterpret_cast<const uint2 *>(xb + TT::koff(it, tig, k));
            uint32_t a[4];
            TT::frag(R, Pp, k, a);
            if (k & 1)
                mma16816(c2, a[0], a[1], a[2], a[3], b.x, b.y);
            else
                mma16816(c, a[0], a[1], a[2], a[3], b.x, b.y);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) c[i] += c2[i];
    if (!ok && P.err) atomicExch(P.err, 1);
    __syncthreads();
    if (abort_flag && threadIdx.x == 0) {
        // a stage never landed: wait (bounded again) for the copies still in
        // flight before the CTA's shared memory is released
        for (int s = 0; s < nst; s++) {
            const unsigned long long t0 = globaltimer_ns();
            while (!tbar_try(&bars[s]) && globaltimer_ns() - t0 < TMA_WAIT_NS) {
            }
        }
    }
    if (!gemv_finish<TT, EPI, TMA_WARPS, TMA_WARPS>(p, tile, by, sh, c, 0.f, 0.f)) return;
    gemv_post_op(p, tma_dyn);
}

// ----------------------------------------------------------------- host ---

typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                             const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// A byte-element tensor map over one plane: dims[0] innermost (contiguous
// bytes), strides in bytes for dims 1.., box as given.  Out-of-range boxes read
// as zero bytes (a zero quant block or scale dequantises to zero weights).
int encode_u8(CUtensorMap *m, const void *base, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
              const cuuint32_t *box, bool swizzle128) {
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            set_error("gemv: cuTensorMapEncodeTiled is not available from the driver");
            return CUQ_ECUDA;
        }
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void *>(base), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("gemv: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return CUQ_ECUDA;
    }
    return CUQ_OK;
}

// The tensor maps of one weight's planes for the stage layout above.
int make_maps(const Planes &w, CUtensorMap (&m)[4]) {
    const uint8_t *q = w.base + w.off_q;
    const cuuint64_t R = w.rows, K = w.cols;
    int rc = CUQ_OK;
    switch (w.type) {
    case CUQ_Q4_K: {
        const cuuint64_t nsb = K / 256;
        const cuuint64_t d0[3] = {128, R, nsb}, s0[2] = {K / 2, 128};
        const cuuint32_t b0[3] = {128, 16, (cuuint32_t)TmaGeo<TQ4K>::ST};
        if ((rc = encode_u8(&m[0], q, 3, d0, s0, b0, true))) return rc;
        const cuuint64_t d1[2] = {R * 16, nsb}, s1[1] = {R * 16};
        const cuuint32_t b1[2] = {256, (cuuint32_t)TmaGeo<TQ4K>::ST};
        return encode_u8(&m[1], w.base + w.off_s, 2, d1, s1, b1, false);
    }
    case CUQ_Q6_K: {
        constexpr cuuint32_t ST = TmaGeo<TQ6K>::ST;
        const cuuint64_t nsb = K / 256;
        const cuuint64_t d0[3] = {128, R, nsb}, s0[2] = {K / 2, 128};
        const cuuint32_t b0[3] = {128, 16, ST};
        if ((rc = encode_u8(&m[0], q, 3, d0, s0, b0, true))) return rc;
        const cuuint64_t d1[3] = {64, R, nsb}, s1[2] = {K / 4, 64};
        const cuuint32_t b1[3] = {64, 16, ST};
        if ((rc = encode_u8(&m[1], w.base + w.off_q2, 3, d1, s1, b1, false))) return rc;
        const cuuint64_t d2[2] = {R * 16, nsb}, s2[1] = {R * 16};
        const cuuint32_t b2[2] = {256, ST};
        if ((rc = encode_u8(&m[2], w.base + w.off_s, 2, d2, s2, b2, false))) return rc;
        const cuuint64_t d3[2] = {R * 2, nsb}, s3[1] = {R * 2};
        const cuuint32_t b3[2] = {32, ST};
        return encode_u8(&m[3], w.base + w.off_s2, 2, d3, s3, b3, false);
    }
    case CUQ_Q8_0: {
        const cuuint64_t d0[2] = {K, R}, s0[1] = {K};
        const cuuint32_t b0[2] = {128, 16};
        if ((rc = encode_u8(&m[0], q, 2, d0, s0, b0, true))) return rc;
        const cuuint64_t d1[2] = {R * 2, K / 32}, s1[1] = {R * 2};
        const cuuint32_t b1[2] = {32, (cuuint32_t)(2 * TmaGeo<TQ8_0>::ST)};
        return encode_u8(&m[1], w.base + w.off_s, 2, d1, s1, b1, false);
    }
    }
    set_error("gemv: no TMA layout for ggml type %d", w.type);
    return CUQ_EUNSUPPORTED;
}

// Iterations, stage size and bytes per iteration (per matrix) of a weight.
void tma_geometry(const Planes &w, int &ni, int &st, uint32_t &it_bytes) {
    switch (w.type) {
    case CUQ_Q4_K: st = TmaGeo<TQ4K>::ST; it_bytes = TmaGeo<TQ4K>::SLICE / st; ni = (int)(w.cols / 256); break;
    case CUQ_Q6_K: st = TmaGeo<TQ6K>::ST; it_bytes = TmaGeo<TQ6K>::SLICE / st; ni = (int)(w.cols / 256); break;
    default: st = TmaGeo<TQ8_0>::ST; it_bytes = TmaGeo<TQ8_0>::SLICE / st; ni = (int)((w.cols + 63) / 64); break;
    }
}

template <class TT, int EPI>
cudaError_t launch_one(const TmaGemvArgs &args, dim3 grid, size_t smem, bool pdl, cudaStream_t s) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(gemv_tma_kernel<TT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set = true;
    }
    return launch_maybe_pdl(gemv_tma_kernel<TT, EPI>, grid, dim3(32 * TMA_WARPS), smem, s, pdl, args);
}

template <class TT>
cudaError_t launch_epi_tma(int epi, const TmaGemvArgs &args, dim3 grid, size_t smem, bool pdl, cudaStream_t s) {
    switch (epi) {
    case EPI_STORE: return launch_one<TT, EPI_STORE>(args, grid, smem, pdl, s);
    case EPI_ADD: return launch_one<TT, EPI_ADD>(args, grid, smem, pdl, s);
    case EPI_SILU_XQ: return launch_one<TT, EPI_SILU_XQ>(args, grid, smem, pdl, s);
    case EPI_ARGMAX: return launch_one<TT, EPI_ARGMAX>(args, grid, smem, pdl, s);
    case EPI_TP_PUSH: return launch_one<TT, EPI_TP_PUSH>(args, grid, smem, pdl, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

// The block types the TMA-fed kernels decode.  CUQ_GEMV_TMA is a bit mask of
// the types that use them (bit 0 Q4_K, bit 1 Q6_K, bit 2 Q8_0; default all);
// the others run the register-prefetch kernel.
bool gemv_tma_supported(int type) {
    static int mask = -1;
    if (mask < 0) {
        const char *e = getenv("CUQ_GEMV_TMA");
        mask = e ? atoi(e) & 7 : 7;
    }
    switch (type) {
    case CUQ_Q4_K: return mask & 1;
    case CUQ_Q6_K: return mask & 2;
    case CUQ_Q8_0: return mask & 4;
    }
    return false;
}

// K parts of a TMA GEMV: enough that a part's weights (both matrices of a
// gate|up pair) fit TMA_CTA_BYTES, and about four CTAs per SM in total when the
// matrix has few tiles, with at least one stage per part.
int gemv_tma_ksplit(const Planes &w, int nmat, int sm_count) {
    int ni, st;
    uint32_t itb;
    tma_geometry(w, ni, st, itb);
    const int tiles = (int)(w.rows / 16);
    const int sm = sm_count > 0 ? sm_count : 148;
    const size_t total = (size_t)ni * itb * nmat;
    int k = (int)((total + TMA_CTA_BYTES - 1) / TMA_CTA_BYTES);
    const int want = (4 * sm + tiles - 1) / tiles;
    if (want > k) k = want;
    const int maxk = (ni + st - 1) / st;  // a stage per part at least
    if (k > maxk) k = maxk;
    if (k > 16) k = 16;
    if (k < 1) k = 1;
    // parts of whole stages
    const int per = ((ni + k - 1) / k + st - 1) / st * st;
    return (ni + per - 1) / per;
}

int launch_gemv_tma(const GemvArgs &a, int epi, cudaStream_t s) {
    const Planes &w = *a.w;
    if (!gemv_tma_supported(w.type) || (a.pre_w && !a.ss_in)) return CUQ_EUNSUPPORTED;
    if (a.ss_in && (!a.pre_x || !a.pre_w || a.pre_n != w.cols || a.pre_n % 16)) {
        set_error("gemv: the input norm needs x and its weight of cols (%u) floats", w.cols);
        return CUQ_EINVAL;
    }
    const bool dual = epi == EPI_SILU_XQ;
    TmaGemvArgs args;
    memset(&args, 0, sizeof(args));
    int rc = make_maps(w, args.map[0]);
    if (rc) return rc;
    if (dual && (rc = make_maps(*a.w2, args.map[1]))) return rc;
    args.k = make_kargs(a);
    int st;
    uint32_t itb;
    tma_geometry(w, args.ni, st, itb);
    const int ksplit = a.ksplit < 1 ? 1 : a.ksplit;
    args.per = ((args.ni + ksplit - 1) / ksplit + st - 1) / st * st;
    args.k.ksplit = ksplit;
    args.err = a.err;
    const int nst = (args.per + st - 1) / st;
    if (nst > TMA_MAX_STAGES) {
        set_error("gemv: %d stages per CTA exceed the %d barriers (ksplit %d too small)", nst, TMA_MAX_STAGES, ksplit);
        return CUQ_EINVAL;
    }
    uint32_t slice;
    switch (w.type) {
    case CUQ_Q4_K: slice = TmaGeo<TQ4K>::SLICE; break;
    case CUQ_Q6_K: slice = TmaGeo<TQ6K>::SLICE; break;
    default: slice = TmaGeo<TQ8_0>::SLICE; break;
    }
    size_t smem = (size_t)nst * (dual ? 2 : 1) * slice;
    if (a.ss_in) {  // the staged input: klen hi + klen lo halves
        args.xs_off = (uint32_t)((smem + 15) & ~(size_t)15);
        smem = args.xs_off + 2 * sizeof(__half) * (size_t)args.per * (w.type == CUQ_Q8_0 ? 64 : 256);
    }
    const bool norm = a.post.op == POST_RMSNORM || a.post.op == POST_TP_REDUCE;
    if (norm && a.post.n % 16 == 0 && a.post.n <= RN_MAX && smem < sizeof(float) * a.post.n)
        smem = sizeof(float) * a.post.n;
    smem += 1024;  // alignment slack of the swizzled boxes
    dim3 grid(w.rows / 16, ksplit);
    cudaError_t e;
    switch (w.type) {
    case CUQ_Q4_K: e = launch_epi_tma<TQ4K>(epi, args, grid, smem, a.pdl, s); break;
    case CUQ_Q6_K: e = launch_epi_tma<TQ6K>(epi, args, grid, smem, a.pdl, s); break;
    default: e = launch_epi_tma<TQ8_0>(epi, args, grid, smem, a.pdl, s); break;
    }
    if (e != cudaSuccess) {
        set_error("gemv (TMA) launch: %s", cudaGetErrorString(e));
        return CUQ_ECUDA;
    }
    return CUQ_OK;
}

}  // namespace cuq
