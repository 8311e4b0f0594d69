// gemv.cu -- batch-1 quantized GEMV, the decode projection (engine.zig:547-819 qkv/o/ffn/head).
//
// Design (HBM-bound; one pass over the quantized bytes, nothing else):
//   * A warp owns 16 rows.  Each lane streams 128-bit, L1-bypassing loads of
//     its rows' quant bytes from the planes layout and dequantises them in
//     registers to fp16 -- for Q8_0/Q4_0/Q4_1/Q5_x/F16/BF16 exactly the
//     reference's fp16 weight RN16(dequant_f32) (load_gguf.zig:371); for the
//     K-quants as RN16 of the exact scaled quant, with Q4_K's minimum term
//     subtracted in fp32 after the MMA (see TQ4K).
//   * The fp16 weights are the A operand of mma.sync m16n8k16 (fp32
//     accumulate).  B holds the activation split as x = hi + lo (two fp16
//     columns, ~22 bits), so the tensor core does the dot products and the
//     CUDA cores only unpack bits: 1-2 ALU ops per weight.
//   * Within each group of 4 columns a lane feeds the pairs (0,2) and (1,3),
//     which is what PRMT/LOP3 produce from packed bytes without shuffles; the
//     activation is stored in the same permuted order ("xq", common.cuh).
//   * 4 warps per CTA split the CTA's K range; split-K across CTAs (ksplit)
//     reduces deterministically through a workspace: the last CTA of a tile
//     (atomic ticket) sums the partials in a fixed order and resets the ticket.
#include <type_traits>

#include "common.cuh"
#include "gemv_impl.cuh"
#include "tp.cuh"

namespace cuq {

namespace {

template <class TT, int EPI, int KW, int D>
__global__ void __launch_bounds__(128) gemv_kernel(const KArgs p) {
    __shared__ GemvShared sh;
    // the pre-norm's x stage and xq (before the body), the post-op's x stage (after)
    extern __shared__ __align__(16) uint8_t gemv_dyn[];
    const bool pre = p.pre_w != nullptr;
    float4 *pre_stage = reinterpret_cast<float4 *>(gemv_dyn);
    __half *pre_xq = reinterpret_cast<__half *>(gemv_dyn + sizeof(float) * p.pre_n);
    if (!gemv_body<TT, EPI, KW, D>(
            p, blockIdx.x, blockIdx.y, sh,
            [&] {
                griddep_wait();
                griddep_launch();
                if (pre) {  // the RMSNorm this GEMV reads, computed by every CTA
                    reduce_norm_xq_block(const_cast<float *>(p.pre_x), nullptr, 0, nullptr, p.pre_w, p.pre_n,
                                         p.pre_eps, pre_xq, p.kpad, pre_stage);
                    __syncthreads();
                }
            },
            pre ? pre_xq : nullptr, pre ? xq_sums(pre_xq, p.kpad) : nullptr))
        return;
    gemv_post_op(p, gemv_dyn);
}

template <class TT, int EPI, int KW>
cudaError_t launch_kw(const GemvArgs &a, const KArgs &k, cudaStream_t s) {
    constexpr int D = TT::DEPTH;
    constexpr int TPC = EPI == EPI_SILU_XQ ? 1 : 4 / KW;
    dim3 grid((a.w->rows / 16 + TPC - 1) / TPC, k.ksplit);
    // the RMSNorm post-ops stage x in dynamic shared memory (reduce_norm_xq_block)
    const bool norm = a.post.op == POST_RMSNORM || a.post.op == POST_TP_REDUCE;
    size_t smem = norm && a.post.n % 16 == 0 && a.post.n <= RN_MAX ? sizeof(float) * a.post.n : 0;
    if (a.pre_w) {
        const size_t pre = sizeof(float) * a.pre_n + sizeof(__half) * xq_halves(a.pre_n);
        if (pre > smem) smem = pre;
    }
    return launch_maybe_pdl(gemv_kernel<TT, EPI, KW, D>, grid, dim3(128), smem, s, a.pdl, k);
}

template <class TT, int EPI>
cudaError_t launch_epi(const GemvArgs &a, const KArgs &k, int kw, cudaStream_t s) {
    if (EPI == EPI_SILU_XQ) return launch_kw<TT, EPI, 2>(a, k, s);  // dual: 2 warps per matrix, one tile per CTA
    if (std::is_same<TT, TRaw>::value) return launch_kw<TT, EPI, 4>(a, k, s);
    switch (kw) {
    case 1: return launch_kw<TT, EPI, 1>(a, k, s);
    case 2: return launch_kw<TT, EPI, 2>(a, k, s);
    default: return launch_kw<TT, EPI, 4>(a, k, s);
    }
}

template <class TT>
int launch_t(const GemvArgs &a, int epi, cudaStream_t s) {
    const KArgs k = make_kargs(a);
    // the raw-block decoder runs one shape of CTA (four warps per tile)
    const int kw = std::is_same<TT, TRaw>::value ? 4 : gemv_pick_plan(*a.w, 0).kw;
    cudaError_t e;
    switch (epi) {
    case EPI_STORE: e = launch_epi<TT, EPI_STORE>(a, k, kw, s); break;
    case EPI_ADD: e = launch_epi<TT, EPI_ADD>(a, k, kw, s); break;
    case EPI_SILU_XQ: e = launch_epi<TT, EPI_SILU_XQ>(a, k, kw, s); break;
    case EPI_ARGMAX: e = launch_epi<TT, EPI_ARGMAX>(a, k, kw, s); break;
    case EPI_TP_PUSH: e = launch_epi<TT, EPI_TP_PUSH>(a, k, kw, s); break;
    default: set_error("bad epilogue %d", epi); return CUQ_EINVAL;
    }
    if (e != cudaSuccess) {
        set_error("gemv launch: %s", cudaGetErrorString(e));
        return CUQ_ECUDA;
    }
    return CUQ_OK;
}

// -------------------------------------------------------------- xq makers --

__global__ void to_xq_kernel(const float *__restrict__ x, uint32_t n, uint32_t x_stride, __half *__restrict__ xq,
                             uint32_t kpad, size_t vec_stride) {
    const uint32_t v = blockIdx.y;
    const float *xv = x + (size_t)v * x_stride;
    __half *o = xq + (size_t)v * vec_stride;
    float *sums = xq_sums(o, kpad);
    // launched with exactly kpad threads per vector (kpad % 256 == 0): one
    // column each, and 16 consecutive columns in each aligned group of 16 lanes
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < kpad; i += gridDim.x * blockDim.x) {
        float f = i < n ? xv[i] : 0.f;
        __half hi = __float2half_rn(f);
        __half lo = __float2half_rn(f - __half2float(hi));
        uint32_t pos = xq_pos(i);
        o[pos] = hi;
        o[kpad + pos] = lo;
        float a = f;
#pragma unroll
        for (int o2 = 1; o2 < 16; o2 <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o2);
        if ((i & 15u) == 0) sums[i >> 4] = a;
    }
}

// One CTA per row: cpu.rmsnorm (cpu.zig:11-18), then the xq split.
__global__ void rmsnorm_xq_kernel(const float *__restrict__ x, const float *__restrict__ w, uint32_t n, float eps,
                                  __half *__restrict__ xq, uint32_t kpad, size_t vec_stride, float *h_out) {
    griddep_wait();
    griddep_launch();
    rmsnorm_xq_block(x + (size_t)blockIdx.x * n, w, n, eps, xq + (size_t)blockIdx.x * vec_stride, kpad,
                     h_out ? h_out + (size_t)blockIdx.x * n : nullptr);
}

}  // namespace

int launch_to_xq(const float *x, uint32_t n, uint32_t n_vec, uint32_t x_stride, __half *xq, cudaStream_t s) {
    uint32_t kpad = xq_pad(n);
    dim3 grid((kpad + 255) / 256, n_vec);
    to_xq_kernel<<<grid, 256, 0, s>>>(x, n, x_stride, xq, kpad, xq_halves(n));
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_rmsnorm_xq_pdl(const float *x, const float *w, uint32_t n, float eps, __half *xq, cudaStream_t s) {
    cudaError_t e = launch_maybe_pdl(rmsnorm_xq_kernel, dim3(1), dim3(1024), 0, s, true, x, w, n, eps, xq, xq_pad(n),
                                     xq_halves(n), (float *)nullptr);
    if (e != cudaSuccess) {
        set_error("rmsnorm launch: %s", cudaGetErrorString(e));
        return CUQ_ECUDA;
    }
    return CUQ_OK;
}

int launch_rmsnorm_xq(const float *x, const float *w, uint32_t n, uint32_t n_rows, float eps, __half *xq,
                      float *h_out, cudaStream_t s) {
    rmsnorm_xq_kernel<<<n_rows, 256, 0, s>>>(x, w, n, eps, xq, xq_pad(n), xq_halves(n), h_out);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

// Work split of a GEMV: KW warps per 16-row tile inside a CTA and ksplit CTAs
// along K (chosen from a sweep of both over the decode shapes of the benchmark
// configs).  KW depends on the shape only (not on sm_count), so callers that
// size the split-K workspace with one sm_count and launch with another agree.
GemvPlan gemv_pick_plan(const Planes &w, int sm_count) {
    int span;
    switch (w.type) {
    case CUQ_Q8_0: case CUQ_F16: case CUQ_BF16: span = 64; break;
    case CUQ_Q4_K: case CUQ_Q6_K: span = 256; break;
    default: span = planes_raw_type(w.type) ? 64 : 128; break;
    }
    const int ni = (int)((w.cols + span - 1) / span);
    const int tiles = (int)(w.rows / 16);
    GemvPlan pl;
    // Very tall matrices (lm_head, embeddings) have tiles enough to fill the GPU
    // many times over: two tiles per CTA with two warps each measured best.
    pl.kw = tiles >= 2048 ? 2 : 4;
    const int sm = sm_count > 0 ? sm_count : 148;
    int want, maxk;
    if (tiles >= sm) {
        // A tile per SM or more: about two CTAs per SM, and K parts of >= 16
        // iterations (4 per warp), which a sweep of the c4/c5 shapes measured
        // best: a split's partial store, ticket and reload cost more than the
        // extra parallelism returns (14336x4096 Q4_K 24.7 -> 18.9 us unsplit).
        want = (2 * sm + tiles - 1) / tiles;
        maxk = ni / 16;
    } else {
        want = (sm * 8 + tiles - 1) / tiles;  // ~8 CTAs of 4 warps per SM
        maxk = ni / 8;                        // keep >= 2 iterations per warp
    }
    if (want > maxk) want = maxk;
    if (want > 16) want = 16;
    if (want < 1) want = 1;
    pl.ksplit = want;
    return pl;
}

int gemv_pick_ksplit(const Planes &w, int sm_count, int nmat, bool tma) {
    if (tma && gemv_tma_supported(w.type)) return gemv_tma_ksplit(w, nmat, sm_count);
    return gemv_pick_plan(w, sm_count).ksplit;
}

int launch_gemv(const GemvArgs &a, int epi, cudaStream_t s) {
    const Planes &w = *a.w;
    if (!gemv_supported(w.type)) {
        set_error("UnsupportedType: no GEMV for ggml type %d", w.type);
        return CUQ_EUNSUPPORTED;
    }
    if (w.rows % 16 || w.rows == 0) {
        set_error("gemv: rows (%u) must be a positive multiple of 16", w.rows);
        return CUQ_EINVAL;
    }
    if ((w.type == CUQ_F16 || w.type == CUQ_BF16) && w.cols % 16) {
        set_error("gemv: 16-bit weights need cols %% 16 == 0 (cols %u)", w.cols);
        return CUQ_EINVAL;
    }
    if (epi == EPI_SILU_XQ && (!a.w2 || a.w2->type != w.type || a.w2->rows != w.rows || a.w2->cols != w.cols)) {
        set_error("gemv: gate/up must share type and shape");
        return CUQ_EINVAL;
    }
    if (a.pre_w && (!a.pre_x || a.pre_n != w.cols || a.pre_n % 16 || a.pre_n > RN_MAX)) {
        set_error("gemv: the pre-norm needs x of cols (%u) floats, a multiple of 16 up to %u", w.cols, RN_MAX);
        return CUQ_EINVAL;
    }
    if (a.ksplit > 1 && (!a.ws || !a.counters)) {
        set_error("gemv: split-K needs a workspace");
        return CUQ_EINVAL;
    }
    if (a.tma && (!a.pre_w || a.ss_in) && gemv_tma_supported(w.type)) return launch_gemv_tma(a, epi, s);
    switch (w.type) {
    case CUQ_Q8_0: return launch_t<TQ8_0>(a, epi, s);
    case CUQ_Q4_0: return launch_t<TQ4L<CUQ_Q4_0>>(a, epi, s);
    case CUQ_Q4_1: return launch_t<TQ4L<CUQ_Q4_1>>(a, epi, s);
    case CUQ_Q5_0: return launch_t<TQ4L<CUQ_Q5_0>>(a, epi, s);
    case CUQ_Q5_1: return launch_t<TQ4L<CUQ_Q5_1>>(a, epi, s);
    case CUQ_Q4_K: return launch_t<TQ4K>(a, epi, s);
    case CUQ_Q6_K: return launch_t<TQ6K>(a, epi, s);
    case CUQ_F16: return launch_t<T16<CUQ_F16>>(a, epi, s);
    case CUQ_BF16: return launch_t<T16<CUQ_BF16>>(a, epi, s);
    }
    if (planes_raw_type(w.type)) return launch_t<TRaw>(a, epi, s);
    return CUQ_EUNSUPPORTED;
}

}  // namespace cuq
