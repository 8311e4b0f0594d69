// common.cuh -- shared definitions for the sm_100a kernels and the C ABI.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>
#include <utility>

#include "../../include/cuq.h"

namespace cuq {

// ---------------------------------------------------------------- errors ---

// Thread-local last error, like ane_shim_last_error (src/ane/shim.h:60).
void set_error(const char *fmt, ...);
const char *get_error();

#define CUQ_CUDA_TRY(expr)                                                                      \
    do {                                                                                        \
        cudaError_t e_ = (expr);                                                                \
        if (e_ != cudaSuccess) {                                                                \
            ::cuq::set_error("%s:%d %s: %s", __FILE__, __LINE__, #expr, cudaGetErrorString(e_)); \
            return CUQ_ECUDA;                                                                   \
        }                                                                                       \
    } while (0)

#define CUQ_CHECK_ARG(cond, ...)            \
    do {                                    \
        if (!(cond)) {                      \
            ::cuq::set_error(__VA_ARGS__);  \
            return CUQ_EINVAL;              \
        }                                   \
    } while (0)

// --------------------------------------------------------------- geometry --

__host__ __device__ inline int block_elems(int t) {
    switch (t) {
    case CUQ_F32: case CUQ_F16: case CUQ_BF16: return 1;
    case CUQ_Q4_0: case CUQ_Q4_1: case CUQ_Q5_0: case CUQ_Q5_1: case CUQ_Q8_0: case CUQ_Q8_1: return 32;
    case CUQ_Q2_K: case CUQ_Q3_K: case CUQ_Q4_K: case CUQ_Q5_K: case CUQ_Q6_K: case CUQ_Q8_K: return 256;
    default: return 0;
    }
}

__host__ __device__ inline int block_bytes(int t) {
    switch (t) {
    case CUQ_F32: return 4;
    case CUQ_F16: case CUQ_BF16: return 2;
    case CUQ_Q4_0: return 18;
    case CUQ_Q4_1: return 20;
    case CUQ_Q5_0: return 22;
    case CUQ_Q5_1: return 24;
    case CUQ_Q8_0: return 34;
    case CUQ_Q8_1: return 36;
    case CUQ_Q2_K: return 84;
    case CUQ_Q3_K: return 110;
    case CUQ_Q4_K: return 144;
    case CUQ_Q5_K: return 176;
    case CUQ_Q6_K: return 210;
    case CUQ_Q8_K: return 292;
    default: return 0;
    }
}

// ------------------------------------------------------------ plane layout -
//
// A weight's device copy ("planes"): the raw GGUF blocks of a [rows][cols]
// matrix regrouped field by field, losslessly and with the same byte count.
// Quant bytes stay row-major with each row's blocks in file order, so a row's
// quants are one contiguous, 16-byte aligned run; per-block scale fields are
// stored block-major ([block][row]) so the 16 rows a warp works on read one
// contiguous 32-byte sector per block.
//
//   Q8_0 : qs  int8  [rows][cols]           d    fp16  [nb][rows]
//   Q4_0 : qs  u8    [rows][cols/2]         d    fp16  [nb][rows]
//   Q4_1 : qs  u8    [rows][cols/2]         dm   half2 [nb][rows]   (d, m)
//   Q5_0 : qs  u8    [rows][cols/2]         qh   u32   [nb][rows]   d fp16 [nb][rows]
//   Q5_1 : qs  u8    [rows][cols/2]         qh   u32   [nb][rows]   dm half2 [nb][rows]
//   Q4_K : qs  u8    [rows][cols/2]         meta 16 B  [nsb][rows]  (d, dmin, scales[12])
//   Q6_K : ql  u8    [rows][cols/2]         qh   u8    [rows][cols/4]
//          sc  int8  [nsb][rows][16]        d    fp16  [nsb][rows]
//   F16/BF16 : [rows][cols] 16-bit
// Other types (F32, Q8_1, Q2_K, Q3_K, Q5_K, Q8_K) keep the raw blocks as-is
// ("raw": one plane, the GGUF payload unchanged); their GEMV decodes each
// weight with the element dequantiser, and their prefill GEMM expands the
// weight to fp16 in a scratch buffer first.
struct Planes {
    int type = -1;
    uint32_t rows = 0, cols = 0;
    uint8_t *base = nullptr;  // one allocation
    size_t nbytes = 0;        // == rows*cols/elems*bytes (the GGUF payload size)
    // field offsets into base (bytes); unused = SIZE_MAX
    size_t off_q = 0, off_q2 = SIZE_MAX, off_s = SIZE_MAX, off_s2 = SIZE_MAX;
    bool raw = false;         // true: base holds the GGUF payload unchanged
};

// Types with a field-regrouped planes layout and their own register decoders.
inline bool planes_fast_type(int t) {
    switch (t) {
    case CUQ_Q8_0: case CUQ_Q4_0: case CUQ_Q4_1: case CUQ_Q5_0: case CUQ_Q5_1:
    case CUQ_Q4_K: case CUQ_Q6_K: case CUQ_F16: case CUQ_BF16: return true;
    default: return false;
    }
}
// Types kept as raw GGUF blocks (gguf.zig:842-949, 998-1034, 1061-1071, 751-761).
inline bool planes_raw_type(int t) {
    switch (t) {
    case CUQ_F32: case CUQ_Q8_1: case CUQ_Q2_K: case CUQ_Q3_K: case CUQ_Q5_K: case CUQ_Q8_K: return true;
    default: return false;
    }
}
// Every type a projection may have: all 15 block types of gguf.zig:30-77.
inline bool gemv_supported(int t) { return planes_fast_type(t) || planes_raw_type(t); }

// Compute plane offsets for a type/shape; returns false for non-GEMV types.
bool plan_planes(Planes &p);

// Launchers (defined in the .cu files).
int launch_dequant_raw(int type, const uint8_t *raw, size_t raw_bytes, uint64_t elem_offset, float *out,
                       size_t n, cudaStream_t s);
int launch_repack(const uint8_t *raw, const Planes &p, cudaStream_t s);
int launch_unpack(const Planes &p, uint8_t *raw, cudaStream_t s);
int launch_dequant_planes_f16(const Planes &p, __half *out, cudaStream_t s);

// The activation vector a GEMV consumes, pre-split into fp16 hi/lo parts
// (x = hi + lo to ~22 bits) in the k-permuted order the MMA fragments read:
// within each group of 4 consecutive columns the order is (0, 2, 1, 3).
// Layout: hi at [0, kpad), lo at [kpad, 2*kpad); kpad = round_up(cols, 256),
// tail zero-filled; then kpad/16 float32 sums of x over each aligned group of
// 16 columns (the K-quant GEMV subtracts its per-sub-block minimum as
// m1 * sum(x) in fp32).  `n_vec` vectors are stored back to back with a stride
// of xq_halves(cols) halves.
__host__ __device__ inline uint32_t xq_pad(uint32_t cols) { return (cols + 255u) & ~255u; }
inline size_t xq_halves(uint32_t cols) {
    size_t k = xq_pad(cols);
    return 2 * k + k / 8;
}
__host__ __device__ inline float *xq_sums(__half *xq, uint32_t kpad) { return (float *)(xq + 2 * (size_t)kpad); }
__host__ __device__ inline const float *xq_sums(const __half *xq, uint32_t kpad) {
    return (const float *)(xq + 2 * (size_t)kpad);
}

int launch_to_xq(const float *x, uint32_t n, uint32_t n_vec, uint32_t x_stride, __half *xq, cudaStream_t s);
// Fused RMSNorm producer: xq = split(x * rsqrt(mean(x^2)+eps) * w); also writes
// the fp32 result to h_out when non-null.
int launch_rmsnorm_xq(const float *x, const float *w, uint32_t n, uint32_t n_rows, float eps, __half *xq,
                      float *h_out, cudaStream_t s);
// One row, one CTA of 1024 threads, launched as a programmatic dependent of the
// previous kernel (its own dependents may start as soon as it does).
int launch_rmsnorm_xq_pdl(const float *x, const float *w, uint32_t n, float eps, __half *xq, cudaStream_t s);

// Device-side decode-step state, read and advanced by the step's kernels.
struct StepState {
    int token;      // token fed to the next step
    int pos;        // its position
    int step;       // steps run since the state was last set by the host
    int n_forced;   // steps whose next token comes from forced[] (prompt ids)
    unsigned long long argmax64;  // packed (value, index) max of the lm_head
};

// Programmatic dependent launch: wait for the preceding kernel's results
// (no-op when launched without the attribute) / let the next kernel start.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch `kernel` with the programmatic-stream-serialization attribute when pdl is set.
template <typename... KArgsT, typename... ActT>
cudaError_t launch_maybe_pdl(void (*kernel)(KArgsT...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                             ActT &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<ActT>(args)...);
}

// ------------------------------------------------------------------ GEMV ---

// Tensor parallelism (Megatron column/row split, one rank per GPU): every rank
// maps every other rank's communication buffer (CUDA IPC over NVLink) and
// pushes its partial sums into a slot of each peer's buffer with plain stores,
// then counts its arrival with a system-scope atomic on each peer.  Layout of
// one buffer: two phase regions (o and down projections alternate, so a rank
// is never more than one phase ahead of its peers) of [size][slot_floats]
// fp32, then [size] packed argmax keys, then arrival counters.
constexpr int TP_MAX = 8;
enum TpCounter : int { TP_CTR_PH0 = 0, TP_CTR_PH1 = 1, TP_CTR_ARGMAX = 2 };
struct TpComm {
    int rank = 0, size = 1;
    uint8_t *peer[TP_MAX] = {};   // each rank's buffer as mapped in this process (own at [rank])
    size_t slot_floats = 0;       // floats per source-rank slot
    size_t off_phase[2] = {0, 0}; // byte offsets of the two phase regions
    size_t off_am = 0;            // byte offset of the argmax keys
    size_t off_ctr = 0;           // byte offset of the counters
    int *err = nullptr;           // this rank's error flag: set when a wait gives up
    unsigned long long wait_ns = 10000000000ull;  // a wait for the peers gives up after this long
};

// Work the CTA that completes a GEMV's last tile does after the whole output is
// written: the next RMSNorm (of the residual x into xq), or the end of a decode
// step (argmax -> next token); with tensor parallelism, first the cross-rank
// reduction of the pushed partials (POST_TP_REDUCE) or argmax keys (POST_TP_FINISH).
enum GemvPostOp : int { POST_NONE = 0, POST_RMSNORM = 1, POST_FINISH = 2, POST_TP_REDUCE = 3, POST_TP_FINISH = 4 };

struct GemvPost {
    int op = POST_NONE;
    unsigned int *done = nullptr;  // grid completion counter (self-resetting)
    // POST_RMSNORM: xq_out = split(rmsnorm(x, w, eps)), n = len(x)
    const float *x = nullptr, *w = nullptr;
    uint32_t n = 0;
    float eps = 0.f;
    __half *xq = nullptr;
    // POST_FINISH
    StepState *state = nullptr;
    const uint32_t *forced = nullptr;
    uint32_t *out_tokens = nullptr;
    // POST_TP_REDUCE: x += sum over ranks of the phase-`tp_phase` partials (+ bias),
    // then the RMSNorm above.  POST_TP_FINISH: argmax across ranks, then POST_FINISH.
    TpComm tp;
    int tp_phase = 0;
    float *xr = nullptr;          // residual updated by POST_TP_REDUCE
    const float *bias = nullptr;
};

enum GemvEpilogue : int {
    EPI_STORE = 0,     // y = acc (+ bias)
    EPI_ADD = 1,       // y += (acc + bias)        (residual add, engine.zig:607-620)
    EPI_SILU_XQ = 2,   // dual weight: act = silu(gate) * up, written as xq (+ fp32)
    EPI_ARGMAX = 3,    // y = acc; packed (value, row_base + index) max into *argmax64
    EPI_TP_PUSH = 4,   // partial -> slot [rank] of phase post.tp_phase on every rank (see TpComm)
};

struct GemvArgs {
    const Planes *w = nullptr;    // weight (gate for EPI_SILU_XQ)
    const Planes *w2 = nullptr;   // up weight for EPI_SILU_XQ
    const __half *xq = nullptr;   // activation in xq form
    float *y = nullptr;           // output (fp32), or act fp32 for SILU (may be null)
    const float *bias = nullptr;
    __half *xq_out = nullptr;     // EPI_SILU_XQ: act in xq form (kpad of w->rows)
    unsigned long long *argmax64 = nullptr;
    uint32_t row_base = 0;        // EPI_ARGMAX: global index of this weight's row 0
    float *ws = nullptr;          // split-K partials [ksplit][rows]
    unsigned int *counters = nullptr;  // one per 16-row tile, self-resetting
    int ksplit = 1;
    bool pdl = false;             // launch as a programmatic dependent of the previous kernel
    // Input from the residual instead of xq: every CTA computes
    // xq = split(rmsnorm(pre_x, pre_w, pre_eps)) into its own shared memory once
    // the previous kernel is done (pre_n == cols, a multiple of 16, <= RN_MAX).
    const float *pre_x = nullptr, *pre_w = nullptr;
    uint32_t pre_n = 0;
    float pre_eps = 0.f;
    // With ss_in (TMA-fed GEMV): the mean square comes from the producer's
    // per-16-row sums of squares ss_in[0 .. pre_n/16), and each CTA normalises
    // only its own K range.
    const float *ss_in = nullptr;
    // EPI_ADD: the sum of squares of each 16-row tile of the updated output
    // (the residual) into ss_out[tile], for the next GEMV's ss_in.
    float *ss_out = nullptr;
    bool tma = true;              // the TMA-fed kernels may run it (else the register-prefetch kernel)
    int *err = nullptr;           // set to 1 when a bounded wait of the TMA GEMV gave up (may be null)
    GemvPost post;
};

// Position of column i inside an xq half-vector: (0, 2, 1, 3) in each group of 4.
__device__ __forceinline__ uint32_t xq_pos(uint32_t i) { return (i & ~3u) | ((i & 1u) << 1) | ((i >> 1) & 1u); }

// The block-level RMSNorm -> xq writer shared by the standalone kernel, the
// GEMV post-op and the embedding kernel: cpu.rmsnorm (cpu.zig:11-18),
// out = (x * (1 / sqrt(mean(x^2) + eps))) * w, then the xq split and per-16
// sums.  Reads x through L2 (it may have been written by other SMs).  Every
// thread of the block must call it.
__device__ __forceinline__ void rmsnorm_xq_block(const float *x, const float *w, uint32_t n, float eps, __half *xq,
                                                 uint32_t kpad, float *h_out) {
    __shared__ float part[32];
    float acc = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        float v = __ldcg(x + i);
        acc += v * v;
    }
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o2);
    __syncthreads();  // `part` may still be in use by a previous call in this block
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float s = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o2);
        if (threadIdx.x == 0) part[0] = s;
    }
    __syncthreads();
    const float mean = part[0] / (float)n;
    const float inv = 1.0f / sqrtf(mean + eps);
    float *sums = xq_sums(xq, kpad);
    // kpad is a multiple of 256 and blockDim a multiple of 16, so every thread
    // runs the same number of iterations and each aligned group of 16 lanes
    // holds 16 consecutive columns: their sum is a 16-lane shuffle reduction.
    for (uint32_t i = threadIdx.x; i < kpad; i += blockDim.x) {
        float f = 0.f;
        if (i < n) {
            f = (__ldcg(x + i) * inv) * w[i];
            if (h_out) h_out[i] = f;
        }
        __half hi = __float2half_rn(f);
        __half lo = __float2half_rn(f - __half2float(hi));
        uint32_t pos = xq_pos(i);
        xq[pos] = hi;
        xq[kpad + pos] = lo;
        float a = f;
#pragma unroll
        for (int o2 = 1; o2 < 16; o2 <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o2);
        if ((i & 15u) == 0) sums[i >> 4] = a;
    }
}

int launch_gemv(const GemvArgs &a, int epilogue, cudaStream_t s);
// K parts (CTAs along K) of a GEMV of this weight; nmat 2 for a gate|up pair.
// Callers size the split-K workspace with the same value they launch with.
// tma: the caller lets the TMA-fed kernels run this weight (GemvArgs::tma).
int gemv_pick_ksplit(const Planes &w, int sm_count, int nmat = 1, bool tma = true);
// The TMA-fed GEMV (gemv_tma.cu): the types it covers, its K split, and its
// launcher (CUQ_EUNSUPPORTED for a type or form it does not cover; then the
// register-prefetch kernel runs).
bool gemv_tma_supported(int type);
int gemv_tma_ksplit(const Planes &w, int nmat, int sm_count);
int launch_gemv_tma(const GemvArgs &a, int epilogue, cudaStream_t s);
struct GemvPlan {
    int kw = 4;      // warps per 16-row tile
    int ksplit = 1;  // CTAs along K
};
GemvPlan gemv_pick_plan(const Planes &w, int sm_count);

}  // namespace cuq
