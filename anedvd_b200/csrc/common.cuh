// common.cuh -- shared definitions for the sm_100a kernels and the C ABI.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

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
// ("raw" plane only) and are served by the dequantiser, not the GEMV.
struct Planes {
    int type = -1;
    uint32_t rows = 0, cols = 0;
    uint8_t *base = nullptr;  // one allocation
    size_t nbytes = 0;        // == rows*cols/elems*bytes (the GGUF payload size)
    // field offsets into base (bytes); unused = SIZE_MAX
    size_t off_q = 0, off_q2 = SIZE_MAX, off_s = SIZE_MAX, off_s2 = SIZE_MAX;
    bool raw = false;         // true: base holds the GGUF payload unchanged
};

inline bool gemv_supported(int t) {
    switch (t) {
    case CUQ_Q8_0: case CUQ_Q4_0: case CUQ_Q4_1: case CUQ_Q5_0: case CUQ_Q5_1:
    case CUQ_Q4_K: case CUQ_Q6_K: case CUQ_F16: case CUQ_BF16: return true;
    default: return false;
    }
}

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
inline uint32_t xq_pad(uint32_t cols) { return (cols + 255u) & ~255u; }
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

// ------------------------------------------------------------------ GEMV ---

enum GemvEpilogue : int {
    EPI_STORE = 0,     // y = acc (+ bias)
    EPI_ADD = 1,       // y += (acc + bias)        (residual add, engine.zig:607-620)
    EPI_SILU_XQ = 2,   // dual weight: act = silu(gate) * up, written as xq (+ fp32)
    EPI_ARGMAX = 3,    // y = acc; packed (value, index) max into *argmax64
};

struct GemvArgs {
    const Planes *w = nullptr;    // weight (gate for EPI_SILU_XQ)
    const Planes *w2 = nullptr;   // up weight for EPI_SILU_XQ
    const __half *xq = nullptr;   // activation in xq form
    float *y = nullptr;           // output (fp32), or act fp32 for SILU (may be null)
    const float *bias = nullptr;
    __half *xq_out = nullptr;     // EPI_SILU_XQ: act in xq form (kpad of w->rows)
    unsigned long long *argmax64 = nullptr;
    float *ws = nullptr;          // split-K partials [ksplit][rows]
    unsigned int *counters = nullptr;  // one per 16-row tile, self-resetting
    int ksplit = 1;
};

int launch_gemv(const GemvArgs &a, int epilogue, cudaStream_t s);
// Scratch a GEMV of this weight needs for a given ksplit (floats, counters).
int gemv_pick_ksplit(const Planes &w, int sm_count);

}  // namespace cuq
