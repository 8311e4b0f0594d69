// qgemm.cuh -- the tensor-core (tcgen05) quantized GEMM of the prefill path.
#pragma once
#include "common.cuh"

namespace cuq {

struct QgemmArgs {
    const Planes *w = nullptr;    // weight (gate for EPI_SILU_XQ)
    const Planes *w2 = nullptr;   // up weight for EPI_SILU_XQ
    const __half *xh = nullptr;   // [n][cols] activation, fp16 hi part
    const __half *xl = nullptr;   // [n][cols] fp16 lo part (x = hi + lo)
    uint32_t n = 0;               // tokens
    float *y = nullptr;           // EPI_STORE / EPI_ADD: [n][ldy] fp32
    uint32_t ldy = 0;             // 0 = rows
    const float *bias = nullptr;  // [rows] or null
    __half *oh = nullptr, *ol = nullptr;  // EPI_SILU_XQ: act hi / lo [n][rows]
    int *err = nullptr;           // device int, set to 1 if a bounded wait timed out
    // raw-block weights (Q8_1, Q2_K, Q3_K, Q5_K, Q8_K, F32): rows * cols fp16
    // (twice that for a gate|up pair) the weight is first dequantised into,
    // exactly as Gguf.readF16 rounds; the GEMM then runs on those fp16 values
    __half *f16_scratch = nullptr;
};

// fp16 elements of scratch a GEMM of this weight (pair) needs: 0 for the
// types the GEMM decodes itself.
size_t qgemm_scratch_halves(const Planes &w, bool dual);

// Y = X W^T on tcgen05/TMEM (cols % 64 == 0).  Epilogues: EPI_STORE (+bias),
// EPI_ADD (y += ... + bias), EPI_SILU_XQ (act = silu(X Wg^T) * (X Wu^T) as hi/lo).
int launch_qgemm(const QgemmArgs &g, int epi, cudaStream_t s);
int launch_split_hilo(const float *x, size_t count, __half *hi, __half *lo, cudaStream_t s);

}  // namespace cuq
