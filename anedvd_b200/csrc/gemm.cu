// gemm.cu -- cuq_gemm, the prefill projection Y[n][rows] = X[n][cols] W^T.
//
// First version: each token is a batch-1 GEMV over the quantized planes (the
// weight is re-streamed per token).  Correct, and the reference for the
// tensor-core prefill path that replaces it.
#include "common.cuh"

struct cuq_weight;

namespace cuq {
const Planes *weight_planes(const cuq_weight *w, float **ws, unsigned int **counters, int *ksplit);
}

using namespace cuq;

extern "C" int cuq_gemm(const cuq_weight *w, const float *x_dev, uint32_t n, float *y_dev, void *stream) {
    CUQ_CHECK_ARG(w && x_dev && y_dev, "cuq_gemm: null argument");
    float *ws = nullptr;
    unsigned int *ctr = nullptr;
    int ksplit = 1;
    const Planes *p = weight_planes(w, &ws, &ctr, &ksplit);
    if (!p || p->raw) {
        set_error("UnsupportedType: no GEMM for this weight");
        return CUQ_EUNSUPPORTED;
    }
    if (n == 0) return CUQ_OK;
    cudaStream_t s = (cudaStream_t)stream;
    size_t kp = xq_halves(p->cols);
    __half *xq = nullptr;
    CUQ_CUDA_TRY(cudaMallocAsync(&xq, sizeof(__half) * kp * n, s));
    int rc = launch_to_xq(x_dev, p->cols, n, p->cols, xq, s);
    for (uint32_t t = 0; rc == CUQ_OK && t < n; t++) {
        GemvArgs a;
        a.w = p;
        a.xq = xq + kp * t;
        a.y = y_dev + (size_t)t * p->rows;
        a.ws = ws;
        a.counters = ctr;
        a.ksplit = ksplit;
        rc = launch_gemv(a, EPI_STORE, s);
    }
    cudaFreeAsync(xq, s);
    return rc;
}
