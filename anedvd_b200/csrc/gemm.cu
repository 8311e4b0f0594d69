// gemm.cu -- cuq_gemm, the prefill projection Y[n][rows] = X[n][cols] W^T, on
// the tcgen05 tensor-core kernel (qgemm_tc.cu).
#include "common.cuh"
#include "qgemm.cuh"

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
    if (!p) {
        set_error("UnsupportedType: no GEMM for this weight");
        return CUQ_EUNSUPPORTED;
    }
    if (n == 0) return CUQ_OK;
    cudaStream_t s = (cudaStream_t)stream;
    size_t cnt = (size_t)n * p->cols;
    const size_t scratch = qgemm_scratch_halves(*p, false);
    __half *xh = nullptr;
    int *err = nullptr;
    // x hi | x lo | (raw-block weights) the fp16 expansion
    CUQ_CUDA_TRY(cudaMallocAsync(&xh, sizeof(__half) * (2 * cnt + scratch) + 16, s));
    CUQ_CUDA_TRY(cudaMallocAsync(&err, sizeof(int), s));
    CUQ_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), s));
    int rc = launch_split_hilo(x_dev, cnt, xh, xh + cnt, s);
    if (rc == CUQ_OK) {
        QgemmArgs g;
        g.w = p;
        g.xh = xh;
        g.xl = xh + cnt;
        g.n = n;
        g.y = y_dev;
        g.err = err;
        if (scratch) g.f16_scratch = xh + 2 * cnt;
        rc = launch_qgemm(g, EPI_STORE, s);
    }
    int herr = 0;
    if (rc == CUQ_OK) {
        cudaError_t e = cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            set_error("cuq_gemm: %s", cudaGetErrorString(e));
            rc = CUQ_ECUDA;
        } else if (herr) {
            set_error("cuq_gemm: a tensor-core pipeline wait timed out");
            rc = CUQ_ETIMEOUT;
        }
    }
    cudaFreeAsync(xh, s);
    cudaFreeAsync(err, s);
    return rc;
}
