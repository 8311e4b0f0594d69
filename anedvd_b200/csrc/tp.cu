// tp.cu -- tensor-parallel pieces that are not part of a GEMV: the prefill
// all-reduce kernels and the host-side slicing of raw GGUF tensors into a
// rank's shard (column-parallel = a row range, row-parallel = a column range
// of whole blocks).
#include <cstring>

#include "tp.cuh"

namespace cuq {

namespace {

// Push: every CTA stores its share of src into slot [rank] of phase ph on
// every rank, then counts one arrival on each of them.
__global__ void __launch_bounds__(256) tp_push_kernel(const TpComm t, int ph, const float4 *__restrict__ src,
                                                       size_t n4) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        for (int p = 0; p < t.size; p++) reinterpret_cast<float4 *>(tp_slot(t, p, ph, t.rank))[i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) tp_signal(t, ph);
}

// Reduce: wait for every rank's push, then x += (sum over ranks + bias).  The
// CTA that finishes last sets the phase counter back to 0.
__global__ void __launch_bounds__(256) tp_reduce_add_kernel(const TpComm t, int ph, unsigned int expected,
                                                             float *__restrict__ x, const float *__restrict__ bias,
                                                             uint32_t hidden, size_t count, unsigned int *done) {
    __shared__ int ok, last;
    if (threadIdx.x == 0) ok = tp_wait(t, ph, expected);
    __syncthreads();
    if (ok) {
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count;
             i += (size_t)gridDim.x * blockDim.x) {
            float s = tp_sum(t, ph, i);
            if (bias) s = s + bias[i % hidden];
            x[i] = x[i] + s;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(done, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (last && threadIdx.x == 0) {
        tp_reset(t, ph);
        *done = 0u;
    }
}

constexpr int TP_PUSH_GRID_MAX = 264;

}  // namespace

int launch_tp_push(const TpComm &t, int ph, const float *src, size_t count, int *grid_out, cudaStream_t s) {
    if (count % 4) {
        set_error("tp push: %zu floats is not a multiple of 4", count);
        return CUQ_EINVAL;
    }
    if (count > t.slot_floats) {
        set_error("tp push: %zu floats exceed the slot of %zu", count, t.slot_floats);
        return CUQ_EINVAL;
    }
    const size_t n4 = count / 4;
    int grid = (int)((n4 + 255) / 256);
    if (grid > TP_PUSH_GRID_MAX) grid = TP_PUSH_GRID_MAX;
    if (grid < 1) grid = 1;
    tp_push_kernel<<<grid, 256, 0, s>>>(t, ph, reinterpret_cast<const float4 *>(src), n4);
    CUQ_CUDA_TRY(cudaGetLastError());
    *grid_out = grid;
    return CUQ_OK;
}

int launch_tp_reduce_add(const TpComm &t, int ph, unsigned int expected, float *x, const float *bias, uint32_t hidden,
                         size_t count, unsigned int *done, cudaStream_t s) {
    int grid = (int)((count + 1023) / 1024);
    if (grid > 296) grid = 296;
    if (grid < 1) grid = 1;
    tp_reduce_add_kernel<<<grid, 256, 0, s>>>(t, ph, expected, x, bias, hidden, count, done);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

}  // namespace cuq

using namespace cuq;

extern "C" {

// Rows [r0, r1) of a raw [rows][cols] tensor: one contiguous byte range.
int cuq_shard_rows(int ggml_type, uint32_t rows, uint32_t cols, uint32_t r0, uint32_t r1, const void *raw, void *out) {
    CUQ_CHECK_ARG(raw && out, "cuq_shard_rows: null argument");
    const int epb = block_elems(ggml_type), bpb = block_bytes(ggml_type);
    if (!epb) {
        set_error("UnsupportedType: ggml type %d", ggml_type);
        return CUQ_EUNSUPPORTED;
    }
    if (cols % epb || r0 > r1 || r1 > rows) {
        set_error("cuq_shard_rows: rows [%u, %u) of %u x %u (block %d)", r0, r1, rows, cols, epb);
        return CUQ_EINVAL;
    }
    const size_t row_bytes = (size_t)(cols / epb) * bpb;
    memcpy(out, static_cast<const uint8_t *>(raw) + r0 * row_bytes, (r1 - r0) * row_bytes);
    return CUQ_OK;
}

// Columns [c0, c1) of every row, whole blocks only (c0, c1 multiples of the
// block size): the shard is [rows][c1 - c0] in the same block format.
int cuq_shard_cols(int ggml_type, uint32_t rows, uint32_t cols, uint32_t c0, uint32_t c1, const void *raw, void *out) {
    CUQ_CHECK_ARG(raw && out, "cuq_shard_cols: null argument");
    const int epb = block_elems(ggml_type), bpb = block_bytes(ggml_type);
    if (!epb) {
        set_error("UnsupportedType: ggml type %d", ggml_type);
        return CUQ_EUNSUPPORTED;
    }
    if (cols % epb || c0 % epb || c1 % epb || c0 > c1 || c1 > cols) {
        set_error("cuq_shard_cols: columns [%u, %u) of %u x %u are not whole blocks of %d", c0, c1, rows, cols, epb);
        return CUQ_EINVAL;
    }
    const size_t row_bytes = (size_t)(cols / epb) * bpb, off = (size_t)(c0 / epb) * bpb,
                 len = (size_t)((c1 - c0) / epb) * bpb;
    const uint8_t *src = static_cast<const uint8_t *>(raw);
    uint8_t *dst = static_cast<uint8_t *>(out);
    for (uint32_t r = 0; r < rows; r++) memcpy(dst + r * len, src + r * row_bytes + off, len);
    return CUQ_OK;
}

}  // extern "C"
