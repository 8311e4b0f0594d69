// dequant.cu -- bit-exact ggml dequantisation, and the lossless raw <-> planes regrouping.
//
// Element formulas restate src/gguf.zig:751-1071 (the reference's dequantisers).
// Every multiply/add is an explicit round-to-nearest intrinsic so the compiler
// cannot contract `a*b - c` into one FMA: the reference rounds after each op.
#include "common.cuh"
#include "dequant_impl.cuh"
#include "ops.cuh"

namespace cuq {

namespace {

__global__ void dequant_raw_kernel(int type, const uint8_t *__restrict__ raw, uint64_t elem_offset, float *out,
                                   size_t n, int epb, int bpb) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        uint64_t e = elem_offset + i;
        uint64_t b = e / (uint64_t)epb;
        int j = (int)(e - b * (uint64_t)epb);
        out[i] = dq_elem(type, raw + b * (uint64_t)bpb, j);
    }
}

__global__ void repack_kernel(PlanesView p, const uint8_t *__restrict__ raw, uint8_t *raw_out, int dir, int epb,
                              int bpb) {
    uint32_t nb = p.cols / epb;
    size_t total = (size_t)p.rows * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t r = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
        uint8_t *blk = (dir == 0 ? (uint8_t *)raw : raw_out) + i * bpb;
        block_move(p, blk, r, b, dir);
    }
}

// Dequantise planes to fp16 exactly like Gguf.readF16: rebuild the raw block in
// registers, take the reference fp32 value, round to nearest even.
__global__ void dequant_planes_f16_kernel(PlanesView p, __half *__restrict__ out, int epb, int bpb) {
    uint32_t nb = p.cols / epb;
    size_t total = (size_t)p.rows * nb;
    uint8_t blk[296];  // the largest block (Q8_K, 292 bytes)
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t r = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
        block_move(p, blk, r, b, 1);
        __half *o = out + (size_t)r * p.cols + (size_t)b * epb;
        for (int j = 0; j < epb; j++) o[j] = __float2half_rn(dq_elem(p.type, blk, j));
    }
}

// Embedding row: x[c] = f32(RN16(dequant(row token)))[c] * 1.0 -- the fp16
// token_embd of loadRuntime (load_gguf.zig:578-647) read by Engine.forward
// (engine.zig:561-564).  One CTA.
__global__ void embed_row_kernel(PlanesView p, const int *__restrict__ token_ptr, float *__restrict__ x, int epb) {
    extern __shared__ __align__(16) uint8_t stage[];
    embed_row_staged(p, (uint32_t)*token_ptr, x, epb, stage);
}

// Decode-step start: the embedding row of state->token (as embed_row_kernel)
// followed by the first layer's RMSNorm into the qkv projection's xq input.
__global__ void embed_norm_kernel(PlanesView p, const StepState *__restrict__ st, float *__restrict__ x,
                                  const float *__restrict__ nw, uint32_t n, float eps, __half *__restrict__ xq,
                                  int epb) {
    griddep_wait();
    griddep_launch();
    extern __shared__ __align__(16) uint8_t stage[];
    embed_row_staged(p, (uint32_t)st->token, x, epb, stage);
    __threadfence();
    __syncthreads();
    rmsnorm_xq_block(x, nw, n, eps, xq, xq_pad(n), nullptr);
}

// Prefill: embedding rows of ids[0..n) into x[n][cols], one CTA per token.
__global__ void embed_rows_kernel(PlanesView p, const uint32_t *__restrict__ ids, float *__restrict__ x, int epb) {
    embed_row_block(p, ids[blockIdx.x], x + (size_t)blockIdx.x * p.cols, epb);
}

PlanesView view(const Planes &p) {
    return PlanesView{p.type, p.rows, p.cols, p.base, p.off_q, p.off_q2, p.off_s, p.off_s2};
}

int grid_for(size_t n, int threads) {
    size_t g = (n + threads - 1) / threads;
    if (g > 148 * 64) g = 148 * 64;
    if (g < 1) g = 1;
    return (int)g;
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

bool plan_planes(Planes &p) {
    size_t rows = p.rows, cols = p.cols;
    int epb = block_elems(p.type);
    if (!epb) return false;
    size_t nb = cols / epb;
    p.off_q2 = p.off_s = p.off_s2 = SIZE_MAX;
    p.off_q = 0;
    switch (p.type) {
    case CUQ_Q8_0: p.off_s = align256(rows * cols); p.nbytes = p.off_s + nb * rows * 2; break;
    case CUQ_Q4_0: p.off_s = align256(rows * cols / 2); p.nbytes = p.off_s + nb * rows * 2; break;
    case CUQ_Q4_1: p.off_s = align256(rows * cols / 2); p.nbytes = p.off_s + nb * rows * 4; break;
    case CUQ_Q5_0:
        p.off_q2 = align256(rows * cols / 2);
        p.off_s = align256(p.off_q2 + nb * rows * 4);
        p.nbytes = p.off_s + nb * rows * 2;
        break;
    case CUQ_Q5_1:
        p.off_q2 = align256(rows * cols / 2);
        p.off_s = align256(p.off_q2 + nb * rows * 4);
        p.nbytes = p.off_s + nb * rows * 4;
        break;
    case CUQ_Q4_K: p.off_s = align256(rows * cols / 2); p.nbytes = p.off_s + nb * rows * 16; break;
    case CUQ_Q6_K:
        p.off_q2 = align256(rows * cols / 2);
        p.off_s = align256(p.off_q2 + rows * cols / 4);
        p.off_s2 = align256(p.off_s + nb * rows * 16);
        p.nbytes = p.off_s2 + nb * rows * 2;
        break;
    case CUQ_F16: case CUQ_BF16: p.nbytes = rows * cols * 2; break;
    default:
        if (!planes_raw_type(p.type)) return false;
        p.raw = true;  // the GGUF payload unchanged
        p.nbytes = rows * nb * (size_t)block_bytes(p.type);
        break;
    }
    return true;
}

int launch_dequant_raw(int type, const uint8_t *raw, size_t raw_bytes, uint64_t elem_offset, float *out, size_t n,
                       cudaStream_t s) {
    int epb = block_elems(type), bpb = block_bytes(type);
    if (!epb) {
        set_error("UnsupportedType: ggml type %d", type);
        return CUQ_EUNSUPPORTED;
    }
    if (n == 0) return CUQ_OK;
    if (n % epb || elem_offset % epb) {
        set_error("InvalidTensorShape: %zu elements at offset %llu, block of %d", n,
                  (unsigned long long)elem_offset, epb);
        return CUQ_EINVAL;
    }
    uint64_t need = (elem_offset + n) / epb * (uint64_t)bpb;
    if (need > raw_bytes) {
        set_error("TruncatedFile: need %llu bytes, have %zu", (unsigned long long)need, raw_bytes);
        return CUQ_EINVAL;
    }
    dequant_raw_kernel<<<grid_for(n, 256), 256, 0, s>>>(type, raw, elem_offset, out, n, epb, bpb);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_repack(const uint8_t *raw, const Planes &p, cudaStream_t s) {
    if (p.raw || p.type == CUQ_F16 || p.type == CUQ_BF16) {
        CUQ_CUDA_TRY(cudaMemcpyAsync(p.base, raw, p.nbytes, cudaMemcpyDeviceToDevice, s));
        return CUQ_OK;
    }
    int epb = block_elems(p.type), bpb = block_bytes(p.type);
    size_t total = (size_t)p.rows * (p.cols / epb);
    repack_kernel<<<grid_for(total, 128), 128, 0, s>>>(view(p), raw, nullptr, 0, epb, bpb);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_unpack(const Planes &p, uint8_t *raw, cudaStream_t s) {
    if (p.raw || p.type == CUQ_F16 || p.type == CUQ_BF16) {
        CUQ_CUDA_TRY(cudaMemcpyAsync(raw, p.base, p.nbytes, cudaMemcpyDeviceToDevice, s));
        return CUQ_OK;
    }
    int epb = block_elems(p.type), bpb = block_bytes(p.type);
    size_t total = (size_t)p.rows * (p.cols / epb);
    repack_kernel<<<grid_for(total, 128), 128, 0, s>>>(view(p), nullptr, raw, 1, epb, bpb);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

// Shared memory of the single-CTA embedding kernels: the row's raw blocks.
static int embed_stage_bytes(const Planes &p, size_t &bytes) {
    bytes = (size_t)(p.cols / block_elems(p.type)) * block_bytes(p.type);
    if (bytes > 200 * 1024) {
        set_error("embedding row of %u columns does not fit shared memory", p.cols);
        return CUQ_EUNSUPPORTED;
    }
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(embed_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(embed_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr = true;
    }
    return CUQ_OK;
}

int launch_embed_norm(const Planes &p, const StepState *state, float *x, const float *norm_w, uint32_t n, float eps,
                      __half *xq, bool pdl, cudaStream_t s) {
    size_t smem;
    if (int rc = embed_stage_bytes(p, smem)) return rc;
    cudaError_t e = launch_maybe_pdl(embed_norm_kernel, dim3(1), dim3(256), smem, s, pdl, view(p), state, x, norm_w,
                                     n, eps, xq, block_elems(p.type));
    if (e != cudaSuccess) {
        set_error("embed launch: %s", cudaGetErrorString(e));
        return CUQ_ECUDA;
    }
    return CUQ_OK;
}

int launch_embed_rows(const Planes &p, const uint32_t *ids, uint32_t n, float *x, cudaStream_t s) {
    if (n == 0) return CUQ_OK;
    embed_rows_kernel<<<n, 128, 0, s>>>(view(p), ids, x, block_elems(p.type));
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_embed_row(const Planes &p, const int *token_ptr, float *x, cudaStream_t s) {
    size_t smem;
    if (int rc = embed_stage_bytes(p, smem)) return rc;
    embed_row_kernel<<<1, 256, smem, s>>>(view(p), token_ptr, x, block_elems(p.type));
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_dequant_planes_f16(const Planes &p, __half *out, cudaStream_t s) {
    int epb = block_elems(p.type), bpb = block_bytes(p.type);
    if (p.type == CUQ_F16) {
        CUQ_CUDA_TRY(cudaMemcpyAsync(out, p.base, p.nbytes, cudaMemcpyDeviceToDevice, s));
        return CUQ_OK;
    }
    size_t total = (size_t)p.rows * (p.cols / epb);
    dequant_planes_f16_kernel<<<grid_for(total, 128), 128, 0, s>>>(view(p), out, epb, bpb);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

}  // namespace cuq
