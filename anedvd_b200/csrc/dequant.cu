// dequant.cu -- bit-exact ggml dequantisation, and the lossless raw <-> planes regrouping.
//
// Element formulas restate src/gguf.zig:751-1071 (the reference's dequantisers).
// Every multiply/add is an explicit round-to-nearest intrinsic so the compiler
// cannot contract `a*b - c` into one FMA: the reference rounds after each op.
#include "common.cuh"
#include "ops.cuh"

namespace cuq {

namespace {

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t rd16(const uint8_t *b) { return (uint16_t)(b[0] | (b[1] << 8)); }
__device__ __forceinline__ uint32_t rd32(const uint8_t *b) {
    return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}

// getScaleMinK4 (gguf.zig:952-960)
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *q, int &d, int &m) {
    if (j < 4) {
        d = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Element j of one raw block (gguf.zig:751-1071).
__device__ float dq_elem(int type, const uint8_t *blk, int j) {
    switch (type) {
    case CUQ_F32: return __uint_as_float(rd32(blk));
    case CUQ_F16: return h2f_bits(rd16(blk));
    case CUQ_BF16: return __uint_as_float((uint32_t)rd16(blk) << 16);
    case CUQ_Q4_0: {  // gguf.zig:763-776
        float d = h2f_bits(rd16(blk));
        int x = j < 16 ? (blk[2 + j] & 0x0F) : (blk[2 + j - 16] >> 4);
        return __fmul_rn((float)(x - 8), d);
    }
    case CUQ_Q4_1: {  // gguf.zig:778-792
        float d = h2f_bits(rd16(blk)), m = h2f_bits(rd16(blk + 2));
        int x = j < 16 ? (blk[4 + j] & 0x0F) : (blk[4 + j - 16] >> 4);
        return __fadd_rn(__fmul_rn((float)x, d), m);
    }
    case CUQ_Q5_0:
    case CUQ_Q5_1: {  // gguf.zig:795-825 (shared body adds m, 0.0 for Q5_0)
        bool has_min = type == CUQ_Q5_1;
        int qh_off = has_min ? 4 : 2, qs_off = qh_off + 4;
        float d = h2f_bits(rd16(blk));
        float m = has_min ? h2f_bits(rd16(blk + 2)) : 0.0f;
        uint32_t qh = rd32(blk + qh_off);
        int v;
        if (j < 16) {
            v = (blk[qs_off + j] & 0x0F) | (int)(((qh >> j) << 4) & 0x10u);
        } else {
            int jj = j - 16;
            v = (blk[qs_off + jj] >> 4) | (int)((qh >> (jj + 12)) & 0x10u);
        }
        float x = (float)(v - (has_min ? 0 : 16));
        return __fadd_rn(__fmul_rn(x, d), m);
    }
    case CUQ_Q8_0: return __fmul_rn(h2f_bits(rd16(blk)), (float)(int8_t)blk[2 + j]);  // gguf.zig:827-840
    case CUQ_Q8_1: return __fmul_rn((float)(int8_t)blk[4 + j], h2f_bits(rd16(blk)));  // gguf.zig:842-853
    case CUQ_Q2_K: {  // gguf.zig:855-893
        int half = j >> 7, jj = j & 127, g = jj >> 5, part = (jj >> 4) & 1, l = jj & 15;
        float d = h2f_bits(rd16(blk + 80)), mn = h2f_bits(rd16(blk + 82));
        uint8_t sc = blk[half * 8 + g * 2 + part];
        float dl = __fmul_rn(d, (float)(sc & 0x0F)), ml = __fmul_rn(mn, (float)(sc >> 4));
        float v = (float)((blk[16 + half * 32 + part * 16 + l] >> (2 * g)) & 3);
        return __fsub_rn(__fmul_rn(dl, v), ml);
    }
    case CUQ_Q3_K: {  // gguf.zig:895-949
        const uint32_t kmask1 = 0x03030303u, kmask2 = 0x0f0f0f0fu;
        int half = j >> 7, jj = j & 127, g = jj >> 5, part = (jj >> 4) & 1, l = jj & 15;
        int is = half * 8 + g * 2 + part;
        uint32_t a0 = rd32(blk + 96), a1 = rd32(blk + 100), tmp = rd32(blk + 104);
        uint32_t aux;
        switch (is >> 2) {
        case 0: aux = (a0 & kmask2) | (((tmp >> 0) & kmask1) << 4); break;
        case 1: aux = (a1 & kmask2) | (((tmp >> 2) & kmask1) << 4); break;
        case 2: aux = ((a0 >> 4) & kmask2) | (((tmp >> 4) & kmask1) << 4); break;
        default: aux = ((a1 >> 4) & kmask2) | (((tmp >> 6) & kmask1) << 4); break;
        }
        int8_t s = (int8_t)(uint8_t)(aux >> (8 * (is & 3)));
        float d_all = h2f_bits(rd16(blk + 108));
        float dl = __fmul_rn(d_all, (float)((int)s - 32));
        uint8_t mbit = (uint8_t)(1u << (4 * half + g));
        int low = (blk[32 + half * 32 + part * 16 + l] >> (2 * g)) & 3;
        int v = low - ((blk[l + 16 * part] & mbit) ? 0 : 4);
        return __fmul_rn(dl, (float)v);
    }
    case CUQ_Q4_K: {  // gguf.zig:962-996
        int c = j >> 6, part = (j >> 5) & 1, l = j & 31;
        int sc, mm;
        scale_min_k4(2 * c + part, blk + 4, sc, mm);
        float d = h2f_bits(rd16(blk)), dmin = h2f_bits(rd16(blk + 2));
        float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mm);
        uint8_t byte = blk[16 + 32 * c + l];
        float q = (float)(part ? (byte >> 4) : (byte & 0x0F));
        return __fsub_rn(__fmul_rn(d1, q), m1);
    }
    case CUQ_Q5_K: {  // gguf.zig:998-1034
        int c = j >> 6, part = (j >> 5) & 1, l = j & 31;
        int sc, mm;
        scale_min_k4(2 * c + part, blk + 4, sc, mm);
        float d = h2f_bits(rd16(blk)), dmin = h2f_bits(rd16(blk + 2));
        float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mm);
        uint8_t byte = blk[48 + 32 * c + l];
        uint8_t mask = (uint8_t)((part ? 2u : 1u) << (2 * c));
        int v = (part ? (byte >> 4) : (byte & 0x0F)) + ((blk[16 + l] & mask) ? 16 : 0);
        return __fsub_rn(__fmul_rn(d1, (float)v), m1);
    }
    case CUQ_Q6_K: {  // gguf.zig:1036-1059
        int half = j >> 7, jj = j & 127, t = jj >> 5, l = jj & 31;
        const uint8_t *ql = blk + half * 64, *qh = blk + 128 + half * 32;
        const int8_t *sc = (const int8_t *)(blk + 192 + half * 8);
        int q;
        switch (t) {
        case 0: q = (ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4); break;
        case 1: q = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4); break;
        case 2: q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4); break;
        default: q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4); break;
        }
        float d = h2f_bits(rd16(blk + 208));
        float s = __fmul_rn(d, (float)sc[(l >> 4) + 2 * t]);
        return __fmul_rn(s, (float)(q - 32));
    }
    case CUQ_Q8_K: return __fmul_rn((float)(int8_t)blk[4 + j], __uint_as_float(rd32(blk)));  // gguf.zig:1061-1071
    default: return 0.0f;
    }
}

__global__ void dequant_raw_kernel(int type, const uint8_t *__restrict__ raw, uint64_t elem_offset, float *out,
                                   size_t n, int epb, int bpb) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        uint64_t e = elem_offset + i;
        uint64_t b = e / (uint64_t)epb;
        int j = (int)(e - b * (uint64_t)epb);
        out[i] = dq_elem(type, raw + b * (uint64_t)bpb, j);
    }
}

// ---------------------------------------------------------------- planes ---

// Copy one block between its raw form and the planes. dir = 0: raw -> planes.
__device__ __forceinline__ void mv(uint8_t *planes_p, uint8_t *raw_p, int n, int dir) {
    if (dir == 0)
        for (int i = 0; i < n; i++) planes_p[i] = raw_p[i];
    else
        for (int i = 0; i < n; i++) raw_p[i] = planes_p[i];
}

struct PlanesView {
    int type;
    uint32_t rows, cols;
    uint8_t *base;
    size_t off_q, off_q2, off_s, off_s2;
};

__device__ void block_move(const PlanesView &p, uint8_t *rawblk, uint32_t r, uint32_t b, int dir) {
    uint8_t *B = p.base;
    size_t rows = p.rows, cols = p.cols;
    switch (p.type) {
    case CUQ_Q8_0:
        mv(B + p.off_s + ((size_t)b * rows + r) * 2, rawblk, 2, dir);
        mv(B + p.off_q + r * cols + (size_t)b * 32, rawblk + 2, 32, dir);
        break;
    case CUQ_Q4_0:
        mv(B + p.off_s + ((size_t)b * rows + r) * 2, rawblk, 2, dir);
        mv(B + p.off_q + r * (cols / 2) + (size_t)b * 16, rawblk + 2, 16, dir);
        break;
    case CUQ_Q4_1:
        mv(B + p.off_s + ((size_t)b * rows + r) * 4, rawblk, 4, dir);
        mv(B + p.off_q + r * (cols / 2) + (size_t)b * 16, rawblk + 4, 16, dir);
        break;
    case CUQ_Q5_0:
        mv(B + p.off_s + ((size_t)b * rows + r) * 2, rawblk, 2, dir);
        mv(B + p.off_q2 + ((size_t)b * rows + r) * 4, rawblk + 2, 4, dir);
        mv(B + p.off_q + r * (cols / 2) + (size_t)b * 16, rawblk + 6, 16, dir);
        break;
    case CUQ_Q5_1:
        mv(B + p.off_s + ((size_t)b * rows + r) * 4, rawblk, 4, dir);
        mv(B + p.off_q2 + ((size_t)b * rows + r) * 4, rawblk + 4, 4, dir);
        mv(B + p.off_q + r * (cols / 2) + (size_t)b * 16, rawblk + 8, 16, dir);
        break;
    case CUQ_Q4_K:
        mv(B + p.off_s + ((size_t)b * rows + r) * 16, rawblk, 16, dir);
        mv(B + p.off_q + r * (cols / 2) + (size_t)b * 128, rawblk + 16, 128, dir);
        break;
    case CUQ_Q6_K:
        mv(B + p.off_q + r * (cols / 2) + (size_t)b * 128, rawblk, 128, dir);
        mv(B + p.off_q2 + r * (cols / 4) + (size_t)b * 64, rawblk + 128, 64, dir);
        mv(B + p.off_s + ((size_t)b * rows + r) * 16, rawblk + 192, 16, dir);
        mv(B + p.off_s2 + ((size_t)b * rows + r) * 2, rawblk + 208, 2, dir);
        break;
    case CUQ_F16:
    case CUQ_BF16: mv(B + ((size_t)r * cols + b) * 2, rawblk, 2, dir); break;
    default: break;
    }
}

// One thread per (row, block).
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
    uint8_t blk[212];
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t r = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
        block_move(p, blk, r, b, 1);
        __half *o = out + (size_t)r * p.cols + (size_t)b * epb;
        for (int j = 0; j < epb; j++) o[j] = __float2half_rn(dq_elem(p.type, blk, j));
    }
}

// Embedding row: x[c] = f32(RN16(dequant(row token)))[c] * 1.0 -- the fp16
// token_embd of loadRuntime (load_gguf.zig:578-647) read by Engine.forward
// (engine.zig:561-564).  One CTA, one thread per block of the row.
__global__ void embed_row_kernel(PlanesView p, const int *__restrict__ token_ptr, float *__restrict__ x, int epb) {
    const uint32_t r = (uint32_t)*token_ptr;
    if (r >= p.rows) return;
    uint8_t blk[212];
    for (uint32_t b = threadIdx.x; b < p.cols / epb; b += blockDim.x) {
        block_move(p, blk, r, b, 1);
        for (int j = 0; j < epb; j++) x[(size_t)b * epb + j] = __half2float(__float2half_rn(dq_elem(p.type, blk, j)));
    }
}

// Decode-step start: the embedding row of state->token (as embed_row_kernel)
// followed by the first layer's RMSNorm into the qkv projection's xq input.
__global__ void embed_norm_kernel(PlanesView p, const StepState *__restrict__ st, float *__restrict__ x,
                                  const float *__restrict__ nw, uint32_t n, float eps, __half *__restrict__ xq,
                                  int epb) {
    griddep_wait();
    griddep_launch();
    const uint32_t r = (uint32_t)st->token;
    uint8_t blk[212];
    if (r < p.rows) {
        for (uint32_t b = threadIdx.x; b < p.cols / epb; b += blockDim.x) {
            block_move(p, blk, r, b, 1);
            for (int j = 0; j < epb; j++)
                x[(size_t)b * epb + j] = __half2float(__float2half_rn(dq_elem(p.type, blk, j)));
        }
    }
    __threadfence();
    __syncthreads();
    rmsnorm_xq_block(x, nw, n, eps, xq, xq_pad(n), nullptr);
}

// Prefill: embedding rows of ids[0..n) into x[n][cols], one CTA per token.
__global__ void embed_rows_kernel(PlanesView p, const uint32_t *__restrict__ ids, float *__restrict__ x, int epb) {
    const uint32_t r = ids[blockIdx.x];
    float *xr = x + (size_t)blockIdx.x * p.cols;
    if (r >= p.rows) return;
    uint8_t blk[212];
    for (uint32_t b = threadIdx.x; b < p.cols / epb; b += blockDim.x) {
        block_move(p, blk, r, b, 1);
        for (int j = 0; j < epb; j++) xr[(size_t)b * epb + j] = __half2float(__float2half_rn(dq_elem(p.type, blk, j)));
    }
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
    default: return false;
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
    if (p.type == CUQ_F16 || p.type == CUQ_BF16) {
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
    if (p.type == CUQ_F16 || p.type == CUQ_BF16) {
        CUQ_CUDA_TRY(cudaMemcpyAsync(raw, p.base, p.nbytes, cudaMemcpyDeviceToDevice, s));
        return CUQ_OK;
    }
    int epb = block_elems(p.type), bpb = block_bytes(p.type);
    size_t total = (size_t)p.rows * (p.cols / epb);
    repack_kernel<<<grid_for(total, 128), 128, 0, s>>>(view(p), nullptr, raw, 1, epb, bpb);
    CUQ_CUDA_TRY(cudaGetLastError());
    return CUQ_OK;
}

int launch_embed_norm(const Planes &p, const StepState *state, float *x, const float *norm_w, uint32_t n, float eps,
                      __half *xq, bool pdl, cudaStream_t s) {
    cudaError_t e = launch_maybe_pdl(embed_norm_kernel, dim3(1), dim3(256), 0, s, pdl, view(p), state, x, norm_w, n,
                                     eps, xq, block_elems(p.type));
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
    embed_row_kernel<<<1, 256, 0, s>>>(view(p), token_ptr, x, block_elems(p.type));
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
