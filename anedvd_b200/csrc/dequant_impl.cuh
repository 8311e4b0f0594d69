// dequant_impl.cuh -- device-side block decoding shared by dequant.cu and the
// persistent decode kernel: bit-exact element dequantisation (gguf.zig:751-1071)
// and the planes <-> raw block regrouping.
#pragma once

#include "common.cuh"

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

// ---------------------------------------------------------------- planes ---

// Copy one block between its raw form and the planes. dir = 0: raw -> planes.
__device__ __forceinline__ void mv(uint8_t *planes_p, uint8_t *raw_p, int n, int dir) {
    if (dir == 1 && (n & 15) == 0 && (reinterpret_cast<uintptr_t>(planes_p) & 15) == 0) {
        // an aligned plane segment: four 16-byte loads in flight, then the byte stores
        for (int i = 0; i < n; i += 64) {
            uint4 v[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
                v[k] = i + 16 * k < n ? *reinterpret_cast<const uint4 *>(planes_p + i + 16 * k) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (i + 16 * k >= n) break;
                const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
                for (int j = 0; j < 16; j++) raw_p[i + 16 * k + j] = (uint8_t)(w[j >> 2] >> (8 * (j & 3)));
            }
        }
        return;
    }
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
    default: {  // raw blocks: the payload itself, row-major
        const int bpb = block_bytes(p.type);
        mv(B + ((size_t)r * (cols / block_elems(p.type)) + b) * bpb, rawblk, bpb, dir);
        break;
    }
    }
}

// One thread per (row, block).
// Embedding row r of planes p (fp16-rounded dequant, load_gguf.zig:578-647 +
// engine.zig:561-564) into x[0..cols), by every thread of the block: S threads
// share one GGUF block, each decoding a contiguous share of its elements.
__device__ __forceinline__ void embed_row_block(const PlanesView &p, uint32_t r, float *x, int epb) {
    if (r >= p.rows) return;
    const int S = epb >= 256 ? 8 : 1;
    const uint32_t nb = p.cols / epb;
    uint8_t blk[296];  // the largest block (Q8_K, 292 bytes)
    for (uint32_t idx = threadIdx.x; idx < nb * S; idx += blockDim.x) {
        const uint32_t b = idx / S;
        const int part = idx % S, per = epb / S;
        block_move(p, blk, r, b, 1);
        for (int j = part * per; j < (part + 1) * per; j++)
            x[(size_t)b * epb + j] = __half2float(__float2half_rn(dq_elem(p.type, blk, j)));
    }
}

// The same row by one CTA with its raw blocks staged in shared memory (`stage`:
// cols / epb * block_bytes bytes): one thread rebuilds each block once, then
// every thread decodes elements out of shared memory.  For the decode step's
// single-CTA embedding, where one thread per block share would rebuild every
// block several times in local memory.
__device__ __forceinline__ void embed_row_staged(const PlanesView &p, uint32_t r, float *x, int epb, uint8_t *stage) {
    if (r >= p.rows) return;  // r is the same for the whole CTA
    const int bpb = block_bytes(p.type);
    const uint32_t nb = p.cols / epb;
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) block_move(p, stage + (size_t)b * bpb, r, b, 1);
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < p.cols; i += blockDim.x)
        x[i] = __half2float(__float2half_rn(dq_elem(p.type, stage + (size_t)(i / epb) * bpb, (int)(i % epb))));
}

}  // namespace

}  // namespace cuq
