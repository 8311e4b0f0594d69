// gemv_impl.cuh -- the batch-1 quantized GEMV's per-type register decoders and
// its CTA body, shared by gemv.cu (one kernel per projection) and the
// persistent decode kernel.
#pragma once

#include "common.cuh"
#include "dequant_impl.cuh"
#include "tp.cuh"

namespace cuq {

namespace {

// A weight as the decoders see it: the planes of a whole matrix in global
// memory, or one pipeline stage of a tile in shared memory (rows = 16, cols =
// the stage's valid columns, qs / q2s = padded row strides).
struct W {
    const uint8_t *q, *q2, *s, *s2;  // plane pointers (see common.cuh)
    uint32_t rows, cols;
    uint32_t qs, q2s;                // bytes per row of the row-major q plane and of Q6_K's qh plane
    int type;                        // ggml type (the raw-block decoder reads it)
};

W wview(const Planes &p) {
    W w;
    w.q = p.base + p.off_q;
    w.q2 = p.off_q2 == SIZE_MAX ? nullptr : p.base + p.off_q2;
    w.s = p.off_s == SIZE_MAX ? nullptr : p.base + p.off_s;
    w.s2 = p.off_s2 == SIZE_MAX ? nullptr : p.base + p.off_s2;
    w.rows = p.rows;
    w.cols = p.cols;
    switch (p.type) {
    case CUQ_Q8_0: w.qs = p.cols; break;
    case CUQ_F16: case CUQ_BF16: w.qs = p.cols * 2; break;
    default: w.qs = p.cols / 2; break;
    }
    w.q2s = p.type == CUQ_Q6_K ? p.cols / 4 : 0;
    w.type = p.type;
    return w;
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Where a decoder's 16-byte quant loads come from: the planes in global memory,
// streamed past L1.
struct SrcGlobal {
    __device__ static uint4 ld16(const void *p) { return ldg_stream(p); }
};

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Packed fp32 pairs (lane 0 in the low word) for the f32x2 instructions.
__device__ __forceinline__ unsigned long long pack_f2(float a, float b) {
    return (unsigned long long)__float_as_uint(a) | ((unsigned long long)__float_as_uint(b) << 32);
}
__device__ __forceinline__ unsigned long long ffma_f2(unsigned long long a, unsigned long long b,
                                                      unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long fsub_f2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// RN16 of both lanes -> half2 (lane 0 low)
__device__ __forceinline__ uint32_t cvt_rn_h2(unsigned long long v) {
    return h2u(__floats2half2_rn(__uint_as_float((uint32_t)v), __uint_as_float((uint32_t)(v >> 32))));
}
// two bytes of w (small unsigned integers, selected by byte_perm selectors
// 0x744b) as the floats 2^23 + byte, packed
__device__ __forceinline__ unsigned long long magic23_bytes(uint32_t w, uint32_t sel0, uint32_t sel1) {
    return (unsigned long long)__byte_perm(w, 0x4B000000u, sel0) |
           ((unsigned long long)__byte_perm(w, 0x4B000000u, sel1) << 32);
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// half2 with 0x6400 exponent over the low bits of both 16-bit lanes: 1024 + field.
__device__ __forceinline__ uint32_t magic(uint32_t v, uint32_t mask) { return (v & mask) | 0x64006400u; }

// ------------------------------------------------------------- per type ---
// Each type provides SPAN (columns per lane-row per iteration x 4 lanes),
// KSTEPS (MMA k-steps per iteration), load() of one iteration's bytes for rows
// r0 and r0+8, frag() giving the A registers of k-step s, and koff() giving
// the first column of the 4-column group the lane feeds at k-step s.

struct TQ8_0 {
    static constexpr int SPAN = 64, KSTEPS = 4, DEPTH = 3;  // 3 x 16 rows x 64 columns in flight per warp
    static constexpr bool HAS_CORR = false;
    template <class R_>
    __device__ static void correct(const R_ &, const float *, int, int, float &, float &) {}
    struct Raw { uint4 q[2]; __half2 d[2]; };
    struct Prep {};
    __device__ static void prep(const Raw &, int, Prep &) {}
    template <class Src = SrcGlobal>
    __device__ static void load(Raw &R, const W &w, uint32_t r0, int it, int tig) {
        uint32_t k = it * SPAN + tig * 16;
        if (k < w.cols) {
            R.q[0] = Src::ld16(w.q + (size_t)r0 * w.qs + k);
            R.q[1] = Src::ld16(w.q + (size_t)(r0 + 8) * w.qs + k);
            const __half *d = reinterpret_cast<const __half *>(w.s) + (size_t)(k >> 5) * w.rows;
            R.d[0] = __half2half2(d[r0]);
            R.d[1] = __half2half2(d[r0 + 8]);
        } else {
            R.q[0] = R.q[1] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // q = 0
            R.d[0] = R.d[1] = __float2half2_rn(0.f);
        }
    }
    __device__ static uint32_t word(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
    __device__ static void frag(const Raw &R, const Prep &P, int s, uint32_t (&a)[4]) {
        const __half2 off = __float2half2_rn(1152.f);
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            uint32_t u = word(R.q[rr], s) ^ 0x80808080u;  // int8 q -> q + 128 (unsigned byte)
            __half2 p02 = u2h(__byte_perm(u, 0x64646464u, 0x4240u));  // 1152 + q for bytes 0, 2
            __half2 p13 = u2h(__byte_perm(u, 0x64646464u, 0x4341u));
            a[rr] = h2u(__hmul2(__hsub2(p02, off), R.d[rr]));        // RN16(q * d)
            a[rr + 2] = h2u(__hmul2(__hsub2(p13, off), R.d[rr]));
        }
    }
    __device__ static uint32_t koff(int it, int tig, int s) { return it * SPAN + tig * 16 + s * 4; }
};

// Legacy 32-blocks with 4-bit nibbles: one block per lane per iteration.
template <int T>
struct TQ4L {
    static constexpr int SPAN = 128, KSTEPS = 8, DEPTH = 2;
    static constexpr bool HAS_CORR = false;
    template <class R_>
    __device__ static void correct(const R_ &, const float *, int, int, float &, float &) {}
    struct Raw { uint4 q[2]; __half2 d[2], m[2]; uint32_t qh[2]; };
    struct Prep {};
    __device__ static void prep(const Raw &, int, Prep &) {}
    template <class Src = SrcGlobal>
    __device__ static void load(Raw &R, const W &w, uint32_t r0, int it, int tig) {
        uint32_t k = it * SPAN + tig * 32;
        if (k < w.cols) {
            uint32_t b = k >> 5;
            R.q[0] = Src::ld16(w.q + (size_t)r0 * w.qs + b * 16);
            R.q[1] = Src::ld16(w.q + (size_t)(r0 + 8) * w.qs + b * 16);
            if (T == CUQ_Q4_0 || T == CUQ_Q5_0) {
                const __half *d = reinterpret_cast<const __half *>(w.s) + (size_t)b * w.rows;
                R.d[0] = __half2half2(d[r0]);
                R.d[1] = __half2half2(d[r0 + 8]);
                R.m[0] = R.m[1] = __float2half2_rn(0.f);
            } else {
                const __half2 *dm = reinterpret_cast<const __half2 *>(w.s) + (size_t)b * w.rows;
                __half2 x0 = dm[r0], x1 = dm[r0 + 8];
                R.d[0] = __low2half2(x0);
                R.m[0] = __high2half2(x0);
                R.d[1] = __low2half2(x1);
                R.m[1] = __high2half2(x1);
            }
            if (T == CUQ_Q5_0 || T == CUQ_Q5_1) {
                const uint32_t *qh = reinterpret_cast<const uint32_t *>(w.q2) + (size_t)b * w.rows;
                R.qh[0] = qh[r0];
                R.qh[1] = qh[r0 + 8];
            } else {
                R.qh[0] = R.qh[1] = 0;
            }
        } else {
            R.q[0] = R.q[1] = make_uint4(0, 0, 0, 0);
            R.d[0] = R.d[1] = R.m[0] = R.m[1] = __float2half2_rn(0.f);
            R.qh[0] = R.qh[1] = 0;
        }
    }
    // k-step s: word i = s >> 1 of the block, low nibbles (s even) or high (s odd).
    __device__ static void frag(const Raw &R, const Prep &P, int s, uint32_t (&a)[4]) {
        const int i = s >> 1;
        const bool hi = s & 1;
        constexpr bool five = (T == CUQ_Q5_0 || T == CUQ_Q5_1);
        constexpr bool has_min = (T == CUQ_Q4_1 || T == CUQ_Q5_1);
        // offset removed before scaling: 1024 + (8 | 16 for the signed types)
        const float offv = 1024.f + (T == CUQ_Q4_0 ? 8.f : T == CUQ_Q5_0 ? 16.f : 0.f);
        const __half2 off = __float2half2_rn(offv);
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            uint32_t u = TQ8_0::word(R.q[rr], i);
            uint32_t v02 = hi ? (u >> 4) : u, v13 = hi ? (u >> 12) : (u >> 8);
            uint32_t p02 = magic(v02, 0x000F000Fu), p13 = magic(v13, 0x000F000Fu);
            if (five) {
                // 5th bits: weight j (< 16) uses qh bit j, weight 16+j uses bit 16+j.
                uint32_t t = R.qh[rr] >> (4 * i);
                if (!hi) {
                    p02 |= ((t << 4) & 0x10u) | ((t << 18) & 0x100000u);
                    p13 |= ((t << 3) & 0x10u) | ((t << 17) & 0x100000u);
                } else {
                    p02 |= ((t >> 12) & 0x10u) | ((t << 2) & 0x100000u);
                    p13 |= ((t >> 13) & 0x10u) | ((t << 1) & 0x100000u);
                }
            }
            __half2 x02 = __hsub2(u2h(p02), off), x13 = __hsub2(u2h(p13), off);
            if (has_min) {
                a[rr] = h2u(__hfma2(x02, R.d[rr], R.m[rr]));          // RN16(q*d + m)
                a[rr + 2] = h2u(__hfma2(x13, R.d[rr], R.m[rr]));
            } else {
                a[rr] = h2u(__hmul2(x02, R.d[rr]));                    // RN16((q - 8|16) * d)
                a[rr + 2] = h2u(__hmul2(x13, R.d[rr]));
            }
        }
    }
    __device__ static uint32_t koff(int it, int tig, int s) { return it * SPAN + tig * 32 + (s & 1) * 16 + (s >> 1) * 4; }
};

// Q4_K: one 256-superblock per iteration; lane tig owns the 32-byte group tig
// (sub-blocks 2tig in the low nibbles and 2tig+1 in the high nibbles).
// The reference weight is RN16 of the fp32 value d1*q - m1 with d1 = d*sc and
// m1 = dmin*m, both exact in fp32 (gguf.zig:975-992, load_gguf.zig:371); d1*q
// is exact too, so one fp32 fma(d1, q, -m1) rounds exactly where the
// reference's subtraction rounds, and cvt.rn.f16x2 then rounds like readF16.
// q becomes an exact float through the 2^23 exponent (bits 0x4B0000qq minus
// 2^23), two weights per packed f32x2 operation.
struct TQ4K {
    static constexpr int SPAN = 256, KSTEPS = 16, DEPTH = 1;
    static constexpr bool HAS_CORR = false;
    template <class R_>
    __device__ static void correct(const R_ &, const float *, int, int, float &, float &) {}
    // prefetched: the quant bytes and the 16-byte scale record of rows r0, r0+8
    struct Raw { uint4 q[2][2]; uint4 meta[2]; };
    // derived at compute time (keeps the prefetch ring small): packed (d1, d1)
    // and (-m1, -m1) per row and sub-block part
    struct Prep { unsigned long long d1[2][2], nm1[2][2]; };
    template <class Src = SrcGlobal>
    __device__ static void load(Raw &R, const W &w, uint32_t r0, int it, int tig) {
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            uint32_t r = r0 + rr * 8;
            const uint8_t *qp = w.q + (size_t)r * w.qs + (size_t)it * 128 + tig * 32;
            R.q[rr][0] = Src::ld16(qp);
            R.q[rr][1] = Src::ld16(qp + 16);
            R.meta[rr] = *reinterpret_cast<const uint4 *>(w.s + ((size_t)it * w.rows + r) * 16);
        }
    }
    // get_scale_min_k4 (gguf.zig:960-973) for this lane's sub-blocks j0 = 2*tig and
    // j0 + 1, all four 6-bit fields at once: V = [sc(j0), sc(j0+1), m(j0), m(j0+1)]
    // as bytes.  Scale bytes b0..b11 are the words y, z, w of the record.
    //   j < 4 : sc = b[j] & 63,                        m = b[j+4] & 63
    //   j >= 4: sc = (b[j+4] & 15) | (b[j-4] >> 6) << 4, m = (b[j+4] >> 4) | (b[j] >> 6) << 4
    __device__ static uint32_t scale_bytes(const uint4 &meta, int tig) {
        const bool lo = tig < 2;
        const uint32_t j0 = 2u * tig, j1 = j0 + 1u;
        const uint32_t selA = lo ? (j0 | j1 << 4 | (j0 + 4u) << 8 | (j1 + 4u) << 12)
                                 : ((j0 - 4u) | (j1 - 4u) << 4 | (j0 - 4u) << 8 | (j1 - 4u) << 12);
        const uint32_t a = __byte_perm(lo ? meta.y : meta.w, lo ? meta.z : meta.w, selA);
        const uint32_t a2 = __byte_perm(a, a >> 4, lo ? 0x3210u : 0x7610u);  // m bytes: high nibbles
        const uint32_t b = __byte_perm(meta.y, meta.z, (j0 - 4u) | (j1 - 4u) << 4 | j0 << 8 | j1 << 12);
        const uint32_t hb = (b >> 2) & (lo ? 0u : 0x30303030u);  // (x >> 6) << 4 in every byte
        return (a2 & (lo ? 0x3F3F3F3Fu : 0x0F0F0F0Fu)) | hb;
    }
    __device__ static void prep(const Raw &R, int tig, Prep &P) {
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const uint4 meta = R.meta[rr];
            const uint32_t v = scale_bytes(meta, tig);
            const float d = __half2float(__ushort_as_half((unsigned short)(meta.x & 0xFFFFu)));
            const float dmin = __half2float(__ushort_as_half((unsigned short)(meta.x >> 16)));
#pragma unroll
            for (int part = 0; part < 2; part++) {
                const float d1 = __fmul_rn(d, (float)((v >> (8 * part)) & 0xFFu));          // exact
                const float m1 = __fmul_rn(dmin, (float)((v >> (8 * (part + 2))) & 0xFFu));  // exact
                P.d1[rr][part] = pack_f2(d1, d1);
                P.nm1[rr][part] = pack_f2(-m1, -m1);
            }
        }
    }
    // k-step s: word i = s & 7 of the group, part = s >> 3 (low nibbles, then high).
    __device__ static void frag(const Raw &R, const Prep &P, int s, uint32_t (&a)[4]) {
        const int i = s & 7, part = s >> 3;
        const unsigned long long mg = pack_f2(8388608.f, 8388608.f);
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const uint32_t u = TQ8_0::word(R.q[rr][i >> 2], i & 3);
            const uint32_t nib = part ? ((u >> 4) & 0x0F0F0F0Fu) : (u & 0x0F0F0F0Fu);
            // columns 0, 2 and 1, 3 of the word's four (the fragment's pairs)
            const unsigned long long q02 = fsub_f2(magic23_bytes(nib, 0x7440u, 0x7442u), mg);
            const unsigned long long q13 = fsub_f2(magic23_bytes(nib, 0x7441u, 0x7443u), mg);
            a[rr] = cvt_rn_h2(ffma_f2(P.d1[rr][part], q02, P.nm1[rr][part]));  // RN16(fp32(d1*q - m1))
            a[rr + 2] = cvt_rn_h2(ffma_f2(P.d1[rr][part], q13, P.nm1[rr][part]));
        }
    }
    __device__ static uint32_t koff(int it, int tig, int s) { return it * SPAN + tig * 64 + (s >> 3) * 32 + (s & 7) * 4; }
};

// Q6_K: one superblock per iteration; lane tig owns half h = tig/2 and the
// 16 l-values starting at 16*(tig&1): ql bytes [64h+lh, +16) and [64h+32+lh, +16),
// qh bytes [32h+lh, +16); it produces 64 weights per row.
// The sub-block scale d*sc is exact in fp32 (11 x 8 bits); it is carried as
// an fp16 pair s_hi + s_lo so each weight RN16((q-32) * d * sc) is rounded
// once, like the reference's fp16 weight (gguf.zig:1036-1059, load_gguf.zig:371).
struct TQ6K {
    static constexpr int SPAN = 256, KSTEPS = 16, DEPTH = 1;
    static constexpr bool HAS_CORR = false;
    template <class R_>
    __device__ static void correct(const R_ &, const float *, int, int, float &, float &) {}
    // prefetched: ql/qh bytes, the 16 int8 scales and d of rows r0, r0+8
    struct Raw { uint4 a[2], b[2], h[2], scv[2]; __half d[2]; };
    // derived at compute time: d*sc as an fp16 hi + lo pair per quarter
    struct Prep { __half2 s[2][4], sl[2][4]; };
    template <class Src = SrcGlobal>
    __device__ static void load(Raw &R, const W &w, uint32_t r0, int it, int tig) {
        const int hh = tig >> 1, lh = (tig & 1) * 16;
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            uint32_t r = r0 + rr * 8;
            const uint8_t *ql = w.q + (size_t)r * w.qs + (size_t)it * 128 + hh * 64 + lh;
            R.a[rr] = Src::ld16(ql);
            R.b[rr] = Src::ld16(ql + 32);
            R.h[rr] = Src::ld16(w.q2 + (size_t)r * w.q2s + (size_t)it * 64 + hh * 32 + lh);
            R.scv[rr] = *reinterpret_cast<const uint4 *>(w.s + ((size_t)it * w.rows + r) * 16);
            R.d[rr] = reinterpret_cast<const __half *>(w.s2)[(size_t)it * w.rows + r];
        }
    }
    __device__ static void prep(const Raw &R, int tig, Prep &P) {
        const int hh = tig >> 1;
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const float d = __half2float(R.d[rr]);
            const uint4 scv = R.scv[rr];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                // int8 scale hh*8 + 2t + (tig&1), picked with a select and a runtime
                // shift (no local-memory indexing)
                const uint32_t wd = t < 2 ? (hh ? scv.z : scv.x) : (hh ? scv.w : scv.y);
                const int sc = (int)(int8_t)((wd >> (8 * (2 * (t & 1) + (tig & 1)))) & 0xFFu);
                const float scale = d * (float)sc;  // exact
                const __half hi = __float2half_rn(scale);
                P.s[rr][t] = __half2half2(hi);
                P.sl[rr][t] = __float2half2_rn(scale - __half2float(hi));
            }
        }
    }
    // k-step s: t = s >> 2 (which quarter), word i = s & 3.
    __device__ static void frag(const Raw &R, const Prep &P, int s, uint32_t (&a)[4]) {
        const int t = s >> 2, i = s & 3;
        const __half2 off = __float2half2_rn(1056.f);  // 1024 + 32
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            uint32_t A = TQ8_0::word(R.a[rr], i), B = TQ8_0::word(R.b[rr], i), Q = TQ8_0::word(R.h[rr], i);
            uint32_t p02, p13;
            switch (t) {
            case 0:
                p02 = (A & 0x000F000Fu) | ((Q << 4) & 0x00300030u);
                p13 = ((A >> 8) & 0x000F000Fu) | ((Q >> 4) & 0x00300030u);
                break;
            case 1:
                p02 = (B & 0x000F000Fu) | ((Q << 2) & 0x00300030u);
                p13 = ((B >> 8) & 0x000F000Fu) | ((Q >> 6) & 0x00300030u);
                break;
            case 2:
                p02 = ((A >> 4) & 0x000F000Fu) | (Q & 0x00300030u);
                p13 = ((A >> 12) & 0x000F000Fu) | ((Q >> 8) & 0x00300030u);
                break;
            default:
                p02 = ((B >> 4) & 0x000F000Fu) | ((Q >> 2) & 0x00300030u);
                p13 = ((B >> 12) & 0x000F000Fu) | ((Q >> 10) & 0x00300030u);
                break;
            }
            __half2 x02 = __hsub2(u2h(p02 | 0x64006400u), off), x13 = __hsub2(u2h(p13 | 0x64006400u), off);
            a[rr] = h2u(__hfma2(x02, P.s[rr][t], __hmul2(x02, P.sl[rr][t])));  // ~RN16((q-32) * scale)
            a[rr + 2] = h2u(__hfma2(x13, P.s[rr][t], __hmul2(x13, P.sl[rr][t])));
        }
    }
    __device__ static uint32_t koff(int it, int tig, int s) {
        return it * SPAN + (tig >> 1) * 128 + (s >> 2) * 32 + (tig & 1) * 16 + (s & 3) * 4;
    }
};

// F16 / BF16: 16 weights per lane-row per iteration.
template <int T>
struct T16 {
    static constexpr int SPAN = 64, KSTEPS = 4, DEPTH = 2;
    static constexpr bool HAS_CORR = false;
    template <class R_>
    __device__ static void correct(const R_ &, const float *, int, int, float &, float &) {}
    struct Raw { uint4 q[2][2]; };
    struct Prep {};
    __device__ static void prep(const Raw &, int, Prep &) {}
    template <class Src = SrcGlobal>
    __device__ static void load(Raw &R, const W &w, uint32_t r0, int it, int tig) {
        uint32_t k = it * SPAN + tig * 16;
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            if (k < w.cols) {
                const uint8_t *p = w.q + (size_t)(r0 + rr * 8) * w.qs + (size_t)k * 2;
                R.q[rr][0] = Src::ld16(p);
                R.q[rr][1] = Src::ld16(p + 16);
            } else {
                R.q[rr][0] = R.q[rr][1] = make_uint4(0, 0, 0, 0);
            }
        }
    }
    __device__ static uint32_t cvt(uint32_t lo16src, uint32_t hi16src) {
        // two bf16 (low halves of the sources) -> fp16x2, RN (Gguf.readF16 of a bf16 tensor)
        float a = __uint_as_float(lo16src << 16), b = __uint_as_float(hi16src << 16);
        return h2u(__floats2half2_rn(a, b));
    }
    __device__ static void frag(const Raw &R, const Prep &P, int s, uint32_t (&a)[4]) {
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const uint4 &v = R.q[rr][s >> 1];
            uint32_t w0 = (s & 1) ? v.z : v.x, w1 = (s & 1) ? v.w : v.y;  // (e0,e1), (e2,e3)
            if (T == CUQ_F16) {
                a[rr] = __byte_perm(w0, w1, 0x5410u);      // (e0, e2)
                a[rr + 2] = __byte_perm(w0, w1, 0x7632u);  // (e1, e3)
            } else {
                a[rr] = cvt(w0, w1);
                a[rr + 2] = cvt(w0 >> 16, w1 >> 16);
            }
        }
    }
    __device__ static uint32_t koff(int it, int tig, int s) { return it * SPAN + tig * 16 + s * 4; }
};

// Raw GGUF blocks of any other type (F32, Q8_1, Q2_K, Q3_K, Q5_K, Q8_K): each
// weight is the element dequantiser's bit-exact fp32 value (dq_elem,
// gguf.zig:751-1071) rounded to fp16 as readF16 does.  64 columns per
// iteration; the lane's 32 weights (4 k-steps x rows r0, r0 + 8 x 4 columns)
// are decoded by load(), so the prefetch ring carries finished fragments.
// These types have no bandwidth target; this path is for correctness.
struct TRaw {
    static constexpr int SPAN = 64, KSTEPS = 4, DEPTH = 1;
    static constexpr bool HAS_CORR = false;
    template <class R_>
    __device__ static void correct(const R_ &, const float *, int, int, float &, float &) {}
    struct Raw { uint32_t f[4][4]; };
    struct Prep {};
    __device__ static void prep(const Raw &, int, Prep &) {}
    template <class Src = SrcGlobal>
    __device__ static void load(Raw &R, const W &w, uint32_t r0, int it, int tig) {
        const int epb = block_elems(w.type), bpb = block_bytes(w.type);
        const uint32_t nb = w.cols / (uint32_t)epb;
#pragma unroll
        for (int s = 0; s < 4; s++) {
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const uint8_t *row = w.q + (size_t)(r0 + 8 * rr) * nb * bpb;
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const uint32_t c = (uint32_t)it * SPAN + tig * 16 + s * 4 + e;
                    v[e] = c < w.cols ? __half2float(__float2half_rn(dq_elem(w.type, row + (size_t)(c / epb) * bpb,
                                                                             (int)(c % epb))))
                                      : 0.f;
                }
                R.f[s][rr] = h2u(__floats2half2_rn(v[0], v[2]));      // columns (0, 2) of the group
                R.f[s][rr + 2] = h2u(__floats2half2_rn(v[1], v[3]));  // columns (1, 3)
            }
        }
    }
    __device__ static void frag(const Raw &R, const Prep &, int s, uint32_t (&a)[4]) {
#pragma unroll
        for (int i = 0; i < 4; i++) a[i] = R.f[s][i];
    }
    __device__ static uint32_t koff(int it, int tig, int s) { return it * SPAN + tig * 16 + s * 4; }
};

// ------------------------------------------------------------------ kernel -

struct KArgs {
    W w, w2;
    const __half *xq;
    const float *xsum;  // per-16-column sums of x (xq_sums)
    uint32_t kpad;
    float *y;
    const float *bias;
    __half *xq_out;
    uint32_t kpad_out;
    unsigned long long *argmax64;
    uint32_t row_base;
    float *ws;
    unsigned int *counters;
    int ksplit;
    const float *pre_x, *pre_w;  // GemvArgs::pre_* (pre_w null: input is xq)
    uint32_t pre_n;
    float pre_eps;
    const float *ss_in;          // GemvArgs::ss_in / ss_out
    float *ss_out;
    GemvPost post;
};

// Kernel arguments of a GEMV described by GemvArgs (host).
inline KArgs make_kargs(const GemvArgs &a) {
    KArgs k;
    k.w = wview(*a.w);
    if (a.w2) k.w2 = wview(*a.w2);
    k.xq = a.xq;
    k.kpad = xq_pad(a.w->cols);
    k.xsum = a.xq ? xq_sums(a.xq, k.kpad) : nullptr;
    k.y = a.y;
    k.bias = a.bias;
    k.xq_out = a.xq_out;
    k.kpad_out = xq_pad(a.w->rows);
    k.argmax64 = a.argmax64;
    k.row_base = a.row_base;
    k.ws = a.ws;
    k.counters = a.counters;
    k.ksplit = a.ksplit < 1 ? 1 : a.ksplit;
    k.pre_x = a.pre_x;
    k.pre_w = a.pre_w;
    k.pre_n = a.pre_n;
    k.pre_eps = a.pre_eps;
    k.ss_in = a.ss_in;
    k.ss_out = a.ss_out;
    k.post = a.post;
    return k;
}

__device__ __forceinline__ unsigned long long pack_argmax(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v);
    uint32_t key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

// End of a decode step (engine.zig:865-900 + generate.zig:217-244, greedy):
// the packed argmax becomes the step's output token and, past the forced
// prompt, the next step's input.
__device__ void finish_step(StepState *st, const uint32_t *forced, uint32_t *out_tokens) {
    unsigned long long a = st->argmax64;
    uint32_t idx = 0xFFFFFFFFu - (uint32_t)(a & 0xFFFFFFFFull);
    st->argmax64 = 0ull;
    int s = st->step;
    out_tokens[s] = idx;
    st->step = s + 1;
    st->pos = st->pos + 1;
    st->token = (s + 1 < st->n_forced) ? (int)forced[s + 1] : (int)idx;
}

// Shared memory of gemv_body, owned by the calling kernel so that the body's
// instantiations share one copy.
struct GemvShared {
    float red[8][16];    // per-warp partial sums (up to 8 warps)
    float gu[4][32];     // EPI_SILU_XQ: gate and up values of a tile
    float act16[4][16];  // EPI_SILU_XQ: activations of a tile
    int is_last;
};

// Everything after a CTA's main loop: the cross-warp sum of the tile's rows,
// the split-K reduction and the epilogue.  c / k0 / k1: this lane's MMA
// accumulators and K-quant corrections.  Returns false for a CTA whose split-K
// partial was not the tile's last.
// Barrier of the threads running a GEMV epilogue: the whole CTA (N = 0), or
// its first N threads on named barrier 1 (a CTA whose other warps do
// something else, e.g. a producer warp that streams the weights).
template <int N>
__device__ __forceinline__ void cta_sync() {
    if constexpr (N == 0)
        __syncthreads();
    else
        asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}

// nparts: CTAs contributing partial sums to this tile (0: p.ksplit); by is this
// CTA's slot among them.
template <class TT, int EPI, int KW, int NW = 4, int SYNC_N = 0>
__device__ __forceinline__ bool gemv_finish(const KArgs &p, uint32_t bx, uint32_t by, GemvShared &sh, float (&c)[4],
                                            float k0, float k1, int nparts = 0) {
    // NW warps per CTA: TPC tiles of KW warps each, or (gate|up) one tile whose
    // first NW/2 warps hold the gate rows and the others the up rows
    constexpr bool DUAL = (EPI == EPI_SILU_XQ);
    constexpr int TPC = DUAL ? 1 : NW / KW;
    constexpr int KWE = DUAL ? NW / 2 : KW;
    constexpr int NV = DUAL ? 32 : 16;
    float(&red)[8][16] = sh.red;
    int &is_last = sh.is_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const uint32_t ntiles = p.w.rows / 16;
    if (TT::HAS_CORR) {  // the four lanes of a row hold different sub-blocks: sum them
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            k0 += __shfl_xor_sync(0xffffffffu, k0, o);
            k1 += __shfl_xor_sync(0xffffffffu, k1, o);
        }
    }
    if (SYNC_N) cta_sync<SYNC_N>();  // the previous unit's readers of `sh` are done
    if (tig == 0) {
        red[warp][g] = (c[0] + c[1]) - k0;
        red[warp][g + 8] = (c[2] + c[3]) - k1;
    }
    cta_sync<SYNC_N>();
    // thread t < TPC * NV owns value vi of local tile tl (dual: vi < 16 gate, >= 16 up)
    const int t = threadIdx.x;
    const int tl = t / NV, vi = t % NV;
    const bool own = t < TPC * NV && bx * TPC + tl < ntiles;
    const uint32_t row = (bx * TPC + tl) * 16 + (vi & 15);
    float v = 0.f;
    if (own) {
        const int w0 = DUAL ? KWE * (vi >> 4) : tl * KW;
#pragma unroll
        for (int w = 0; w < KWE; w++) v += red[w0 + w][vi & 15];
    }
    const uint32_t rows = p.w.rows;
    const int np = nparts > 0 ? nparts : p.ksplit;
    if (np > 1) {
        // split-K: publish the partials, the last CTA of this column of the grid
        // (atomic ticket per tile group) reduces them in a fixed order.
        if (own) p.ws[((size_t)by * (DUAL ? 2 : 1) + (vi >> 4)) * rows + row] = v;
        __threadfence();
        cta_sync<SYNC_N>();
        if (t == 0) {
            unsigned int prev = atomicAdd(&p.counters[bx], 1u);
            is_last = (prev == (unsigned)np - 1u);
        }
        cta_sync<SYNC_N>();
        if (!is_last) return false;
        __threadfence();
        if (own) {
            float acc = 0.f;
            for (int ky = 0; ky < np; ky++)
                acc += __ldcg(&p.ws[((size_t)ky * (DUAL ? 2 : 1) + (vi >> 4)) * rows + row]);
            v = acc;
        }
        if (t == 0) p.counters[bx] = 0u;
    }
    if (EPI == EPI_SILU_XQ) {
        float(&gu)[4][32] = sh.gu;
        float(&act16)[4][16] = sh.act16;
        if (own) gu[tl][vi] = v;
        cta_sync<SYNC_N>();
        if (own && vi < 16) {
            float gt = gu[tl][vi], ut = gu[tl][16 + vi];
            // cpu.siluMul (cpu.zig:65-70): g * (1 / (1 + exp(-g))) * u
            float sg = 1.0f / (1.0f + expf(-gt));
            float act = (gt * sg) * ut;
            if (p.y) p.y[row] = act;
            __half hi = __float2half_rn(act);
            __half lo = __float2half_rn(act - __half2float(hi));
            uint32_t pos = xq_pos(row);
            p.xq_out[pos] = hi;
            p.xq_out[p.kpad_out + pos] = lo;
            act16[tl][vi] = act;
        }
        cta_sync<SYNC_N>();
        if (t < TPC && bx * TPC + t < ntiles) {  // a tile's 16 rows are exactly one xq sum group
            float acc = 0.f;
            for (int j = 0; j < 16; j++) acc += act16[t][j];
            xq_sums(p.xq_out, p.kpad_out)[bx * TPC + t] = acc;
        }
    } else if (EPI == EPI_TP_PUSH) {
        // this rank's partial of rows [row] into slot [rank] of every rank's buffer
        if (own)
            for (int q = 0; q < p.post.tp.size; q++) tp_slot(p.post.tp, q, p.post.tp_phase, p.post.tp.rank)[row] = v;
        // the barrier orders every thread's stores before thread 0's system fence
        // in tp_signal (a cumulative release), which publishes them to the peers
        // before its arrival is counted
        cta_sync<SYNC_N>();
        if (t == 0) tp_signal(p.post.tp, p.post.tp_phase);
    } else {
        if (own) {
            if (EPI == EPI_STORE || EPI == EPI_ARGMAX) {
                if (p.bias) v = v + p.bias[row];
                p.y[row] = v;
            } else if (EPI == EPI_ADD) {
                if (p.bias) v = v + p.bias[row];
                v = p.y[row] + v;
                p.y[row] = v;
            }
        }
        if (EPI == EPI_ADD && p.ss_out && t < TPC * 16) {
            // the tile's sum of squares of the updated rows (16 lanes, fixed order)
            float q = own ? v * v : 0.f;
            const unsigned mask = 0xFFFFu << (t & 16);
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) q += __shfl_xor_sync(mask, q, o);
            if (own && (t & 15) == 0) p.ss_out[bx * TPC + tl] = q;
        }
        if (EPI == EPI_ARGMAX) {
            // first index of the maximum (cpu.zig:477-483) as a packed 64-bit max
            // across the CTA, then across CTAs: larger value wins, then smaller index.
            if (t < TPC * 16) {  // TPC * 16 is 16, 32 or 64 threads
                unsigned long long key = own ? pack_argmax(v, p.row_base + row) : 0ull;
                constexpr unsigned mask = TPC == 1 ? 0x0000ffffu : 0xffffffffu;
#pragma unroll
                for (int o = TPC == 1 ? 8 : 16; o > 0; o >>= 1) {
                    unsigned long long other = __shfl_xor_sync(mask, key, o);
                    key = other > key ? other : key;
                }
                if ((t & 31) == 0) atomicMax(p.argmax64, key);
            }
        }
    }
    return true;
}

// Grid completion of a GEMV: the CTA that finishes last runs the post-op
// (the next RMSNorm, the end of a decode step, or the cross-rank reduction
// before them).  `dyn`: dynamic shared memory of at least post.n floats when the
// post-op is a norm with post.n % 16 == 0 and post.n <= RN_MAX (staging), free
// for reuse at this point.  Every thread of the CTA calls it.
__device__ __forceinline__ void gemv_post_op(const KArgs &p, uint8_t *gemv_dyn) {
    const int t = threadIdx.x;
    __shared__ int is_last;
    if (p.post.op == POST_NONE) return;
    // Grid completion: the CTA that finishes last runs the post-op.
    __threadfence();
    __syncthreads();
    if (t == 0) {
        unsigned int prev = atomicAdd(p.post.done, 1u);
        is_last = (prev == gridDim.x - 1u);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float4 *rn_stage = reinterpret_cast<float4 *>(gemv_dyn);  // n floats when the launch gave them (fast path)
    const bool fast = p.post.n % 16 == 0 && p.post.n <= RN_MAX;
    if (p.post.op == POST_TP_REDUCE) {
        // every rank's CTAs pushed once: x += sum over ranks (+ bias), then the RMSNorm
        const TpComm &tp = p.post.tp;
        __shared__ int ok;
        if (t == 0) ok = tp_wait(tp, p.post.tp_phase, (unsigned)tp.size * gridDim.x);
        __syncthreads();
        if (fast) {
            reduce_norm_xq_block(p.post.xr, ok ? &tp : nullptr, p.post.tp_phase, p.post.bias, p.post.w, p.post.n,
                                 p.post.eps, p.post.xq, xq_pad(p.post.n), rn_stage);
        } else {
            if (ok) {
                for (uint32_t i = t; i < p.post.n; i += blockDim.x) {
                    float sum = tp_sum(tp, p.post.tp_phase, i);
                    if (p.post.bias) sum = sum + p.post.bias[i];
                    p.post.xr[i] = __ldcg(p.post.xr + i) + sum;
                }
            }
            __threadfence();
            __syncthreads();
            rmsnorm_xq_block(p.post.x, p.post.w, p.post.n, p.post.eps, p.post.xq, xq_pad(p.post.n), nullptr);
        }
        __syncthreads();
        if (t == 0) tp_reset(tp, p.post.tp_phase);
    } else if (p.post.op == POST_RMSNORM) {
        if (fast)
            reduce_norm_xq_block(const_cast<float *>(p.post.x), nullptr, 0, nullptr, p.post.w, p.post.n, p.post.eps,
                                 p.post.xq, xq_pad(p.post.n), rn_stage);
        else
            rmsnorm_xq_block(p.post.x, p.post.w, p.post.n, p.post.eps, p.post.xq, xq_pad(p.post.n), nullptr);
    } else if (p.post.op == POST_FINISH) {
        if (t == 0) finish_step(p.post.state, p.post.forced, p.post.out_tokens);
    } else if (p.post.op == POST_TP_FINISH) {
        // cross-rank argmax: every rank publishes its packed key, all take the max
        // (the packing keeps the reference's first-index tie rule, cpu.zig:477-483)
        if (t == 0) {
            const TpComm &tp = p.post.tp;
            const unsigned long long mine = __ldcg(&p.post.state->argmax64);
            for (int q = 0; q < tp.size; q++) tp_am(tp, q)[tp.rank] = mine;
            tp_signal(tp, TP_CTR_ARGMAX);
            unsigned long long best = mine;
            if (tp_wait(tp, TP_CTR_ARGMAX, (unsigned)tp.size)) {
                for (int r = 0; r < tp.size; r++) {
                    const unsigned long long k = __ldcv(tp_am(tp, tp.rank) + r);
                    best = k > best ? k : best;
                }
            }
            tp_reset(tp, TP_CTR_ARGMAX);
            p.post.state->argmax64 = best;
            finish_step(p.post.state, p.post.forced, p.post.out_tokens);
        }
    }
    if (t == 0) *p.post.done = 0u;
}

// CTA of 4 warps = TPC = 4 / KW tiles of 16 rows, KW warps per tile splitting
// the CTA's K range (iteration it goes to warp it % KW of the tile).  Each warp
// keeps D iterations of loads in flight ahead of the one it computes.
// One CTA's share of a GEMV: tile group bx, K split part by.  `before_x()` is
// called by every thread once the first weight loads are in flight and before
// anything written by earlier work (the activation) is read: the standalone
// kernel waits there for its predecessor (PDL), the persistent decode kernel
// for its grid barrier.  Returns false for a CTA that published a split-K
// partial and is not the tile's last (its epilogue ran elsewhere); true once
// the epilogue is done.

template <class TT, int EPI, int KW, int D, class BeforeX>
__device__ __forceinline__ bool gemv_body(const KArgs &p, uint32_t bx, uint32_t by, GemvShared &sh,
                                          BeforeX &&before_x, const __half *xq_in = nullptr,
                                          const float *xsum_in = nullptr) {
    // Dual (gate|up): one tile per CTA, warps 0-1 stream the gate rows and
    // warps 2-3 the same rows of up (KW = 2 per matrix), so no warp holds both.
    constexpr bool DUAL = (EPI == EPI_SILU_XQ);
    constexpr int TPC = DUAL ? 1 : 4 / KW;  // tiles per CTA
    constexpr int KWE = DUAL ? 2 : KW;      // warps per tile and matrix
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const int lt = DUAL ? 0 : warp / KW, kw = warp % KWE;
    const W &wm = (DUAL && warp >= 2) ? p.w2 : p.w;
    const uint32_t ntiles = p.w.rows / 16;
    const uint32_t tile = bx * TPC + lt;
    const bool active = tile < ntiles;
    const uint32_t r0 = tile * 16 + g;
    const int ni = (int)((p.w.cols + TT::SPAN - 1) / TT::SPAN);
    const int per = (ni + p.ksplit - 1) / p.ksplit;
    const int it0 = by * per, it1 = active ? min(ni, it0 + per) : it0;

    // The weights do not depend on the previous kernel: start streaming the
    // warp's first D iterations before waiting for the activation.
    typename TT::Raw ring[D];
#pragma unroll
    for (int j = 0; j < D; j++) {
        const int itj = it0 + kw + KWE * j;
        if (itj < it1) TT::load(ring[j], wm, r0, itj, tig);
    }
    before_x();

    // B fragments (L1-cached, shared by the SM's CTAs): p.xq, or xq_in / xsum_in
    // when the caller built the input itself (shared memory)
    const __half *xb = (xq_in ? xq_in : p.xq) + (g == 1 ? p.kpad : 0);
    const float *xsum = xsum_in ? xsum_in : p.xsum;
    const bool bl = g < 2;

    float c[4] = {0.f, 0.f, 0.f, 0.f};
    float k0 = 0.f, k1 = 0.f;  // fp32 corrections (rows r0, r0+8), K-quants only
    for (int base = it0 + kw; base < it1; base += KWE * D) {
#pragma unroll
        for (int j = 0; j < D; j++) {
            const int it = base + KWE * j;
            if (it >= it1) break;  // uniform across the warp
            typename TT::Raw R = ring[j];
            const int itn = it + KWE * D;
            if (itn < it1) TT::load(ring[j], wm, r0, itn, tig);  // refill this slot while the iteration computes
            typename TT::Prep P;
            TT::prep(R, tig, P);
#pragma unroll
            for (int s = 0; s < TT::KSTEPS; s++) {
                uint2 b = make_uint2(0u, 0u);
                if (bl) b = *reinterpret_cast<const uint2 *>(xb + TT::koff(it, tig, s));
                uint32_t a[4];
                TT::frag(R, P, s, a);
                mma16816(c, a[0], a[1], a[2], a[3], b.x, b.y);
            }
            if (TT::HAS_CORR) TT::correct(P, xsum, it, tig, k0, k1);
        }
    }
    return gemv_finish<TT, EPI, KW>(p, bx, by, sh, c, k0, k1);
}

}  // namespace

}  // namespace cuq
