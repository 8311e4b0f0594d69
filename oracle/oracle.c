/* oracle.c -- CPU restatement of ANEDVD's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; see oracle.h).  Compiled with
 * -O2 -ffp-contract=off so that `a * b + c` rounds twice, as the reference's
 * Zig code does in its default (strict) float mode.
 *
 * Every function names the reference lines it restates.  Paths are relative to
 * the midasdf/ANEDVD source tree.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ geometry --- */

int orc_block_elems(int t) {
    switch (t) {
    case ORC_F32: case ORC_F16: case ORC_BF16: return 1;
    case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q5_1: case ORC_Q8_0: case ORC_Q8_1: return 32;
    case ORC_Q2_K: case ORC_Q3_K: case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: case ORC_Q8_K: return 256;
    default: return 0;
    }
}

int orc_block_bytes(int t) {
    switch (t) {
    case ORC_F32: return 4;
    case ORC_F16: case ORC_BF16: return 2;
    case ORC_Q4_0: return 18;
    case ORC_Q4_1: return 20;
    case ORC_Q5_0: return 22;
    case ORC_Q5_1: return 24;
    case ORC_Q8_0: return 34;
    case ORC_Q8_1: return 36;
    case ORC_Q2_K: return 84;
    case ORC_Q3_K: return 110;
    case ORC_Q4_K: return 144;
    case ORC_Q5_K: return 176;
    case ORC_Q6_K: return 210;
    case ORC_Q8_K: return 292;
    default: return 0;
    }
}

/* --------------------------------------------------------- fp16 / bf16 --- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0x1F) return u2f(sign | 0x7F800000u | (man << 13));   /* inf / nan */
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal: man * 2^-24, exact in binary32 */
        float v = (float)man * u2f(0x33800000u); /* 2^-24 */
        return sign ? -v : v;
    }
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* Round-to-nearest-even binary32 -> binary16 (the conversion Zig's
 * @floatCast performs, gguf.zig:682-692). */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) {                      /* inf or nan */
        if (ax == 0x7F800000u) return sign | 0x7C00u;
        return sign | 0x7E00u | (uint16_t)((ax >> 13) & 0x3FFu);
    }
    if (ax >= 0x477FF000u) return sign | 0x7C00u; /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                       /* below 2^-14: subnormal or zero */
        if (ax < 0x33000000u) return sign;        /* < 2^-25: rounds to zero */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e;                /* result = m >> (shift) with rounding */
        /* value = m * 2^(e-150); subnormal unit = 2^-24 -> q = m * 2^(e-126) */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return sign | (uint16_t)q;
    }
    uint32_t e = (ax >> 23) - 112u;               /* rebias 127 -> 15 */
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;  /* carry may bump exponent: fine */
    return sign | (uint16_t)q;
}

void orc_f32_to_f16_n(const float *src, uint16_t *dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = orc_f32_to_f16(src[i]);
}

static float f16tab[65536];
static pthread_once_t f16tab_once = PTHREAD_ONCE_INIT;
static void f16tab_init(void) {
    for (uint32_t i = 0; i < 65536; i++) f16tab[i] = orc_f16_to_f32((uint16_t)i);
}
static inline float h2f(uint16_t h) { return f16tab[h]; }

/* ------------------------------------------------------------- dequant --- */

static inline uint16_t rd16(const uint8_t *b) { return (uint16_t)(b[0] | ((uint16_t)b[1] << 8)); }
static inline uint32_t rd32(const uint8_t *b) {
    return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}

/* gguf.zig:751-761 */
static void dq_f32(const uint8_t *b, float *o, size_t n) { for (size_t i = 0; i < n; i++) o[i] = u2f(rd32(b + 4 * i)); }
static void dq_f16(const uint8_t *b, float *o, size_t n) { for (size_t i = 0; i < n; i++) o[i] = h2f(rd16(b + 2 * i)); }
static void dq_bf16(const uint8_t *b, float *o, size_t n) { for (size_t i = 0; i < n; i++) o[i] = u2f((uint32_t)rd16(b + 2 * i) << 16); }

/* gguf.zig:763-776: (nibble - 8) * d, low nibbles first then high. */
static void dq_q4_0(const uint8_t *b, float *o, size_t n) {
    for (size_t i = 0; i < n / 32; i++) {
        const uint8_t *blk = b + i * 18;
        float d = h2f(rd16(blk));
        for (int j = 0; j < 16; j++) {
            uint8_t byte = blk[2 + j];
            float x0 = (float)((int)(byte & 0x0F) - 8);
            float x1 = (float)((int)(byte >> 4) - 8);
            o[i * 32 + j] = x0 * d;
            o[i * 32 + j + 16] = x1 * d;
        }
    }
}

/* gguf.zig:778-792: nibble * d + m (two roundings). */
static void dq_q4_1(const uint8_t *b, float *o, size_t n) {
    for (size_t i = 0; i < n / 32; i++) {
        const uint8_t *blk = b + i * 20;
        float d = h2f(rd16(blk)), m = h2f(rd16(blk + 2));
        for (int j = 0; j < 16; j++) {
            uint8_t byte = blk[4 + j];
            float x0 = (float)(byte & 0x0F), x1 = (float)(byte >> 4);
            float p0 = x0 * d, p1 = x1 * d;
            o[i * 32 + j] = p0 + m;
            o[i * 32 + j + 16] = p1 + m;
        }
    }
}

/* gguf.zig:795-825: 5th bit from the u32 qh word; Q5_0 subtracts 16, Q5_1 adds m. */
static void dq_q5(const uint8_t *b, float *o, size_t n, int bb, int has_min) {
    int qh_off = has_min ? 4 : 2, qs_off = qh_off + 4, minus = has_min ? 0 : 16;
    for (size_t i = 0; i < n / 32; i++) {
        const uint8_t *blk = b + i * (size_t)bb;
        float d = h2f(rd16(blk));
        float m = has_min ? h2f(rd16(blk + 2)) : 0.0f;
        uint32_t qh = rd32(blk + qh_off);
        for (int j = 0; j < 16; j++) {
            uint8_t byte = blk[qs_off + j];
            uint32_t xh0 = ((qh >> j) << 4) & 0x10u;
            uint32_t xh1 = (qh >> (j + 12)) & 0x10u;
            float x0 = (float)((int)((byte & 0x0Fu) | xh0) - minus);
            float x1 = (float)((int)((byte >> 4) | xh1) - minus);
            if (has_min) {
                float p0 = x0 * d, p1 = x1 * d;
                o[i * 32 + j] = p0 + m;
                o[i * 32 + j + 16] = p1 + m;
            } else {
                /* gguf.zig:814-816 adds m = 0.0 in the shared body; x*d + 0.0
                 * only differs from x*d for -0.0, which d > 0 never yields. */
                float p0 = x0 * d, p1 = x1 * d;
                o[i * 32 + j] = p0 + m;
                o[i * 32 + j + 16] = p1 + m;
            }
        }
    }
}

/* gguf.zig:827-840 */
static void dq_q8_0(const uint8_t *b, float *o, size_t n) {
    for (size_t i = 0; i < n / 32; i++) {
        const uint8_t *blk = b + i * 34;
        float d = h2f(rd16(blk));
        for (int j = 0; j < 32; j++) o[i * 32 + j] = d * (float)(int8_t)blk[2 + j];
    }
}

/* gguf.zig:842-853 (s at offset 2 is unused) */
static void dq_q8_1(const uint8_t *b, float *o, size_t n) {
    for (size_t i = 0; i < n / 32; i++) {
        const uint8_t *blk = b + i * 36;
        float d = h2f(rd16(blk));
        for (int j = 0; j < 32; j++) o[i * 32 + j] = (float)(int8_t)blk[4 + j] * d;
    }
}

/* gguf.zig:855-893 */
static void dq_q2_k(const uint8_t *b, float *o, size_t n) {
    for (size_t ib = 0; ib < n / 256; ib++) {
        const uint8_t *blk = b + ib * 84;
        float d = h2f(rd16(blk + 80)), mn = h2f(rd16(blk + 82));
        const uint8_t *sc = blk;
        size_t q = 16, y = ib * 256;
        int is = 0;
        for (int half = 0; half < 2; half++) {
            int shift = 0;
            for (int g = 0; g < 4; g++) {
                for (int part = 0; part < 2; part++) {
                    uint8_t s = sc[is++];
                    float dl = d * (float)(s & 0x0F);
                    float ml = mn * (float)(s >> 4);
                    for (int l = 0; l < 16; l++) {
                        float v = (float)((blk[q + l + 16 * part] >> shift) & 3);
                        float p = dl * v;
                        o[y + l] = p - ml;
                    }
                    y += 16;
                }
                shift += 2;
            }
            q += 32;
        }
    }
}

/* gguf.zig:895-949 */
static void dq_q3_k(const uint8_t *b, float *o, size_t n) {
    const uint32_t kmask1 = 0x03030303u, kmask2 = 0x0f0f0f0fu;
    for (size_t ib = 0; ib < n / 256; ib++) {
        const uint8_t *blk = b + ib * 110;
        float d_all = h2f(rd16(blk + 108));
        const uint8_t *hm = blk, *qs = blk + 32;
        uint32_t aux[4] = {rd32(blk + 96), rd32(blk + 100), rd32(blk + 104), 0};
        uint32_t tmp = aux[2];
        aux[2] = ((aux[0] >> 4) & kmask2) | (((tmp >> 4) & kmask1) << 4);
        aux[3] = ((aux[1] >> 4) & kmask2) | (((tmp >> 6) & kmask1) << 4);
        aux[0] = (aux[0] & kmask2) | (((tmp >> 0) & kmask1) << 4);
        aux[1] = (aux[1] & kmask2) | (((tmp >> 2) & kmask1) << 4);
        int8_t scales[16];
        for (int k = 0; k < 4; k++)
            for (int bi = 0; bi < 4; bi++) scales[k * 4 + bi] = (int8_t)(uint8_t)(aux[k] >> (8 * bi));
        uint8_t m = 1;
        int is = 0;
        size_t q = 0, y = ib * 256;
        for (int half = 0; half < 2; half++) {
            int shift = 0;
            for (int g = 0; g < 4; g++) {
                for (int part = 0; part < 2; part++) {
                    float dl = d_all * (float)((int)scales[is++] - 32);
                    for (int l = 0; l < 16; l++) {
                        int low = (qs[q + l + 16 * part] >> shift) & 3;
                        int v = low - ((hm[l + 16 * part] & m) ? 0 : 4);
                        o[y + l] = dl * (float)v;
                    }
                    y += 16;
                }
                shift += 2;
                m = (uint8_t)(m << 1);
            }
            q += 32;
        }
    }
}

/* getScaleMinK4, gguf.zig:952-960 */
static inline void scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* gguf.zig:962-996: per 64-chunk d1 = d*sc, m1 = dmin*m; y = d1*q - m1. */
static void dq_q4_k(const uint8_t *b, float *o, size_t n) {
    for (size_t ib = 0; ib < n / 256; ib++) {
        const uint8_t *blk = b + ib * 144;
        float d = h2f(rd16(blk)), mn = h2f(rd16(blk + 2));
        const uint8_t *scales = blk + 4;
        size_t q = 16;
        for (int is = 0; is < 8; is += 2) {
            uint8_t s0, m0, s1, m1;
            scale_min_k4(is, scales, &s0, &m0);
            scale_min_k4(is + 1, scales, &s1, &m1);
            float d1 = d * (float)s0, mm1 = mn * (float)m0;
            float d2 = d * (float)s1, mm2 = mn * (float)m1;
            size_t y = ib * 256 + (size_t)(is / 2) * 64;
            for (int l = 0; l < 32; l++) {
                float lo = (float)(blk[q + l] & 0x0F), hi = (float)(blk[q + l] >> 4);
                float p0 = d1 * lo, p1 = d2 * hi;
                o[y + l] = p0 - mm1;
                o[y + 32 + l] = p1 - mm2;
            }
            q += 32;
        }
    }
}

/* gguf.zig:998-1034 */
static void dq_q5_k(const uint8_t *b, float *o, size_t n) {
    for (size_t ib = 0; ib < n / 256; ib++) {
        const uint8_t *blk = b + ib * 176;
        float d = h2f(rd16(blk)), mn = h2f(rd16(blk + 2));
        const uint8_t *scales = blk + 4, *qh = blk + 16;
        size_t ql = 48;
        uint8_t mask1 = 1, mask2 = 2;
        for (int is = 0; is < 8; is += 2) {
            uint8_t s0, m0, s1, m1;
            scale_min_k4(is, scales, &s0, &m0);
            scale_min_k4(is + 1, scales, &s1, &m1);
            float d1 = d * (float)s0, mm1 = mn * (float)m0;
            float d2 = d * (float)s1, mm2 = mn * (float)m1;
            size_t y = ib * 256 + (size_t)(is / 2) * 64;
            for (int l = 0; l < 32; l++) {
                int h = (qh[l] & mask1) ? 16 : 0;
                float v = (float)((blk[ql + l] & 0x0F) + h);
                float p = d1 * v;
                o[y + l] = p - mm1;
            }
            for (int l = 0; l < 32; l++) {
                int h = (qh[l] & mask2) ? 16 : 0;
                float v = (float)((blk[ql + l] >> 4) + h);
                float p = d2 * v;
                o[y + 32 + l] = p - mm2;
            }
            ql += 32;
            mask1 = (uint8_t)(mask1 << 2);
            mask2 = (uint8_t)(mask2 << 2);
        }
    }
}

/* gguf.zig:1036-1059: y = (d * f32(sc)) * f32(q - 32). */
static void dq_q6_k(const uint8_t *b, float *o, size_t n) {
    for (size_t ib = 0; ib < n / 256; ib++) {
        const uint8_t *blk = b + ib * 210;
        float d = h2f(rd16(blk + 208));
        for (int half = 0; half < 2; half++) {
            const uint8_t *ql = blk + half * 64, *qh = blk + 128 + half * 32;
            const int8_t *sc = (const int8_t *)(blk + 192 + half * 8);
            size_t y = ib * 256 + (size_t)half * 128;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                float s0 = d * (float)sc[is + 0], s2 = d * (float)sc[is + 2];
                float s4 = d * (float)sc[is + 4], s6 = d * (float)sc[is + 6];
                o[y + l] = s0 * (float)q1;
                o[y + l + 32] = s2 * (float)q2;
                o[y + l + 64] = s4 * (float)q3;
                o[y + l + 96] = s6 * (float)q4;
            }
        }
    }
}

/* gguf.zig:1061-1071 (d is a binary32) */
static void dq_q8_k(const uint8_t *b, float *o, size_t n) {
    for (size_t ib = 0; ib < n / 256; ib++) {
        const uint8_t *blk = b + ib * 292;
        float d = u2f(rd32(blk));
        for (int j = 0; j < 256; j++) o[ib * 256 + j] = (float)(int8_t)blk[4 + j] * d;
    }
}

int orc_dequant_range(int type, const uint8_t *src, size_t src_len, uint64_t elem_offset,
                      float *out, size_t out_n) {
    pthread_once(&f16tab_once, f16tab_init);
    int epb = orc_block_elems(type), bpb = orc_block_bytes(type);
    if (!epb || !bpb) return ORC_EUNSUPPORTED;
    if (out_n == 0) return ORC_OK;
    if (out_n % (size_t)epb || elem_offset % (uint64_t)epb) return ORC_ESHAPE;
    uint64_t start = elem_offset / (uint64_t)epb * (uint64_t)bpb;
    if (start > src_len) return ORC_ETRUNC;
    uint64_t need = (uint64_t)(out_n / (size_t)epb) * (uint64_t)bpb;
    if (src_len - start < need) return ORC_ETRUNC;
    const uint8_t *b = src + start;
    switch (type) {
    case ORC_F32: dq_f32(b, out, out_n); break;
    case ORC_F16: dq_f16(b, out, out_n); break;
    case ORC_BF16: dq_bf16(b, out, out_n); break;
    case ORC_Q4_0: dq_q4_0(b, out, out_n); break;
    case ORC_Q4_1: dq_q4_1(b, out, out_n); break;
    case ORC_Q5_0: dq_q5(b, out, out_n, 22, 0); break;
    case ORC_Q5_1: dq_q5(b, out, out_n, 24, 1); break;
    case ORC_Q8_0: dq_q8_0(b, out, out_n); break;
    case ORC_Q8_1: dq_q8_1(b, out, out_n); break;
    case ORC_Q2_K: dq_q2_k(b, out, out_n); break;
    case ORC_Q3_K: dq_q3_k(b, out, out_n); break;
    case ORC_Q4_K: dq_q4_k(b, out, out_n); break;
    case ORC_Q5_K: dq_q5_k(b, out, out_n); break;
    case ORC_Q6_K: dq_q6_k(b, out, out_n); break;
    case ORC_Q8_K: dq_q8_k(b, out, out_n); break;
    default: return ORC_EUNSUPPORTED;
    }
    return ORC_OK;
}

/* Gguf.readF16 (gguf.zig:554-578): 2048-element chunks, f32 -> f16 RNE. */
int orc_read_f16(int type, const uint8_t *src, size_t src_len, uint16_t *out, size_t n) {
    pthread_once(&f16tab_once, f16tab_init);
    if (type == ORC_F16) {
        if (src_len < 2 * n) return ORC_ETRUNC;
        for (size_t i = 0; i < n; i++) out[i] = rd16(src + 2 * i);
        return ORC_OK;
    }
    float buf[2048];
    size_t done = 0;
    while (done < n) {
        size_t m = n - done < 2048 ? n - done : 2048;
        int rc = orc_dequant_range(type, src, src_len, done, buf, m);
        if (rc) return rc;
        orc_f32_to_f16_n(buf, out + done, m);
        done += m;
    }
    return ORC_OK;
}

/* -------------------------------------------------------------- matvec --- */

typedef struct {
    float *out;
    const uint16_t *w;
    const float *x;
    size_t r0, r1, cols;
} mv_job;

/* Eight rows at a time, one accumulator per row, columns ascending: every
 * row sees exactly the scalar order of main.zig:320-326. */
static void mv_rows(float *out, const uint16_t *w, const float *x, size_t r0, size_t r1, size_t cols) {
    size_t r = r0;
    for (; r + 8 <= r1; r += 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const uint16_t *rows[8];
        for (int j = 0; j < 8; j++) rows[j] = w + (r + (size_t)j) * cols;
        for (size_t i = 0; i < cols; i++) {
            float xi = x[i];
            for (int j = 0; j < 8; j++) {
                float p = h2f(rows[j][i]) * xi;
                acc[j] = acc[j] + p;
            }
        }
        for (int j = 0; j < 8; j++) out[r + (size_t)j] = acc[j];
    }
    for (; r < r1; r++) {
        float acc = 0;
        const uint16_t *row = w + r * cols;
        for (size_t i = 0; i < cols; i++) {
            float p = h2f(row[i]) * x[i];
            acc = acc + p;
        }
        out[r] = acc;
    }
}

static void *mv_thread(void *arg) {
    mv_job *j = (mv_job *)arg;
    mv_rows(j->out, j->w, j->x, j->r0, j->r1, j->cols);
    return NULL;
}

void orc_matvec_f16(float *out, const uint16_t *w, const float *x, size_t rows, size_t cols, int threads) {
    pthread_once(&f16tab_once, f16tab_init);
    if (threads <= 1 || rows < 64) {
        mv_rows(out, w, x, 0, rows, cols);
        return;
    }
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    mv_job jobs[256];
    size_t per = (rows + (size_t)threads - 1) / (size_t)threads;
    per = (per + 7) & ~(size_t)7;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        size_t r0 = (size_t)t * per, r1 = r0 + per;
        if (r0 >= rows) break;
        if (r1 > rows) r1 = rows;
        jobs[t] = (mv_job){out, w, x, r0, r1, cols};
        if (pthread_create(&tid[t], NULL, mv_thread, &jobs[t]) != 0) {
            mv_rows(out, w, x, r0, r1, cols);
            jobs[t].cols = 0;
            continue;
        }
        started = t + 1;
        (void)started;
    }
    for (int t = 0; t < threads; t++) {
        if ((size_t)t * per >= rows) break;
        if (jobs[t].cols) pthread_join(tid[t], NULL);
    }
}

/* ----------------------------------------------------------- dense ops --- */

/* cpu.zig:11-18 */
void orc_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps) {
    float acc = 0;
    for (size_t i = 0; i < n; i++) {
        float p = x[i] * x[i];
        acc = acc + p;
    }
    float mean = acc / (float)n;
    float inv = 1.0f / sqrtf(mean + eps);
    for (size_t i = 0; i < n; i++) {
        float t = x[i] * inv;
        out[i] = t * w[i];
    }
}

/* cpu.zig:22-38: pairs (i, i + hd/2). freq = 1 / pow(theta, 2i/hd) in f32. */
void orc_rope(float *v, uint32_t heads, uint32_t hd, uint32_t pos, float theta) {
    uint32_t half = hd / 2;
    for (uint32_t h = 0; h < heads; h++) {
        size_t base = (size_t)h * hd;
        for (uint32_t i = 0; i < half; i++) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / (float)hd);
            float angle = (float)pos * freq;
            float c = cosf(angle), s = sinf(angle);
            float a = v[base + i], b = v[base + i + half];
            float ac = a * c, bs = b * s, as = a * s, bc = b * c;
            v[base + i] = ac - bs;
            v[base + i + half] = as + bc;
        }
    }
}

/* cpu.zig:46-62: pairs (2j, 2j+1). */
void orc_rope_adjacent(float *v, uint32_t heads, uint32_t hd, uint32_t pos, float theta) {
    uint32_t half = hd / 2;
    for (uint32_t h = 0; h < heads; h++) {
        size_t base = (size_t)h * hd;
        for (uint32_t j = 0; j < half; j++) {
            float freq = 1.0f / powf(theta, (float)(2 * j) / (float)hd);
            float angle = (float)pos * freq;
            float c = cosf(angle), s = sinf(angle);
            float a = v[base + 2 * j], b = v[base + 2 * j + 1];
            float ac = a * c, bs = b * s, as = a * s, bc = b * c;
            v[base + 2 * j] = ac - bs;
            v[base + 2 * j + 1] = as + bc;
        }
    }
}

/* cpu.zig:65-70: g * (1 / (1 + exp(-g))) * u */
void orc_silu_mul(float *out, const float *g, const float *u, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float s = 1.0f / (1.0f + expf(-g[i]));
        float t = g[i] * s;
        out[i] = t * u[i];
    }
}

/* cpu.zig:269-283: the reference's own range-reduced degree-5 polynomial. */
float orc_exp_approx(float x) {
    if (x != x) return x;
    if (x < -87.0f) return 0;
    const float inv_ln2 = 1.4426950408889634f;
    float n_f = roundf(x * inv_ln2);
    int n = (int)n_f;
    float r = x - (float)n * 0.6931471805599453f;
    float p = 1.0f + r * (1.0f + r * (0.5f + r * (0.16666667f + r * (0.041666668f + r * 0.008333334f))));
    float scale = u2f((uint32_t)(n + 127) << 23);
    return p * scale;
}

/* cpu.zig:220-249: vector max, exp on full 8-lane chunks (the vector @exp,
 * here libm expf), the reference's polynomial on the tail, one reciprocal. */
void orc_softmax(float *s, size_t n) {
    if (n == 0) return;
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = s[i] > mx ? s[i] : mx;
    float sum = 0;
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        float e[8];
        for (int j = 0; j < 8; j++) e[j] = expf(s[i + (size_t)j] - mx);
        float cs = e[0];
        for (int j = 1; j < 8; j++) cs = cs + e[j];
        for (int j = 0; j < 8; j++) s[i + (size_t)j] = e[j];
        sum = sum + cs;
    }
    for (; i < n; i++) {
        float e = orc_exp_approx(s[i] - mx);
        s[i] = e;
        sum = sum + e;
    }
    if (sum == 0) return;
    float inv = 1.0f / sum;
    for (size_t k = 0; k < n; k++) s[k] = s[k] * inv;
}

/* dotF32F16, cpu.zig:123-135: 8 lane accumulators, lane-ordered reduce, tail. */
static float dot_f32_f16(const float *a, const uint16_t *b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; j++) {
            float p = a[i + (size_t)j] * h2f(b[i + (size_t)j]);
            acc[j] = acc[j] + p;
        }
    float sum = acc[0];
    for (int j = 1; j < 8; j++) sum = sum + acc[j];
    for (; i < n; i++) {
        float p = a[i] * h2f(b[i]);
        sum = sum + p;
    }
    return sum;
}

/* cpu.zig:323-395 (window = 0, softcap = 0, scale = 1/sqrt(hd)). */
/* One query head of cpu.attentionDecode: qh [hd]; kh / vh point at its KV
 * head's first column, rows `row_stride` halves apart. */
void orc_attention_decode_strided(float *oh, const float *qh, const uint16_t *kh, const uint16_t *vh,
                                  size_t row_stride, size_t n_past, uint32_t hd) {
    pthread_once(&f16tab_once, f16tab_init);
    float scale = 1.0f / sqrtf((float)hd);
    float *scores = (float *)malloc((n_past ? n_past : 1) * sizeof(float));
    if (!scores) return;
    for (size_t t = 0; t < n_past; t++) {
        float d = dot_f32_f16(qh, kh + t * row_stride, hd);
        scores[t] = d * scale;
    }
    orc_softmax(scores, n_past);
    for (uint32_t d = 0; d < hd; d++) oh[d] = 0;
    for (size_t t = 0; t < n_past; t++) {
        const uint16_t *vt = vh + t * row_stride;
        float w = scores[t];
        for (uint32_t d = 0; d < hd; d++) {
            float p = w * h2f(vt[d]);
            oh[d] = oh[d] + p;
        }
    }
    free(scores);
}

void orc_attention_decode(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                          size_t n_past, uint32_t heads, uint32_t kv_heads, uint32_t hd) {
    size_t kv_dim = (size_t)kv_heads * hd;
    uint32_t group = heads / kv_heads;
    for (uint32_t h = 0; h < heads; h++) {
        uint32_t kvh = h / group;
        orc_attention_decode_strided(out + (size_t)h * hd, q + (size_t)h * hd, k_cache + (size_t)kvh * hd,
                                     v_cache + (size_t)kvh * hd, kv_dim, n_past, hd);
    }
}

/* orc_attention_decode with the query heads split across threads: each head's
 * scores, softmax and weighted sum are computed exactly as above, by one
 * thread, so the result does not depend on the split. */
typedef struct {
    float *out;
    const float *q;
    const uint16_t *k_cache, *v_cache;
    size_t n_past;
    uint32_t heads, kv_heads, hd, h0, h1;
} att_job;

static void *att_thread(void *arg) {
    att_job *j = (att_job *)arg;
    const uint32_t group = j->heads / j->kv_heads;
    const size_t kv_dim = (size_t)j->kv_heads * j->hd;
    for (uint32_t h = j->h0; h < j->h1; h++) {
        /* one query head at a time through the single-threaded routine, on a
         * one-head view (its KV head's columns at their offset in the row) */
        const uint32_t kvh = h / group;
        orc_attention_decode_strided(j->out + (size_t)h * j->hd, j->q + (size_t)h * j->hd,
                                     j->k_cache + (size_t)kvh * j->hd, j->v_cache + (size_t)kvh * j->hd, kv_dim,
                                     j->n_past, j->hd);
    }
    return NULL;
}

static void attention_decode_threads(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                     size_t n_past, uint32_t heads, uint32_t kv_heads, uint32_t hd, int threads) {
    if (threads <= 1 || n_past < 256) {
        orc_attention_decode(out, q, k_cache, v_cache, n_past, heads, kv_heads, hd);
        return;
    }
    if ((uint32_t)threads > heads) threads = (int)heads;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    att_job jobs[256];
    int ok[256];
    uint32_t per = (heads + (uint32_t)threads - 1) / (uint32_t)threads;
    for (int t = 0; t < threads; t++) {
        uint32_t h0 = (uint32_t)t * per, h1 = h0 + per < heads ? h0 + per : heads;
        jobs[t] = (att_job){out, q, k_cache, v_cache, n_past, heads, kv_heads, hd, h0, h0 < heads ? h1 : h0};
        ok[t] = pthread_create(&tid[t], NULL, att_thread, &jobs[t]) == 0;
        if (!ok[t]) att_thread(&jobs[t]);
    }
    for (int t = 0; t < threads; t++)
        if (ok[t]) pthread_join(tid[t], NULL);
}

/* cpu.attentionPrefill (cpu.zig:165-217): causal attention of n_q prompt
 * queries starting at position q_pos0.  Query qi, head h, dim d is
 * q[(h * hd + d) * chan_stride + qi * col_stride] (the engine's channel-major
 * layout when chan_stride > 1; position-major with chan_stride 1, col_stride
 * heads * hd); out uses the same layout.  Query qi sees cache positions
 * [0, min(n_past, q_pos0 + qi + 1)), with the same dot / softmax / fp16 axpy
 * as attentionDecode.  Queries are split across threads (each query's result
 * is computed by one thread, so the split does not change it). */
typedef struct {
    float *out;
    const float *q;
    size_t chan_stride, col_stride;
    const uint16_t *k_cache, *v_cache;
    size_t n_past, q_pos0, qi0, qi1;
    uint32_t heads, kv_heads, hd;
} pf_job;

static void *pf_thread(void *arg) {
    pf_job *j = (pf_job *)arg;
    const size_t hd = j->hd, kv_dim = (size_t)j->kv_heads * hd;
    const uint32_t group = j->heads / j->kv_heads;
    float *qs = (float *)malloc(hd * sizeof(float)), *os = (float *)malloc(hd * sizeof(float));
    if (!qs || !os) {
        free(qs);
        free(os);
        return NULL;
    }
    for (size_t qi = j->qi0; qi < j->qi1; qi++) {
        const size_t pos = j->q_pos0 + qi;
        const size_t visible = j->n_past < pos + 1 ? j->n_past : pos + 1;
        const size_t col = qi * j->col_stride;
        for (uint32_t h = 0; h < j->heads; h++) {
            const uint32_t kvh = h / group;
            const size_t base = (size_t)h * hd * j->chan_stride + col;
            for (size_t d = 0; d < hd; d++) qs[d] = j->q[base + d * j->chan_stride];
            orc_attention_decode_strided(os, qs, j->k_cache + (size_t)kvh * hd, j->v_cache + (size_t)kvh * hd,
                                         kv_dim, visible, (uint32_t)hd);
            for (size_t d = 0; d < hd; d++) j->out[base + d * j->chan_stride] = os[d];
        }
    }
    free(qs);
    free(os);
    return NULL;
}

void orc_attention_prefill(float *out, const float *q, size_t chan_stride, size_t col_stride,
                           const uint16_t *k_cache, const uint16_t *v_cache, size_t n_past, size_t n_q,
                           size_t q_pos0, uint32_t heads, uint32_t kv_heads, uint32_t hd, int threads) {
    pthread_once(&f16tab_once, f16tab_init);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((size_t)threads > n_q) threads = n_q ? (int)n_q : 1;
    pthread_t tid[256];
    pf_job jobs[256];
    int ok[256];
    /* interleaved ranges would balance the causal work better; contiguous
     * ranges of equal length keep it simple */
    size_t per = (n_q + (size_t)threads - 1) / (size_t)threads;
    for (int t = 0; t < threads; t++) {
        size_t a = (size_t)t * per, b = a + per < n_q ? a + per : n_q;
        if (a > n_q) a = n_q;
        jobs[t] = (pf_job){out, q, chan_stride, col_stride, k_cache, v_cache, n_past, q_pos0, a, b,
                           heads, kv_heads, hd};
        ok[t] = threads > 1 && pthread_create(&tid[t], NULL, pf_thread, &jobs[t]) == 0;
        if (!ok[t]) pf_thread(&jobs[t]);
    }
    for (int t = 0; t < threads; t++)
        if (ok[t]) pthread_join(tid[t], NULL);
}

/* cpu.zig:477-483: first index of the maximum (strict >). */
uint32_t orc_argmax(const float *v, size_t n) {
    size_t best = 0;
    for (size_t i = 0; i < n; i++)
        if (v[i] > v[best]) best = i;
    return (uint32_t)best;
}

/* ------------------------------------------------------------- sampler --- */

/* cpu.zig:529-547: each occurrence in the window (in window order) divides a
 * positive logit by the repetition penalty or multiplies a non-positive one,
 * then subtracts the frequency penalty; the presence penalty is subtracted at
 * a token's first occurrence only. */
void orc_apply_penalties(float *logits, size_t n, const orc_sampler_params *p, const uint32_t *recent,
                         size_t n_recent) {
    if (p->repetition_penalty == 1.0f && p->presence_penalty == 0.0f && p->frequency_penalty == 0.0f) return;
    const float rep = p->repetition_penalty > 0.0f ? p->repetition_penalty : 1.0f;
    for (size_t i = 0; i < n_recent; i++) {
        const uint32_t id = recent[i];
        if (id >= n) continue;
        float v = logits[id];
        if (rep != 1.0f) v = v > 0 ? v / rep : v * rep;
        if (p->frequency_penalty != 0) v -= p->frequency_penalty;
        if (p->presence_penalty != 0) {
            int seen = 0;
            for (size_t j = 0; j < i; j++)
                if (recent[j] == id) { seen = 1; break; }
            if (!seen) v -= p->presence_penalty;
        }
        logits[id] = v;
    }
}

typedef struct { float logit; uint32_t index; } orc_cand;

/* cpu.zig:573-604 selectTopK: the k largest in items[0..k), descending, by an
 * insertion scan that moves an item only past strictly smaller ones, so equal
 * logits keep their scan (index) order. */
static void select_top_k(orc_cand *items, size_t n, size_t k) {
    size_t held = 0;
    for (size_t i = 0; i < n; i++) {
        const orc_cand c = items[i];
        if (held < k) {
            size_t j = held;
            while (j > 0 && items[j - 1].logit < c.logit) { items[j] = items[j - 1]; j--; }
            items[j] = c;
            held++;
        } else {
            if (c.logit <= items[k - 1].logit) continue;
            const orc_cand victim = items[k - 1];
            size_t j = k - 1;
            while (j > 0 && items[j - 1].logit < c.logit) { items[j] = items[j - 1]; j--; }
            items[j] = c;
            items[i] = victim;
        }
    }
}

/* std.mem.sort is stable: with the candidates in index order, "value
 * descending, then index ascending" is the same order. */
static int cand_desc(const void *a, const void *b) {
    const orc_cand *x = (const orc_cand *)a, *y = (const orc_cand *)b;
    if (x->logit != y->logit) return x->logit > y->logit ? -1 : 1;
    return x->index < y->index ? -1 : (x->index > y->index);
}

uint32_t orc_sample(float *logits, size_t n, const orc_sampler_params *p, const uint32_t *recent, size_t n_recent,
                    uint32_t *rng, orc_sampler_info *info) {
    orc_sampler_info tmp;
    if (!info) info = &tmp;
    memset(info, 0, sizeof(*info));
    info->top_p_margin = 1.0f;
    info->topk_gap = INFINITY;
    orc_apply_penalties(logits, n, p, recent, n_recent);
    const float top_p = p->top_p > 0.0f ? (p->top_p < 1.0f ? p->top_p : 1.0f) : 1.0f;
    float max_v = -INFINITY;
    for (size_t i = 0; i < n; i++) max_v = logits[i] > max_v ? logits[i] : max_v;  /* @max */
    info->max_logit = max_v;
    if (p->temperature <= 0) return orc_argmax(logits, n);
    const float cut = max_v - p->min_keep_delta * p->temperature;
    orc_cand *c = (orc_cand *)malloc(sizeof(orc_cand) * (n ? n : 1));
    size_t nc = 0;
    for (size_t i = 0; i < n; i++)
        if (logits[i] >= cut) { c[nc].logit = logits[i]; c[nc].index = (uint32_t)i; nc++; }
    info->candidates = (uint32_t)nc;
    uint32_t out;
    if (nc == 0) {
        info->path = 1;
        out = orc_argmax(logits, n);
        free(c);
        return out;
    }
    size_t keep = nc;
    const int topk = p->top_k > 0 && p->top_k < nc;
    if (topk) {
        select_top_k(c, nc, p->top_k);
        keep = p->top_k;
        /* the k-th kept logit against the best one left out (ties resolve by index on both sides) */
        float next = -INFINITY;
        for (size_t i = keep; i < nc; i++) next = c[i].logit > next ? c[i].logit : next;
        info->topk_gap = c[keep - 1].logit - next;
    }
    /* probabilities replace the logits in place (cpu.zig:677-681), so the
     * top-p sort below orders by probability */
    float sum = 0;
    for (size_t i = 0; i < keep; i++) {
        c[i].logit = expf((c[i].logit - max_v) / p->temperature);
        sum += c[i].logit;
    }
    if (sum <= 0) {
        info->path = 2;
        out = orc_argmax(logits, n);
        goto done;
    }
    if (top_p < 1.0f) {
        info->sorted_for_top_p = 1;
        if (!topk && keep > 1) qsort(c, keep, sizeof(orc_cand), cand_desc);
        float acc = 0, prev = 0;
        size_t cut_n = keep;
        info->top_p_margin = INFINITY;
        for (size_t i = 0; i < keep; i++) {
            prev = acc;
            acc += c[i].logit / sum;
            if (acc >= top_p) {
                cut_n = i + 1;
                float a = acc - top_p, b = top_p - prev;
                info->top_p_margin = a < b ? a : b;
                break;
            }
        }
        keep = cut_n;
        sum = 0;
        for (size_t i = 0; i < keep; i++) sum += c[i].logit;
        if (sum <= 0) {
            info->path = 2;
            out = orc_argmax(logits, n);
            goto done;
        }
    }
    info->kept = (uint32_t)keep;
    info->sum = sum;
    *rng = *rng * 1664525u + 1013904223u;
    {
        const float r = (float)(*rng >> 8) / 16777216.0f;
        float target = r * sum;
        info->target = target;
        info->path = 3;
        out = c[0].index;
        double cum = 0;
        for (size_t i = 0; i < keep; i++) {
            const double lo = cum;
            cum += c[i].logit;
            target -= c[i].logit;
            if (target <= 0) {
                out = c[i].index;
                const double a = (double)info->target - lo, b = cum - (double)info->target;
                info->draw_margin = (float)((a < b ? a : b) / sum);
                break;
            }
        }
    }
done:
    free(c);
    return out;
}

/* --------------------------------------------------------------- model --- */

typedef struct {
    uint16_t *qkv, *o, *gate, *up, *down;   /* fp16 [out][in]; qkv = q||k||v rows */
    float *attn_norm, *ffn_norm, *qkv_bias, *o_bias;
    uint16_t *k_cache, *v_cache;            /* [max_seq][kv_dim] fp16 */
} orc_layer;

struct orc_model {
    orc_config c;
    orc_layer *layers;
    uint16_t *embed, *output;               /* [vocab][hidden] */
    float *final_norm;
    float *x, *h, *qkv, *attn, *proj, *gate, *up, *act;
};

static size_t q_dim(const orc_config *c) { return (size_t)c->heads * c->head_dim; }
static size_t kv_dim(const orc_config *c) { return (size_t)c->kv_heads * c->head_dim; }

orc_model *orc_model_create(const orc_config *cfg) {
    pthread_once(&f16tab_once, f16tab_init);
    if (!cfg || !cfg->hidden || !cfg->layers || !cfg->heads || !cfg->kv_heads || !cfg->head_dim ||
        cfg->heads % cfg->kv_heads || !cfg->max_seq)
        return NULL;
    orc_model *m = (orc_model *)calloc(1, sizeof(*m));
    if (!m) return NULL;
    m->c = *cfg;
    m->layers = (orc_layer *)calloc(cfg->layers, sizeof(orc_layer));
    size_t qd = q_dim(cfg), kvd = kv_dim(cfg), qkvd = qd + 2 * kvd;
    size_t widest = qkvd > cfg->inter ? qkvd : cfg->inter;
    if (widest < cfg->hidden) widest = cfg->hidden;
    m->x = (float *)calloc(cfg->hidden, 4);
    m->h = (float *)calloc(cfg->hidden, 4);
    m->qkv = (float *)calloc(qkvd, 4);
    m->attn = (float *)calloc(qd, 4);
    m->proj = (float *)calloc(cfg->hidden, 4);
    m->gate = (float *)calloc(cfg->inter, 4);
    m->up = (float *)calloc(cfg->inter, 4);
    m->act = (float *)calloc(cfg->inter, 4);
    if (!m->layers || !m->x || !m->h || !m->qkv || !m->attn || !m->proj || !m->gate || !m->up || !m->act) {
        orc_model_free(m);
        return NULL;
    }
    for (uint32_t l = 0; l < cfg->layers; l++) {
        m->layers[l].k_cache = (uint16_t *)calloc((size_t)cfg->max_seq * kvd, 2);
        m->layers[l].v_cache = (uint16_t *)calloc((size_t)cfg->max_seq * kvd, 2);
        if (!m->layers[l].k_cache || !m->layers[l].v_cache) {
            orc_model_free(m);
            return NULL;
        }
    }
    (void)widest;
    return m;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    if (m->layers) {
        for (uint32_t l = 0; l < m->c.layers; l++) {
            orc_layer *L = &m->layers[l];
            free(L->qkv); free(L->o); free(L->gate); free(L->up); free(L->down);
            free(L->attn_norm); free(L->ffn_norm); free(L->qkv_bias); free(L->o_bias);
            free(L->k_cache); free(L->v_cache);
        }
        free(m->layers);
    }
    free(m->embed); free(m->output); free(m->final_norm);
    free(m->x); free(m->h); free(m->qkv); free(m->attn); free(m->proj);
    free(m->gate); free(m->up); free(m->act);
    free(m);
}

/* load_gguf.loadLinear (load_gguf.zig:358-386) for a tensor whose dims are
 * already [in][out] in ggml order (payload row-major [out][in]). */
/* orc_read_f16 split into contiguous element ranges across threads.  Every
 * element is dequantised and rounded on its own, so the result does not depend
 * on the split; ranges start on multiples of 2048 elements (whole blocks of
 * every type, the chunking of gguf.zig:554-578). */
typedef struct {
    int type;
    const uint8_t *src;
    size_t src_len, e0, e1;
    uint16_t *out;
    int rc;
} rf16_job;

static void *rf16_thread(void *arg) {
    rf16_job *j = (rf16_job *)arg;
    float buf[2048];
    j->rc = ORC_OK;
    for (size_t done = j->e0; done < j->e1;) {
        size_t k = j->e1 - done < 2048 ? j->e1 - done : 2048;
        int rc = orc_dequant_range(j->type, j->src, j->src_len, done, buf, k);
        if (rc) {
            j->rc = rc;
            break;
        }
        orc_f32_to_f16_n(buf, j->out + done, k);
        done += k;
    }
    return NULL;
}

static int read_f16_threads(int type, const uint8_t *src, size_t src_len, uint16_t *out, size_t n, int threads) {
    if (threads <= 1 || type == ORC_F16 || n < (size_t)1 << 20) return orc_read_f16(type, src, src_len, out, n);
    pthread_once(&f16tab_once, f16tab_init);
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    rf16_job jobs[256];
    size_t per = (n + (size_t)threads - 1) / (size_t)threads;
    per = (per + 2047) & ~(size_t)2047;
    int started = 0, rc = ORC_OK;
    for (int t = 0; t < threads; t++) {
        size_t e0 = (size_t)t * per, e1 = e0 + per < n ? e0 + per : n;
        if (e0 >= n) break;
        jobs[t] = (rf16_job){type, src, src_len, e0, e1, out, ORC_OK};
        if (pthread_create(&tid[t], NULL, rf16_thread, &jobs[t]) != 0) {
            rf16_thread(&jobs[t]);  /* no thread: do it here */
            if (jobs[t].rc) rc = jobs[t].rc;
            jobs[t].src = NULL;
            continue;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++) {
        if (!jobs[t].src) continue;
        pthread_join(tid[t], NULL);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    return rc;
}

int orc_model_set_linear(orc_model *m, int layer, int role, int type, const uint8_t *raw, size_t nbytes,
                         uint32_t rows, uint32_t cols) {
    const orc_config *c = &m->c;
    if (role != ORC_ROLE_EMBED && role != ORC_ROLE_OUTPUT && (layer < 0 || (uint32_t)layer >= c->layers))
        return ORC_ESHAPE;
    size_t qd = q_dim(c), kvd = kv_dim(c), n = (size_t)rows * cols;
    uint16_t *dst = NULL;
    orc_layer *L = (role == ORC_ROLE_EMBED || role == ORC_ROLE_OUTPUT) ? NULL : &m->layers[layer];
    switch (role) {
    case ORC_ROLE_Q: case ORC_ROLE_K: case ORC_ROLE_V: {
        size_t want = role == ORC_ROLE_Q ? qd : kvd;
        if (rows != want || cols != c->hidden) return ORC_ESHAPE;
        if (!L->qkv) L->qkv = (uint16_t *)calloc((qd + 2 * kvd) * c->hidden, 2);
        if (!L->qkv) return ORC_ENOMEM;
        size_t row0 = role == ORC_ROLE_Q ? 0 : role == ORC_ROLE_K ? qd : qd + kvd;  /* q||k||v, load_gguf.zig:677-682 */
        dst = L->qkv + row0 * c->hidden;
        break;
    }
    case ORC_ROLE_O:
        if (rows != c->hidden || cols != qd) return ORC_ESHAPE;
        dst = L->o = (uint16_t *)malloc(n * 2); break;
    case ORC_ROLE_GATE:
        if (rows != c->inter || cols != c->hidden) return ORC_ESHAPE;
        dst = L->gate = (uint16_t *)malloc(n * 2); break;
    case ORC_ROLE_UP:
        if (rows != c->inter || cols != c->hidden) return ORC_ESHAPE;
        dst = L->up = (uint16_t *)malloc(n * 2); break;
    case ORC_ROLE_DOWN:
        if (rows != c->hidden || cols != c->inter) return ORC_ESHAPE;
        dst = L->down = (uint16_t *)malloc(n * 2); break;
    case ORC_ROLE_EMBED:
        if (rows != c->vocab || cols != c->hidden) return ORC_ESHAPE;
        dst = m->embed = (uint16_t *)malloc(n * 2); break;
    case ORC_ROLE_OUTPUT:
        if (rows != c->vocab || cols != c->hidden) return ORC_ESHAPE;
        dst = m->output = (uint16_t *)malloc(n * 2); break;
    default: return ORC_ESHAPE;
    }
    if (!dst) return ORC_ENOMEM;
    return read_f16_threads(type, raw, nbytes, dst, n, c->threads);
}

int orc_model_set_f32(orc_model *m, int layer, int role, const float *v, size_t n) {
    const orc_config *c = &m->c;
    size_t qd = q_dim(c), kvd = kv_dim(c);
    if (role == ORC_ROLE_FINAL_NORM) {
        if (n != c->hidden) return ORC_ESHAPE;
        free(m->final_norm);
        m->final_norm = (float *)malloc(n * 4);
        if (!m->final_norm) return ORC_ENOMEM;
        memcpy(m->final_norm, v, n * 4);
        return ORC_OK;
    }
    if (layer < 0 || (uint32_t)layer >= c->layers) return ORC_ESHAPE;
    orc_layer *L = &m->layers[layer];
    float **slot = NULL;
    size_t off = 0, want = 0, total = 0;
    switch (role) {
    case ORC_ROLE_ATTN_NORM: slot = &L->attn_norm; want = total = c->hidden; break;
    case ORC_ROLE_FFN_NORM: slot = &L->ffn_norm; want = total = c->hidden; break;
    case ORC_ROLE_O_BIAS: slot = &L->o_bias; want = total = c->hidden; break;
    case ORC_ROLE_Q_BIAS: slot = &L->qkv_bias; want = qd; off = 0; total = qd + 2 * kvd; break;
    case ORC_ROLE_K_BIAS: slot = &L->qkv_bias; want = kvd; off = qd; total = qd + 2 * kvd; break;
    case ORC_ROLE_V_BIAS: slot = &L->qkv_bias; want = kvd; off = qd + kvd; total = qd + 2 * kvd; break;
    default: return ORC_ESHAPE;
    }
    if (n != want) return ORC_ESHAPE;
    if (!*slot) *slot = (float *)calloc(total, 4);
    if (!*slot) return ORC_ENOMEM;
    memcpy(*slot + off, v, n * 4);
    return ORC_OK;
}

/* refForward, main.zig:334-541, for the dense llama/qwen2 path.  The shipped
 * refForward only carries a MoE branch after ffn_norm (main.zig:487-520), so
 * the dense MLP follows the engine's split path (engine.zig:645-668):
 * gate = Wg h, up = Wu h, act = siluMul(gate, up), x += Wd act. */
int orc_model_forward(orc_model *m, uint32_t token, uint32_t pos, float *logits) {
    const orc_config *c = &m->c;
    if (pos >= c->max_seq) return ORC_ESHAPE;  /* error.ContextOverflow, engine.zig:549 */
    if (token >= c->vocab || !m->embed || !m->final_norm) return ORC_ESHAPE;
    size_t H = c->hidden, qd = q_dim(c), kvd = kv_dim(c), qkvd = qd + 2 * kvd, I = c->inter;
    int thr = c->threads;
    for (size_t i = 0; i < H; i++) m->x[i] = h2f(m->embed[(size_t)token * H + i]) * 1.0f;
    for (uint32_t l = 0; l < c->layers; l++) {
        orc_layer *L = &m->layers[l];
        if (!L->qkv || !L->o || !L->gate || !L->up || !L->down || !L->attn_norm || !L->ffn_norm)
            return ORC_ESHAPE;
        orc_rmsnorm(m->h, m->x, L->attn_norm, H, c->eps);
        orc_matvec_f16(m->qkv, L->qkv, m->h, qkvd, H, thr);
        if (L->qkv_bias)
            for (size_t i = 0; i < qkvd; i++) m->qkv[i] = m->qkv[i] + L->qkv_bias[i];
        float *q = m->qkv, *k = m->qkv + qd, *v = m->qkv + qd + kvd;
        if (c->rope_adjacent) {
            orc_rope_adjacent(q, c->heads, c->head_dim, pos, c->rope_theta);
            orc_rope_adjacent(k, c->kv_heads, c->head_dim, pos, c->rope_theta);
        } else {
            orc_rope(q, c->heads, c->head_dim, pos, c->rope_theta);
            orc_rope(k, c->kv_heads, c->head_dim, pos, c->rope_theta);
        }
        for (size_t i = 0; i < kvd; i++) {
            L->k_cache[(size_t)pos * kvd + i] = orc_f32_to_f16(k[i]);
            L->v_cache[(size_t)pos * kvd + i] = orc_f32_to_f16(v[i]);
        }
        attention_decode_threads(m->attn, q, L->k_cache, L->v_cache, (size_t)pos + 1, c->heads, c->kv_heads,
                                 c->head_dim, thr);
        orc_matvec_f16(m->proj, L->o, m->attn, H, qd, thr);
        if (L->o_bias)
            for (size_t i = 0; i < H; i++) m->proj[i] = m->proj[i] + L->o_bias[i];
        for (size_t i = 0; i < H; i++) m->x[i] = m->x[i] + m->proj[i];
        orc_rmsnorm(m->h, m->x, L->ffn_norm, H, c->eps);
        orc_matvec_f16(m->gate, L->gate, m->h, I, H, thr);
        orc_matvec_f16(m->up, L->up, m->h, I, H, thr);
        orc_silu_mul(m->act, m->gate, m->up, I);
        orc_matvec_f16(m->proj, L->down, m->act, H, I, thr);
        for (size_t i = 0; i < H; i++) m->x[i] = m->x[i] + m->proj[i];
    }
    orc_rmsnorm(m->h, m->x, m->final_norm, H, c->eps);
    const uint16_t *head = c->tie_embeddings ? m->embed : m->output;
    if (!head) return ORC_ESHAPE;
    /* logits == NULL: a prompt position whose logits nobody reads (the engine's
     * prefill computes the head for the last position only, engine.zig:1310-1316) */
    if (logits) orc_matvec_f16(logits, head, m->h, c->vocab, H, thr);
    return ORC_OK;
}

const float *orc_model_last_hidden(const orc_model *m) { return m->h; }

/* Overwrite cache rows [pos0, pos0 + n) of `layer` with fp16 rows [n][kv_dim]
 * (test infrastructure: the GPU engine gets the same rows through cuq_kv_write,
 * so both continue from one cache state). */
int orc_model_set_kv(orc_model *m, uint32_t layer, uint32_t pos0, uint32_t n, const uint16_t *k, const uint16_t *v) {
    const orc_config *c = &m->c;
    if (layer >= c->layers || (uint64_t)pos0 + n > c->max_seq) return ORC_ESHAPE;
    size_t kvd = kv_dim(c);
    memcpy(m->layers[layer].k_cache + (size_t)pos0 * kvd, k, (size_t)n * kvd * 2);
    memcpy(m->layers[layer].v_cache + (size_t)pos0 * kvd, v, (size_t)n * kvd * 2);
    return ORC_OK;
}

int orc_model_kv_row(const orc_model *m, uint32_t layer, uint32_t pos, uint16_t *k, uint16_t *v) {
    const orc_config *c = &m->c;
    if (layer >= c->layers || pos >= c->max_seq) return ORC_ESHAPE;
    size_t kvd = kv_dim(c);
    memcpy(k, m->layers[layer].k_cache + (size_t)pos * kvd, kvd * 2);
    memcpy(v, m->layers[layer].v_cache + (size_t)pos * kvd, kvd * 2);
    return ORC_OK;
}
