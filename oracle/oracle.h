/* oracle.h -- CPU restatement of ANEDVD's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in anedvd_b200/: it is loaded by tests/, by __graft_entry__.smoke() and
 * by bench.py's CPU-baseline leg, never by the product path.
 *
 * Parity pin: the dequantisers are checked bit-for-bit against the reference's
 * own golden vectors (the dequant fixture .bin/.f32 pairs in midasdf/ANEDVD,
 * copied with their generator into tests/golden/) and against the reference's
 * hand-computed blocks (src/gguf.zig:1424-1526).  The dense ops restate
 * src/cpu.zig and src/main.zig; each function names the lines it follows.
 *
 * Build: plain C11, -O2 -ffp-contract=off (no FMA contraction, no fast-math),
 * so every float operation rounds exactly where the reference's does.
 */
#ifndef ANEDVD_ORACLE_H
#define ANEDVD_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids as stored in GGUF (src/gguf.zig:30-46). */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q5_0 = 6,
    ORC_Q5_1 = 7, ORC_Q8_0 = 8, ORC_Q8_1 = 9, ORC_Q2_K = 10, ORC_Q3_K = 11,
    ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14, ORC_Q8_K = 15, ORC_BF16 = 30
};

/* Error codes mirror gguf.zig's error set for dequantizeRange. */
enum { ORC_OK = 0, ORC_EUNSUPPORTED = -1, ORC_ESHAPE = -2, ORC_ETRUNC = -3, ORC_ENOMEM = -4 };

int orc_block_elems(int type);          /* gguf.zig:49-56; 0 = unsupported */
int orc_block_bytes(int type);          /* gguf.zig:59-77; 0 = unsupported */

/* dequantizeRange (gguf.zig:694-728): `out_n` elements starting at element
 * `elem_offset` of `src` (both multiples of the block size). */
int orc_dequant_range(int type, const uint8_t *src, size_t src_len,
                      uint64_t elem_offset, float *out, size_t out_n);

/* IEEE binary16 <-> binary32, round-to-nearest-even (gguf.zig:682-692). */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_f16_n(const float *src, uint16_t *dst, size_t n);

/* Gguf.readF16 (gguf.zig:554-578): dequantise then round every weight to fp16. */
int orc_read_f16(int type, const uint8_t *src, size_t src_len, uint16_t *out, size_t n);

/* main.zig:320-326 matmulF16: out[o] = sum_i f32(w[o][i]) * x[i], fp32, i
 * ascending.  `threads` > 1 splits rows across threads; each row keeps the
 * same sequential order, so the result does not depend on `threads`. */
void orc_matvec_f16(float *out, const uint16_t *w, const float *x, size_t rows,
                    size_t cols, int threads);

void orc_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps); /* cpu.zig:11-18 */
void orc_rope(float *v, uint32_t heads, uint32_t hd, uint32_t pos, float theta);    /* cpu.zig:22-38 */
void orc_rope_adjacent(float *v, uint32_t heads, uint32_t hd, uint32_t pos, float theta); /* cpu.zig:46-62 */
void orc_silu_mul(float *out, const float *g, const float *u, size_t n);             /* cpu.zig:65-70 */
float orc_exp_approx(float x);                                                       /* cpu.zig:269-283 */
void orc_softmax(float *s, size_t n);                                                /* cpu.zig:220-249 */
/* cpu.zig:323-395 with the default AttnOpts (no softcap, no window). */
void orc_attention_decode_strided(float *oh, const float *qh, const uint16_t *kh, const uint16_t *vh,
                                  size_t row_stride, size_t n_past, uint32_t hd);
void orc_attention_prefill(float *out, const float *q, size_t chan_stride, size_t col_stride,
                           const uint16_t *k_cache, const uint16_t *v_cache, size_t n_past, size_t n_q,
                           size_t q_pos0, uint32_t heads, uint32_t kv_heads, uint32_t hd, int threads);
void orc_attention_decode(float *out, const float *q, const uint16_t *k_cache,
                          const uint16_t *v_cache, size_t n_past, uint32_t heads,
                          uint32_t kv_heads, uint32_t hd);
uint32_t orc_argmax(const float *v, size_t n);                                       /* cpu.zig:477-483 */

/* cpu.SamplerParams (cpu.zig:502-518), field for field. */
typedef struct {
    float temperature;          /* <= 0: greedy */
    uint32_t top_k;             /* 0: off */
    float top_p;                /* 1: off; <= 0 treated as 1 */
    float repetition_penalty;   /* 1: off; <= 0 treated as 1 */
    float presence_penalty;
    float frequency_penalty;
    float min_keep_delta;       /* logits below max - delta * temperature are dropped */
} orc_sampler_params;

/* What one draw did: cpu.SamplerInfo (cpu.zig:491-500) plus the distances the
 * parity tests use to tell a genuine mismatch from one forced by rounding. */
typedef struct {
    uint32_t candidates;        /* entries >= the min_keep_delta cut */
    uint32_t kept;              /* entries drawn from */
    int32_t sorted_for_top_p;
    int32_t path;               /* 0 greedy, 1 no candidates, 2 sum <= 0, 3 drawn */
    float max_logit;            /* after the penalties */
    float sum;                  /* probability mass of the kept set */
    float target;               /* r * sum before the walk */
    float draw_margin;          /* distance of target from the nearest cumulative edge, / sum */
    float top_p_margin;         /* distance of the nucleus cut from top_p (1 when top_p is off) */
    float topk_gap;             /* logit of the k-th kept minus the next one (inf when top-k is off) */
} orc_sampler_info;

/* cpu.applyPenalties (cpu.zig:529-547), in place. */
void orc_apply_penalties(float *logits, size_t n, const orc_sampler_params *p, const uint32_t *recent,
                         size_t n_recent);
/* cpu.sampleProfiled (cpu.zig:621-721): penalties (in place), greedy for a
 * non-positive temperature, the min_keep_delta cut, top-k by selectTopK
 * (cpu.zig:573-604), probabilities by exp, top-p over the descending order
 * (stable sort), then the LCG draw (rng = rng * 1664525 + 1013904223).
 * info may be NULL. */
uint32_t orc_sample(float *logits, size_t n, const orc_sampler_params *p, const uint32_t *recent, size_t n_recent,
                    uint32_t *rng, orc_sampler_info *info);

/* ------------------------------------------------------------ model ----- */

typedef struct {
    uint32_t hidden, layers, heads, kv_heads, head_dim, inter, vocab, max_seq;
    float eps, rope_theta;
    int rope_adjacent;      /* load_gguf.zig:81-90: llama -> 1, qwen2 -> 0 */
    int tie_embeddings;     /* no output.weight (load_gguf.zig:141) */
    int threads;            /* matvec row threads (1 = reference order, single core) */
} orc_config;

typedef struct orc_model orc_model;

/* Tensor roles for orc_model_set_*. */
enum {
    ORC_ROLE_Q = 0, ORC_ROLE_K = 1, ORC_ROLE_V = 2, ORC_ROLE_O = 3,
    ORC_ROLE_GATE = 4, ORC_ROLE_UP = 5, ORC_ROLE_DOWN = 6,
    ORC_ROLE_ATTN_NORM = 7, ORC_ROLE_FFN_NORM = 8,
    ORC_ROLE_Q_BIAS = 9, ORC_ROLE_K_BIAS = 10, ORC_ROLE_V_BIAS = 11, ORC_ROLE_O_BIAS = 12,
    ORC_ROLE_EMBED = 13, ORC_ROLE_OUTPUT = 14, ORC_ROLE_FINAL_NORM = 15
};

orc_model *orc_model_create(const orc_config *cfg);
void orc_model_free(orc_model *m);
/* Raw GGUF blocks for a [rows][cols] linear; dequantised + fp16-rounded like
 * load_gguf.loadLinear (load_gguf.zig:358-386).  layer is ignored for
 * EMBED/OUTPUT. */
int orc_model_set_linear(orc_model *m, int layer, int role, int type,
                         const uint8_t *raw, size_t nbytes, uint32_t rows, uint32_t cols);
int orc_model_set_f32(orc_model *m, int layer, int role, const float *v, size_t n);
/* refForward (main.zig:334-541, dense MLP from engine.zig:645-668). */
int orc_model_forward(orc_model *m, uint32_t token, uint32_t pos, float *logits);
/* Hidden state after the final RMSNorm of the last forward (for per-stage checks). */
const float *orc_model_last_hidden(const orc_model *m);
/* Read back a fp16 KV-cache row: [layer][pos][kv_dim]. */
int orc_model_set_kv(orc_model *m, uint32_t layer, uint32_t pos0, uint32_t n, const uint16_t *k,
                     const uint16_t *v);
int orc_model_kv_row(const orc_model *m, uint32_t layer, uint32_t pos, uint16_t *k, uint16_t *v);

#ifdef __cplusplus
}
#endif
#endif
