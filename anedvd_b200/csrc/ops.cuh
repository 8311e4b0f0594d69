// ops.cuh -- launchers of the dense decode/prefill ops (ops.cu).
#pragma once
#include "common.cuh"

namespace cuq {

int launch_rmsnorm(float *out, const float *x, const float *w, uint32_t n, uint32_t n_rows, float eps,
                   cudaStream_t s);
// One position's cos | sin row (hd <= 256), passed to the kernel by value.
struct RopeRow {
    float v[256];
};
int launch_rope(float *v, uint32_t heads, uint32_t hd, const RopeRow &cs_row, int adjacent, cudaStream_t s);
// cs: [max_seq][hd] table, each row cos(0..hd/2) then sin(0..hd/2).
int launch_rope_cache(const float *qkv, uint32_t qkv_stride, float *q_out, __half *k_cache, __half *v_cache,
                      uint32_t cache_stride, const float *cs, const int *pos_ptr, uint32_t pos_val, uint32_t n_tok,
                      uint32_t heads, uint32_t kv_heads, uint32_t hd, int adjacent, cudaStream_t s);
int attn_pick_nsplit(uint32_t kv_heads, uint32_t max_seq, int sm_count);
// part: nsplit * heads * (hd + 2) floats of scratch.  n = *pos_ptr + 1 when pos_ptr is set.
int launch_attention_decode(const float *q, const __half *k_cache, const __half *v_cache, uint32_t cache_stride,
                            const int *pos_ptr, uint32_t n_val, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                            float *part, int nsplit, float *out, __half *xq, cudaStream_t s);
// The decode step's fused attention (RoPE, KV write, split attention, combine -> xq).
// tickets: kv_heads counters, zero-initialised once (self-resetting).
int launch_attention_step(const float *qkv, const float *cs, const StepState *state, __half *k_cache,
                          __half *v_cache, uint32_t cache_stride, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                          int adjacent, float *part, int nsplit, unsigned int *tickets, __half *xq, bool pdl,
                          cudaStream_t s);
// Embedding row + the first layer's RMSNorm -> xq, one CTA (decode step start).
int launch_embed_norm(const Planes &p, const StepState *state, float *x, const float *norm_w, uint32_t n, float eps,
                      __half *xq, bool pdl, cudaStream_t s);
// Prefill: RMSNorm rows -> fp16 hi/lo; causal attention for n_q prompt positions
// starting at pos0 (K/V already in the cache) -> hi/lo; SiLU*mul -> hi/lo;
// embedding rows of ids[0..n) -> x[n][hidden].
int launch_rmsnorm_hilo(const float *x, const float *w, uint32_t n, uint32_t n_rows, float eps, __half *hi,
                        __half *lo, cudaStream_t s);
int launch_attention_prefill(const float *q, const __half *k_cache, const __half *v_cache, uint32_t cache_stride,
                             uint32_t pos0, uint32_t n_q, uint32_t heads, uint32_t kv_heads, uint32_t hd,
                             __half *oh, __half *ol, cudaStream_t s);
// out[i] = hi[i] + lo[i] in fp32 (an activation split into fp16 hi and lo planes).
int launch_hilo_sum(const __half *hi, const __half *lo, size_t count, float *out, cudaStream_t s);
int launch_silu_hilo(const float *g, const float *u, size_t count, __half *hi, __half *lo, cudaStream_t s);
int launch_embed_rows(const Planes &p, const uint32_t *ids, uint32_t n, float *x, cudaStream_t s);
int launch_silu_mul(float *out, const float *g, const float *u, uint32_t n, cudaStream_t s);
int launch_argmax(const float *v, uint32_t n, uint32_t *out, cudaStream_t s);
// Embedding row (token from *token_ptr): x = f32(RN16(dequant(row))) (load_gguf.zig:578-647 + engine.zig:561-564).
int launch_embed_row(const Planes &p, const int *token_ptr, float *x, cudaStream_t s);

// RoPE table with the reference formula (cpu.zig:26-31): freq = 1 / powf(theta, 2i/hd),
// angle = f32(pos) * freq, cos/sin in fp32.  Host-side; rows of hd floats.
void build_rope_table(float *out, uint32_t max_seq, uint32_t hd, float theta);

}  // namespace cuq
