/* cuq.h -- C ABI of the B200 (sm_100a) CUDA backend for ANEDVD's quantized-weight path.
 *
 * This header is the drop-in boundary.  It sits where the reference's ANE
 * shim sits (src/ane/shim.h:49-116) and keeps that shim's conventions:
 * opaque handles, int status codes, a thread-local last-error string, plain
 * pointers and sizes, no C++ or torch types.  The engine-level calls mirror
 * src/engine.zig's Engine (init / forward / prefill / reset / stats) so the
 * Zig engine can call them where it evaluates ANE kernels today.
 *
 * Memory conventions:
 *   - "host" arguments are ordinary CPU memory owned by the caller;
 *   - "dev" arguments are CUDA device pointers on the current device;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     op entry points only enqueue work and return (cuq_gemm excepted: it
 *     waits for its stream, see there).
 * Status: CUQ_OK (0) on success, a negative CUQ_E* code on failure, with
 * cuq_last_error() describing it.
 */
#ifndef CUQ_H
#define CUQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status ---- */
#define CUQ_OK 0
#define CUQ_EINVAL (-1)       /* bad argument / shape (engine.zig WrongShape, gguf InvalidTensorShape) */
#define CUQ_ENOMEM (-2)       /* device or host allocation failed */
#define CUQ_ECUDA (-3)        /* a CUDA runtime call failed */
#define CUQ_ECONTEXT (-4)     /* position past max_seq: engine.zig:549,981 error.ContextOverflow */
#define CUQ_EUNSUPPORTED (-5) /* ggml type not handled here: gguf.zig error.UnsupportedType */
#define CUQ_ETIMEOUT (-6)     /* a bounded device-side wait gave up */
#define CUQ_EFORMAT (-7)      /* malformed GGUF: gguf.zig NotGgufFile / TruncatedFile / ... */
#define CUQ_ENOTREADY (-8)    /* cuq_init not called / model not finalized */

/* ggml type ids as stored in GGUF (src/gguf.zig:30-46). */
#define CUQ_F32 0
#define CUQ_F16 1
#define CUQ_Q4_0 2
#define CUQ_Q4_1 3
#define CUQ_Q5_0 6
#define CUQ_Q5_1 7
#define CUQ_Q8_0 8
#define CUQ_Q8_1 9
#define CUQ_Q2_K 10
#define CUQ_Q3_K 11
#define CUQ_Q4_K 12
#define CUQ_Q5_K 13
#define CUQ_Q6_K 14
#define CUQ_Q8_K 15
#define CUQ_BF16 30

/* ------------------------------------------------------- lifecycle ---- */

/* Select `device` and create the library's context on it.
 * Replaces ane_shim_init (src/ane/shim.h:53-54): 0 on success, <0 on failure. */
int cuq_init(int device);
/* 1 if cuq_init succeeded on this thread's current device (ane_shim_ready, shim.h:57). */
int cuq_ready(void);
/* Thread-local description of the last failure (ane_shim_last_error, shim.h:60). */
const char *cuq_last_error(void);
/* Library build string (git-free: compiler + arch). */
const char *cuq_version(void);

/* Block geometry (gguf.zig:49-77); 0 for unsupported types. */
int cuq_block_elems(int ggml_type);
int cuq_block_bytes(int ggml_type);

/* --------------------------------------------------- dequantisation ---- */

/* gguf.dequantizeRange (gguf.zig:694-728) on the device: `out_n` float32
 * values starting at element `elem_offset` of the raw GGUF blocks at
 * `raw_dev` (`raw_bytes` long).  Bit-exact with the reference for all 15
 * types.  All pointers dev. */
int cuq_dequant(int ggml_type, const void *raw_dev, size_t raw_bytes, uint64_t elem_offset,
                float *out_dev, size_t out_n, void *stream);

/* ------------------------------------------------------------ weights --- */

/* A weight matrix resident in HBM in its quantized form.  Replaces the fp16
 * [out][in] expansion of load_gguf.loadLinear (load_gguf.zig:358-386): the raw
 * GGUF payload (row-major [rows][cols], blocks along cols) is copied to the
 * device as-is and losslessly regrouped there into per-field planes (quants,
 * scales) so every warp load is an aligned 128-bit access.  Same byte count as
 * the file; cuq_weight_export_raw gives back the identical bytes. */
typedef struct cuq_weight cuq_weight;

/* raw_host: host pointer to the GGUF payload. NULL on failure (see cuq_last_error). */
cuq_weight *cuq_weight_create(int ggml_type, const void *raw_host, size_t nbytes, uint32_t rows,
                              uint32_t cols);
/* Rebuild the original GGUF payload (host buffer of cuq_weight_nbytes bytes). */
int cuq_weight_export_raw(const cuq_weight *w, void *raw_host, size_t nbytes);
size_t cuq_weight_nbytes(const cuq_weight *w);
void cuq_weight_free(cuq_weight *w);

/* y[rows] = W x: quantized GEMV, batch 1 (the decode projection).  x_dev is
 * float32 [cols], y_dev float32 [rows].  Results follow the reference's
 * matmulF16 (main.zig:320-326) on fp16-rounded weights within 1e-3 relative. */
int cuq_gemv(const cuq_weight *w, const float *x_dev, float *y_dev, void *stream);

/* The GEMV's activation operand, prepared once: x split into fp16 hi + lo
 * parts (x = hi + lo to ~22 bits) in the column order the tensor-core
 * fragments read.  cuq_xq_halves(n) halves of device memory hold it. */
size_t cuq_xq_halves(uint32_t n);
int cuq_prepare_x(const float *x_dev, uint32_t n, uint16_t *xq_dev, void *stream);
/* cuq_gemv on an already prepared activation (one kernel launch). */
int cuq_gemv_prepared(const cuq_weight *w, const uint16_t *xq_dev, float *y_dev, void *stream);

/* Y[n][rows] = X[n][cols] W^T for a chunk of n tokens (the prefill projection,
 * engine.zig:975-1329).  X, Y float32 row-major, dev.  Returns after the GEMM
 * has run (it synchronises `stream`): the tensor-core pipeline's bounded waits
 * report through a device flag, read here, so a wait that gave up comes back
 * as CUQ_ETIMEOUT from this call. */
int cuq_gemm(const cuq_weight *w, const float *x_dev, uint32_t n, float *y_dev, void *stream);

/* Dequantise W to fp16 [rows][cols] exactly as Gguf.readF16 (gguf.zig:554-578) does:
 * reference fp32 value, then round to nearest even. out_dev holds rows*cols halves. */
int cuq_weight_dequant_f16(const cuq_weight *w, uint16_t *out_dev, void *stream);

/* --------------------------------------------------------- dense ops ---- */

/* cpu.rmsnorm (cpu.zig:11-18) on `n_rows` rows of length n: out = x * rsqrt(mean(x^2)+eps) * w. */
int cuq_rmsnorm(float *out_dev, const float *x_dev, const float *w_dev, uint32_t n, uint32_t n_rows,
                float eps, void *stream);
/* cpu.rope / cpu.ropeAdjacent (cpu.zig:22-62), in place on `heads` heads of `hd`. */
int cuq_rope(float *v_dev, uint32_t heads, uint32_t hd, uint32_t pos, float theta, int adjacent,
             void *stream);
/* cpu.siluMul (cpu.zig:65-70). */
int cuq_silu_mul(float *out_dev, const float *g_dev, const float *u_dev, uint32_t n, void *stream);
/* cpu.attentionDecode (cpu.zig:323-395): q [heads*hd] f32; k/v fp16 caches laid
 * out [kv_heads][cache_stride][hd] (position-major inside each head); attends to
 * positions [0, n_past).  Split over positions on the device. */
int cuq_attention_decode(float *out_dev, const float *q_dev, const uint16_t *k_dev,
                         const uint16_t *v_dev, uint32_t n_past, uint32_t cache_stride,
                         uint32_t heads, uint32_t kv_heads, uint32_t hd, void *stream);
/* cpu.attentionPrefill (cpu.zig:165-217): causal attention of `n` prompt
 * queries at positions pos0 .. pos0+n-1.  q [n][heads*hd] f32 (already
 * rotated), out [n][heads*hd] f32; k/v fp16 caches [kv_heads][cache_stride][hd]
 * holding positions [0, pos0 + n).  Query i sees positions [0, pos0 + i].  The
 * tensor-core kernel the engine's prefill runs. */
int cuq_attention_prefill(float *out_dev, const float *q_dev, const uint16_t *k_dev, const uint16_t *v_dev,
                          uint32_t n, uint32_t pos0, uint32_t cache_stride, uint32_t heads, uint32_t kv_heads,
                          uint32_t hd, void *stream);
/* cuq_attention_decode without any allocation.  No counterpart in the
 * reference: it exists for callers that may not allocate device memory while
 * they run (an engine that reserved all device memory up front, or a loop that
 * cannot afford an allocator call between steps).  Its split scratch lives in a
 * fixed 1 MiB array inside the library (262,144 floats, held on every GPU that
 * loads the library until exit); calls whose heads * (hd + 2) exceeds that are
 * rejected with CUQ_EINVAL.  The first call on each device looks the array's
 * device address up (cudaGetSymbolAddress), so make that first call before any
 * stream capture; the first call after the host application reset the device
 * (cudaDeviceReset) looks it up again.  All calls share the one array: calls
 * that overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller. */
int cuq_attention_decode_noalloc(float *out_dev, const float *q_dev, const uint16_t *k_dev,
                                 const uint16_t *v_dev, uint32_t n_past, uint32_t cache_stride,
                                 uint32_t heads, uint32_t kv_heads, uint32_t hd, void *stream);
/* cpu.argmax (cpu.zig:477-483): first index of the maximum, written to *out_dev (u32). */
int cuq_argmax(const float *v_dev, uint32_t n, uint32_t *out_dev, void *stream);

/* cpu.SamplerParams (cpu.zig:502-518), field for field.  The reference's
 * defaults: temperature 1, top_k 0 (off), top_p 1 (off), repetition_penalty 1,
 * presence/frequency 0, min_keep_delta 20; Session.generate's default sampler
 * is temperature 0.7, top_k 40 (generate.zig:36-43). */
typedef struct {
    float temperature;         /* <= 0: greedy (after the penalties) */
    uint32_t top_k;            /* 0: off */
    float top_p;               /* 1: off; <= 0 is treated as 1 */
    float repetition_penalty;  /* 1: off; <= 0 is treated as 1 */
    float presence_penalty;
    float frequency_penalty;
    float min_keep_delta;      /* logits below max - delta * temperature are never drawn */
} cuq_sampler_params;
#define CUQ_SAMPLE_MAX_VOCAB 327680u  /* logits one draw holds on chip */
#define CUQ_SAMPLE_MAX_WINDOW 8192u   /* penalty window ids */
/* cpu.sampleProfiled (cpu.zig:621-721) with cpu.applyPenalties (cpu.zig:529-547)
 * on the device: logits_dev [vocab] f32 is penalised in place, like the
 * reference's slice; recent_dev holds the n_recent window ids; rng_dev is the
 * LCG state (u32, advanced only when a draw happens, as the reference's *rng);
 * the token goes to *token_dev.  One cluster of 8 CTAs.  params is host
 * memory, read at the call. */
int cuq_sample(float *logits_dev, uint32_t vocab, const cuq_sampler_params *params, const uint32_t *recent_dev,
               uint32_t n_recent, uint32_t *rng_dev, uint32_t *token_dev, void *stream);

/* ------------------------------------------------------------ engine ---- */

/* Model geometry: the fields of model.Config (model.zig:10-244) this path uses. */
typedef struct {
    uint32_t hidden, layers, heads, kv_heads, head_dim, inter, vocab;
    float eps, rope_theta;
    int32_t rope_adjacent;   /* load_gguf.zig:81-90: llama -> 1, qwen2 -> 0 */
    int32_t tie_embeddings;  /* no output.weight: lm_head reads token_embd (load_gguf.zig:141) */
} cuq_config;

/* Engine options (engine.zig:28-51 Options, plus device-side knobs). */
typedef struct {
    uint32_t max_seq;        /* KV-cache positions (engine.zig:447-458); default 2048 */
    uint32_t max_chunk;      /* largest prefill chunk; default 512 */
    int32_t use_graphs;      /* capture the decode step in a CUDA graph (default 1) */
    int32_t tp_rank, tp_size;/* tensor parallel slot (tp_size 1 = single GPU; up to 8, one
                              * process per GPU; see cuq_tp_connect) */
    int32_t decode_kernel;   /* CUQ_DECODE_*: how decode steps run (default AUTO) */
    int32_t persistent_ctas; /* CTAs per SM of the persistent decode kernel; 0 = as many as fit */
    uint32_t wait_limit_ms;  /* tensor parallel: a wait for the peers gives up after this long
                              * (CUQ_ETIMEOUT); 0 = 10 s */
} cuq_options;

/* decode_kernel: PER_OP (and AUTO, the default) runs one kernel per op,
 * captured in a CUDA graph when use_graphs; PERSISTENT runs every decode step
 * of a call in one persistent cooperative kernel with grid-wide barriers
 * between the phases (single GPU, gate/up of one type, hidden <= 8192;
 * cuq_model_finalize fails when the model does not allow it).  On B200 the
 * per-op path with programmatic dependent launch is the faster of the two for
 * benchmark models (SmolLM2-135M to Llama-3-8B), so AUTO picks it. */
#define CUQ_DECODE_AUTO 0
#define CUQ_DECODE_PER_OP 1
#define CUQ_DECODE_PERSISTENT 2

/* Tensor roles for cuq_upload_*. */
#define CUQ_ROLE_Q 0
#define CUQ_ROLE_K 1
#define CUQ_ROLE_V 2
#define CUQ_ROLE_O 3
#define CUQ_ROLE_GATE 4
#define CUQ_ROLE_UP 5
#define CUQ_ROLE_DOWN 6
#define CUQ_ROLE_ATTN_NORM 7
#define CUQ_ROLE_FFN_NORM 8
#define CUQ_ROLE_Q_BIAS 9
#define CUQ_ROLE_K_BIAS 10
#define CUQ_ROLE_V_BIAS 11
#define CUQ_ROLE_O_BIAS 12
#define CUQ_ROLE_EMBED 13
#define CUQ_ROLE_OUTPUT 14
#define CUQ_ROLE_FINAL_NORM 15

typedef struct cuq_model cuq_model;

/* Per-call statistics (engine.zig:83-131 Stats): device time per node class. */
typedef struct {
    uint64_t tokens;           /* decode steps run */
    uint64_t prefill_tokens;   /* prompt tokens prefilled */
    double decode_ms;          /* device time in decode steps */
    double prefill_ms;         /* device time in prefill */
    uint64_t weight_bytes;     /* quantized weight bytes resident */
    uint64_t kv_bytes;         /* KV-cache bytes */
    uint64_t graph_replays;
    uint64_t kernels_per_step; /* kernel launches in one decode step */
    uint64_t kernel_launches;  /* all kernels this model has launched (graph nodes counted) */
    uint64_t persistent_ctas;  /* CTAs of the persistent decode kernel; 0 when decode runs per op */
} cuq_stats;

/* Engine.init (engine.zig:320-521) without weights: allocates the KV cache and
 * activation buffers.  NULL on failure. */
cuq_model *cuq_model_create(const cuq_config *cfg, const cuq_options *opts);
/* Upload one tensor's raw GGUF payload (load_gguf.loadLayer, load_gguf.zig:650-713,
 * minus the fp16 expansion).  `layer` is ignored for EMBED/OUTPUT.  Copied; the
 * caller keeps ownership of raw_host (e.g. its mmap). */
int cuq_upload_tensor(cuq_model *m, int layer, int role, int ggml_type, const void *raw_host,
                      size_t nbytes, uint32_t rows, uint32_t cols);
/* Norm weights and biases (float32, host). */
int cuq_upload_f32(cuq_model *m, int layer, int role, const float *v_host, size_t n);
/* Check every tensor is present and build the device-resident step. */
int cuq_model_finalize(cuq_model *m);
/* Parse a GGUF v2/v3 file (gguf.zig:328-656), read its config (load_gguf.loadConfig,
 * load_gguf.zig:96-302) and upload every tensor raw.  Returns a finalized model,
 * except with opts->tp_size > 1: then the caller runs cuq_tp_connect and
 * cuq_model_finalize. */
cuq_model *cuq_model_load_gguf(const char *path, const cuq_options *opts);

/* ----------------------------------------------------- GGUF container --- */
/* The file format the loader reads, as gguf.zig's Gguf exposes it (host only,
 * no GPU needed).  Open errors (cuq_last_error): NotGgufFile,
 * UnsupportedVersion, TruncatedFile, TooManyTensors, TooManyMetadataEntries,
 * InvalidMetadata, InvalidTensorShape (gguf.zig:589-656). */
typedef struct cuq_gguf cuq_gguf;
cuq_gguf *cuq_gguf_open(const char *path);                  /* Gguf.load: maps the file */
cuq_gguf *cuq_gguf_open_bytes(const void *data, size_t n);  /* Gguf.fromBytes: parses a copy */
void cuq_gguf_close(cuq_gguf *g);
uint32_t cuq_gguf_version(const cuq_gguf *g);
uint64_t cuq_gguf_tensor_count(const cuq_gguf *g);
/* Metadata (gguf.zig:198-291): the value type id of `key` (0-12) or -1 when
 * absent; integer, float and bool values converted as the reference's
 * asU64 / asI64 / asF32 do (CUQ_EINVAL when absent or not convertible). */
int cuq_gguf_kv_type(const cuq_gguf *g, const char *key);
int cuq_gguf_get_u64(const cuq_gguf *g, const char *key, uint64_t *out);
int cuq_gguf_get_i64(const cuq_gguf *g, const char *key, int64_t *out);
int cuq_gguf_get_f64(const cuq_gguf *g, const char *key, double *out);
const char *cuq_gguf_get_string(const cuq_gguf *g, const char *key);  /* NULL unless a string */
int cuq_gguf_array_info(const cuq_gguf *g, const char *key, uint64_t *len, int *elem_type);
int cuq_gguf_array_u64(const cuq_gguf *g, const char *key, uint64_t i, uint64_t *out);
const char *cuq_gguf_array_string(const cuq_gguf *g, const char *key, uint64_t i);
/* Tensor table: type, dims in ggml order (dims[0] = row length; up to 8) and
 * offset inside the data section; CUQ_EINVAL (TensorNotFound) when absent. */
int cuq_gguf_tensor_info(const cuq_gguf *g, const char *name, int *ggml_type, uint32_t *n_dims, uint64_t *dims,
                         uint64_t *offset);
/* Gguf.tensorBytes (gguf.zig:448-460): the tensor's payload inside the file
 * (valid until cuq_gguf_close).  CUQ_EUNSUPPORTED (UnsupportedType),
 * CUQ_EINVAL (InvalidTensorShape, TensorNotFound), CUQ_EFORMAT
 * (TensorDataOutOfRange). */
int cuq_gguf_tensor_bytes(const cuq_gguf *g, const char *name, const void **data, size_t *nbytes);

/* ------------------------------------------- HuggingFace directories --- */
/* safetensors files (safetensors.zig): open errors HeaderTooSmall,
 * InvalidHeaderLength, InvalidHeader, InvalidTensorEntry, UnsupportedDtype,
 * DataSizeMismatch (safetensors.zig:104-121).  Host only. */
typedef struct cuq_safetensors cuq_safetensors;
cuq_safetensors *cuq_safetensors_open(const char *path);
cuq_safetensors *cuq_safetensors_open_bytes(const void *data, size_t n);
void cuq_safetensors_close(cuq_safetensors *s);
uint64_t cuq_safetensors_count(const cuq_safetensors *s);                /* tensors, __metadata__ excluded */
const char *cuq_safetensors_name(const cuq_safetensors *s, uint64_t i);   /* in header order */
/* dtype_out: 8 bytes ("F16", "BF16", ...), shape: up to 8 dims; data valid until close. */
int cuq_safetensors_tensor(const cuq_safetensors *s, const char *name, char *dtype_out, uint32_t *rank,
                           uint64_t *shape, const void **data, size_t *nbytes);
/* config.json of a model directory (hf.zig Config -> load_hf.zig toModelConfig):
 * hidden_size, num_hidden_layers, num_attention_heads, num_key_value_heads,
 * head_dim, intermediate_size, vocab_size, rms_norm_eps, rope_theta,
 * tie_word_embeddings; rope_adjacent is 0 (HF's half-split RoPE).  Host only. */
int cuq_hf_read_config(const char *dir, cuq_config *out);
/* load_hf.zig (loadRuntime / loadLayer / loadHead, load_hf.zig:143-230): a
 * model directory (config.json + model*.safetensors shards, or the files of
 * model.safetensors.index.json) uploaded raw: F16 / BF16 / F32 weights as on
 * disk, norms and biases as f32; the head is tied when lm_head.weight is
 * absent.  Returns a finalized model, except with opts->tp_size > 1 (as
 * cuq_model_load_gguf). */
cuq_model *cuq_model_load_hf(const char *dir, const cuq_options *opts);

/* Tensor parallelism (Megatron split, used for the Llama-3-8B shape; the reference engine
 * is single-device, so these have no counterpart there).  One process per GPU,
 * each creating its model with the same config and tp_size and its own tp_rank,
 * uploading the FULL tensors (each rank keeps its shard: q/k/v/gate/up and the
 * lm_head by rows, o/down by whole-block columns; embeddings and norms are
 * replicated).  Before cuq_model_finalize every rank publishes its
 * communication buffer's handle (CUQ_TP_HANDLE_BYTES opaque bytes) and passes
 * all ranks' handles, in rank order, to cuq_tp_connect.  The ranks then exchange
 * partial sums over NVLink inside the step's kernels (no library collective);
 * every rank must make the same calls with the same arguments, in the same
 * order.  A handle of CUQ_TP_HANDLE_BYTES zero bytes stands for a rank that
 * never joins (fault tests on one GPU): every exchange then waits for it until
 * options.wait_limit_ms and the call returns CUQ_ETIMEOUT.  cuq_reset clears
 * this rank's arrival counters, so that after a time-out every rank can reset
 * and carry on.  cuq_forward/cuq_prefill return this rank's slice of the logits
 * (vocab / tp_size values starting at token id tp_rank * vocab / tp_size); the
 * argmax and generated tokens are global.  A peer that does not arrive within
 * options.wait_limit_ms (10 s by default) ends the call with CUQ_ETIMEOUT. */
#define CUQ_TP_HANDLE_BYTES 64
int cuq_tp_comm_handle(cuq_model *m, void *handle_out);
int cuq_tp_connect(cuq_model *m, const void *handles);
/* Host-only helpers (no GPU needed): copy rows [r0, r1), or whole-block columns
 * [c0, c1) of every row, of a raw [rows][cols] GGUF tensor into out. */
int cuq_shard_rows(int ggml_type, uint32_t rows, uint32_t cols, uint32_t r0, uint32_t r1,
                   const void *raw, void *out);
int cuq_shard_cols(int ggml_type, uint32_t rows, uint32_t cols, uint32_t c0, uint32_t c1,
                   const void *raw, void *out);
int cuq_model_get_config(const cuq_model *m, cuq_config *out);

/* Engine.forward (engine.zig:547-819): one decode step for `token` at `pos`.
 * logits_host (vocab floats) may be NULL; argmax_out (host u32) may be NULL. */
int cuq_forward(cuq_model *m, uint32_t token, uint32_t pos, float *logits_host, uint32_t *argmax_out);
/* Engine.prefill (engine.zig:975-1329): run `n` prompt ids starting at start_pos;
 * logits/argmax of the LAST token (engine.zig:1310-1316). */
int cuq_prefill(cuq_model *m, const uint32_t *ids, uint32_t n, uint32_t start_pos,
                float *logits_host, uint32_t *argmax_out);
/* Session.generate (generate.zig:166-250) for greedy decoding: prefill `ids`, then
 * `n_decode` steps entirely on the device (the argmax feeds the next step with
 * no host round-trip).  out_tokens (host, n_decode u32) gets the generated ids. */
int cuq_generate(cuq_model *m, const uint32_t *ids, uint32_t n_prompt, uint32_t n_decode,
                 uint32_t *out_tokens);
/* Session.generate (generate.zig:166-250) with its Params: prefill the prompt
 * `ids`, then draw `n_decode` tokens with `params`, the LCG seeded with `seed`
 * (generate.zig:169) and the penalties looking at the last `penalty_window`
 * ids of prompt and output (generate.zig:205-211, 231-233; at most
 * CUQ_SAMPLE_MAX_WINDOW).  Positions [0, n_cached) of the KV cache already
 * hold ids[0..n_cached) (a session's reused prefix, generate.zig:187-192;
 * 0 = none): only ids[n_cached..n_prompt) are prefilled.  Every draw runs on
 * the device right after its step's lm_head (cuq_sample's kernel, reading the
 * parameters, the LCG state and the window from device memory), so the loop
 * stays on the device.  With temperature <= 0 and no penalty the step's own
 * argmax is used, as in cuq_generate.  Drawing needs a single GPU
 * (CUQ_EUNSUPPORTED under tensor parallelism) and vocab <= CUQ_SAMPLE_MAX_VOCAB. */
int cuq_generate_sampled(cuq_model *m, const uint32_t *ids, uint32_t n_prompt, uint32_t n_cached, uint32_t n_decode,
                         const cuq_sampler_params *params, uint32_t seed, uint32_t penalty_window,
                         uint32_t *out_tokens);
/* Decode `n_steps` greedy tokens from the device-resident state left by a
 * prefill/forward at position `pos` with next token `token` (no prefill). */
int cuq_decode_greedy(cuq_model *m, uint32_t token, uint32_t pos, uint32_t n_steps,
                      uint32_t *out_tokens);
/* The fp16 KV cache of one layer, rows [pos0, pos0 + n) in the reference's
 * layout (engine.zig:447-458, 966-969: row p holds kv_heads * head_dim halves,
 * KV head major), host memory.  cuq_kv_write replaces the rows (a session
 * restored from elsewhere, or a cache shared with another engine); cuq_kv_read
 * copies them out.  Under tensor parallelism the rows are full width and each
 * rank reads / writes its own KV heads (cuq_kv_read leaves the other heads'
 * columns untouched).  Both synchronise the model's stream. */
int cuq_kv_write(cuq_model *m, uint32_t layer, uint32_t pos0, uint32_t n, const uint16_t *k_host,
                 const uint16_t *v_host);
int cuq_kv_read(const cuq_model *m, uint32_t layer, uint32_t pos0, uint32_t n, uint16_t *k_host,
                uint16_t *v_host);
/* Engine.reset (engine.zig:1479): forget the KV cache. */
int cuq_reset(cuq_model *m);
int cuq_model_stats(const cuq_model *m, cuq_stats *out);
/* Per-kernel decode timing, in the shape of the reference's `anedvd kernels`
 * table (main.zig:1729-1791) and its per-node counters (engine.zig:83-131
 * Stats.node_ns): `n_steps` decode steps from (`token`, `pos`) are enqueued one
 * launch at a time (no CUDA graph) with a CUDA event recorded on the model's
 * stream after every launch, and each launch's time (event to event: the
 * kernel plus its launch gap, with no overlap between consecutive kernels) is
 * added to its node.  `bytes` is the node's algorithmic traffic over the steps:
 * weight bytes as stored (this rank's shard), plus the fp16 K/V rows the
 * attention reads.  The KV cache and decode state advance as in cuq_forward;
 * under tensor parallelism every rank makes the call together.  Per-op decode
 * only (CUQ_EUNSUPPORTED with the persistent decode kernel). */
#define CUQ_NODE_EMBED 0    /* embedding row */
#define CUQ_NODE_QKV 1      /* q||k||v projection (+ its RMSNorm) */
#define CUQ_NODE_ATTN 2     /* RoPE + KV write + attention */
#define CUQ_NODE_O 3        /* o projection + residual */
#define CUQ_NODE_GATE_UP 4  /* gate|up projections + SiLU*mul (+ RMSNorm) */
#define CUQ_NODE_DOWN 5     /* down projection + residual */
#define CUQ_NODE_HEAD 6     /* final RMSNorm + lm_head + argmax */
#define CUQ_NODE_NORM 7     /* RMSNorms launched as kernels of their own */
#define CUQ_NODES 8
typedef struct {
    uint64_t launches;  /* kernel launches of this node over the steps */
    double ms;          /* summed launch times */
    double bytes;       /* algorithmic bytes over the steps */
} cuq_node_time;
int cuq_profile_decode(cuq_model *m, uint32_t token, uint32_t pos, uint32_t n_steps, cuq_node_time *out);
/* The stream the model enqueues on (cudaStream_t as void*). */
void *cuq_model_stream(const cuq_model *m);
void cuq_model_free(cuq_model *m);

#ifdef __cplusplus
}
#endif
#endif /* CUQ_H */
