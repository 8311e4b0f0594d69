// model.cu -- the engine: Engine.init / forward / prefill / reset (src/engine.zig)
// and Session.generate's greedy loop (src/generate.zig:166-250), device-resident.
//
// A decode step is one fixed launch sequence (captured once in a CUDA graph),
// 2 + 5 launches per layer:
//   embed row + RMSNorm -> per layer [qkv GEMV (+bias);
//   attention (RoPE, fp16 KV write, split softmax, combine -> xq);
//   o GEMV (+= residual, last CTA: ffn RMSNorm -> xq);
//   gate|up GEMV with the SiLU*mul epilogue -> xq;
//   down GEMV (+= residual, last CTA: next RMSNorm -> xq)] ->
//   lm_head GEMV with the fused argmax (last CTA: next token).
// Every launch is a programmatic dependent of the one before: a GEMV starts
// streaming its weights while its predecessor finishes, then waits for the
// activation (griddepcontrol.wait).  The step reads its token and position from
// device memory and writes the next ones, so consecutive steps (a prompt fed
// token by token, then greedy decoding) replay the graph with no host round-trip.
#include <algorithm>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <string>

#include "model.h"
#include "ops.cuh"
#include "qgemm.cuh"
#include "tp.cuh"

using namespace cuq;

namespace cuq {
int sm_count_current();
}

namespace {

enum { R_Q = 0, R_K, R_V, R_O, R_GATE, R_UP, R_DOWN };

uint32_t q_dim(const cuq_config &c) { return c.heads * c.head_dim; }
size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }
uint32_t kv_dim(const cuq_config &c) { return c.kv_heads * c.head_dim; }

void free_pending(PendingTensor &t) {
    if (t.raw) cudaFree(t.raw);
    t = PendingTensor();
}

void free_planes(Planes &p) {
    if (p.base) cudaFree(p.base);
    p.base = nullptr;
}

// Repack one or more same-typed pending tensors (concatenated by rows) into planes.
int build_proj(Proj &out, std::vector<PendingTensor *> parts, cudaStream_t s) {
    int type = parts[0]->type;
    uint32_t cols = parts[0]->cols, rows = 0;
    size_t nbytes = 0;
    for (auto *t : parts) {
        rows += t->rows;
        nbytes += t->nbytes;
    }
    out.p = Planes();
    out.p.type = type;
    out.p.rows = rows;
    out.p.cols = cols;
    if (!plan_planes(out.p)) {
        set_error("UnsupportedType: ggml type %d has no GEMV here", type);
        return CUQ_EUNSUPPORTED;
    }
    CUQ_CUDA_TRY(cudaMalloc(&out.p.base, out.p.nbytes));
    uint8_t *cat = parts[0]->raw;
    bool own = false;
    if (parts.size() > 1) {
        CUQ_CUDA_TRY(cudaMalloc(&cat, nbytes));
        own = true;
        size_t off = 0;
        for (auto *t : parts) {
            CUQ_CUDA_TRY(cudaMemcpyAsync(cat + off, t->raw, t->nbytes, cudaMemcpyDeviceToDevice, s));
            off += t->nbytes;
        }
    }
    int rc = launch_repack(cat, out.p, s);
    cudaStreamSynchronize(s);
    if (own) cudaFree(cat);
    return rc;
}

}  // namespace

// The lm_head weight: the embedding table when tied on one GPU, else `output`
// (the untied head, or this rank's rows of the tied table).
// The lm_head GEMV runs the register-prefetch kernel: its grid is many waves
// long, so the TMA kernel's early weight requests buy little, and timed in the
// c5 decode step it is 1.5 % faster there (272 against 268 tok/s).
// CUQ_HEAD_TMA=1 puts it on the TMA-fed kernel when the other GEMVs use it.
static bool head_tma(const cuq_model *m) {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("CUQ_HEAD_TMA");
        v = e ? (atoi(e) != 0) : 0;
    }
    return m->use_tma && v;
}

static const Proj &head_proj(const cuq_model *m) {
    return (m->cfg.tie_embeddings && m->opt.tp_size == 1) ? m->embed : m->output;
}

// o / down projection output: on one GPU added into the residual with the next
// RMSNorm as post-op; under tensor parallelism pushed to every rank and reduced
// (+ bias, + residual, RMSNorm) by the post-op.
static void residual_out(cuq_model *m, GemvArgs &a, int &epi, const float *bias, const float *next_norm, int phase) {
    const cuq_config &c = m->cfg;
    a.post.x = m->x;
    a.post.w = next_norm;
    a.post.n = c.hidden;
    a.post.eps = c.eps;
    a.post.xq = m->xq_h;
    if (m->opt.tp_size > 1) {
        epi = EPI_TP_PUSH;
        a.y = nullptr;
        a.bias = nullptr;
        a.post.op = POST_TP_REDUCE;
        a.post.tp = m->tpc;
        a.post.tp_phase = phase;
        a.post.xr = m->x;
        a.post.bias = bias;
    } else {
        epi = EPI_ADD;
        a.y = m->x;
        a.bias = bias;
        a.post.op = POST_RMSNORM;
    }
}

// cuq_profile_decode: record the next event of the pool after a launch, tagged
// with the node being enqueued.
static int prof_mark(cuq_model *m) {
    if (m->prof_n >= m->prof_ev.size()) {
        cudaEvent_t e;
        CUQ_CUDA_TRY(cudaEventCreate(&e));
        m->prof_ev.push_back(e);
        m->prof_tag.push_back(0);
    }
    m->prof_tag[m->prof_n] = m->prof_node;
    CUQ_CUDA_TRY(cudaEventRecord(m->prof_ev[m->prof_n], m->stream));
    m->prof_n++;
    return CUQ_OK;
}

static int enqueue_step(cuq_model *m) {
    const cuq_config &c = m->cfg, &lc = m->lc;
    cudaStream_t s = m->stream;
    const bool pdl = true;  // every launch below waits for its predecessor with griddepcontrol.wait
    int rc;
    uint64_t nk = 0;  // kernel launches in the step
#define TRY(x)                                \
    do {                                      \
        rc = (x);                             \
        if (rc != CUQ_OK) return rc;          \
        nk++;                                 \
        if (m->profiling) {                   \
            if ((rc = prof_mark(m))) return rc; \
        }                                     \
    } while (0)
    auto gemv = [&](const Planes &w, const __half *xq, float *y, const float *bias) {
        GemvArgs a;
        a.w = &w;
        a.xq = xq;
        a.y = y;
        a.bias = bias;
        a.ws = m->ws;
        a.counters = m->counters;
        a.tma = m->use_tma;
        a.ksplit = gemv_pick_ksplit(w, m->sm_count, 1, m->use_tma);
        a.pdl = pdl;
        a.err = m->gemm_err;
        a.post.done = m->done;
        return a;
    };
    // Single GPU with register-prefetch GEMVs: each RMSNorm is computed by every
    // CTA of the GEMV that reads it (pre-norm), after its first weight loads are
    // in flight, instead of by the last CTA of the GEMV that wrote the residual.
    const bool pre = m->opt.tp_size == 1 && c.hidden % 16 == 0 && c.hidden <= RN_MAX && !m->all_tma;
    // TMA-fed GEMVs request all their weights at launch, before the activation
    // exists.  There the GEMV that updates the residual (o, down) also writes the
    // sum of squares of each 16-row tile it produced, and every CTA of the
    // consumer normalises only its own K range with the mean square summed from
    // those partials: no norm kernel, no serial tail.  ss[0]: after o, ss[1]:
    // after down.
    const bool tnorm = m->opt.tp_size == 1 && m->all_tma;
    auto prenorm = [&](GemvArgs &a, const float *w, const float *ss) {
        if (!pre && !(tnorm && ss)) return;
        a.pre_x = m->x;
        a.pre_w = w;
        a.pre_n = c.hidden;
        a.pre_eps = c.eps;
        if (tnorm) a.ss_in = ss;
    };
    float *const ss_o = m->ss, *const ss_down = m->ss + c.hidden / 16;
    // engine.zig:561-564 embedding (then layer 0's attention RMSNorm)
    m->prof_node = CUQ_NODE_EMBED;
    if (pre)
        TRY(launch_embed_row(m->embed.p, &m->state->token, m->x, s));
    else
        TRY(launch_embed_norm(m->embed.p, m->state, m->x, m->layers[0].attn_norm, c.hidden, c.eps, m->xq_h, pdl, s));
    for (uint32_t l = 0; l < c.layers; l++) {
        Layer &L = m->layers[l];
        // qkv projection + bias (main.zig:435-436)
        m->prof_node = CUQ_NODE_QKV;
        for (auto &seg : L.qkv) {
            GemvArgs a = gemv(seg.p, m->xq_h, m->qkv + seg.row_off, L.qkv_bias ? L.qkv_bias + seg.row_off : nullptr);
            prenorm(a, L.attn_norm, l > 0 ? ss_down : nullptr);  // layer 0: the embedding kernel's xq
            TRY(launch_gemv(a, EPI_STORE, s));
        }
        // RoPE + fp16 KV write + attention (main.zig:457-472), this rank's heads
        m->prof_node = CUQ_NODE_ATTN;
        TRY(launch_attention_step(m->qkv, m->rope_cs, m->state, L.k_cache, L.v_cache, m->opt.max_seq, lc.heads,
                                  lc.kv_heads, c.head_dim, c.rope_adjacent, m->attn_part, m->attn_nsplit, m->tickets,
                                  m->xq_attn, pdl, s));
        // o projection + o_bias into the residual (main.zig:477-485), then ffn RMSNorm (main.zig:487)
        m->prof_node = CUQ_NODE_O;
        {
            GemvArgs a = gemv(L.o.p, m->xq_attn, nullptr, nullptr);
            int epi;
            residual_out(m, a, epi, L.o_bias, L.ffn_norm, 0);
            if (pre || tnorm) a.post.op = POST_NONE;
            if (tnorm) a.ss_out = ss_o;  // for the ffn RMSNorm (main.zig:487) in gate|up
            TRY(launch_gemv(a, epi, s));
        }
        // gate/up with the SiLU*mul epilogue (engine.zig:645-668 split path)
        m->prof_node = CUQ_NODE_GATE_UP;
        if (L.gate_up_dual) {
            GemvArgs a = gemv(L.gate.p, m->xq_h, nullptr, nullptr);
            a.ksplit = gemv_pick_ksplit(L.gate.p, m->sm_count, 2, m->use_tma);
            a.w2 = &L.up.p;
            a.xq_out = m->xq_act;
            prenorm(a, L.ffn_norm, ss_o);
            TRY(launch_gemv(a, EPI_SILU_XQ, s));
        } else {
            GemvArgs a = gemv(L.gate.p, m->xq_h, m->gate_buf, nullptr);
            prenorm(a, L.ffn_norm, ss_o);
            TRY(launch_gemv(a, EPI_STORE, s));
            a = gemv(L.up.p, m->xq_h, m->up_buf, nullptr);
            prenorm(a, L.ffn_norm, ss_o);
            TRY(launch_gemv(a, EPI_STORE, s));
            TRY(launch_silu_mul(m->act, m->gate_buf, m->up_buf, lc.inter, s));
            TRY(launch_to_xq(m->act, lc.inter, 1, lc.inter, m->xq_act, s));
        }
        // down projection into the residual, then the next RMSNorm (next layer's
        // attention norm, or the final norm before the lm_head, main.zig:532)
        m->prof_node = CUQ_NODE_DOWN;
        {
            GemvArgs a = gemv(L.down.p, m->xq_act, nullptr, nullptr);
            int epi;
            const float *next_norm = l + 1 < c.layers ? m->layers[l + 1].attn_norm : m->final_norm;
            residual_out(m, a, epi, nullptr, next_norm, 1);
            if (pre || tnorm) a.post.op = POST_NONE;
            if (tnorm) a.ss_out = ss_down;  // for the next attention RMSNorm or the final norm
            TRY(launch_gemv(a, epi, s));
        }
    }
    // lm_head with the fused argmax (main.zig:534, cpu.zig:477-483); the last CTA
    // turns the argmax into the next step's token (generate.zig:217-244), after
    // the cross-rank argmax under tensor parallelism.
    m->prof_node = CUQ_NODE_HEAD;
    {
        // the final RMSNorm (main.zig:532): the lm_head's many waves of CTAs
        // would each repeat a per-CTA norm, so it runs once, as its own kernel
        if (tnorm) {
            m->prof_node = CUQ_NODE_NORM;
            TRY(launch_rmsnorm_xq_pdl(m->x, m->final_norm, c.hidden, c.eps, m->xq_h, s));
            m->prof_node = CUQ_NODE_HEAD;
        }
        GemvArgs a = gemv(head_proj(m).p, m->xq_h, m->logits, nullptr);
        a.tma = head_tma(m);
        a.ksplit = gemv_pick_ksplit(head_proj(m).p, m->sm_count, 1, a.tma);
        prenorm(a, m->final_norm, nullptr);
        a.argmax64 = &m->state->argmax64;
        a.row_base = m->vocab_base;
        a.post.op = m->opt.tp_size > 1 ? POST_TP_FINISH : POST_FINISH;
        a.post.tp = m->tpc;
        a.post.state = m->state;
        a.post.forced = m->forced;
        a.post.out_tokens = m->out_tokens;
        TRY(launch_gemv(a, EPI_ARGMAX, s));
    }
    m->stats.kernels_per_step = nk;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cap);
    if (cap == cudaStreamCaptureStatusNone) m->stats.kernel_launches += nk;
#undef TRY
    return CUQ_OK;
}

static int run_steps(cuq_model *m, uint32_t n) {
    if (m->mega.impl) {
        if (n == 0) return CUQ_OK;
        int rc = mega_launch(m->mega, n, m->stream);
        if (rc) return rc;
        m->mega_ran = true;
        m->stats.kernel_launches += 1;
        return CUQ_OK;
    }
    for (uint32_t i = 0; i < n; i++) {
        if (m->graph_exec) {
            CUQ_CUDA_TRY(cudaGraphLaunch(m->graph_exec, m->stream));
            m->stats.graph_replays++;
            m->stats.kernel_launches += m->stats.kernels_per_step;
        } else {
            int rc = enqueue_step(m);
            if (rc) return rc;
        }
    }
    return CUQ_OK;
}

// A draw right after the step's lm_head: replaces the step's greedy token
// (out_tokens[step], the next token) with one sampled from the logits with the
// call's parameters, LCG state and window, all read from device memory.
static int enqueue_sample(cuq_model *m) {
    SampleArgs a;
    a.logits = m->logits;
    a.vocab = m->lc.vocab;
    a.prm = &m->smp->prm;
    a.rng = &m->smp->rng;
    a.st = m->state;
    a.out_tokens = m->out_tokens;
    a.ring = &m->smp->ring;
    a.ring_ids = m->smp->ids;
    return launch_sample(a, true, m->stream);
}

// n sampled decode steps: the decode step and its draw, replayed as one CUDA
// graph (captured at the first sampled call) when the model uses graphs.
static int run_steps_sampled(cuq_model *m, uint32_t n) {
    if (n == 0) return CUQ_OK;
    if (m->opt.use_graphs && !m->graph_exec_smp) {
        CUQ_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_step(m);
        if (rc == CUQ_OK) rc = enqueue_sample(m);
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (rc != CUQ_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) {
            set_error("graph capture: %s", cudaGetErrorString(e));
            return CUQ_ECUDA;
        }
        m->graph_smp = g;
        CUQ_CUDA_TRY(cudaGraphInstantiate(&m->graph_exec_smp, g, 0));
    }
    for (uint32_t i = 0; i < n; i++) {
        if (m->graph_exec_smp) {
            CUQ_CUDA_TRY(cudaGraphLaunch(m->graph_exec_smp, m->stream));
            m->stats.graph_replays++;
            m->stats.kernel_launches += m->stats.kernels_per_step + 1;
        } else {
            int rc = enqueue_step(m);
            if (rc == CUQ_OK) rc = enqueue_sample(m);
            if (rc) return rc;
            m->stats.kernel_launches += 1;
        }
    }
    return CUQ_OK;
}

// The lm_head over the residual row `x_row` (final RMSNorm first), with the
// argmax and the step-finish post-op (main.zig:532-534, generate.zig:217-244).
static int enqueue_head(cuq_model *m, const float *x_row, bool pdl) {
    const cuq_config &c = m->cfg;
    int rc = launch_rmsnorm_xq(x_row, m->final_norm, c.hidden, 1, c.eps, m->xq_h, nullptr, m->stream);
    if (rc) return rc;
    const Proj &head = head_proj(m);
    GemvArgs a;
    a.w = &head.p;
    a.xq = m->xq_h;
    a.y = m->logits;
    a.argmax64 = &m->state->argmax64;
    a.row_base = m->vocab_base;
    a.ws = m->ws;
    a.counters = m->counters;
    a.tma = head_tma(m);
    a.ksplit = gemv_pick_ksplit(head.p, m->sm_count, 1, a.tma);
    a.pdl = pdl;
    a.err = m->gemm_err;
    a.post.done = m->done;
    a.post.op = m->opt.tp_size > 1 ? POST_TP_FINISH : POST_FINISH;
    a.post.tp = m->tpc;
    a.post.state = m->state;
    a.post.forced = m->forced;
    a.post.out_tokens = m->out_tokens;
    return launch_gemv(a, EPI_ARGMAX, m->stream);
}

// Row-parallel projection output of a prefill chunk under tensor parallelism:
// the partial [n][hidden] goes to every rank, then x += sum + bias.
static int prefill_allreduce(cuq_model *m, uint32_t n, const float *bias, int phase) {
    const size_t count = (size_t)n * m->cfg.hidden;
    int grid = 0;
    int rc = launch_tp_push(m->tpc, phase, m->pf_part, count, &grid, m->stream);
    if (rc) return rc;
    return launch_tp_reduce_add(m->tpc, phase, (unsigned)(m->tpc.size * grid), m->pf_x, bias, m->cfg.hidden, count,
                                m->tp_done, m->stream);
}

// Engine.prefill for one chunk of n <= max_chunk prompt positions starting at
// pos0 (ids already on the device): every projection is one tensor-core GEMM
// over the chunk, attention is causal over the cache.  When `last` is set the
// chunk's final position goes through the lm_head and sets the decode state.
static int prefill_chunk(cuq_model *m, const uint32_t *ids_dev, uint32_t n, uint32_t pos0, bool last) {
    const cuq_config &c = m->cfg, &lc = m->lc;
    const bool tp = m->opt.tp_size > 1;
    cudaStream_t s = m->stream;
    const uint32_t qd = q_dim(lc), kvd = kv_dim(lc), qkvd = qd + 2 * kvd;
    int rc;
#define PTRY(x)                      \
    do {                             \
        rc = (x);                    \
        if (rc != CUQ_OK) return rc; \
        m->stats.kernel_launches++;  \
    } while (0)
    PTRY(launch_embed_rows(m->embed.p, ids_dev, n, m->pf_x, s));
    for (uint32_t l = 0; l < c.layers; l++) {
        Layer &L = m->layers[l];
        PTRY(launch_rmsnorm_hilo(m->pf_x, L.attn_norm, c.hidden, n, c.eps, m->pf_h, m->pf_l, s));
        for (auto &seg : L.qkv) {
            QgemmArgs g;
            g.f16_scratch = m->pf_wscratch;
            g.w = &seg.p;
            g.xh = m->pf_h;
            g.xl = m->pf_l;
            g.n = n;
            g.y = m->pf_qkv + seg.row_off;
            g.ldy = qkvd;
            g.bias = L.qkv_bias ? L.qkv_bias + seg.row_off : nullptr;
            g.err = m->gemm_err;
            PTRY(launch_qgemm(g, EPI_STORE, s));
        }
        PTRY(launch_rope_cache(m->pf_qkv, qkvd, m->pf_q, L.k_cache, L.v_cache, m->opt.max_seq, m->rope_cs, nullptr,
                               pos0, n, lc.heads, lc.kv_heads, c.head_dim, c.rope_adjacent, s));
        PTRY(launch_attention_prefill(m->pf_q, L.k_cache, L.v_cache, m->opt.max_seq, pos0, n, lc.heads, lc.kv_heads,
                                      c.head_dim, m->pf_h, m->pf_l, s));
        {
            QgemmArgs g;
            g.f16_scratch = m->pf_wscratch;
            g.w = &L.o.p;
            g.xh = m->pf_h;
            g.xl = m->pf_l;
            g.n = n;
            g.y = tp ? m->pf_part : m->pf_x;
            g.ldy = c.hidden;
            g.bias = tp ? nullptr : L.o_bias;
            g.err = m->gemm_err;
            PTRY(launch_qgemm(g, tp ? EPI_STORE : EPI_ADD, s));
            if (tp) {
                PTRY(prefill_allreduce(m, n, L.o_bias, 0));
                m->stats.kernel_launches++;  // push + reduce
            }
        }
        PTRY(launch_rmsnorm_hilo(m->pf_x, L.ffn_norm, c.hidden, n, c.eps, m->pf_h, m->pf_l, s));
        if (L.gate_up_dual) {
            QgemmArgs g;
            g.f16_scratch = m->pf_wscratch;
            g.w = &L.gate.p;
            g.w2 = &L.up.p;
            g.xh = m->pf_h;
            g.xl = m->pf_l;
            g.n = n;
            g.oh = m->pf_ah;
            g.ol = m->pf_al;
            g.err = m->gemm_err;
            PTRY(launch_qgemm(g, EPI_SILU_XQ, s));
        } else {
            QgemmArgs g;
            g.f16_scratch = m->pf_wscratch;
            g.xh = m->pf_h;
            g.xl = m->pf_l;
            g.n = n;
            g.err = m->gemm_err;
            g.w = &L.gate.p;
            g.y = m->pf_g;
            PTRY(launch_qgemm(g, EPI_STORE, s));
            g.w = &L.up.p;
            g.y = m->pf_u;
            PTRY(launch_qgemm(g, EPI_STORE, s));
            PTRY(launch_silu_hilo(m->pf_g, m->pf_u, (size_t)n * lc.inter, m->pf_ah, m->pf_al, s));
        }
        {
            QgemmArgs g;
            g.f16_scratch = m->pf_wscratch;
            g.w = &L.down.p;
            g.xh = m->pf_ah;
            g.xl = m->pf_al;
            g.n = n;
            g.y = tp ? m->pf_part : m->pf_x;
            g.ldy = c.hidden;
            g.err = m->gemm_err;
            PTRY(launch_qgemm(g, tp ? EPI_STORE : EPI_ADD, s));
            if (tp) {
                PTRY(prefill_allreduce(m, n, nullptr, 1));
                m->stats.kernel_launches++;  // push + reduce
            }
        }
    }
    if (last) {
        PTRY(enqueue_head(m, m->pf_x + (size_t)(n - 1) * c.hidden, false));
        m->stats.kernel_launches++;  // final norm + lm_head
    }
#undef PTRY
    return CUQ_OK;
}

static int set_state(cuq_model *m, int token, int pos, int n_forced) {
    m->state_host->token = token;
    m->state_host->pos = pos;
    m->state_host->step = 0;
    m->state_host->n_forced = n_forced;
    m->state_host->argmax64 = 0ull;
    CUQ_CUDA_TRY(cudaMemcpyAsync(m->state, m->state_host, sizeof(StepState), cudaMemcpyHostToDevice, m->stream));
    return CUQ_OK;
}


// Prefill ids[0..n) at start_pos in chunks; leaves the state ready for decoding
// (token = argmax of the last position, pos = start_pos + n, step = 1,
// out_tokens[0] = that argmax).
static int prefill_batched(cuq_model *m, const uint32_t *ids, uint32_t n, uint32_t start_pos) {
    int rc;
    const uint32_t C = m->opt.max_chunk;
    for (uint32_t off = 0; off < n; off += C) {
        const uint32_t cn = n - off < C ? n - off : C;
        const bool last = off + cn == n;
        CUQ_CUDA_TRY(cudaMemcpyAsync(m->pf_ids, ids + off, sizeof(uint32_t) * cn, cudaMemcpyHostToDevice, m->stream));
        if (last && (rc = set_state(m, 0, (int)(start_pos + off + cn - 1), 1))) return rc;
        if ((rc = prefill_chunk(m, m->pf_ids, cn, start_pos + off, last))) return rc;
        if (!last) CUQ_CUDA_TRY(cudaStreamSynchronize(m->stream));  // pf_ids is reused by the next chunk
    }
    return CUQ_OK;
}

static int check_gemm_err(cuq_model *m) {
    int herr = 0;
    CUQ_CUDA_TRY(cudaMemcpy(&herr, m->gemm_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) {
        cudaMemset(m->gemm_err, 0, sizeof(int));
        set_error("prefill: a tensor-core pipeline wait timed out");
        return CUQ_ETIMEOUT;
    }
    return CUQ_OK;
}

extern "C" {

cuq_model *cuq_model_create(const cuq_config *cfg, const cuq_options *opts) {
    if (!cfg) {
        set_error("cuq_model_create: null config");
        return nullptr;
    }
    const cuq_config &c = *cfg;
    if (!c.hidden || !c.layers || !c.heads || !c.kv_heads || !c.head_dim || !c.inter || !c.vocab ||
        c.heads % c.kv_heads || (c.head_dim != 64 && c.head_dim != 128) || c.hidden % 16 || c.inter % 16 ||
        c.vocab % 16) {
        set_error("cuq_model_create: unsupported geometry (hidden %u heads %u/%u head_dim %u inter %u vocab %u)",
                  c.hidden, c.heads, c.kv_heads, c.head_dim, c.inter, c.vocab);
        return nullptr;
    }
    cuq_options o{};
    if (opts) o = *opts;
    if (!o.max_seq) o.max_seq = 2048;
    if (!o.max_chunk) o.max_chunk = 512;
    if (!o.tp_size) o.tp_size = 1;
    {
        // Megatron split (column-parallel q/k/v/gate/up and lm_head rows,
        // row-parallel o/down columns): whole KV heads and 16-row tiles per rank
        const uint32_t tp = (uint32_t)o.tp_size;
        if (o.tp_size < 1 || o.tp_size > TP_MAX || o.tp_rank < 0 || o.tp_rank >= o.tp_size || c.kv_heads % tp ||
            (c.inter / tp) % 64 || c.inter % tp || c.vocab % (16 * tp) || (c.heads / tp * c.head_dim) % 64) {
            set_error("cuq_model_create: tensor parallel %d/%d does not divide the model (kv_heads %u, inter %u, "
                      "vocab %u)",
                      o.tp_rank, o.tp_size, c.kv_heads, c.inter, c.vocab);
            return nullptr;
        }
    }
    cuq_model *m = new cuq_model();
    m->cfg = c;
    m->lc = c;
    m->lc.heads = c.heads / o.tp_size;
    m->lc.kv_heads = c.kv_heads / o.tp_size;
    m->lc.inter = c.inter / o.tp_size;
    m->lc.vocab = c.vocab / o.tp_size;
    m->vocab_base = m->lc.vocab * (uint32_t)o.tp_rank;
    m->opt = o;
    m->sm_count = sm_count_current();
    m->layers.resize(c.layers);
    const cuq_config &lc = m->lc;
    const uint32_t qd = q_dim(lc), kvd = kv_dim(lc);
    bool ok = false;
    do {
        if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) break;
        size_t kv_bytes = (size_t)lc.kv_heads * o.max_seq * c.head_dim * sizeof(__half);
        bool bad = false;
        for (auto &L : m->layers) {
            if (cudaMalloc(&L.k_cache, kv_bytes) != cudaSuccess || cudaMalloc(&L.v_cache, kv_bytes) != cudaSuccess ||
                cudaMemset(L.k_cache, 0, kv_bytes) != cudaSuccess || cudaMemset(L.v_cache, 0, kv_bytes) != cudaSuccess) {
                bad = true;
                break;
            }
        }
        if (bad) break;
        m->stats.kv_bytes = 2 * kv_bytes * c.layers;
        m->attn_nsplit = attn_pick_nsplit(lc.kv_heads, o.max_seq, m->sm_count);
        if (cudaMalloc(&m->x, sizeof(float) * c.hidden) != cudaSuccess) break;
        if (cudaMalloc(&m->qkv, sizeof(float) * (qd + 2 * kvd)) != cudaSuccess) break;
        if (cudaMalloc(&m->q_rot, sizeof(float) * qd) != cudaSuccess) break;
        if (cudaMalloc(&m->logits, sizeof(float) * lc.vocab) != cudaSuccess) break;
        if (cudaMalloc(&m->act, sizeof(float) * lc.inter) != cudaSuccess) break;
        if (cudaMalloc(&m->gate_buf, sizeof(float) * lc.inter) != cudaSuccess) break;
        if (cudaMalloc(&m->up_buf, sizeof(float) * lc.inter) != cudaSuccess) break;
        if (cudaMalloc(&m->attn_part, sizeof(float) * (size_t)m->attn_nsplit * lc.heads * (c.head_dim + 2)) !=
            cudaSuccess)
            break;
        size_t xh = xq_halves(c.hidden), xa = xq_halves(qd), xi = xq_halves(lc.inter);
        if (cudaMalloc(&m->xq_h, sizeof(__half) * xh) != cudaSuccess) break;
        if (cudaMalloc(&m->xq_attn, sizeof(__half) * xa) != cudaSuccess) break;
        if (cudaMalloc(&m->xq_act, sizeof(__half) * xi) != cudaSuccess) break;
        cudaMemset(m->xq_h, 0, sizeof(__half) * xh);
        cudaMemset(m->xq_attn, 0, sizeof(__half) * xa);
        cudaMemset(m->xq_act, 0, sizeof(__half) * xi);
        // RoPE table, reference formula (cpu.zig:26-31)
        std::vector<float> cs((size_t)o.max_seq * c.head_dim);
        build_rope_table(cs.data(), o.max_seq, c.head_dim, c.rope_theta);
        if (cudaMalloc(&m->rope_cs, sizeof(float) * cs.size()) != cudaSuccess) break;
        if (cudaMemcpy(m->rope_cs, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice) != cudaSuccess) break;
        if (cudaMalloc(&m->ss, sizeof(float) * 2 * (c.hidden / 16)) != cudaSuccess) break;
        cudaMemset(m->ss, 0, sizeof(float) * 2 * (c.hidden / 16));
        if (cudaMalloc(&m->done, sizeof(unsigned int)) != cudaSuccess) break;
        if (cudaMalloc(&m->tickets, sizeof(unsigned int) * lc.kv_heads) != cudaSuccess) break;
        cudaMemset(m->done, 0, sizeof(unsigned int));
        cudaMemset(m->tickets, 0, sizeof(unsigned int) * lc.kv_heads);
        if (cudaMalloc(&m->state, sizeof(StepState)) != cudaSuccess) break;
        cudaMemset(m->state, 0, sizeof(StepState));
        if (cudaMallocHost(&m->state_host, sizeof(StepState)) != cudaSuccess) break;
        if (cudaMalloc(&m->forced, sizeof(uint32_t) * (o.max_seq + 1)) != cudaSuccess) break;
        if (cudaMalloc(&m->out_tokens, sizeof(uint32_t) * (o.max_seq + 1)) != cudaSuccess) break;
        if (cudaMallocHost(&m->out_host, sizeof(uint32_t) * (o.max_seq + 1)) != cudaSuccess) break;
        if (cudaMallocHost(&m->err_host, sizeof(int)) != cudaSuccess) break;
        *m->err_host = 0;
        {
            const size_t C = o.max_chunk;
            const size_t wide = c.hidden > qd ? c.hidden : qd;
            if (cudaMalloc(&m->pf_x, sizeof(float) * C * c.hidden) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_qkv, sizeof(float) * C * (qd + 2 * kvd)) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_q, sizeof(float) * C * qd) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_g, sizeof(float) * C * lc.inter) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_u, sizeof(float) * C * lc.inter) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_h, sizeof(__half) * C * wide) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_l, sizeof(__half) * C * wide) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_ah, sizeof(__half) * C * lc.inter) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_al, sizeof(__half) * C * lc.inter) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_ids, sizeof(uint32_t) * C) != cudaSuccess) break;
            if (cudaMalloc(&m->gemm_err, sizeof(int)) != cudaSuccess) break;
            cudaMemset(m->gemm_err, 0, sizeof(int));
        }
        if (o.tp_size > 1) {
            // communication buffer: 2 phase regions of [tp][max_chunk * hidden]
            // fp32 slots, [tp] argmax keys, 4 counters (plain cudaMalloc: IPC-exportable)
            const size_t slot = (size_t)o.max_chunk * c.hidden;
            TpComm &t = m->tpc;
            t.rank = o.tp_rank;
            t.size = o.tp_size;
            t.slot_floats = slot;
            t.off_phase[0] = 0;
            t.off_phase[1] = round256(sizeof(float) * slot * o.tp_size);
            t.off_am = t.off_phase[1] + round256(sizeof(float) * slot * o.tp_size);
            t.off_ctr = t.off_am + 256;
            m->tp_bytes = t.off_ctr + 256;
            if (cudaMalloc(&m->tp_buf, m->tp_bytes) != cudaSuccess) break;
            if (cudaMemset(m->tp_buf, 0, m->tp_bytes) != cudaSuccess) break;
            if (cudaMalloc(&m->tp_err, sizeof(int)) != cudaSuccess) break;
            if (cudaMalloc(&m->tp_done, sizeof(unsigned int)) != cudaSuccess) break;
            if (cudaMalloc(&m->pf_part, sizeof(float) * slot) != cudaSuccess) break;
            cudaMemset(m->tp_err, 0, sizeof(int));
            cudaMemset(m->tp_done, 0, sizeof(unsigned int));
            t.err = m->tp_err;
            if (o.wait_limit_ms) t.wait_ns = (unsigned long long)o.wait_limit_ms * 1000000ull;
            t.peer[t.rank] = m->tp_buf;
        }
        if (cudaMalloc(&m->smp, sizeof(SampleState)) != cudaSuccess) break;
        if (cudaMallocHost(&m->smp_host, sizeof(SampleState)) != cudaSuccess) break;
        if (cudaEventCreate(&m->ev0) != cudaSuccess || cudaEventCreate(&m->ev1) != cudaSuccess) break;
        ok = true;
    } while (0);
    if (!ok) {
        set_error("cuq_model_create: allocation failed (%s)", cudaGetErrorString(cudaGetLastError()));
        cuq_model_free(m);
        return nullptr;
    }
    return m;
}

static int check_linear_shape(const cuq_model *m, int role, uint32_t rows, uint32_t cols) {
    const cuq_config &c = m->cfg;
    uint32_t qd = q_dim(c), kvd = kv_dim(c);
    uint32_t er = 0, ec = 0;
    switch (role) {
    case CUQ_ROLE_Q: er = qd; ec = c.hidden; break;
    case CUQ_ROLE_K: case CUQ_ROLE_V: er = kvd; ec = c.hidden; break;
    case CUQ_ROLE_O: er = c.hidden; ec = qd; break;
    case CUQ_ROLE_GATE: case CUQ_ROLE_UP: er = c.inter; ec = c.hidden; break;
    case CUQ_ROLE_DOWN: er = c.hidden; ec = c.inter; break;
    case CUQ_ROLE_EMBED: case CUQ_ROLE_OUTPUT: er = c.vocab; ec = c.hidden; break;
    default: set_error("cuq_upload_tensor: role %d is not a linear tensor", role); return CUQ_EINVAL;
    }
    if (rows != er || cols != ec) {
        set_error("DimensionMismatch: role %d is %u x %u, expected %u x %u", role, rows, cols, er, ec);
        return CUQ_EINVAL;
    }
    return CUQ_OK;
}

int cuq_upload_tensor(cuq_model *m, int layer, int role, int ggml_type, const void *raw_host, size_t nbytes,
                      uint32_t rows, uint32_t cols) {
    CUQ_CHECK_ARG(m && raw_host, "cuq_upload_tensor: null argument");
    if (m->finalized) {
        set_error("cuq_upload_tensor: model already finalized");
        return CUQ_EINVAL;
    }
    int rc = check_linear_shape(m, role, rows, cols);
    if (rc) return rc;
    int epb = block_elems(ggml_type), bpb = block_bytes(ggml_type);
    if (!epb || !gemv_supported(ggml_type)) {
        set_error("UnsupportedType: ggml type %d for role %d", ggml_type, role);
        return CUQ_EUNSUPPORTED;
    }
    if (cols % epb || nbytes != (size_t)rows * (cols / epb) * bpb) {
        set_error("InvalidTensorShape: %zu bytes for %u x %u of type %d", nbytes, rows, cols, ggml_type);
        return CUQ_EINVAL;
    }
    // tensor parallelism: keep this rank's shard only (rows for column-parallel
    // projections and the lm_head, whole-block columns for o and down)
    std::vector<uint8_t> shard;
    if (m->opt.tp_size > 1 && role != CUQ_ROLE_EMBED) {
        const cuq_config &lc = m->lc;
        const uint32_t rank = (uint32_t)m->opt.tp_rank, lqd = q_dim(lc), lkvd = kv_dim(lc);
        uint32_t r0 = 0, r1 = rows, c0 = 0, c1 = cols;
        switch (role) {
        case CUQ_ROLE_Q: r0 = rank * lqd; r1 = r0 + lqd; break;
        case CUQ_ROLE_K: case CUQ_ROLE_V: r0 = rank * lkvd; r1 = r0 + lkvd; break;
        case CUQ_ROLE_GATE: case CUQ_ROLE_UP: r0 = rank * lc.inter; r1 = r0 + lc.inter; break;
        case CUQ_ROLE_OUTPUT: r0 = m->vocab_base; r1 = r0 + lc.vocab; break;
        case CUQ_ROLE_O: c0 = rank * lqd; c1 = c0 + lqd; break;
        case CUQ_ROLE_DOWN: c0 = rank * lc.inter; c1 = c0 + lc.inter; break;
        default: break;
        }
        const size_t row_bytes = (size_t)(cols / epb) * bpb;
        if (c0 % epb || c1 % epb) {
            set_error("tensor parallel: columns [%u, %u) of role %d are not whole blocks of %d", c0, c1, role, epb);
            return CUQ_EINVAL;
        }
        const size_t lrow_bytes = (size_t)((c1 - c0) / epb) * bpb;
        shard.resize((size_t)(r1 - r0) * lrow_bytes);
        const uint8_t *src = static_cast<const uint8_t *>(raw_host);
        for (uint32_t r = r0; r < r1; r++)
            memcpy(shard.data() + (size_t)(r - r0) * lrow_bytes, src + (size_t)r * row_bytes + (size_t)(c0 / epb) * bpb,
                   lrow_bytes);
        raw_host = shard.data();
        nbytes = shard.size();
        rows = r1 - r0;
        cols = c1 - c0;
    }
    PendingTensor *t;
    if (role == CUQ_ROLE_EMBED)
        t = &m->pend_embed;
    else if (role == CUQ_ROLE_OUTPUT)
        t = &m->pend_output;
    else {
        CUQ_CHECK_ARG(layer >= 0 && (uint32_t)layer < m->cfg.layers, "cuq_upload_tensor: layer %d out of range", layer);
        t = &m->layers[layer].pend[role];
    }
    free_pending(*t);
    t->type = ggml_type;
    t->rows = rows;
    t->cols = cols;
    t->nbytes = nbytes;
    CUQ_CUDA_TRY(cudaMalloc(&t->raw, nbytes));  // the GGUF bytes, as they are on disk
    CUQ_CUDA_TRY(cudaMemcpy(t->raw, raw_host, nbytes, cudaMemcpyHostToDevice));
    m->stats.weight_bytes += nbytes;
    return CUQ_OK;
}

int cuq_upload_f32(cuq_model *m, int layer, int role, const float *v, size_t n) {
    CUQ_CHECK_ARG(m && v, "cuq_upload_f32: null argument");
    const cuq_config &c = m->cfg;
    uint32_t qd = q_dim(c), kvd = kv_dim(c);
    // tensor parallelism: q/k/v biases follow their projection's row shard
    const uint32_t lqd = q_dim(m->lc), lkvd = kv_dim(m->lc), rank = (uint32_t)m->opt.tp_rank;
    if (m->opt.tp_size > 1 && (role == CUQ_ROLE_Q_BIAS || role == CUQ_ROLE_K_BIAS || role == CUQ_ROLE_V_BIAS)) {
        const size_t want_full = role == CUQ_ROLE_Q_BIAS ? qd : kvd;
        if (n != want_full) {
            set_error("DimensionMismatch: role %d has %zu values, expected %zu", role, n, want_full);
            return CUQ_EINVAL;
        }
        CUQ_CHECK_ARG(layer >= 0 && (uint32_t)layer < c.layers, "cuq_upload_f32: layer %d out of range", layer);
        float **slot = &m->layers[layer].qkv_bias;
        const size_t total = lqd + 2 * lkvd;
        size_t off = 0, len = lqd, src = (size_t)rank * lqd;
        if (role != CUQ_ROLE_Q_BIAS) {
            off = role == CUQ_ROLE_K_BIAS ? lqd : lqd + lkvd;
            len = lkvd;
            src = (size_t)rank * lkvd;
        }
        if (!*slot) {
            CUQ_CUDA_TRY(cudaMalloc(slot, sizeof(float) * total));
            CUQ_CUDA_TRY(cudaMemset(*slot, 0, sizeof(float) * total));
        }
        CUQ_CUDA_TRY(cudaMemcpy(*slot + off, v + src, sizeof(float) * len, cudaMemcpyHostToDevice));
        return CUQ_OK;
    }
    float **slot = nullptr;
    size_t want = 0, off = 0, total = 0;
    if (role == CUQ_ROLE_FINAL_NORM) {
        slot = &m->final_norm;
        want = total = c.hidden;
    } else {
        CUQ_CHECK_ARG(layer >= 0 && (uint32_t)layer < c.layers, "cuq_upload_f32: layer %d out of range", layer);
        Layer &L = m->layers[layer];
        switch (role) {
        case CUQ_ROLE_ATTN_NORM: slot = &L.attn_norm; want = total = c.hidden; break;
        case CUQ_ROLE_FFN_NORM: slot = &L.ffn_norm; want = total = c.hidden; break;
        case CUQ_ROLE_O_BIAS: slot = &L.o_bias; want = total = c.hidden; break;
        case CUQ_ROLE_Q_BIAS: slot = &L.qkv_bias; want = qd; off = 0; total = qd + 2 * kvd; break;
        case CUQ_ROLE_K_BIAS: slot = &L.qkv_bias; want = kvd; off = qd; total = qd + 2 * kvd; break;
        case CUQ_ROLE_V_BIAS: slot = &L.qkv_bias; want = kvd; off = qd + kvd; total = qd + 2 * kvd; break;
        default: set_error("cuq_upload_f32: role %d is not a vector", role); return CUQ_EINVAL;
        }
    }
    if (n != want) {
        set_error("DimensionMismatch: role %d has %zu values, expected %zu", role, n, want);
        return CUQ_EINVAL;
    }
    if (!*slot) {
        CUQ_CUDA_TRY(cudaMalloc(slot, sizeof(float) * total));
        CUQ_CUDA_TRY(cudaMemset(*slot, 0, sizeof(float) * total));
    }
    CUQ_CUDA_TRY(cudaMemcpy(*slot + off, v, sizeof(float) * n, cudaMemcpyHostToDevice));
    return CUQ_OK;
}

// The decode step as a persistent-kernel program: the phases enqueue_step
// launches as kernels, with the RMSNorms folded into the GEMV phases that
// consume them and the embedding into the first.
static int build_mega(cuq_model *m) {
    const cuq_config &c = m->cfg, &lc = m->lc;
    MegaStepSpec sp;
    sp.embed = &m->embed.p;
    sp.x = m->x;
    sp.hidden = c.hidden;
    sp.eps = c.eps;
    sp.state = m->state;
    sp.forced = m->forced;
    sp.out_tokens = m->out_tokens;
    if (m->opt.tp_size > 1) {
        set_error("persistent decode: single GPU only");
        return CUQ_EUNSUPPORTED;
    }
    auto seg = [](const Planes &w, const __half *xq, float *y, const float *bias, int epi) {
        MegaSegSpec g;
        g.a.w = &w;
        g.a.xq = xq;
        g.a.y = y;
        g.a.bias = bias;
        g.epi = epi;
        return g;
    };
    for (uint32_t l = 0; l < c.layers; l++) {
        Layer &L = m->layers[l];
        if (!L.gate_up_dual) {
            set_error("persistent decode: layer %u gate and up differ in type", l);
            return CUQ_EUNSUPPORTED;
        }
        MegaPhaseSpec q;
        q.norm_w = L.attn_norm;
        q.embed = l == 0;
        for (auto &sg : L.qkv)
            q.segs.push_back(seg(sg.p, nullptr, m->qkv + sg.row_off, L.qkv_bias ? L.qkv_bias + sg.row_off : nullptr,
                                 EPI_STORE));
        sp.phases.push_back(q);
        MegaPhaseSpec at;
        at.kind = MEGA_ATTN;
        at.attn.qkv = m->qkv;
        at.attn.cs = m->rope_cs;
        at.attn.k_cache = L.k_cache;
        at.attn.v_cache = L.v_cache;
        at.attn.cache_stride = m->opt.max_seq;
        at.attn.heads = lc.heads;
        at.attn.kv_heads = lc.kv_heads;
        at.attn.hd = c.head_dim;
        at.attn.adjacent = c.rope_adjacent;
        at.attn.nsplit = m->attn_nsplit;
        at.attn.xq = m->xq_attn;
        sp.phases.push_back(at);
        MegaPhaseSpec o;
        o.segs.push_back(seg(L.o.p, m->xq_attn, m->x, L.o_bias, EPI_ADD));
        sp.phases.push_back(o);
        MegaPhaseSpec gu;
        gu.norm_w = L.ffn_norm;
        MegaSegSpec g = seg(L.gate.p, nullptr, nullptr, nullptr, EPI_SILU_XQ);
        g.a.w2 = &L.up.p;
        g.a.xq_out = m->xq_act;
        gu.segs.push_back(g);
        sp.phases.push_back(gu);
        MegaPhaseSpec dn;
        dn.segs.push_back(seg(L.down.p, m->xq_act, m->x, nullptr, EPI_ADD));
        sp.phases.push_back(dn);
    }
    MegaPhaseSpec hd;
    hd.norm_w = m->final_norm;
    MegaSegSpec h = seg(head_proj(m).p, nullptr, m->logits, nullptr, EPI_ARGMAX);
    h.a.row_base = m->vocab_base;
    hd.segs.push_back(h);
    sp.phases.push_back(hd);
    return mega_build(sp, m->sm_count, m->opt.persistent_ctas, m->mega);
}

int cuq_model_finalize(cuq_model *m) {
    CUQ_CHECK_ARG(m, "cuq_model_finalize: null model");
    if (m->finalized) return CUQ_OK;
    const cuq_config &c = m->cfg;
    const uint32_t qd = q_dim(m->lc), kvd = kv_dim(m->lc);
    cudaStream_t s = m->stream;
    int rc;
    if (m->opt.tp_size > 1 && !m->tp_connected) {
        set_error("cuq_model_finalize: tensor-parallel model not connected (cuq_tp_connect first)");
        return CUQ_ENOTREADY;
    }
    if (!m->pend_embed.raw) {
        set_error("MissingTensor: token_embd.weight");
        return CUQ_EINVAL;
    }
    if (!c.tie_embeddings && !m->pend_output.raw) {
        set_error("MissingTensor: output.weight");
        return CUQ_EINVAL;
    }
    if (!m->final_norm) {
        set_error("MissingTensor: output_norm.weight");
        return CUQ_EINVAL;
    }
    {
        // Decode GEMV kernel.  The TMA-fed kernels (a CTA requests a whole tile's
        // weights at once) pay off when a rank streams gigabytes per token; on
        // smaller models the register-prefetch kernel is faster (measured on
        // B200: SmolLM2-135M 1393 against 1111 tok/s, Qwen2.5-1.5B 551 against
        // 485, Llama-3-8B 234 against 265).
        size_t wb = 0;
        for (auto &L : m->layers)
            for (int r = 0; r < 7; r++) wb += L.pend[r].nbytes;
        wb += c.tie_embeddings ? m->pend_embed.nbytes : m->pend_output.nbytes;
        m->use_tma = wb >= (size_t(2) << 30);  // this rank's bytes (uploads keep only the shard)
    }
    size_t ws_need = 0, ctr_need = 0;
    auto account = [&](const Planes &p, int dual, bool tma) {
        int k = gemv_pick_ksplit(p, m->sm_count, dual ? 2 : 1, tma);
        if (k > 1) {
            size_t need = (size_t)k * p.rows * (dual ? 2 : 1);
            if (need > ws_need) ws_need = need;
        }
        if (p.rows / 16 > ctr_need) ctr_need = p.rows / 16;
    };
    for (uint32_t l = 0; l < c.layers; l++) {
        Layer &L = m->layers[l];
        for (int r = 0; r < 7; r++)
            if (!L.pend[r].raw) {
                static const char *names[] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up",
                                              "ffn_down"};
                set_error("MissingTensor: blk.%u.%s.weight", l, names[r]);
                return CUQ_EINVAL;
            }
        if (!L.attn_norm || !L.ffn_norm) {
            set_error("MissingTensor: blk.%u norm weights", l);
            return CUQ_EINVAL;
        }
        // q||k||v, fused where the types agree (load_gguf.zig:677-682)
        PendingTensor *q = &L.pend[R_Q], *k = &L.pend[R_K], *v = &L.pend[R_V];
        std::vector<std::vector<PendingTensor *>> groups;
        std::vector<uint32_t> offs;
        if (q->type == k->type && k->type == v->type) {
            groups.push_back({q, k, v});
            offs.push_back(0);
        } else if (q->type == k->type) {
            groups.push_back({q, k});
            offs.push_back(0);
            groups.push_back({v});
            offs.push_back(qd + kvd);
        } else {
            groups.push_back({q});
            offs.push_back(0);
            groups.push_back({k});
            offs.push_back(qd);
            groups.push_back({v});
            offs.push_back(qd + kvd);
        }
        L.qkv.resize(groups.size());
        for (size_t gi = 0; gi < groups.size(); gi++) {
            if ((rc = build_proj(L.qkv[gi], groups[gi], s))) return rc;
            L.qkv[gi].row_off = offs[gi];
            account(L.qkv[gi].p, 0, m->use_tma);
        }
        if ((rc = build_proj(L.o, {&L.pend[R_O]}, s))) return rc;
        if ((rc = build_proj(L.gate, {&L.pend[R_GATE]}, s))) return rc;
        if ((rc = build_proj(L.up, {&L.pend[R_UP]}, s))) return rc;
        if ((rc = build_proj(L.down, {&L.pend[R_DOWN]}, s))) return rc;
        L.gate_up_dual = L.gate.p.type == L.up.p.type;
        account(L.o.p, 0, m->use_tma);
        account(L.gate.p, L.gate_up_dual, m->use_tma);
        account(L.up.p, 0, m->use_tma);
        account(L.down.p, 0, m->use_tma);
        for (int r = 0; r < 7; r++) free_pending(L.pend[r]);
    }
    if (c.tie_embeddings && m->opt.tp_size > 1) {
        // tied lm_head under tensor parallelism: this rank's vocab rows of the
        // embedding table become its own head weight
        PendingTensor view = m->pend_embed;
        const size_t row_bytes = view.nbytes / view.rows;
        view.raw += (size_t)m->vocab_base * row_bytes;
        view.rows = m->lc.vocab;
        view.nbytes = (size_t)m->lc.vocab * row_bytes;
        if ((rc = build_proj(m->output, {&view}, s))) return rc;
    }
    if ((rc = build_proj(m->embed, {&m->pend_embed}, s))) return rc;
    free_pending(m->pend_embed);
    if (!c.tie_embeddings) {
        if ((rc = build_proj(m->output, {&m->pend_output}, s))) return rc;
        free_pending(m->pend_output);
    }
    account(head_proj(m).p, 0, head_tma(m));
    {
        // every layer GEMV on the TMA-fed kernels: the norms are computed from
        // the per-tile partials (the lm_head reads its own norm kernel's xq)
        bool all = m->use_tma;
        for (auto &L : m->layers) {
            for (auto &sg : L.qkv) all = all && gemv_tma_supported(sg.p.type);
            all = all && gemv_tma_supported(L.o.p.type) && gemv_tma_supported(L.gate.p.type) &&
                  gemv_tma_supported(L.up.p.type) && gemv_tma_supported(L.down.p.type) && L.gate_up_dual;
        }
        m->all_tma = all;
    }
    {
        // raw-block weights: fp16 expansion scratch of the largest prefill GEMM
        size_t need = 0;
        for (auto &L : m->layers) {
            for (auto &sg : L.qkv) need = std::max(need, qgemm_scratch_halves(sg.p, false));
            need = std::max(need, qgemm_scratch_halves(L.o.p, false));
            need = std::max(need, qgemm_scratch_halves(L.gate.p, L.gate_up_dual));
            need = std::max(need, qgemm_scratch_halves(L.up.p, false));
            need = std::max(need, qgemm_scratch_halves(L.down.p, false));
        }
        if (need) CUQ_CUDA_TRY(cudaMalloc(&m->pf_wscratch, sizeof(__half) * need));
    }
    m->ws_floats = ws_need;
    m->n_counters = ctr_need + 1;
    if (ws_need) CUQ_CUDA_TRY(cudaMalloc(&m->ws, sizeof(float) * ws_need));
    CUQ_CUDA_TRY(cudaMalloc(&m->counters, sizeof(unsigned) * m->n_counters));
    CUQ_CUDA_TRY(cudaMemset(m->counters, 0, sizeof(unsigned) * m->n_counters));
    CUQ_CUDA_TRY(cudaDeviceSynchronize());
    (void)qd;
    (void)kvd;
    m->finalized = true;
    if (m->opt.decode_kernel == CUQ_DECODE_PERSISTENT) {
        rc = build_mega(m);
        if (rc != CUQ_OK) {
            m->finalized = false;
            return rc;
        }
    }
    if (m->opt.use_graphs && !m->mega.impl) {
        CUQ_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_step(m);
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(s, &g);
        if (rc != CUQ_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) {
            set_error("graph capture: %s", cudaGetErrorString(e));
            return CUQ_ECUDA;
        }
        m->graph = g;
        CUQ_CUDA_TRY(cudaGraphInstantiate(&m->graph_exec, g, 0));
    }
    return CUQ_OK;
}

int cuq_tp_comm_handle(cuq_model *m, void *handle_out) {
    CUQ_CHECK_ARG(m && handle_out, "cuq_tp_comm_handle: null argument");
    if (m->opt.tp_size < 2) {
        set_error("cuq_tp_comm_handle: model is not tensor parallel");
        return CUQ_EINVAL;
    }
    cudaIpcMemHandle_t h;
    CUQ_CUDA_TRY(cudaIpcGetMemHandle(&h, m->tp_buf));
    static_assert(sizeof(h) == CUQ_TP_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    return CUQ_OK;
}

int cuq_tp_connect(cuq_model *m, const void *handles) {
    CUQ_CHECK_ARG(m && handles, "cuq_tp_connect: null argument");
    if (m->opt.tp_size < 2 || m->tp_connected) {
        set_error("cuq_tp_connect: model is not tensor parallel or already connected");
        return CUQ_EINVAL;
    }
    const uint8_t *hb = static_cast<const uint8_t *>(handles);
    for (int r = 0; r < m->tpc.size; r++) {
        if (r == m->tpc.rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)r * CUQ_TP_HANDLE_BYTES, sizeof(h));
        bool absent = true;
        for (int i = 0; i < CUQ_TP_HANDLE_BYTES; i++) absent = absent && hb[(size_t)r * CUQ_TP_HANDLE_BYTES + i] == 0;
        if (absent) {
            // a rank that never joins: what this rank sends it lands in a local
            // sink, and every wait for its arrivals runs out (CUQ_ETIMEOUT)
            if (!m->tp_sink) {
                CUQ_CUDA_TRY(cudaMalloc(&m->tp_sink, m->tp_bytes));
                CUQ_CUDA_TRY(cudaMemset(m->tp_sink, 0, m->tp_bytes));
            }
            m->tpc.peer[r] = m->tp_sink;
            continue;
        }
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; q++)
                if (q != m->tpc.rank && m->tpc.peer[q] && m->tpc.peer[q] != m->tp_sink) {
                    cudaIpcCloseMemHandle(m->tpc.peer[q]);
                    m->tpc.peer[q] = nullptr;
                }
            set_error("cuq_tp_connect: rank %d buffer: %s", r, cudaGetErrorString(e));
            return CUQ_ECUDA;
        }
        m->tpc.peer[r] = static_cast<uint8_t *>(p);
    }
    m->tp_connected = true;
    return CUQ_OK;
}

int cuq_model_get_config(const cuq_model *m, cuq_config *out) {
    CUQ_CHECK_ARG(m && out, "cuq_model_get_config: null argument");
    *out = m->cfg;
    return CUQ_OK;
}

static int finish_call(cuq_model *m, uint32_t n_steps, float *logits_host, uint32_t *argmax_out, double *ms_out) {
    CUQ_CUDA_TRY(cudaEventRecord(m->ev1, m->stream));
    const bool mega_ran = m->mega_ran;
    m->mega_ran = false;
    if (mega_ran) {
        int rc = mega_err_copy(m->mega, m->err_host, m->stream);
        if (rc) return rc;
    }
    if (logits_host)
        CUQ_CUDA_TRY(cudaMemcpyAsync(logits_host, m->logits, sizeof(float) * m->lc.vocab, cudaMemcpyDeviceToHost,
                                     m->stream));
    if (n_steps)
        CUQ_CUDA_TRY(cudaMemcpyAsync(m->out_host, m->out_tokens, sizeof(uint32_t) * n_steps, cudaMemcpyDeviceToHost,
                                     m->stream));
    CUQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, m->ev0, m->ev1);
    if (ms_out) *ms_out += ms;
    if (argmax_out && n_steps) *argmax_out = m->out_host[n_steps - 1];
    if (mega_ran && *m->err_host) {
        set_error("persistent decode: a grid barrier was not reached within its wait limit");
        return CUQ_ETIMEOUT;
    }
    if (m->gemm_err) {
        int herr = 0;
        CUQ_CUDA_TRY(cudaMemcpy(&herr, m->gemm_err, sizeof(int), cudaMemcpyDeviceToHost));
        if (herr) {
            cudaMemset(m->gemm_err, 0, sizeof(int));
            set_error("decode: a weight-stream wait timed out");
            return CUQ_ETIMEOUT;
        }
    }
    if (m->tp_err) {
        int herr = 0;
        CUQ_CUDA_TRY(cudaMemcpy(&herr, m->tp_err, sizeof(int), cudaMemcpyDeviceToHost));
        if (herr) {
            cudaMemset(m->tp_err, 0, sizeof(int));
            set_error("tensor parallel: a peer did not arrive within the wait limit");
            return CUQ_ETIMEOUT;
        }
    }
    return CUQ_OK;
}

static int check_token(const cuq_model *m, uint32_t t) {
    if (t >= m->cfg.vocab) {
        set_error("token %u out of range (vocab %u)", t, m->cfg.vocab);
        return CUQ_EINVAL;
    }
    return CUQ_OK;
}

int cuq_forward(cuq_model *m, uint32_t token, uint32_t pos, float *logits_host, uint32_t *argmax_out) {
    CUQ_CHECK_ARG(m, "cuq_forward: null model");
    if (!m->finalized) {
        set_error("cuq_forward: model not finalized");
        return CUQ_ENOTREADY;
    }
    if (pos >= m->opt.max_seq) {  // engine.zig:549
        set_error("ContextOverflow: position %u >= max_seq %u", pos, m->opt.max_seq);
        return CUQ_ECONTEXT;
    }
    int rc = check_token(m, token);
    if (rc) return rc;
    CUQ_CUDA_TRY(cudaMemcpyAsync(m->forced, &token, sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
    if ((rc = set_state(m, (int)token, (int)pos, 1))) return rc;
    CUQ_CUDA_TRY(cudaEventRecord(m->ev0, m->stream));
    if ((rc = run_steps(m, 1))) return rc;
    m->stats.tokens += 1;
    return finish_call(m, 1, logits_host, argmax_out, &m->stats.decode_ms);
}

int cuq_prefill(cuq_model *m, const uint32_t *ids, uint32_t n, uint32_t start_pos, float *logits_host,
                uint32_t *argmax_out) {
    CUQ_CHECK_ARG(m && (ids || n == 0), "cuq_prefill: null argument");
    if (!m->finalized) {
        set_error("cuq_prefill: model not finalized");
        return CUQ_ENOTREADY;
    }
    if (n == 0) return CUQ_OK;
    if ((uint64_t)start_pos + n > m->opt.max_seq) {  // engine.zig:981
        set_error("ContextOverflow: %u + %u > max_seq %u", start_pos, n, m->opt.max_seq);
        return CUQ_ECONTEXT;
    }
    int rc;
    for (uint32_t i = 0; i < n; i++)
        if ((rc = check_token(m, ids[i]))) return rc;
    CUQ_CUDA_TRY(cudaEventRecord(m->ev0, m->stream));
    if (n == 1) {  // a single position is one decode step
        CUQ_CUDA_TRY(cudaMemcpyAsync(m->forced, ids, sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
        if ((rc = set_state(m, (int)ids[0], (int)start_pos, 1))) return rc;
        if ((rc = run_steps(m, 1))) return rc;
    } else if ((rc = prefill_batched(m, ids, n, start_pos))) {
        return rc;
    }
    m->stats.prefill_tokens += n;
    if ((rc = finish_call(m, 1, logits_host, argmax_out, &m->stats.prefill_ms))) return rc;
    return check_gemm_err(m);
}

int cuq_generate(cuq_model *m, const uint32_t *ids, uint32_t n_prompt, uint32_t n_decode, uint32_t *out_tokens) {
    CUQ_CHECK_ARG(m && ids && n_prompt > 0 && (out_tokens || n_decode == 0), "cuq_generate: bad argument");
    if (!m->finalized) {
        set_error("cuq_generate: model not finalized");
        return CUQ_ENOTREADY;
    }
    if (n_decode == 0) return cuq_prefill(m, ids, n_prompt, 0, nullptr, nullptr);
    uint32_t steps = n_prompt + n_decode - 1;  // the last generated token is not fed back
    if (steps > m->opt.max_seq) {
        set_error("ContextOverflow: %u prompt + %u decode > max_seq %u", n_prompt, n_decode, m->opt.max_seq);
        return CUQ_ECONTEXT;
    }
    int rc;
    for (uint32_t i = 0; i < n_prompt; i++)
        if ((rc = check_token(m, ids[i]))) return rc;
    CUQ_CUDA_TRY(cudaEventRecord(m->ev0, m->stream));
    if (n_prompt == 1) {
        CUQ_CUDA_TRY(cudaMemcpyAsync(m->forced, ids, sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
        if ((rc = set_state(m, (int)ids[0], 0, 1))) return rc;
        if ((rc = run_steps(m, 1))) return rc;
    } else if ((rc = prefill_batched(m, ids, n_prompt, 0))) {
        return rc;
    }
    // the prefill left token = first generated id, step = 1: decode the rest on the device
    if ((rc = run_steps(m, n_decode - 1))) return rc;
    m->stats.prefill_tokens += n_prompt;
    m->stats.tokens += n_decode;
    if ((rc = finish_call(m, n_decode, nullptr, nullptr, &m->stats.decode_ms))) return rc;
    memcpy(out_tokens, m->out_host, sizeof(uint32_t) * n_decode);
    return check_gemm_err(m);
}

int cuq_generate_sampled(cuq_model *m, const uint32_t *ids, uint32_t n_prompt, uint32_t n_cached, uint32_t n_decode,
                         const cuq_sampler_params *params, uint32_t seed, uint32_t penalty_window,
                         uint32_t *out_tokens) {
    CUQ_CHECK_ARG(m && ids && n_prompt > 0 && n_cached < n_prompt && params && (out_tokens || n_decode == 0),
                  "cuq_generate_sampled: bad argument");
    CUQ_CHECK_ARG(penalty_window <= CUQ_SAMPLE_MAX_WINDOW, "cuq_generate_sampled: penalty window %u exceeds %u",
                  penalty_window, (unsigned)CUQ_SAMPLE_MAX_WINDOW);
    if (!m->finalized) {
        set_error("cuq_generate_sampled: model not finalized");
        return CUQ_ENOTREADY;
    }
    const cuq_sampler_params &P = *params;
    const bool pen = !(P.repetition_penalty == 1.0f && P.presence_penalty == 0.0f && P.frequency_penalty == 0.0f);
    const bool draw = P.temperature > 0.0f || pen;  // otherwise the step's own argmax is the reference's choice
    if (draw && m->opt.tp_size > 1) {
        set_error("cuq_generate_sampled: sampling under tensor parallelism is not supported (greedy only)");
        return CUQ_EUNSUPPORTED;
    }
    if (draw && m->lc.vocab > CUQ_SAMPLE_MAX_VOCAB) {
        set_error("cuq_generate_sampled: vocab %u exceeds %u", m->lc.vocab, (unsigned)CUQ_SAMPLE_MAX_VOCAB);
        return CUQ_EINVAL;
    }
    const uint32_t n_new = n_prompt - n_cached;
    if (n_decode == 0) return cuq_prefill(m, ids + n_cached, n_new, n_cached, nullptr, nullptr);
    if (n_prompt + n_decode - 1 > m->opt.max_seq) {
        set_error("ContextOverflow: %u prompt + %u decode > max_seq %u", n_prompt, n_decode, m->opt.max_seq);
        return CUQ_ECONTEXT;
    }
    int rc;
    for (uint32_t i = n_cached; i < n_prompt; i++)
        if ((rc = check_token(m, ids[i]))) return rc;
    if (draw) {
        // parameters, the LCG seed (generate.zig:169) and the window: the last
        // `penalty_window` prompt ids (generate.zig:205-211)
        SampleState &h = *m->smp_host;
        h.prm = P;
        h.rng = seed;
        const uint32_t nw = n_prompt < penalty_window ? n_prompt : penalty_window;
        memcpy(h.ids, ids + (n_prompt - nw), sizeof(uint32_t) * nw);
        h.ring.len = nw;
        h.ring.head = 0;
        h.ring.cap = penalty_window;
        CUQ_CUDA_TRY(cudaMemcpyAsync(m->smp, m->smp_host, offsetof(SampleState, ids) + sizeof(uint32_t) * nw,
                                     cudaMemcpyHostToDevice, m->stream));
    }
    CUQ_CUDA_TRY(cudaEventRecord(m->ev0, m->stream));
    if (n_new == 1) {
        CUQ_CUDA_TRY(cudaMemcpyAsync(m->forced, ids + n_cached, sizeof(uint32_t), cudaMemcpyHostToDevice,
                                     m->stream));
        if ((rc = set_state(m, (int)ids[n_cached], (int)n_cached, 1))) return rc;
        if ((rc = run_steps(m, 1))) return rc;
    } else if ((rc = prefill_batched(m, ids + n_cached, n_new, n_cached))) {
        return rc;
    }
    if (draw) {
        // the first token is drawn from the prompt's last logits, the rest after each step
        if ((rc = enqueue_sample(m))) return rc;
        m->stats.kernel_launches += 1;
        if ((rc = run_steps_sampled(m, n_decode - 1))) return rc;
    } else if ((rc = run_steps(m, n_decode - 1))) {
        return rc;
    }
    m->stats.prefill_tokens += n_new;
    m->stats.tokens += n_decode;
    if ((rc = finish_call(m, n_decode, nullptr, nullptr, &m->stats.decode_ms))) return rc;
    memcpy(out_tokens, m->out_host, sizeof(uint32_t) * n_decode);
    return check_gemm_err(m);
}

int cuq_decode_greedy(cuq_model *m, uint32_t token, uint32_t pos, uint32_t n_steps, uint32_t *out_tokens) {
    CUQ_CHECK_ARG(m && (out_tokens || n_steps == 0), "cuq_decode_greedy: bad argument");
    if (!m->finalized) {
        set_error("cuq_decode_greedy: model not finalized");
        return CUQ_ENOTREADY;
    }
    if (n_steps == 0) return CUQ_OK;
    if ((uint64_t)pos + n_steps > m->opt.max_seq) {
        set_error("ContextOverflow: %u + %u > max_seq %u", pos, n_steps, m->opt.max_seq);
        return CUQ_ECONTEXT;
    }
    int rc = check_token(m, token);
    if (rc) return rc;
    CUQ_CUDA_TRY(cudaMemcpyAsync(m->forced, &token, sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
    if ((rc = set_state(m, (int)token, (int)pos, 1))) return rc;
    CUQ_CUDA_TRY(cudaEventRecord(m->ev0, m->stream));
    if ((rc = run_steps(m, n_steps))) return rc;
    m->stats.tokens += n_steps;
    if ((rc = finish_call(m, n_steps, nullptr, nullptr, &m->stats.decode_ms))) return rc;
    memcpy(out_tokens, m->out_host, sizeof(uint32_t) * n_steps);
    return CUQ_OK;
}

// Rows [pos0, pos0 + n) of one layer's cache between the reference's host
// layout [pos][kv_heads * hd] (full width) and the device's [kv_head][max_seq][hd]
// (this rank's heads): one strided copy per local KV head and tensor.
static int kv_copy(const cuq_model *m, uint32_t layer, uint32_t pos0, uint32_t n, uint16_t *k_host, uint16_t *v_host,
                   bool to_device) {
    CUQ_CHECK_ARG(m && k_host && v_host, "cuq_kv_%s: null argument", to_device ? "write" : "read");
    CUQ_CHECK_ARG(layer < m->cfg.layers && (uint64_t)pos0 + n <= m->opt.max_seq,
                  "cuq_kv_%s: layer %u rows [%u, %u) outside the cache (%u layers, max_seq %u)",
                  to_device ? "write" : "read", layer, pos0, pos0 + n, m->cfg.layers, m->opt.max_seq);
    if (n == 0) return CUQ_OK;
    const uint32_t hd = m->cfg.head_dim, kvd = m->cfg.kv_heads * hd;
    const uint32_t h0 = (uint32_t)m->opt.tp_rank * m->lc.kv_heads;  // this rank's first KV head
    const cuq::Layer &L = m->layers[layer];
    for (uint32_t h = 0; h < m->lc.kv_heads; h++) {
        __half *kd = L.k_cache + ((size_t)h * m->opt.max_seq + pos0) * hd;
        __half *vd = L.v_cache + ((size_t)h * m->opt.max_seq + pos0) * hd;
        uint16_t *kh = k_host + (size_t)(h0 + h) * hd, *vh = v_host + (size_t)(h0 + h) * hd;
        const size_t w = sizeof(__half) * hd, hp = sizeof(uint16_t) * kvd;
        if (to_device) {
            CUQ_CUDA_TRY(cudaMemcpy2DAsync(kd, w, kh, hp, w, n, cudaMemcpyHostToDevice, m->stream));
            CUQ_CUDA_TRY(cudaMemcpy2DAsync(vd, w, vh, hp, w, n, cudaMemcpyHostToDevice, m->stream));
        } else {
            CUQ_CUDA_TRY(cudaMemcpy2DAsync(kh, hp, kd, w, w, n, cudaMemcpyDeviceToHost, m->stream));
            CUQ_CUDA_TRY(cudaMemcpy2DAsync(vh, hp, vd, w, w, n, cudaMemcpyDeviceToHost, m->stream));
        }
    }
    CUQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return CUQ_OK;
}

int cuq_kv_write(cuq_model *m, uint32_t layer, uint32_t pos0, uint32_t n, const uint16_t *k_host,
                 const uint16_t *v_host) {
    return kv_copy(m, layer, pos0, n, const_cast<uint16_t *>(k_host), const_cast<uint16_t *>(v_host), true);
}

int cuq_kv_read(const cuq_model *m, uint32_t layer, uint32_t pos0, uint32_t n, uint16_t *k_host, uint16_t *v_host) {
    return kv_copy(m, layer, pos0, n, k_host, v_host, false);
}

int cuq_reset(cuq_model *m) {
    CUQ_CHECK_ARG(m, "cuq_reset: null model");
    // Engine.reset (engine.zig:1479): the cache is simply overwritten from position 0
    // by the next prefill; clearing it keeps stale rows from ever being read.
    size_t kv_bytes = (size_t)m->lc.kv_heads * m->opt.max_seq * m->cfg.head_dim * sizeof(__half);
    for (auto &L : m->layers) {
        CUQ_CUDA_TRY(cudaMemsetAsync(L.k_cache, 0, kv_bytes, m->stream));
        CUQ_CUDA_TRY(cudaMemsetAsync(L.v_cache, 0, kv_bytes, m->stream));
    }
    if (m->tp_buf) {
        // after a call that gave up on a peer: this rank's arrival counters and
        // error flag start from zero again (every rank resets before the next call)
        CUQ_CUDA_TRY(cudaMemsetAsync(m->tp_buf + m->tpc.off_ctr, 0, m->tp_bytes - m->tpc.off_ctr, m->stream));
        CUQ_CUDA_TRY(cudaMemsetAsync(m->tp_err, 0, sizeof(int), m->stream));
        CUQ_CUDA_TRY(cudaMemsetAsync(m->counters, 0, sizeof(unsigned) * m->n_counters, m->stream));
        CUQ_CUDA_TRY(cudaMemsetAsync(m->done, 0, sizeof(unsigned), m->stream));
    }
    CUQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return CUQ_OK;
}

int cuq_model_stats(const cuq_model *m, cuq_stats *out) {
    CUQ_CHECK_ARG(m && out, "cuq_model_stats: null argument");
    *out = m->stats;
    out->persistent_ctas = m->mega.impl ? (uint64_t)m->mega.grid : 0;
    return CUQ_OK;
}

int cuq_profile_decode(cuq_model *m, uint32_t token, uint32_t pos, uint32_t n_steps, cuq_node_time *out) {
    CUQ_CHECK_ARG(m && out && n_steps > 0, "cuq_profile_decode: bad argument");
    if (!m->finalized) {
        set_error("cuq_profile_decode: model not finalized");
        return CUQ_ENOTREADY;
    }
    if (m->mega.impl) {
        set_error("cuq_profile_decode: per-op decode only (not the persistent kernel)");
        return CUQ_EUNSUPPORTED;
    }
    if ((uint64_t)pos + n_steps > m->opt.max_seq) {
        set_error("ContextOverflow: %u + %u > max_seq %u", pos, n_steps, m->opt.max_seq);
        return CUQ_ECONTEXT;
    }
    int rc = check_token(m, token);
    if (rc) return rc;
    CUQ_CUDA_TRY(cudaMemcpyAsync(m->forced, &token, sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
    if ((rc = set_state(m, (int)token, (int)pos, 1))) return rc;
    m->prof_n = 0;
    m->prof_node = -1;
    m->profiling = true;
    rc = prof_mark(m);  // the start of the first launch
    for (uint32_t i = 0; i < n_steps && rc == CUQ_OK; i++) rc = enqueue_step(m);
    m->profiling = false;
    if (rc) {
        cudaStreamSynchronize(m->stream);
        return rc;
    }
    CUQ_CUDA_TRY(cudaStreamSynchronize(m->stream));
    for (int k = 0; k < CUQ_NODES; k++) out[k] = cuq_node_time{0, 0.0, 0.0};
    for (size_t i = 1; i < m->prof_n; i++) {
        float ms = 0.f;
        CUQ_CUDA_TRY(cudaEventElapsedTime(&ms, m->prof_ev[i - 1], m->prof_ev[i]));
        const int k = m->prof_tag[i];
        if (k < 0 || k >= CUQ_NODES) continue;
        out[k].launches++;
        out[k].ms += ms;
    }
    // algorithmic bytes: the weights as stored, and the K/V rows attention reads
    const cuq_config &c = m->cfg, &lc = m->lc;
    double wq = 0, wo = 0, wgu = 0, wd = 0;
    for (auto &L : m->layers) {
        for (auto &sg : L.qkv) wq += (double)sg.p.nbytes;
        wo += (double)L.o.p.nbytes;
        wgu += (double)L.gate.p.nbytes + (double)L.up.p.nbytes;
        wd += (double)L.down.p.nbytes;
    }
    double kv = 0;
    for (uint32_t i = 0; i < n_steps; i++) kv += 2.0 * (pos + i + 1) * kv_dim(lc) * sizeof(__half) * c.layers;
    const double n = n_steps;
    out[CUQ_NODE_EMBED].bytes = n * (double)m->embed.p.nbytes / c.vocab;
    out[CUQ_NODE_QKV].bytes = n * wq;
    out[CUQ_NODE_ATTN].bytes = kv;
    out[CUQ_NODE_O].bytes = n * wo;
    out[CUQ_NODE_GATE_UP].bytes = n * wgu;
    out[CUQ_NODE_DOWN].bytes = n * wd;
    out[CUQ_NODE_HEAD].bytes = n * (double)head_proj(m).p.nbytes;
    m->stats.tokens += n_steps;
    return CUQ_OK;
}

void *cuq_model_stream(const cuq_model *m) { return m ? (void *)m->stream : nullptr; }

void cuq_model_free(cuq_model *m) {
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph_exec) cudaGraphExecDestroy(m->graph_exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    if (m->graph_exec_smp) cudaGraphExecDestroy(m->graph_exec_smp);
    if (m->graph_smp) cudaGraphDestroy(m->graph_smp);
    if (m->smp_host) cudaFreeHost(m->smp_host);
    for (auto &L : m->layers) {
        for (int r = 0; r < 7; r++) free_pending(L.pend[r]);
        for (auto &seg : L.qkv) free_planes(seg.p);
        free_planes(L.o.p);
        free_planes(L.gate.p);
        free_planes(L.up.p);
        free_planes(L.down.p);
        cudaFree(L.attn_norm);
        cudaFree(L.ffn_norm);
        cudaFree(L.qkv_bias);
        cudaFree(L.o_bias);
        cudaFree(L.k_cache);
        cudaFree(L.v_cache);
    }
    free_pending(m->pend_embed);
    free_pending(m->pend_output);
    free_planes(m->embed.p);
    free_planes(m->output.p);
    void *bufs[] = {m->final_norm, m->x,      m->qkv,  m->q_rot,   m->logits,     m->attn_part, m->act,
                    m->gate_buf,   m->up_buf, m->xq_h, m->xq_attn, m->xq_act,     m->rope_cs,   m->ws,
                    m->counters,   m->state,  m->forced, m->out_tokens, m->done, m->tickets,
                    m->pf_x,       m->pf_qkv, m->pf_q, m->pf_g, m->pf_u, m->pf_h, m->pf_l, m->pf_ah, m->pf_al,
                    m->pf_ids,     m->gemm_err, m->tp_err, m->tp_done, m->pf_part, m->pf_wscratch, m->smp, m->ss, m->tp_sink};
    for (void *b : bufs)
        if (b) cudaFree(b);
    for (int r = 0; r < m->tpc.size && m->tp_connected; r++)
        if (r != m->tpc.rank && m->tpc.peer[r] && m->tpc.peer[r] != m->tp_sink) cudaIpcCloseMemHandle(m->tpc.peer[r]);
    if (m->tp_buf) cudaFree(m->tp_buf);
    if (m->state_host) cudaFreeHost(m->state_host);
    if (m->out_host) cudaFreeHost(m->out_host);
    if (m->err_host) cudaFreeHost(m->err_host);
    mega_free(m->mega);
    for (cudaEvent_t e : m->prof_ev) cudaEventDestroy(e);
    if (m->ev0) cudaEventDestroy(m->ev0);
    if (m->ev1) cudaEventDestroy(m->ev1);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

}  // extern "C"
