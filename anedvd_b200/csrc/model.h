// model.h -- the device-resident engine behind cuq_model_* (include/cuq.h).
#pragma once

#include <vector>

#include "common.cuh"
#include "mega.h"
#include "sample.cuh"

namespace cuq {

// One linear projection, possibly the row-concatenation of several GGUF
// tensors of the same type (q||k||v like load_gguf.zig:677-682).
struct Proj {
    Planes p;
    uint32_t row_off = 0;  // first output row inside the destination vector
};

struct PendingTensor {
    int type = -1;
    uint32_t rows = 0, cols = 0;
    uint8_t *raw = nullptr;  // device staging copy of the GGUF payload
    size_t nbytes = 0;
};

struct Layer {
    PendingTensor pend[7];      // q k v o gate up down, until finalize
    std::vector<Proj> qkv;      // 1..3 segments writing into the qkv vector
    Proj o, gate, up, down;
    bool gate_up_dual = false;  // same type/shape: one dual GEMV with the SiLU epilogue
    float *attn_norm = nullptr, *ffn_norm = nullptr, *qkv_bias = nullptr, *o_bias = nullptr;
    __half *k_cache = nullptr, *v_cache = nullptr;  // [kv_heads][max_seq][head_dim]
};

}  // namespace cuq

struct cuq_model {
    cuq_config cfg{};
    cuq_config lc{};             // this rank's geometry: heads, kv_heads, inter, vocab divided by tp_size
    uint32_t vocab_base = 0;     // first lm_head row (global token id) held by this rank
    cuq_options opt{};
    bool finalized = false;
    bool use_tma = false;        // the decode GEMVs may run the TMA-fed kernels (large models)
    bool all_tma = false;        // every decode GEMV runs the TMA-fed kernel
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    std::vector<cuq::Layer> layers;
    cuq::PendingTensor pend_embed, pend_output;
    cuq::Proj embed, output;     // output unused when tied
    float *final_norm = nullptr;

    // activations
    float *x = nullptr, *qkv = nullptr, *q_rot = nullptr, *logits = nullptr, *attn_part = nullptr, *act = nullptr;
    float *gate_buf = nullptr, *up_buf = nullptr;
    __half *xq_h = nullptr, *xq_attn = nullptr, *xq_act = nullptr;
    float *rope_cs = nullptr;                    // [max_seq][head_dim]
    float *ws = nullptr;                         // split-K partials
    unsigned int *counters = nullptr;
    unsigned int *done = nullptr;                // GEMV grid-completion counter (post-ops)
    float *ss = nullptr;                         // [2][hidden/16] per-tile sums of squares of the residual
    unsigned int *tickets = nullptr;             // attention combine tickets, one per KV head
    size_t ws_floats = 0, n_counters = 0;
    int attn_nsplit = 1;
    cuq::StepState *state = nullptr;             // device
    cuq::StepState *state_host = nullptr;        // pinned
    uint32_t *forced = nullptr, *out_tokens = nullptr;  // device, [max_seq]
    uint32_t *out_host = nullptr;                // pinned [max_seq]

    // batched prefill (chunks of opt.max_chunk tokens)
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_g = nullptr, *pf_u = nullptr;
    __half *pf_h = nullptr, *pf_l = nullptr, *pf_ah = nullptr, *pf_al = nullptr;
    uint32_t *pf_ids = nullptr;
    __half *pf_wscratch = nullptr;               // fp16 expansion of a raw-block weight (its prefill GEMM)
    int *gemm_err = nullptr;

    // tensor parallelism (opt.tp_size > 1)
    uint8_t *tp_buf = nullptr;                   // this rank's communication buffer (IPC-exported)
    uint8_t *tp_sink = nullptr;                  // stands in for the buffer of a rank that never joins
    size_t tp_bytes = 0;
    cuq::TpComm tpc;                             // peers mapped by cuq_tp_connect
    bool tp_connected = false;
    int *tp_err = nullptr;                       // wait time-outs (device)
    unsigned int *tp_done = nullptr;             // grid completion of the prefill reduce kernel
    float *pf_part = nullptr;                    // [max_chunk][hidden] partial of o / down

    cuq::MegaProgram mega;                       // persistent decode kernel (decode_kernel != PER_OP)
    bool mega_ran = false;                       // launched since the last finish_call
    int *err_host = nullptr;                     // pinned: its error flag read back by finish_call

    // cuq_profile_decode: an event after every launch, tagged with its node
    bool profiling = false;
    int prof_node = 0;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_tag;
    size_t prof_n = 0;

    // sampled decoding (cuq_generate_sampled): parameters, LCG state and the
    // penalty window on the device, staged from pinned memory once per call
    cuq::SampleState *smp = nullptr;             // device
    cuq::SampleState *smp_host = nullptr;        // pinned
    cudaGraph_t graph_smp = nullptr;             // decode step + draw
    cudaGraphExec_t graph_exec_smp = nullptr;

    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cuq_stats stats{};
};
