// mega.h -- host interface of the persistent decode kernel (mega.cu).
//
// A decode step is a fixed program of phases separated by grid-wide barriers:
// per layer the qkv GEMVs, the fused attention, the o GEMV, the gate|up GEMV
// and the down GEMV, then the lm_head.  The persistent kernel runs every step
// of a call in one cooperative launch; each CTA works through its share of
// every phase, waiting at a barrier only before it reads what the previous
// phase wrote (its first weight loads are already in flight by then).  The
// RMSNorm feeding a GEMV is recomputed by every CTA into its own shared memory
// from the residual, so norms cost no phase of their own.
#pragma once

#include <vector>

#include "common.cuh"

namespace cuq {

enum MegaKind : int { MEGA_GEMV = 0, MEGA_ATTN = 1 };

struct MegaSegSpec {     // one GEMV of a phase
    GemvArgs a;          // a.xq is ignored when the phase has a norm; ksplit/ws/counters are chosen by mega_build
    int epi = EPI_STORE; // EPI_STORE, EPI_ADD, EPI_SILU_XQ (a.w2 = up) or EPI_ARGMAX
};

struct MegaAttnSpec {
    const float *qkv = nullptr, *cs = nullptr;
    __half *k_cache = nullptr, *v_cache = nullptr;
    uint32_t cache_stride = 0, heads = 0, kv_heads = 0, hd = 0;
    int adjacent = 0, nsplit = 1;
    __half *xq = nullptr;  // o-projection input
};

struct MegaPhaseSpec {
    int kind = MEGA_GEMV;
    std::vector<MegaSegSpec> segs;  // MEGA_GEMV: 1..3 GEMVs run as one phase
    const float *norm_w = nullptr;  // MEGA_GEMV: input = rmsnorm(x, norm_w), per CTA
    bool embed = false;             // x is the step token's embedding row (first phase of a step)
    MegaAttnSpec attn;              // MEGA_ATTN
};

struct MegaStepSpec {
    std::vector<MegaPhaseSpec> phases;  // the last one is the lm_head (EPI_ARGMAX)
    const Planes *embed = nullptr;
    float *x = nullptr;                 // residual [hidden]
    uint32_t hidden = 0;
    float eps = 0.f;
    StepState *state = nullptr;
    const uint32_t *forced = nullptr;
    uint32_t *out_tokens = nullptr;
};

struct MegaImpl;
struct MegaProgram {
    MegaImpl *impl = nullptr;
    int grid = 0;  // CTAs of the cooperative launch
};

// Why the step cannot run persistently ("" when it can).
std::string mega_unsupported(const MegaStepSpec &spec);
// Upload the step program; ctas_per_sm 0 = as many as fit.
int mega_build(const MegaStepSpec &spec, int sm_count, int ctas_per_sm, MegaProgram &out);
// Run n_steps decode steps (state, forced and out_tokens as the per-op path
// uses them).  A barrier that waits longer than its limit sets the error flag
// and ends the kernel; mega_err_copy queues its read into *err_host.
int mega_launch(MegaProgram &p, uint32_t n_steps, cudaStream_t s);
int mega_err_copy(const MegaProgram &p, int *err_host, cudaStream_t s);
void mega_free(MegaProgram &p);

}  // namespace cuq
