// mega.cu -- the persistent decode kernel (host interface in mega.h).
//
// One cooperative launch runs every decode step of a call: Engine.forward's
// layer loop (engine.zig:547-819) followed by the greedy pick of the next token
// (generate.zig:217-244), for as many steps as the call asks.  The work of a
// phase is cut into units (a 16-row tile group and K part of a GEMV, or a KV
// group and position split of the attention) that CTA b takes as units b,
// b + grid, ...; the GEMV and attention bodies are the ones the per-op kernels
// run (gemv_impl.cuh, attn_impl.cuh).
//
// Grid barrier: one arrival counter, zeroed before the launch.  A CTA arrives
// (__syncthreads, then one release add) when it has finished a phase, and waits
// (acquire loads, then __syncthreads) for gen * grid arrivals before it reads
// anything phase gen wrote; no full fence is taken on the waiting side, so the
// weight loads a CTA issued before waiting need not land first.  Every CTA
// arrives once per phase and waits for each generation before arriving at the
// next, so the count cannot run ahead of a generation.  The wait is bounded by
// %globaltimer: past MEGA_WAIT_NS the CTA sets the error flag and every CTA
// leaves the kernel at its next barrier.
#include <cmath>

#include "attn_impl.cuh"
#include "common.cuh"
#include "dequant_impl.cuh"
#include "gemv_impl.cuh"
#include "mega.h"
#include "tp.cuh"

namespace cuq {

namespace {

constexpr int MEGA_THREADS = 128;
constexpr int MEGA_MAX_SEGS = 3;
constexpr int MEGA_MIN_BLOCKS = 4;  // register cap: 128 per thread
constexpr unsigned long long MEGA_WAIT_NS = 4ull * 1000 * 1000 * 1000;

struct MSeg {
    KArgs k;
    int type, epi;
    uint32_t groups, units;  // 16-row tiles, tiles * ksplit
};

struct MPhase {
    int kind, nseg;
    uint32_t units;
    const float *norm_w;
    int embed;
    MSeg seg[MEGA_MAX_SEGS];
    AttnStepArgs attn;
    int hd, g;
};

struct MArgs {
    const MPhase *ph;
    int nph;
    PlanesView embed;
    int epb;
    float *x;
    uint32_t hidden, kpad;
    float eps;
    StepState *state;
    const uint32_t *forced;
    uint32_t *out_tokens;
    unsigned long long *am;  // [2] packed lm_head argmax, alternating steps
    unsigned int *bar;
    int *err;
    uint32_t n_steps;
};

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool grid_wait(const MArgs &a, unsigned int target) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        if (ld_acquire_gpu(a.bar) < target) {
            const unsigned long long t0 = globaltimer_ns();
            while (ld_acquire_gpu(a.bar) < target) {
                if (*reinterpret_cast<volatile int *>(a.err)) {
                    good = 0;
                    break;
                }
                if (globaltimer_ns() - t0 > MEGA_WAIT_NS) {
                    atomicExch(a.err, 1);
                    good = 0;
                    break;
                }
                __nanosleep(20);
            }
        }
        ok = good;
    }
    __syncthreads();
    return ok != 0;
}

__device__ __forceinline__ void grid_arrive(const MArgs &a) {
    __syncthreads();
    if (threadIdx.x == 0) {
        // release: this CTA's writes (ordered before by __syncthreads) are visible
        // to whoever acquires the count
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
    }
}

// One GEMV unit.  Each (type, epilogue) body is a separate function so that
// register allocation sees one body at a time.
template <class TT, int EPI, int KW, class BX>
__device__ __noinline__ void mega_unit(const KArgs *gk, const __half *xq, const float *xsum, unsigned long long *am,
                                       uint32_t bx, uint32_t by, GemvShared &sh, BX &bxf) {
    KArgs k = *gk;
    if (xq) {
        k.xq = xq;
        k.xsum = xsum;
    }
    if (am) k.argmax64 = am;
    gemv_body<TT, EPI, KW, TT::DEPTH>(k, bx, by, sh, bxf);
}

template <class BX>
__device__ __forceinline__ void mega_gemv(const KArgs *gk, int type, int epi, const __half *xq, const float *xsum,
                                          unsigned long long *am, uint32_t bx, uint32_t by, GemvShared &sh, BX &bxf) {
#define MG_EPI(TT)                                                                              \
    switch (epi) {                                                                              \
    case EPI_STORE: mega_unit<TT, EPI_STORE, 4>(gk, xq, xsum, am, bx, by, sh, bxf); break;      \
    case EPI_ADD: mega_unit<TT, EPI_ADD, 4>(gk, xq, xsum, am, bx, by, sh, bxf); break;          \
    case EPI_SILU_XQ: mega_unit<TT, EPI_SILU_XQ, 2>(gk, xq, xsum, am, bx, by, sh, bxf); break;  \
    default: mega_unit<TT, EPI_ARGMAX, 4>(gk, xq, xsum, am, bx, by, sh, bxf); break;            \
    }
    switch (type) {
    case CUQ_Q8_0: MG_EPI(TQ8_0) break;
    case CUQ_Q4_0: MG_EPI(TQ4L<CUQ_Q4_0>) break;
    case CUQ_Q4_1: MG_EPI(TQ4L<CUQ_Q4_1>) break;
    case CUQ_Q5_0: MG_EPI(TQ4L<CUQ_Q5_0>) break;
    case CUQ_Q5_1: MG_EPI(TQ4L<CUQ_Q5_1>) break;
    case CUQ_Q4_K: MG_EPI(TQ4K) break;
    case CUQ_Q6_K: MG_EPI(TQ6K) break;
    case CUQ_F16: MG_EPI(T16<CUQ_F16>) break;
    default: MG_EPI(T16<CUQ_BF16>) break;
    }
#undef MG_EPI
}

template <int HD, int G>
__device__ __noinline__ void mega_attn_unit(const AttnStepArgs *a, uint32_t kvh, uint32_t split, uint32_t pos,
                                            float *scr) {
    attn_step_body<HD, G>(*a, kvh, split, pos, scr);
}

__device__ __forceinline__ void mega_attn(const MPhase &P, uint32_t kvh, uint32_t split, uint32_t pos, float *scr) {
#define MA(HDV, GV) \
    case HDV * 16 + GV: mega_attn_unit<HDV, GV>(&P.attn, kvh, split, pos, scr); break;
    switch (P.hd * 16 + P.g) {
        MA(64, 1) MA(64, 2) MA(64, 3) MA(64, 4) MA(64, 6) MA(64, 7) MA(64, 8)
        MA(128, 1) MA(128, 2) MA(128, 3) MA(128, 4) MA(128, 6) MA(128, 7) MA(128, 8)
    default: break;
    }
#undef MA
}

__global__ void __launch_bounds__(MEGA_THREADS, MEGA_MIN_BLOCKS) decode_persistent_kernel(const MArgs a) {
    extern __shared__ float4 dsm[];
    __shared__ GemvShared sh;
    float4 *stage = dsm;                                         // residual row, hidden floats
    __half *sxq = reinterpret_cast<__half *>(dsm + a.hidden / 4);  // its RMSNorm in xq form
    const float *sxs = xq_sums(sxq, a.kpad);
    float *scr = reinterpret_cast<float *>(dsm);                 // attention phases reuse the region
    const unsigned int G = gridDim.x;
    uint32_t token = (uint32_t)a.state->token, pos = (uint32_t)a.state->pos;
    const int step0 = a.state->step, n_forced = a.state->n_forced;
    unsigned int arrived = 0, passed = 0;  // barrier generations arrived at / waited for
    bool ok = true;

    for (uint32_t s = 0; s < a.n_steps; s++) {
        for (int ph = 0; ph < a.nph; ph++) {
            const MPhase &P = a.ph[ph];
            const bool has_units = blockIdx.x < P.units;
            bool ready = false;
            // Wait for the previous phase, then (GEMV phases with a norm) build
            // the input: xq = split(rmsnorm(x)) in shared memory.
            auto before_x = [&]() {
                if (ready) return;
                ready = true;
                if (arrived > passed) {
                    ok = grid_wait(a, arrived * G);
                    passed = arrived;
                }
                if (!P.norm_w || !ok) return;
                if (P.embed) {
                    // the step's token embedding (engine.zig:561-564); CTA 0 also stores it as x
                    if (!has_units && blockIdx.x != 0) return;
                    embed_row_block(a.embed, token, reinterpret_cast<float *>(stage), a.epb);
                    __syncthreads();
                    float ss = 0.f;
                    for (uint32_t i4 = threadIdx.x; i4 < a.hidden / 4; i4 += blockDim.x) {
                        const float4 v = stage[i4];
                        ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
                        if (blockIdx.x == 0) reinterpret_cast<float4 *>(a.x)[i4] = v;
                    }
                    stage_norm_xq(stage, ss, P.norm_w, a.hidden, a.eps, sxq, a.kpad);
                } else {
                    if (!has_units) return;
                    reduce_norm_xq_block(a.x, nullptr, 0, nullptr, P.norm_w, a.hidden, a.eps, sxq, a.kpad, stage);
                }
                __syncthreads();
            };
            if (P.kind == MEGA_GEMV) {
                for (uint32_t u = blockIdx.x; u < P.units; u += G) {
                    uint32_t uu = u;
                    int si = 0;
                    while (si + 1 < P.nseg && uu >= P.seg[si].units) {
                        uu -= P.seg[si].units;
                        si++;
                    }
                    const MSeg &S = P.seg[si];
                    const int type = S.type, epi = S.epi;
                    const uint32_t groups = S.groups;
                    mega_gemv(&S.k, type, epi, P.norm_w ? sxq : nullptr, sxs,
                              epi == EPI_ARGMAX ? a.am + (s & 1u) : nullptr, uu % groups, uu / groups, sh,
                              before_x);
                    __syncthreads();  // the body's shared reduction buffers are reused by the next unit
                }
            } else {
                for (uint32_t u = blockIdx.x; u < P.units; u += G) {
                    before_x();
                    mega_attn(P, u % P.attn.kv_heads, u / P.attn.kv_heads, pos, scr);
                    __syncthreads();
                }
            }
            before_x();  // a CTA without units still waits before it arrives
            if (!ok) return;
            grid_arrive(a);
            arrived++;
        }
        // End of the step: the lm_head phase's argmax is complete once every
        // CTA has arrived; every CTA derives the next token itself.
        ok = grid_wait(a, arrived * G);
        passed = arrived;
        if (!ok) return;
        const unsigned long long key = __ldcg(a.am + (s & 1u));
        const uint32_t idx = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
        const int sidx = step0 + (int)s;
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            a.out_tokens[sidx] = idx;
            a.am[(s + 1u) & 1u] = 0ull;  // last read at the end of the previous step
        }
        token = (sidx + 1 < n_forced) ? a.forced[sidx + 1] : idx;
        pos++;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        a.state->token = (int)token;
        a.state->pos = (int)pos;
        a.state->step = step0 + (int)a.n_steps;
        a.state->argmax64 = 0ull;
    }
}

int span_of(int type) {
    switch (type) {
    case CUQ_Q8_0: case CUQ_F16: case CUQ_BF16: return 64;
    case CUQ_Q4_K: case CUQ_Q6_K: return 256;
    default: return 128;
    }
}

bool attn_combo_ok(uint32_t hd, uint32_t g) {
    return (hd == 64 || hd == 128) && g >= 1 && g <= 8 && g != 5;
}

size_t round256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace

struct MegaImpl {
    MPhase *d_phases = nullptr;
    uint8_t *scratch = nullptr;
    size_t zero_bytes = 0;
    size_t smem = 0;
    MArgs args{};
};

std::string mega_unsupported(const MegaStepSpec &sp) {
    if (!sp.embed || !sp.x || !sp.state || !sp.forced || !sp.out_tokens) return "incomplete step description";
    if (sp.hidden == 0 || sp.hidden % 16 || sp.hidden > RN_MAX) return "hidden must be a multiple of 16, <= 8192";
    if (block_elems(sp.embed->type) == 0 || sp.embed->cols != sp.hidden) return "embedding table";
    if (sp.phases.empty() || sp.phases.back().kind != MEGA_GEMV || sp.phases.back().segs.size() != 1 ||
        sp.phases.back().segs[0].epi != EPI_ARGMAX)
        return "the last phase must be the lm_head";
    for (const MegaPhaseSpec &p : sp.phases) {
        if (p.kind == MEGA_ATTN) {
            const MegaAttnSpec &t = p.attn;
            if (t.kv_heads == 0 || t.heads % t.kv_heads || !attn_combo_ok(t.hd, t.heads / t.kv_heads))
                return "attention head_dim / group";
            if (t.nsplit < 1 || t.nsplit > ATT_MAX_SPLIT) return "attention split count";
            continue;
        }
        if (p.segs.empty() || p.segs.size() > (size_t)MEGA_MAX_SEGS) return "GEMV phase with 1-3 projections";
        if (p.embed && !p.norm_w) return "embedding phase without a norm";
        for (const MegaSegSpec &g : p.segs) {
            const Planes &w = *g.a.w;
            if (!planes_fast_type(w.type)) return "projection type without a register decoder";
            if (w.rows == 0 || w.rows % 16) return "projection rows not a multiple of 16";
            if ((w.type == CUQ_F16 || w.type == CUQ_BF16) && w.cols % 16) return "16-bit projection cols";
            if (p.norm_w && w.cols != sp.hidden) return "normed projection input must be the residual";
            if (g.epi == EPI_SILU_XQ &&
                (!g.a.w2 || g.a.w2->type != w.type || g.a.w2->rows != w.rows || g.a.w2->cols != w.cols))
                return "gate/up of different type or shape";
            if (g.epi != EPI_STORE && g.epi != EPI_ADD && g.epi != EPI_SILU_XQ && g.epi != EPI_ARGMAX)
                return "epilogue";
        }
    }
    return "";
}

int mega_build(const MegaStepSpec &sp, int sm_count, int ctas_per_sm, MegaProgram &out) {
    const std::string why = mega_unsupported(sp);
    if (!why.empty()) {
        set_error("persistent decode: %s", why.c_str());
        return CUQ_EUNSUPPORTED;
    }
    mega_free(out);
    // shared memory: the residual stage + its xq, or the largest attention scratch
    const uint32_t kpad = xq_pad(sp.hidden);
    size_t smem = sizeof(float) * sp.hidden + sizeof(__half) * xq_halves(sp.hidden);
    for (const MegaPhaseSpec &p : sp.phases)
        if (p.kind == MEGA_ATTN) {
            const uint32_t g = p.attn.heads / p.attn.kv_heads;
            const size_t need = sizeof(float) * (size_t)attn_step_floats((int)p.attn.hd, (int)g);
            if (need > smem) smem = need;
        }
    smem = (smem + 15) & ~(size_t)15;
    CUQ_CUDA_TRY(cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    int per_sm = 0;
    CUQ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent_kernel, MEGA_THREADS, smem));
    if (per_sm < 1) {
        set_error("persistent decode: kernel does not fit on an SM (%zu B shared memory)", smem);
        return CUQ_EUNSUPPORTED;
    }
    if (ctas_per_sm > 0 && ctas_per_sm < per_sm) per_sm = ctas_per_sm;
    const int grid = sm_count * per_sm;

    // phases, with split-K chosen so a phase's units fill the grid evenly
    std::vector<MPhase> ph(sp.phases.size());
    size_t max_counters = 0, max_ws = 0, part_floats = 0;
    uint32_t max_kv = 0;
    for (size_t i = 0; i < sp.phases.size(); i++) {
        const MegaPhaseSpec &p = sp.phases[i];
        MPhase &d = ph[i];
        d.kind = p.kind;
        d.norm_w = p.norm_w;
        d.embed = p.embed ? 1 : 0;
        if (p.kind == MEGA_ATTN) {
            const MegaAttnSpec &t = p.attn;
            d.attn = AttnStepArgs{t.qkv, t.cs, nullptr, t.k_cache, t.v_cache, t.cache_stride, t.heads, t.kv_heads,
                                  t.adjacent, t.nsplit, nullptr, nullptr, t.xq};
            d.hd = (int)t.hd;
            d.g = (int)(t.heads / t.kv_heads);
            d.units = t.kv_heads * (uint32_t)t.nsplit;
            if (t.kv_heads > max_kv) max_kv = t.kv_heads;
            const size_t pf = (size_t)t.nsplit * t.heads * (t.hd + 2);
            if (pf > part_floats) part_floats = pf;
            continue;
        }
        // the phase's tiles, and the fewest K iterations any of its GEMVs has per warp
        uint32_t tiles = 0;
        int kmax = 16;
        for (const MegaSegSpec &g : p.segs) {
            tiles += g.a.w->rows / 16;
            const int ni = (int)((g.a.w->cols + span_of(g.a.w->type) - 1) / span_of(g.a.w->type));
            const int kwe = g.epi == EPI_SILU_XQ ? 2 : 4;
            const int km = ni / (2 * kwe);  // keep >= 2 iterations per warp
            if (km < kmax) kmax = km;
        }
        if (kmax < 1) kmax = 1;
        int ks = 1;
        double best = -1.0;
        for (int k = 1; k <= kmax; k++) {
            const double units = (double)tiles * k;
            const double rounds = std::ceil(units / grid);
            const double eff = units / (rounds * grid);
            if (eff > best + 0.05) {  // a larger split must pay for its partial traffic
                best = eff;
                ks = k;
            }
            if (eff >= 0.9) break;
        }
        d.nseg = (int)p.segs.size();
        size_t cbase = 0, wbase = 0;
        for (size_t j = 0; j < p.segs.size(); j++) {
            const MegaSegSpec &g = p.segs[j];
            MSeg &m = d.seg[j];
            GemvArgs a = g.a;
            a.ksplit = ks;
            a.pdl = false;
            a.post = GemvPost();
            m.k = make_kargs(a);
            m.type = g.a.w->type;
            m.epi = g.epi;
            m.groups = g.a.w->rows / 16;
            m.units = m.groups * (uint32_t)ks;
            d.units += m.units;
            // ws / counters are filled in once the scratch is allocated: record offsets
            m.k.counters = reinterpret_cast<unsigned int *>(cbase);
            m.k.ws = reinterpret_cast<float *>(wbase);
            cbase += m.groups;
            wbase += (size_t)ks * g.a.w->rows * (g.epi == EPI_SILU_XQ ? 2 : 1);
        }
        if (cbase > max_counters) max_counters = cbase;
        if (wbase > max_ws) max_ws = wbase;
    }
    // scratch: [bar | err | am[2] | counters | tickets] (zeroed per launch), ws, part
    const size_t off_counters = 64;
    const size_t off_tickets = off_counters + sizeof(unsigned int) * max_counters;
    const size_t zero_bytes = round256(off_tickets + sizeof(unsigned int) * max_kv);
    const size_t off_ws = zero_bytes;
    const size_t off_part = round256(off_ws + sizeof(float) * max_ws);
    const size_t total = round256(off_part + sizeof(float) * part_floats);
    MegaImpl *im = new MegaImpl();
    out.impl = im;
    cudaError_t e = cudaMalloc(&im->scratch, total);
    if (e == cudaSuccess) e = cudaMemset(im->scratch, 0, total);
    if (e != cudaSuccess) {
        mega_free(out);
        set_error("persistent decode scratch: %s", cudaGetErrorString(e));
        return CUQ_ENOMEM;
    }
    uint8_t *S = im->scratch;
    for (MPhase &d : ph) {
        if (d.kind == MEGA_ATTN) {
            d.attn.part = reinterpret_cast<float *>(S + off_part);
            d.attn.tickets = reinterpret_cast<unsigned int *>(S + off_tickets);
            continue;
        }
        for (int j = 0; j < d.nseg; j++) {
            KArgs &k = d.seg[j].k;
            k.counters = reinterpret_cast<unsigned int *>(S + off_counters) + reinterpret_cast<size_t>(k.counters);
            k.ws = reinterpret_cast<float *>(S + off_ws) + reinterpret_cast<size_t>(k.ws);
        }
    }
    e = cudaMalloc(&im->d_phases, sizeof(MPhase) * ph.size());
    if (e == cudaSuccess) e = cudaMemcpy(im->d_phases, ph.data(), sizeof(MPhase) * ph.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        mega_free(out);
        set_error("persistent decode program: %s", cudaGetErrorString(e));
        return CUQ_ENOMEM;
    }
    im->zero_bytes = zero_bytes;
    im->smem = smem;
    MArgs &A = im->args;
    A.ph = im->d_phases;
    A.nph = (int)ph.size();
    const Planes &E = *sp.embed;
    A.embed = PlanesView{E.type, E.rows, E.cols, E.base, E.off_q, E.off_q2, E.off_s, E.off_s2};
    A.epb = block_elems(E.type);
    A.x = sp.x;
    A.hidden = sp.hidden;
    A.kpad = kpad;
    A.eps = sp.eps;
    A.state = sp.state;
    A.forced = sp.forced;
    A.out_tokens = sp.out_tokens;
    A.bar = reinterpret_cast<unsigned int *>(S);
    A.err = reinterpret_cast<int *>(S + 4);
    A.am = reinterpret_cast<unsigned long long *>(S + 8);
    out.grid = grid;
    return CUQ_OK;
}

int mega_launch(MegaProgram &p, uint32_t n_steps, cudaStream_t s) {
    if (!p.impl) {
        set_error("persistent decode: no program");
        return CUQ_EINVAL;
    }
    if (n_steps == 0) return CUQ_OK;
    MegaImpl &im = *p.impl;
    CUQ_CUDA_TRY(cudaMemsetAsync(im.scratch, 0, im.zero_bytes, s));
    MArgs a = im.args;
    a.n_steps = n_steps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(MEGA_THREADS);
    cfg.dynamicSmemBytes = im.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, decode_persistent_kernel, a);
    if (e != cudaSuccess) {
        set_error("persistent decode launch: %s", cudaGetErrorString(e));
        return CUQ_ECUDA;
    }
    return CUQ_OK;
}

int mega_err_copy(const MegaProgram &p, int *err_host, cudaStream_t s) {
    if (!p.impl) return CUQ_OK;
    CUQ_CUDA_TRY(cudaMemcpyAsync(err_host, p.impl->args.err, sizeof(int), cudaMemcpyDeviceToHost, s));
    return CUQ_OK;
}

void mega_free(MegaProgram &p) {
    if (!p.impl) return;
    if (p.impl->d_phases) cudaFree(p.impl->d_phases);
    if (p.impl->scratch) cudaFree(p.impl->scratch);
    delete p.impl;
    p.impl = nullptr;
    p.grid = 0;
}

}  // namespace cuq
