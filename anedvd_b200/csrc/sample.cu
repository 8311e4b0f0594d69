// sample.cu -- the token sampler of Session.generate on the device:
// cpu.applyPenalties (src/cpu.zig:529-547) and cpu.sampleProfiled
// (src/cpu.zig:621-721) -- repetition / presence / frequency penalties,
// greedy for a non-positive temperature, the min_keep_delta cut, top-k,
// probabilities, top-p and the LCG draw.
//
// One draw is one thread-block cluster of 8 CTAs x 512 threads.  CTA r keeps
// the logits [r*S, r*S + S) in its shared memory (S = vocab / 8, rounded up to
// a multiple of 4), so after the one coalesced read every pass over the
// vocabulary is on chip; the CTAs combine their partial results (maxima,
// counts, histograms, prefix sums) through distributed shared memory, with the
// cluster barrier between the steps.  Nothing here waits on a flag.
//
// Order.  The reference draws from its candidates in one of two orders:
// descending (after selectTopK, or the top-p sort) or vocabulary order (no
// top-k, no top-p).  Descending means "logit descending, equal logits by
// index", which is the order of the 64-bit key (orderable logit bits << 32 |
// ~index).  Positions in that order are found without sorting the whole
// vocabulary: a histogram of the values over 2048 equal-width bins between the
// current bounds finds the bin where the running weight (a count for top-k,
// probability mass for top-p and the draw) crosses the target; a bin small
// enough (<= 4096 entries) is gathered into CTA 0, sorted there and walked,
// a larger one narrows the bounds to its own minimum and maximum for the next
// pass; equal values resolve by index with a prefix sum over the CTAs.
//
// Exactness.  With top-k active and k <= 4096 (the reference's default
// sampler is temperature 0.7, top_k 40) the k kept entries are gathered into
// CTA 0 in the reference's order and one thread repeats the reference's fp32
// arithmetic step by step (probabilities, their sum, the top-p accumulation,
// r * sum and the walk): the token equals the reference's unless expf rounds a
// probability differently.  Otherwise probability mass is summed in 64-bit
// fixed point (2^-40 units), which is order-independent and deterministic but
// rounds differently from the reference's sequential fp32 sums; the drawn token
// then differs from the reference's only when the draw lands within that
// rounding of a boundary between two tokens.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "sample.cuh"

namespace cg = cooperative_groups;

namespace cuq {
namespace {

constexpr int CL = 8;                  // CTAs per cluster (the portable maximum)
constexpr int NT = 512;                // threads per CTA
constexpr int NW = NT / 32;
constexpr int NB = 2048;               // value bins per histogram pass
constexpr int BPT = NB / NT;           // bins per thread
constexpr uint32_t LMAX = 4096;        // entries CTA 0 gathers and sorts
constexpr int EPT = LMAX / NT;         // gathered entries per thread
constexpr double WUNIT = 1099511627776.0;  // 2^40: fixed-point unit of probability mass
typedef unsigned long long u64;

static_assert(SAMPLE_MAX_WINDOW <= 2 * LMAX, "window ids share the gather list");
static_assert(SAMPLE_MAX_VOCAB % (4 * CL) == 0, "slice bound");

struct Smem {
    u64 list[LMAX];        // CTA 0: gathered keys.  Every CTA: its slice's window ids (as u32) first
    u64 hmass[NB];         // histogram: probability mass per bin (fixed point)
    uint32_t hcnt[NB];     // histogram: entries per bin
    u64 red[NW];           // block reductions and scans
    u64 slot[2];           // this CTA's partial of a cluster reduction (double buffered)
    u64 gather[CL];        // the CTAs' partials, read back
    u64 res[3];            // CTA 0: result of a search (key, weight before, weight through)
    u64 bsel[2];           // search: weight above the chosen bin, its entry count
    uint32_t list_n;       // CTA 0: entries gathered
    uint32_t wl_n;         // window ids of this slice
};
constexpr size_t SMEM_HDR = (sizeof(Smem) + 15) & ~(size_t)15;

struct Found {
    u64 key, before, through;
    bool ok;
};

struct Ctx {
    Smem *sh;
    float *sv;            // this CTA's slice of the logits
    uint32_t rank, base, cnt;
    uint32_t c0, c1;      // this thread's contiguous range of the slice
    int phase;            // cluster-reduction buffer parity
    float maxv, T, cut;
    u64 lo_key;           // entries below this key are out of the kept set (0: none)
};

__device__ __forceinline__ uint32_t ord32(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord32(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
__device__ __forceinline__ u64 key64(float v, uint32_t idx) {
    return ((u64)ord32(v) << 32) | (u64)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ float key_val(u64 k) { return unord32((uint32_t)(k >> 32)); }
__device__ __forceinline__ uint32_t key_idx(u64 k) { return 0xFFFFFFFFu - (uint32_t)k; }

// exp((v - max) / T) in the reference's order of operations (cpu.zig:678)
__device__ __forceinline__ float prob(float v, float maxv, float T) {
    return expf(__fdiv_rn(__fsub_rn(v, maxv), T));
}
__device__ __forceinline__ u64 weight(bool mass, float v, const Ctx &x) {
    if (!mass) return 1ull;
    return __double2ull_rn((double)prob(v, x.maxv, x.T) * WUNIT);
}
__device__ __forceinline__ bool in_set(const Ctx &x, float v, uint32_t gi) {
    return v >= x.cut && key64(v, gi) >= x.lo_key;   // false for NaN
}
// The histogram bin of v between lo and lo + NB/scale: monotone in v (every
// step is a correctly rounded double operation), so bins split the order.
__device__ __forceinline__ int bin_of(float v, double dlo, double scale) {
    const int b = (int)(((double)v - dlo) * scale);
    return b < NB - 1 ? b : NB - 1;
}

enum { OP_SUM = 0, OP_MAX = 1, OP_MIN = 2 };
template <int OP>
__device__ __forceinline__ u64 op2(u64 a, u64 b) {
    if (OP == OP_SUM) return a + b;
    if (OP == OP_MAX) return a > b ? a : b;
    return a < b ? a : b;
}

template <int OP>
__device__ u64 block_reduce(Smem &sh, u64 v) {
    for (int o = 16; o; o >>= 1) v = op2<OP>(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    __syncthreads();  // red[] is free
    if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
    __syncthreads();
    u64 r = sh.red[0];
    for (int w = 1; w < NW; w++) r = op2<OP>(r, sh.red[w]);
    return r;
}

// Exclusive prefix sum over the CTA's threads (thread order); *total = CTA sum.
__device__ u64 block_excl_scan(Smem &sh, u64 v, u64 *total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    u64 inc = v;
    for (int o = 1; o < 32; o <<= 1) {
        const u64 y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += y;
    }
    __syncthreads();
    if (lane == 31) sh.red[w] = inc;
    __syncthreads();
    u64 ex = 0, tot = 0;
    for (int j = 0; j < NW; j++) {
        const u64 s = sh.red[j];
        if (j < w) ex += s;
        tot += s;
    }
    *total = tot;
    return ex + inc - v;
}

// Publish this CTA's value and read every CTA's back into gather[] (one
// cluster barrier; the slot alternates so the next reduction may write while a
// slow CTA still reads this one).
__device__ void cluster_gather(Ctx &x, u64 cta_value) {
    Smem &sh = *x.sh;
    cg::cluster_group cl = cg::this_cluster();
    const int ph = x.phase++ & 1;
    if (threadIdx.x == 0) sh.slot[ph] = cta_value;
    cl.sync();
    if (threadIdx.x < CL) sh.gather[threadIdx.x] = *cl.map_shared_rank(&sh.slot[ph], (unsigned)threadIdx.x);
    __syncthreads();
}

template <int OP>
__device__ u64 cluster_reduce(Ctx &x, u64 v) {
    cluster_gather(x, block_reduce<OP>(*x.sh, v));
    u64 r = x.sh->gather[0];
    for (int j = 1; j < CL; j++) r = op2<OP>(r, x.sh->gather[j]);
    return r;
}

// Bitonic sort of a[0..n) (n <= LMAX), descending, by the CTA's threads.
__device__ void sort_desc(u64 *a, uint32_t n) {
    uint32_t n2 = 2;
    while (n2 < n) n2 <<= 1;
    for (uint32_t i = n + threadIdx.x; i < n2; i += NT) a[i] = 0ull;
    __syncthreads();
    for (uint32_t k = 2; k <= n2; k <<= 1)
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            for (uint32_t i = threadIdx.x; i < n2; i += NT) {
                const uint32_t ixj = i ^ j;
                if (ixj > i) {
                    const u64 A = a[i], B = a[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (A < B) : (A > B)) {
                        a[i] = B;
                        a[ixj] = A;
                    }
                }
            }
            __syncthreads();
        }
}

// Every CTA reads CTA 0's search result (written before the caller's last
// cluster barrier).  CTA 0 rewrites res only after at least one more cluster
// barrier, which every CTA reaches after this read.
__device__ Found read_result(Ctx &x) {
    cg::cluster_group cl = cg::this_cluster();
    if (threadIdx.x < 3) x.sh->gather[threadIdx.x] = *cl.map_shared_rank(&x.sh->res[threadIdx.x], 0u);
    __syncthreads();
    Found f;
    f.key = x.sh->gather[0];
    f.before = x.sh->gather[1];
    f.through = x.sh->gather[2];
    f.ok = f.key != 0ull;
    __syncthreads();
    return f;
}

// The first entry in vocabulary order among those with `pred` (the kept set,
// and for ties the value tie_v) whose running weight, starting from `above`,
// reaches W.
__device__ __noinline__ Found search_index(Ctx &x, bool mass, u64 W, u64 above, bool tie, float tie_v) {
    Smem &sh = *x.sh;
    cg::cluster_group cl = cg::this_cluster();
    auto pred = [&](float v, uint32_t i) { return in_set(x, v, x.base + i) && (!tie || v == tie_v); };
    u64 s = 0;
    for (uint32_t i = x.c0; i < x.c1; i++) {
        const float v = x.sv[i];
        if (pred(v, i)) s += weight(mass, v, x);
    }
    u64 btot;
    const u64 ex = block_excl_scan(sh, s, &btot);
    cluster_gather(x, btot);
    u64 cex = 0;
    for (uint32_t j = 0; j < x.rank; j++) cex += sh.gather[j];
    u64 mine = ~0ull, b0 = 0, b1 = 0;
    u64 acc = above + cex + ex;
    if (s > 0 && acc + s >= W) {
        for (uint32_t i = x.c0; i < x.c1; i++) {
            const float v = x.sv[i];
            if (!pred(v, i)) continue;
            const u64 w = weight(mass, v, x);
            if (acc + w >= W) {
                mine = x.base + i;
                b0 = acc;
                b1 = acc + w;
                break;
            }
            acc += w;
        }
    }
    const u64 first = cluster_reduce<OP_MIN>(x, mine);
    if (first == ~0ull) return Found{0, 0, 0, false};
    if (mine == first) {
        // the owner publishes the entry into CTA 0
        u64 *r = cl.map_shared_rank(&sh.res[0], 0u);
        r[0] = key64(x.sv[first - x.base], (uint32_t)first);
        r[1] = b0;
        r[2] = b1;
    }
    if (x.rank == 0 && threadIdx.x == 0) sh.list_n = 0;
    cl.sync();
    return read_result(x);
}

// The first entry in descending key order among the kept set whose running
// weight reaches W (see the top of the file).
__device__ __noinline__ Found search_sorted(Ctx &x, bool mass, u64 W) {
    Smem &sh = *x.sh;
    cg::cluster_group cl = cg::this_cluster();
    const int t = threadIdx.x;
    float lo = x.cut, hi = x.maxv;
    if (x.lo_key) lo = fmaxf(lo, key_val(x.lo_key));
    u64 above = 0;
    for (int it = 0; it < 24 && lo < hi; it++) {
        const double dlo = lo, scale = (double)NB / ((double)hi - dlo);
        for (int b = t; b < NB; b += NT) {
            sh.hcnt[b] = 0u;
            sh.hmass[b] = 0ull;
        }
        __syncthreads();
        for (uint32_t i = x.c0; i < x.c1; i++) {
            const float v = x.sv[i];
            if (!(v >= lo && v <= hi) || !in_set(x, v, x.base + i)) continue;
            const int b = bin_of(v, dlo, scale);
            atomicAdd(&sh.hcnt[b], 1u);
            if (mass) atomicAdd(&sh.hmass[b], weight(true, v, x));
        }
        cl.sync();  // every CTA's histogram is complete
        // thread t owns bins NB-1-BPT*t ... NB-BPT*(t+1): thread order is descending bin order
        uint32_t c[BPT];
        u64 w[BPT], wsum = 0;
        for (int j = 0; j < BPT; j++) {
            const int b = NB - 1 - BPT * t - j;
            uint32_t cc = 0;
            u64 ww = 0;
            for (unsigned r = 0; r < CL; r++) {
                cc += *cl.map_shared_rank(&sh.hcnt[b], r);
                if (mass) ww += *cl.map_shared_rank(&sh.hmass[b], r);
            }
            c[j] = cc;
            w[j] = mass ? ww : (u64)cc;
            wsum += w[j];
        }
        cl.sync();  // every CTA has read every histogram
        u64 tot;
        u64 ex = above + block_excl_scan(sh, wsum, &tot);
        // the highest non-empty bin whose running weight (from the top) reaches W
        u64 pos = NB, pabove = 0, pcount = 0;
        for (int j = 0; j < BPT; j++) {
            if (c[j] > 0 && ex + w[j] >= W) {
                pos = BPT * t + j;
                pabove = ex;
                pcount = c[j];
                break;
            }
            ex += w[j];
        }
        const u64 best = block_reduce<OP_MIN>(sh, pos);
        if (best == NB) return Found{0, 0, 0, false};  // W exceeds the set's weight
        if (pos == best) {
            sh.bsel[0] = pabove;
            sh.bsel[1] = pcount;
        }
        __syncthreads();
        const int bsel = NB - 1 - (int)best;
        const u64 babove = sh.bsel[0];
        const u64 bcount = sh.bsel[1];
        if (bcount <= LMAX) {
            // gather the bin into CTA 0, sort it there and walk it
            uint32_t *ln = cl.map_shared_rank(&sh.list_n, 0u);
            u64 *lst = cl.map_shared_rank(&sh.list[0], 0u);
            for (uint32_t i = x.c0; i < x.c1; i++) {
                const float v = x.sv[i];
                if (!(v >= lo && v <= hi) || !in_set(x, v, x.base + i) || bin_of(v, dlo, scale) != bsel) continue;
                const uint32_t slot = atomicAdd(ln, 1u);
                if (slot < LMAX) lst[slot] = key64(v, x.base + i);
            }
            cl.sync();
            if (x.rank == 0) {
                const uint32_t n = min(sh.list_n, LMAX);
                sort_desc(sh.list, n);
                // each thread takes EPT consecutive entries; scan their weights
                u64 wv[EPT], s = 0;
                for (int j = 0; j < EPT; j++) {
                    const uint32_t e = EPT * t + j;
                    wv[j] = e < n ? weight(mass, key_val(sh.list[e]), x) : 0ull;
                    s += wv[j];
                }
                u64 tot2;
                u64 acc = babove + block_excl_scan(sh, s, &tot2);
                u64 first = ~0ull, f0 = 0, f1 = 0;
                for (int j = 0; j < EPT; j++) {
                    const uint32_t e = EPT * t + j;
                    if (e < n && acc + wv[j] >= W) {
                        first = e;
                        f0 = acc;
                        f1 = acc + wv[j];
                        break;
                    }
                    acc += wv[j];
                }
                const u64 g = block_reduce<OP_MIN>(sh, first);
                if (t == 0) {
                    sh.res[0] = 0ull;
                    sh.res[1] = sh.res[2] = 0ull;
                }
                __syncthreads();
                if (g != ~0ull && first == g) {
                    sh.res[0] = sh.list[g];
                    sh.res[1] = f0;
                    sh.res[2] = f1;
                }
                if (t == 0) sh.list_n = 0;
            }
            cl.sync();
            return read_result(x);
        }
        // narrow the bounds to the bin's own extremes
        u64 mn = ~0ull, mx = 0ull;
        for (uint32_t i = x.c0; i < x.c1; i++) {
            const float v = x.sv[i];
            if (!(v >= lo && v <= hi) || !in_set(x, v, x.base + i) || bin_of(v, dlo, scale) != bsel) continue;
            const u64 o = ord32(v);
            mn = o < mn ? o : mn;
            mx = o > mx ? o : mx;
        }
        mn = cluster_reduce<OP_MIN>(x, mn);
        mx = cluster_reduce<OP_MAX>(x, mx);
        lo = unord32((uint32_t)mn);
        hi = unord32((uint32_t)mx);
        above = babove;
    }
    // one value left: equal values are ordered by index
    return search_index(x, mass, W, above, true, lo);
}

__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(NT, 1) sample_kernel(SampleArgs a) {
    extern __shared__ __align__(16) unsigned char smp_dyn[];
    Smem &sh = *reinterpret_cast<Smem *>(smp_dyn);
    cg::cluster_group cl = cg::this_cluster();
    const int t = threadIdx.x;
    griddep_wait();
    int step = -1;
    if (a.st) {
        step = a.st->step - 1;
        if (step + 1 < a.st->n_forced) return;  // a prompt position: its next token is given (every CTA alike)
    }
    const cuq_sampler_params P = a.prm ? *a.prm : a.pv;
    const uint32_t *recent = a.ring ? a.ring_ids : a.recent;
    uint32_t n_recent = a.n_recent;
    if (a.ring) n_recent = min(a.ring->len, a.ring->cap);

    Ctx x;
    x.sh = &sh;
    x.sv = reinterpret_cast<float *>(smp_dyn + SMEM_HDR);
    x.rank = cl.block_rank();
    x.base = x.rank * a.slice;
    x.cnt = x.base < a.vocab ? min(a.slice, a.vocab - x.base) : 0u;
    x.phase = 0;
    x.lo_key = 0ull;
    {
        const float *src = a.logits + x.base;
        if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
            const uint32_t n4 = x.cnt / 4;
            for (uint32_t i = t; i < n4; i += NT)
                reinterpret_cast<float4 *>(x.sv)[i] = __ldcg(reinterpret_cast<const float4 *>(src) + i);
            for (uint32_t i = 4 * n4 + t; i < x.cnt; i += NT) x.sv[i] = __ldcg(src + i);
        } else {
            for (uint32_t i = t; i < x.cnt; i += NT) x.sv[i] = __ldcg(src + i);
        }
    }
    if (x.rank == 0 && t == 0) sh.list_n = 0;
    if (t == 0) sh.wl_n = 0;
    __syncthreads();

    // cpu.zig:529-547.  A token's result depends only on how many times it
    // occurs in the window, not where: each occurrence divides a positive logit
    // by the repetition penalty (multiplies a non-positive one) and subtracts
    // the frequency penalty; the first also subtracts the presence penalty.
    const bool pen = !(P.repetition_penalty == 1.0f && P.presence_penalty == 0.0f && P.frequency_penalty == 0.0f);
    if (pen && n_recent) {
        uint32_t *wl = reinterpret_cast<uint32_t *>(sh.list);
        for (uint32_t j = t; j < n_recent; j += NT) {
            const uint32_t id = recent[j];
            if (id - x.base < x.cnt) wl[atomicAdd(&sh.wl_n, 1u)] = id;
        }
        __syncthreads();
        const uint32_t m = sh.wl_n;
        const float rep = P.repetition_penalty > 0.0f ? P.repetition_penalty : 1.0f;
        for (uint32_t j = t; j < m; j += NT) {
            const uint32_t id = wl[j];
            uint32_t c = 0;
            bool first = true;
            for (uint32_t q = 0; q < m; q++)
                if (wl[q] == id) {
                    if (q < j) {
                        first = false;
                        break;
                    }
                    c++;
                }
            if (!first) continue;
            float v = x.sv[id - x.base];
            for (uint32_t o = 0; o < c; o++) {
                if (rep != 1.0f) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
                if (P.frequency_penalty != 0.0f) v = __fsub_rn(v, P.frequency_penalty);
                if (P.presence_penalty != 0.0f && o == 0) v = __fsub_rn(v, P.presence_penalty);
            }
            x.sv[id - x.base] = v;
            a.logits[id] = v;  // in place, like the reference
        }
        __syncthreads();
    }

    // this thread's contiguous range; an odd length keeps the strided shared
    // memory reads free of bank conflicts
    {
        const uint32_t C = ((x.cnt + NT - 1) / NT) | 1u;
        x.c0 = min((uint32_t)t * C, x.cnt);
        x.c1 = min(x.c0 + C, x.cnt);
    }

    // maximum and first index of the maximum (cpu.zig:648-649, 477-483)
    u64 best = 0ull;
    for (uint32_t i = x.c0; i < x.c1; i++) {
        const float v = x.sv[i];
        if (v == v) {
            const u64 k = key64(v, x.base + i);
            best = k > best ? k : best;
        }
    }
    best = cluster_reduce<OP_MAX>(x, best);
    const uint32_t am = best ? key_idx(best) : 0u;
    x.maxv = best ? key_val(best) : 0.0f;
    x.T = P.temperature;

    uint32_t token = am, n_cand = 0, kept = 0, rng = *a.rng;
    bool drew = false;
    if (P.temperature > 0.0f) {
        x.cut = __fsub_rn(x.maxv, __fmul_rn(P.min_keep_delta, P.temperature));
        u64 nc = 0;
        for (uint32_t i = x.c0; i < x.c1; i++) nc += x.sv[i] >= x.cut;
        n_cand = (uint32_t)cluster_reduce<OP_SUM>(x, nc);
        const float top_p = P.top_p > 0.0f ? fminf(P.top_p, 1.0f) : 1.0f;
        const bool topk = n_cand > 0 && P.top_k > 0 && P.top_k < n_cand;
        bool done = n_cand == 0;  // nothing survives the cut: argmax
        if (topk) {
            const Found f = search_sorted(x, false, P.top_k);
            x.lo_key = f.ok ? f.key : 0ull;
            if (f.ok && P.top_k <= LMAX) {
                // the k kept entries into CTA 0, then the reference's own fp32 steps
                uint32_t *ln = cl.map_shared_rank(&sh.list_n, 0u);
                u64 *lst = cl.map_shared_rank(&sh.list[0], 0u);
                for (uint32_t i = x.c0; i < x.c1; i++) {
                    const float v = x.sv[i];
                    if (in_set(x, v, x.base + i)) {
                        const uint32_t slot = atomicAdd(ln, 1u);
                        if (slot < LMAX) lst[slot] = key64(v, x.base + i);
                    }
                }
                cl.sync();
                if (x.rank == 0) {
                    const uint32_t k = min(sh.list_n, LMAX);
                    sort_desc(sh.list, k);
                    float *pf = reinterpret_cast<float *>(sh.hmass);  // LMAX floats
                    for (uint32_t j = t; j < k; j += NT) pf[j] = prob(key_val(sh.list[j]), x.maxv, x.T);
                    __syncthreads();
                    if (t == 0) {
                        float sum = 0.0f;
                        for (uint32_t j = 0; j < k; j++) sum = __fadd_rn(sum, pf[j]);
                        uint32_t keep = k;
                        bool ok = !(sum <= 0.0f);
                        if (ok && top_p < 1.0f) {
                            float acc = 0.0f;
                            uint32_t cut_n = keep;
                            for (uint32_t j = 0; j < keep; j++) {
                                acc = __fadd_rn(acc, __fdiv_rn(pf[j], sum));
                                if (acc >= top_p) {
                                    cut_n = j + 1;
                                    break;
                                }
                            }
                            keep = cut_n;
                            sum = 0.0f;
                            for (uint32_t j = 0; j < keep; j++) sum = __fadd_rn(sum, pf[j]);
                            ok = !(sum <= 0.0f);
                        }
                        if (ok) {
                            rng = rng * 1664525u + 1013904223u;
                            const float r = (float)(rng >> 8) / 16777216.0f;
                            float target = __fmul_rn(r, sum);
                            token = key_idx(sh.list[0]);
                            for (uint32_t j = 0; j < keep; j++) {
                                target = __fsub_rn(target, pf[j]);
                                if (target <= 0.0f) {
                                    token = key_idx(sh.list[j]);
                                    break;
                                }
                            }
                            kept = keep;
                            drew = true;
                        }
                    }
                }
                done = true;
            }
        }
        if (!done) {
            // probability mass of the kept set, in fixed point
            u64 s = 0;
            for (uint32_t i = x.c0; i < x.c1; i++) {
                const float v = x.sv[i];
                if (in_set(x, v, x.base + i)) s += weight(true, v, x);
            }
            u64 S = cluster_reduce<OP_SUM>(x, s);
            if (S > 0) {
                const bool sorted = topk || top_p < 1.0f;
                if (top_p < 1.0f) {
                    // the nucleus: descending order up to the first running mass >= top_p * sum
                    const u64 Wp = (u64)ceil((double)top_p * (double)S);
                    const Found f = search_sorted(x, true, Wp);
                    if (f.ok) {
                        x.lo_key = f.key;
                        S = f.through;
                    }
                }
                rng = rng * 1664525u + 1013904223u;
                const float r = (float)(rng >> 8) / 16777216.0f;
                const u64 Wd = (u64)ceil((double)r * (double)S);
                Found f = sorted ? search_sorted(x, true, Wd) : search_index(x, true, Wd, 0, false, 0.0f);
                if (!f.ok && !sorted) f = search_index(x, true, 0, 0, false, 0.0f);  // cpu.zig:719
                token = f.ok ? key_idx(f.key) : am;
                drew = true;
                if (a.info) {
                    u64 kc = 0;
                    for (uint32_t i = x.c0; i < x.c1; i++) kc += in_set(x, x.sv[i], x.base + i);
                    kept = (uint32_t)cluster_reduce<OP_SUM>(x, kc);
                }
            }
        }
    }
    if (x.rank == 0 && t == 0) {
        if (drew) *a.rng = rng;
        if (a.out) *a.out = token;
        if (a.info) {
            a.info[0] = n_cand;
            a.info[1] = kept;
        }
        if (a.st) {
            // the step's output and the next step's input (generate.zig:217-236)
            a.out_tokens[step] = token;
            a.st->token = (int)token;
            const uint32_t cap = a.ring ? a.ring->cap : 0u;
            if (cap) {  // the window drops its oldest id when full
                const uint32_t len = a.ring->len;
                if (len < cap) {
                    a.ring_ids[len] = token;
                    a.ring->len = len + 1;
                } else {
                    a.ring_ids[a.ring->head] = token;
                    a.ring->head = (a.ring->head + 1) % cap;
                }
            }
        }
    }
    cl.sync();  // no CTA leaves while another may still read its shared memory
}

}  // namespace

uint32_t sample_slice(uint32_t vocab) {
    const uint32_t s = (vocab + CL - 1) / CL;
    return (s + 3u) & ~3u;
}

size_t sample_smem_bytes(uint32_t vocab) { return SMEM_HDR + sizeof(float) * (size_t)sample_slice(vocab); }

int launch_sample(const SampleArgs &a, bool pdl, cudaStream_t s) {
    if (a.vocab == 0 || a.vocab > SAMPLE_MAX_VOCAB) {
        set_error("sample: vocab %u outside 1..%u", a.vocab, (unsigned)SAMPLE_MAX_VOCAB);
        return CUQ_EINVAL;
    }
    const size_t smem = sample_smem_bytes(a.vocab);
    // raise the kernel's dynamic shared memory limit once per device
    static std::mutex mu;
    static bool raised[64] = {};
    int dev = 0;
    CUQ_CUDA_TRY(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> g(mu);
        if (dev >= 0 && dev < 64 && !raised[dev]) {
            CUQ_CUDA_TRY(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)sample_smem_bytes(SAMPLE_MAX_VOCAB)));
            raised[dev] = true;
        }
    }
    SampleArgs k = a;
    k.slice = sample_slice(a.vocab);
    CUQ_CUDA_TRY(launch_maybe_pdl(sample_kernel, dim3(CL), dim3(NT), smem, s, pdl, k));
    return CUQ_OK;
}

}  // namespace cuq

using namespace cuq;

extern "C" int cuq_sample(float *logits_dev, uint32_t vocab, const cuq_sampler_params *params,
                          const uint32_t *recent_dev, uint32_t n_recent, uint32_t *rng_dev, uint32_t *token_dev,
                          void *stream) {
    CUQ_CHECK_ARG(logits_dev && params && rng_dev && token_dev && (recent_dev || n_recent == 0),
                  "cuq_sample: null argument");
    CUQ_CHECK_ARG(n_recent <= SAMPLE_MAX_WINDOW, "cuq_sample: window of %u ids exceeds %u", n_recent,
                  (unsigned)SAMPLE_MAX_WINDOW);
    SampleArgs a;
    a.logits = logits_dev;
    a.vocab = vocab;
    a.pv = *params;
    a.recent = recent_dev;
    a.n_recent = n_recent;
    a.rng = rng_dev;
    a.out = token_dev;
    return launch_sample(a, false, (cudaStream_t)stream);
}
