// tp.cuh -- device side of the tensor-parallel exchange (TpComm, common.cuh).
//
// Protocol for one reduction of phase ph (o or down projection):
//   producer CTA: plain stores of its partial values into slot [rank] of phase
//     ph in every rank's buffer; __threadfence_system() by each storing thread;
//     __syncthreads(); one thread adds 1 to counter ph of every rank
//     (atomicAdd_system, which NVLink carries to the peer's memory);
//   consumer (one CTA, or the CTAs of a reduce kernel): wait until its own
//     counter ph reaches size * producer CTAs, read the slots in rank order
//     (identical sums on every rank), then set the counter back to 0.
// Waits are bounded by wall time (%globaltimer): on timeout the rank's error
// flag is set and the kernel carries on, so no GPU is left spinning; the host
// reports CUQ_ETIMEOUT after the call.
#pragma once

#include "common.cuh"

namespace cuq {

constexpr unsigned long long TP_TIMEOUT_NS = 10ull * 1000 * 1000 * 1000;  // 10 s

__device__ __forceinline__ float *tp_slot(const TpComm &t, int dst, int ph, int src) {
    return reinterpret_cast<float *>(t.peer[dst] + t.off_phase[ph]) + (size_t)src * t.slot_floats;
}
__device__ __forceinline__ unsigned int *tp_ctr(const TpComm &t, int dst, int c) {
    return reinterpret_cast<unsigned int *>(t.peer[dst] + t.off_ctr) + c;
}
__device__ __forceinline__ unsigned long long *tp_am(const TpComm &t, int dst) {
    return reinterpret_cast<unsigned long long *>(t.peer[dst] + t.off_am);
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long v;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(v));
    return v;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread: count this CTA's arrival on every rank (after the block's stores
// were fenced by the threads that made them and a __syncthreads()).
__device__ __forceinline__ void tp_signal(const TpComm &t, int c) {
    __threadfence_system();
    for (int p = 0; p < t.size; p++) atomicAdd_system(tp_ctr(t, p, c), 1u);
}

// One thread: wait until this rank's counter c reaches `expected`; false (and
// the error flag set) if it does not within t.wait_ns (TP_TIMEOUT_NS unless the
// model's options set a limit).
__device__ __forceinline__ bool tp_wait(const TpComm &t, int c, unsigned int expected) {
    const unsigned int *ctr = tp_ctr(t, t.rank, c);
    if (ld_acquire_sys(ctr) >= expected) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (ld_acquire_sys(ctr) < expected) {
        if (globaltimer_ns() - t0 > t.wait_ns) {
            atomicExch(t.err, 1);
            return false;
        }
        __nanosleep(64);
    }
    __threadfence_system();
    return true;
}

// One thread: counter c back to 0 once its phase has been consumed.
__device__ __forceinline__ void tp_reset(const TpComm &t, int c) {
    *tp_ctr(t, t.rank, c) = 0u;
    __threadfence_system();
}

// Sum of element i of phase ph over the source ranks, in rank order.
__device__ __forceinline__ float tp_sum(const TpComm &t, int ph, size_t i) {
    float s = 0.f;
    for (int r = 0; r < t.size; r++) s += __ldcv(tp_slot(t, t.rank, ph, r) + i);
    return s;
}

// Residual update + RMSNorm -> xq for the GEMV post-ops (one CTA, n % 16 == 0,
// n <= RN_MAX): x += (sum over ranks of the phase-ph partials + bias) when tp
// is set, then cpu.rmsnorm (cpu.zig:11-18) of x split into xq hi/lo with per-16
// sums.  x goes through `stage` (n floats of dynamic shared memory) so it is
// read from global memory once; loads are issued four float4 at a time per
// thread, so the post-op costs a few memory round trips, not one per element.
constexpr uint32_t RN_MAX = 8192;
__device__ __forceinline__ void stage_norm_xq(const float4 *stage, float ss, const float *w, uint32_t n, float eps,
                                              __half *xq, uint32_t kpad);
__device__ __forceinline__ void reduce_norm_xq_block(float *x, const TpComm *tp, int ph, const float *bias,
                                                     const float *w, uint32_t n, float eps, __half *xq,
                                                     uint32_t kpad, float4 *stage) {
    constexpr int U = 4;
    const int t = threadIdx.x, B = blockDim.x;
    const uint32_t n4 = n / 4;
    float ss = 0.f;
    for (uint32_t base = 0; base < n4; base += U * B) {
        float4 v[U];
#pragma unroll
        for (int k = 0; k < U; k++) {
            const uint32_t i4 = base + t + k * B;
            v[k] = i4 < n4 ? __ldcg(reinterpret_cast<const float4 *>(x) + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (tp) {
            float4 sm[U];
#pragma unroll
            for (int k = 0; k < U; k++) sm[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < tp->size; r++) {  // rank order: identical sums on every rank
                const float4 *src = reinterpret_cast<const float4 *>(tp_slot(*tp, tp->rank, ph, r));
#pragma unroll
                for (int k = 0; k < U; k++) {
                    const uint32_t i4 = base + t + k * B;
                    if (i4 < n4) {
                        const float4 q = __ldcv(src + i4);
                        sm[k].x += q.x;
                        sm[k].y += q.y;
                        sm[k].z += q.z;
                        sm[k].w += q.w;
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < U; k++) {
                const uint32_t i4 = base + t + k * B;
                if (i4 < n4) {
                    if (bias) {
                        const float4 b = reinterpret_cast<const float4 *>(bias)[i4];
                        sm[k].x = sm[k].x + b.x;
                        sm[k].y = sm[k].y + b.y;
                        sm[k].z = sm[k].z + b.z;
                        sm[k].w = sm[k].w + b.w;
                    }
                    v[k].x = v[k].x + sm[k].x;
                    v[k].y = v[k].y + sm[k].y;
                    v[k].z = v[k].z + sm[k].z;
                    v[k].w = v[k].w + sm[k].w;
                    reinterpret_cast<float4 *>(x)[i4] = v[k];
                }
            }
        }
#pragma unroll
        for (int k = 0; k < U; k++) {
            const uint32_t i4 = base + t + k * B;
            if (i4 < n4) stage[i4] = v[k];
            ss += (v[k].x * v[k].x + v[k].y * v[k].y) + (v[k].z * v[k].z + v[k].w * v[k].w);
        }
    }
    stage_norm_xq(stage, ss, w, n, eps, xq, kpad);
}

// Second half of the above, for x already staged in shared memory: `ss` is
// this thread's share of sum(x^2) (any split of the elements across threads).
__device__ __forceinline__ void stage_norm_xq(const float4 *stage, float ss, const float *w, uint32_t n, float eps,
                                              __half *xq, uint32_t kpad) {
    const int t = threadIdx.x, B = blockDim.x;
    const uint32_t n4 = n / 4;
    __shared__ float part[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    __syncthreads();
    if ((t & 31) == 0) part[t >> 5] = ss;
    __syncthreads();
    if (t < 32) {
        float a = t < (B >> 5) ? part[t] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (t == 0) part[0] = a;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(part[0] / (float)n + eps);
    float *sums = xq_sums(xq, kpad);
    for (uint32_t base = 0; base < n4; base += B) {  // uniform trip count: shuffles below
        const uint32_t i4 = base + t;
        float grp = 0.f;
        if (i4 < n4) {
            const float4 v = stage[i4];
            const float4 wv = reinterpret_cast<const float4 *>(w)[i4];
            const float f[4] = {(v.x * inv) * wv.x, (v.y * inv) * wv.y, (v.z * inv) * wv.z, (v.w * inv) * wv.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const uint32_t i = 4 * i4 + e;
                const __half hi = __float2half_rn(f[e]);
                xq[xq_pos(i)] = hi;
                xq[kpad + xq_pos(i)] = __float2half_rn(f[e] - __half2float(hi));
            }
            grp = (f[0] + f[1]) + (f[2] + f[3]);
        }
        // 16 consecutive columns = the float4s of 4 consecutive threads
        grp += __shfl_xor_sync(0xffffffffu, grp, 1);
        grp += __shfl_xor_sync(0xffffffffu, grp, 2);
        if (i4 < n4 && (i4 & 3u) == 0) sums[i4 >> 2] = grp;
    }
    for (uint32_t i = n + t; i < kpad; i += B) {  // zero tail (and its sums)
        xq[xq_pos(i)] = __float2half_rn(0.f);
        xq[kpad + xq_pos(i)] = __float2half_rn(0.f);
        if ((i & 15u) == 0) sums[i >> 4] = 0.f;
    }
}

// Prefill all-reduce: push a [count] fp32 partial to every rank (phase ph), then
// x[i] += sum + bias[i % hidden] once every rank's push has arrived.
int launch_tp_push(const TpComm &t, int ph, const float *src, size_t count, int *grid_out, cudaStream_t s);
int launch_tp_reduce_add(const TpComm &t, int ph, unsigned int expected, float *x, const float *bias,
                         uint32_t hidden, size_t count, unsigned int *done, cudaStream_t s);

}  // namespace cuq
