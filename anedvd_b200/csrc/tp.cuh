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
// the error flag set) if it does not within TP_TIMEOUT_NS.
__device__ __forceinline__ bool tp_wait(const TpComm &t, int c, unsigned int expected) {
    const unsigned int *ctr = tp_ctr(t, t.rank, c);
    if (ld_acquire_sys(ctr) >= expected) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (ld_acquire_sys(ctr) < expected) {
        if (globaltimer_ns() - t0 > TP_TIMEOUT_NS) {
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

// Prefill all-reduce: push a [count] fp32 partial to every rank (phase ph), then
// x[i] += sum + bias[i % hidden] once every rank's push has arrived.
int launch_tp_push(const TpComm &t, int ph, const float *src, size_t count, int *grid_out, cudaStream_t s);
int launch_tp_reduce_add(const TpComm &t, int ph, unsigned int expected, float *x, const float *bias,
                         uint32_t hidden, size_t count, unsigned int *done, cudaStream_t s);

}  // namespace cuq
