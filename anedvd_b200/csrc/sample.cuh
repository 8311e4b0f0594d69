// sample.cuh -- the device sampler (sample.cu): cpu.sampleProfiled and
// cpu.applyPenalties (src/cpu.zig:529-721).
#pragma once
#include "common.cuh"

namespace cuq {

constexpr uint32_t SAMPLE_MAX_VOCAB = CUQ_SAMPLE_MAX_VOCAB;    // 8 CTAs x 40960 logits in shared memory
constexpr uint32_t SAMPLE_MAX_WINDOW = CUQ_SAMPLE_MAX_WINDOW;  // penalty window ids

// The penalty window of a decode loop: `len` valid ids in ids[0..min(len, cap)),
// the oldest at `head` once full.  Only the multiset matters to the penalties.
struct SampleRing {
    uint32_t len, head, cap;
};

// Everything a decode loop's draws read from device memory, in one block (the
// host stages the same layout in pinned memory and copies it once per call).
struct SampleState {
    cuq_sampler_params prm;
    uint32_t rng;
    SampleRing ring;
    uint32_t ids[CUQ_SAMPLE_MAX_WINDOW];
};

struct SampleArgs {
    float *logits = nullptr;      // [vocab], penalised in place
    uint32_t vocab = 0;
    uint32_t slice = 0;           // logits per CTA (set by launch_sample)
    cuq_sampler_params pv{};      // parameters by value, used when prm is null
    const cuq_sampler_params *prm = nullptr;  // device copy (decode loop: changeable between calls)
    const uint32_t *recent = nullptr;         // window ids (standalone)
    uint32_t n_recent = 0;
    uint32_t *rng = nullptr;      // device LCG state, advanced by a draw
    uint32_t *out = nullptr;      // standalone: the token
    uint32_t *info = nullptr;     // optional: [candidates, kept]
    // decode loop: replaces the greedy token of the step that just finished
    StepState *st = nullptr;
    uint32_t *out_tokens = nullptr;
    SampleRing *ring = nullptr;
    uint32_t *ring_ids = nullptr;
};

uint32_t sample_slice(uint32_t vocab);
size_t sample_smem_bytes(uint32_t vocab);
int launch_sample(const SampleArgs &a, bool pdl, cudaStream_t s);

}  // namespace cuq
