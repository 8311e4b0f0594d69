// attn_noalloc.cu -- decode attention that allocates nothing.
//
// cuq_attention_decode gets its split-K scratch (one partial softmax state per
// position split and query head) from the stream-ordered allocator on every
// call.  Some callers of this library cannot let it allocate: an engine that
// reserves all device memory up front for its weights and KV cache and hands out
// nothing afterwards, or a host loop that must not risk the synchronisation an
// allocator call can cause between decode steps.  For them this file keeps the
// scratch in one fixed array compiled into the library; the caller still passes
// its own q, K/V and output buffers.
#include <mutex>

#include "common.cuh"
#include "ops.cuh"

namespace cuq {
int sm_count_current();
}

namespace {

// The scratch: 262,144 floats (1 MiB).  Every GPU that loads the library holds
// this array until the process exits.  A call needs heads * (head_dim + 2)
// floats per position split; splits are capped to fit, and a head count whose
// single split does not fit is rejected.
constexpr size_t kScratchFloats = 262144;
static __device__ __align__(256) float g_attn_scratch[kScratchFloats];

// Host code cannot use the name g_attn_scratch as a device address: it must ask
// the runtime for the array's address on each device, once, with that device
// current.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
float *g_scratch_dev[kMaxDevices] = {};

}  // namespace

using namespace cuq;

extern "C" int cuq_attention_decode_noalloc(float *out_dev, const float *q_dev, const uint16_t *k_dev,
                                            const uint16_t *v_dev, uint32_t n_past, uint32_t cache_stride,
                                            uint32_t heads, uint32_t kv_heads, uint32_t hd, void *stream) {
    CUQ_CHECK_ARG(out_dev && q_dev && k_dev && v_dev && n_past >= 1 && n_past <= cache_stride,
                  "cuq_attention_decode_noalloc: bad argument (n_past %u, stride %u)", n_past, cache_stride);
    CUQ_CHECK_ARG(kv_heads > 0 && heads % kv_heads == 0, "cuq_attention_decode_noalloc: heads %% kv_heads != 0");
    const size_t per_split = (size_t)heads * (hd + 2);
    if (per_split > kScratchFloats) {
        set_error("cuq_attention_decode_noalloc: %u heads x head_dim %u need %zu scratch floats, more than the "
                  "library's fixed %zu (heads * (head_dim + 2) must be <= %zu)",
                  heads, hd, per_split, kScratchFloats, kScratchFloats);
        return CUQ_EINVAL;
    }
    int dev = 0;
    CUQ_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("cuq_attention_decode_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
        return CUQ_EINVAL;
    }
    float *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_scratch_dev[dev]) {  // first call on this device: look the array up
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
            if (e != cudaSuccess || !p) {
                set_error("cuq_attention_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                          cudaGetErrorString(e));
                return CUQ_ECUDA;
            }
            g_scratch_dev[dev] = (float *)p;
        }
        scratch = g_scratch_dev[dev];
    }
    int nsplit = attn_pick_nsplit(kv_heads, n_past, sm_count_current());
    const int cap = (int)(kScratchFloats / per_split);
    if (nsplit > cap) nsplit = cap;
    // Every (split, head) state the combine step reads is written by the split
    // kernel first (empty splits write -inf / 0), so nothing has to be cleared.
    return launch_attention_decode(q_dev, (const __half *)k_dev, (const __half *)v_dev, cache_stride, nullptr, n_past,
                                   heads, kv_heads, hd, scratch, nsplit, out_dev, nullptr, (cudaStream_t)stream);
}
