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
#include <cuda.h>  // CUcontext / CUresult types of the two driver calls fetched below

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
// the runtime for the array's address on each device, with that device
// current.  The answer is cached per device together with the id of the
// context it was taken in; a context the host application destroyed and
// recreated (cudaDeviceReset) has a new id, and the address is looked up again.
constexpr int kMaxDevices = 64;
struct ScratchSlot {
    unsigned long long ctx_id = 0;
    float *ptr = nullptr;
};
std::mutex g_mu;
ScratchSlot g_slot[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long *);

// Id of the calling thread's current context (0 when none or unknown).
unsigned long long current_ctx_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault) == cudaSuccess)
            get_current = (CtxGetCurrentFn)f;
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault) == cudaSuccess) get_id = (CtxGetIdFn)f;
    });
    if (!get_current || !get_id) return 0;
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

}  // namespace

using namespace cuq;

extern "C" int cuq_attention_decode_noalloc(float *out_dev, const float *q_dev, const uint16_t *k_dev,
                                            const uint16_t *v_dev, uint32_t n_past, uint32_t cache_stride,
                                            uint32_t heads, uint32_t kv_heads, uint32_t hd, void *stream) {
    CUQ_CHECK_ARG(out_dev && q_dev && k_dev && v_dev && n_past >= 1 && n_past <= cache_stride,
                  "cuq_attention_decode_noalloc: bad argument (n_past %u, stride %u)", n_past, cache_stride);
    CUQ_CHECK_ARG(heads > 0 && kv_heads > 0 && heads % kv_heads == 0,
                  "cuq_attention_decode_noalloc: heads (%u) must be a positive multiple of kv_heads (%u)", heads,
                  kv_heads);
    if (hd != 64 && hd != 128) {
        set_error("cuq_attention_decode_noalloc: unsupported head_dim %u (64 or 128)", hd);
        return CUQ_EUNSUPPORTED;
    }
    const size_t per_split = (size_t)heads * ((size_t)hd + 2);
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
        ScratchSlot &slot = g_slot[dev];
        unsigned long long id = current_ctx_id();
        if (!slot.ptr || id == 0 || id != slot.ctx_id) {  // set-up on this device (or in a new context)
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
            if (e != cudaSuccess || !p) {
                set_error("cuq_attention_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                          cudaGetErrorString(e));
                return CUQ_ECUDA;
            }
            slot.ptr = (float *)p;
            slot.ctx_id = current_ctx_id();  // the lookup made the primary context current if it was not
        }
        scratch = slot.ptr;
    }
    int nsplit = attn_pick_nsplit(kv_heads, n_past, sm_count_current());
    const int cap = (int)(kScratchFloats / per_split);
    if (nsplit > cap) nsplit = cap;
    // Every (split, head) state the combine step reads is written by the split
    // kernel first (empty splits write -inf / 0), so nothing has to be cleared.
    return launch_attention_decode(q_dev, (const __half *)k_dev, (const __half *)v_dev, cache_stride, nullptr, n_past,
                                   heads, kv_heads, hd, scratch, nsplit, out_dev, nullptr, (cudaStream_t)stream);
}
