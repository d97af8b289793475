// noalloc.cu -- du_flash_decode_noalloc: split-K flash-decode whose scratch
// lives in a fixed, file-scope device array, so the call allocates nothing.
//
// Who needs it: callers that must not call cudaMalloc / cudaFree.  The typical
// one is a game engine plugin invoked from the engine's render or job thread:
// the engine owns the GPU memory budget, and cudaMalloc / cudaFree may
// synchronise the whole device, which stalls the frame.  Hosts whose device
// memory is managed by another allocator have the same constraint.
//
// The scratch is DU_NOALLOC_SCRATCH_FLOATS fp32 partials plus
// DU_NOALLOC_MAX_COUNTERS split counters (about 4 MiB), held by every GPU that
// loads the library until the process exits.  All calls on a device share it:
// calls whose kernels overlap on the GPU (different streams without ordering)
// race on it.  The counters are cleared before each launch; the partials are
// always written before they are read.
#include <mutex>

#include "attn_impl.cuh"
#include "internal.h"

namespace du {

constexpr size_t DU_NOALLOC_SCRATCH_FLOATS = (size_t)1 << 20;   // 4 MiB of split partials
constexpr int DU_NOALLOC_MAX_COUNTERS = 8192;                   // batch * kv heads

// Device-side storage.  In host code these names are only stand-ins for the
// device symbols; the real addresses come from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_noalloc_partials[DU_NOALLOC_SCRATCH_FLOATS];
static __device__ __align__(256) unsigned g_noalloc_counters[DU_NOALLOC_MAX_COUNTERS];

struct NoallocPtrs {
    float *partials = nullptr;
    unsigned *counters = nullptr;
};

// Resolves the device addresses of the scratch arrays once per device (the
// calling thread's current device).  The cached addresses belong to the
// device's primary context: after cudaDeviceReset in this process they are
// stale, so a host that resets a device must not call this entry point on it
// again.
static int noalloc_ptrs(NoallocPtrs *out)
{
    static std::mutex mu;
    static NoallocPtrs cache[64];
    static bool ready[64] = {};
    int dev = 0;
    DU_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(DU_EINVAL, "du_flash_decode_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lk(mu);
    if (!ready[dev]) {
        NoallocPtrs p;
        DU_CUDA_TRY(cudaGetSymbolAddress((void **)&p.partials, g_noalloc_partials));
        DU_CUDA_TRY(cudaGetSymbolAddress((void **)&p.counters, g_noalloc_counters));
        cache[dev] = p;
        ready[dev] = true;
    }
    *out = cache[dev];
    return DU_OK;
}

}  // namespace du

using namespace du;

extern "C" DU_API int du_flash_decode_noalloc(float *out, const float *q, const uint16_t *k_cache,
                                              const uint16_t *v_cache, const int32_t *kv_len, int batch, int hq,
                                              int hkv, int hd, int capacity, float scale, void *stream)
{
    DU_CHECK_ARG(out && q && k_cache && v_cache && kv_len, "du_flash_decode_noalloc: null pointer");
    DU_CHECK_ARG(batch >= 0 && hq > 0 && hkv > 0 && capacity > 0, "du_flash_decode_noalloc: bad sizes");
    DU_CHECK_ARG(hq % hkv == 0, "du_flash_decode_noalloc: hq must be a multiple of hkv");
    DU_CHECK_ARG(hd == 64 || hd == 128, "du_flash_decode_noalloc: head_dim must be 64 or 128");
    DU_CHECK_ARG(hq / hkv <= FD_MAXG, "du_flash_decode_noalloc: num_heads_q / num_heads_kv must be at most 8");
    if (batch == 0) return DU_OK;
    const int G = hq / hkv;
    if ((size_t)batch * hkv > (size_t)DU_NOALLOC_MAX_COUNTERS)
        return fail(DU_EINVAL, "du_flash_decode_noalloc: batch * num_heads_kv exceeds the fixed limit of 8192");
    const size_t per_split = fd_scratch_floats(batch, hkv, G, hd, 1);
    if (per_split > DU_NOALLOC_SCRATCH_FLOATS)
        return fail(DU_EINVAL, "du_flash_decode_noalloc: batch * num_heads_q * (head_dim + 2) exceeds the fixed "
                               "scratch of 1048576 floats");
    int ns = fd_choose_splits(batch, hkv, capacity);
    const int fit = (int)(DU_NOALLOC_SCRATCH_FLOATS / per_split);
    if (ns > fit) ns = fit;
    NoallocPtrs s;
    int rc = noalloc_ptrs(&s);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DU_CUDA_TRY(cudaMemsetAsync(s.counters, 0, sizeof(unsigned) * (size_t)batch * hkv, st));
    return launch_flash_decode(q, reinterpret_cast<const __half *>(k_cache), reinterpret_cast<const __half *>(v_cache),
                               nullptr, kv_len, 0, batch, hq, hkv, hd, capacity, scale, out, s.partials, s.counters,
                               ns, st);
}
