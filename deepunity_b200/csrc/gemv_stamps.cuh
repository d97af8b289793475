// gemv_stamps.cuh -- timing build of the decode GEMV (compiled into
// libdeepunity_cuda_stamps.so only, with DU_GEMV_STAMPS defined; the library
// proper has no hook).
//
// Every launch of the standalone GEMV kernel records, per CTA (CTA index below
// GVS_CTAS), %globaltimer at the phases GV_STAMP marks:
//   0 entry (first instruction), 1 first ring stages issued, 2 dependency met
//   (griddepcontrol.wait returned), 3 activations staged, 4 stream done (the
//   last warp; word 6 holds the first warp), 5 exit (thread 0),
// and in word 7 the shape and SM: N << 40 | K << 16 | %smid.
// Records go to slot (launch count of this CTA index) % GVS_SLOTS, taken with one
// atomic at entry after the entry time is read, so that launches of one CTA index
// that overlap under programmatic dependent launch get distinct slots.
#pragma once

#include "gemv.cuh"

namespace du {

constexpr int GVS_SLOTS = 512;
constexpr int GVS_CTAS = 320;
__device__ unsigned long long gvs_buf[GVS_SLOTS * GVS_CTAS * 8];
__device__ unsigned gvs_cnt[GVS_CTAS];

__device__ __forceinline__ unsigned long long gvs_now()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned &gvs_slot()
{
    __shared__ unsigned s;
    return s;
}

// Event 4 is recorded by lane 0 of every warp; the others by thread 0.  Events 1..5
// follow a block barrier after event 0 (activation staging), which publishes the slot.
template <int E>
__device__ __forceinline__ void gvs_stamp(const GemvParams &p)
{
    if (blockIdx.x >= GVS_CTAS) return;
    const unsigned long long t = gvs_now();
    if (E == 4) {
        if ((threadIdx.x & 31) == 0) {
            unsigned long long *b = gvs_buf + ((size_t)gvs_slot() * GVS_CTAS + blockIdx.x) * 8;
            atomicMax(b + 4, t);
            atomicMin(b + 6, t);
        }
        return;
    }
    if (threadIdx.x != 0) return;
    if (E == 0) gvs_slot() = atomicAdd(&gvs_cnt[blockIdx.x], 1u) % GVS_SLOTS;
    unsigned long long *b = gvs_buf + ((size_t)gvs_slot() * GVS_CTAS + blockIdx.x) * 8;
    b[E] = t;
    if (E == 0) {
        unsigned sm;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
        b[4] = 0ull;
        b[6] = ~0ull;
        b[7] = ((unsigned long long)p.N << 40) | ((unsigned long long)p.K << 16) | sm;
    }
}

}  // namespace du

#define GV_STAMP(e) ::du::gvs_stamp<(e)>(p)

// Host access (exported by the timing build only).
extern "C" __attribute__((visibility("default"))) int du_gemv_stamps_reset(void)
{
    void *b = nullptr, *c = nullptr;
    if (cudaGetSymbolAddress(&b, du::gvs_buf) != cudaSuccess) return 1;
    if (cudaGetSymbolAddress(&c, du::gvs_cnt) != cudaSuccess) return 1;
    if (cudaMemset(b, 0, sizeof(du::gvs_buf)) != cudaSuccess) return 1;
    if (cudaMemset(c, 0, sizeof(du::gvs_cnt)) != cudaSuccess) return 1;
    return cudaDeviceSynchronize() != cudaSuccess;
}

// buf: GVS_SLOTS x GVS_CTAS x 8 words; cnt: GVS_CTAS launch counts.
extern "C" __attribute__((visibility("default"))) int du_gemv_stamps_read(unsigned long long *buf, unsigned *cnt,
                                                                         int *slots, int *ctas)
{
    *slots = du::GVS_SLOTS;
    *ctas = du::GVS_CTAS;
    if (buf && cudaMemcpyFromSymbol(buf, du::gvs_buf, sizeof(du::gvs_buf)) != cudaSuccess) return 1;
    if (cnt && cudaMemcpyFromSymbol(cnt, du::gvs_cnt, sizeof(du::gvs_cnt)) != cudaSuccess) return 1;
    return 0;
}
