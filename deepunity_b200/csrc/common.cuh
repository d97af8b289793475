// common.cuh -- shared helpers for libdeepunity_cuda (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace du {

// Thread-local error message surfaced by du_last_error().
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);

#define DU_CUDA_TRY(expr)                                              \
    do {                                                               \
        cudaError_t _e = (expr);                                       \
        if (_e != cudaSuccess) return ::du::cuda_fail(_e, #expr);      \
    } while (0)

#define DU_CHECK_ARG(cond, msg)                                        \
    do {                                                               \
        if (!(cond)) return ::du::fail(DU_EINVAL, msg);                \
    } while (0)

enum QuantKind { Q_F16 = 0, Q_I8 = 1, Q_I4 = 2 };

constexpr int TP_MAX_RANKS = 8;

// Device-side handles of the peer-memory tensor-parallel reduction (device
// memory, written when the peers are opened; device code in tp_fuse.cuh).
struct TpFuse {
    uint2 *peer_recv[TP_MAX_RANKS];  // rank r's receive words [2 parities][TP_MAX_RANKS][maxn]
    unsigned *seq;                   // this rank's last completed sequence number
    unsigned *done;                  // CTAs finished in the current launch (the last one resets it)
    int *err;                        // set on a timed-out wait
    size_t maxn;                     // elements per slot
    int rank, nranks;
    unsigned spin_limit;             // polls of one peer word before a wait gives up
};

// INT8 KV cache of one layer: uint8 rows [seq][cap][hkv][hd] and one word per
// (seq, position, kv head): fp16 scale | fp16 zero point << 16 (KVCache.hlsl:46-82).
struct Kv8Cache {
    uint8_t *k8, *v8;
    uint32_t *ksz, *vsz;
};

// 16-byte streaming load: weights are read exactly once per launch, so they
// bypass L1 (no_allocate) and come through the read-only path.
__device__ __forceinline__ uint4 ldg_stream(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Programmatic dependent launch: wait for the producer grid's memory, and
// allow the next grid in the stream to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Greedy tie-break of the reference's ArgMax (Gemma3CS.compute:911-928): 256
// threads stride the vocabulary keeping their first strict maximum (lowest
// index of the thread's stride set), then a tree over threads where slot t
// absorbs slot t + s (s = 128, 64, .., 1) only on a strictly larger value.  Among
// tied maxima the winner is therefore the thread whose id, read from bit 0
// upwards, is smallest (the bit-reversed thread id), then the lowest index of
// that thread.  am_rank orders vocabulary indices by that rule.
__device__ __forceinline__ unsigned am_rank(int i)
{
    return (__brev((unsigned)i & 255u) & 0xFF000000u) | ((unsigned)i >> 8);
}

// (v, i) beats (bv, bi): larger value, or an equal value with the reference's tie-break.
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi)
{
    return v > bv || (v == bv && am_rank(i) < am_rank(bi));
}

}  // namespace du
