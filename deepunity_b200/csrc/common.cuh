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

// WriteCacheFull's INT8 quantization (Gemma3CS.compute:300-380) of one (position,
// kv head) row held by a warp, lane values v[0 .. epl) = elements lane * epl + e:
// min / max (exact in any order), scale = (max - min) / 255 floored at 1e-9, zp =
// round(-min / scale) clamped to [0, 255], q = clamp(round(x * (1 / scale)) + zp,
// 0, 255), round half to even, IEEE division and reciprocal; the row's word is
// fp16 scale | fp16 zp << 16.  All 32 lanes call it.
__device__ __forceinline__ void kv8_store_row(const float (&v)[8], int epl, int lane, uint8_t *row, uint32_t *word)
{
    float mn = 3.0e38f, mx = -3.0e38f;
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (e < epl) {
            mn = fminf(mn, v[e]);
            mx = fmaxf(mx, v[e]);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    float scale = (mx - mn) / 255.0f;
    if (scale < 1e-9f) scale = 1e-9f;
    const float zp = fminf(fmaxf(rintf(-mn / scale), 0.0f), 255.0f);
    const float inv = 1.0f / scale;
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (e < epl) row[lane * epl + e] = (uint8_t)fminf(fmaxf(rintf(v[e] * inv) + zp, 0.0f), 255.0f);
    if (lane == 0)
        *word = (uint32_t)__half_as_ushort(__float2half_rn(scale)) | ((uint32_t)__half_as_ushort(__float2half_rn(zp)) << 16);
}

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

// gelu of the reference (Gemma3CS.compute:162-172): tanh form, tanh through
// exp(-2|t|) with sign(0) = 0.
__device__ __forceinline__ float gelu_tanh(float x)
{
    const float t = 0.7978845608f * (x + 0.044715f * x * x * x);
    const float e = expf(-2.0f * fabsf(t));
    const float sg = t > 0.0f ? 1.0f : (t < 0.0f ? -1.0f : 0.0f);
    return 0.5f * x * (1.0f + sg * ((1.0f - e) / (1.0f + e)));
}

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
