// gemv.cuh -- weight-only INT8 / INT4 / FP16 dequant GEMV for decode (M <= 8).
//
// Replaces the coalesced decode GEMVs of Gemma3CS.compute (QKVProj1VecCoal,
// OProj1VecCoal, GateUp1VecCoal, Down1VecCoal, LmHeadPredict1VecCoal,
// G3CS:1183-1302) with one templated kernel plus fused prologues (RMSNorm,
// G3CS:204-223) and epilogues (split + RoPE + fp16 KV write, G3CS:249-411;
// SwiGLU, G3CS:1244-1267; residual add, G3CS:1163-1169; logits + argmax
// partials, G3CS:911-928).
//
// Design (B200, HBM-bound at M = 1):
//  * Each CTA owns a contiguous range of row groups (RW rows) so every SM
//    streams the same number of bytes; its 8 warps take the groups
//    round-robin and never synchronise with each other after the prologue.
//  * A lane streams its 16-byte weight chunks (one per row of the group, 512
//    contiguous bytes per row across the warp) through a private D-stage ring
//    in shared memory with cp.async (L2 only), so D - 1 steps per warp are in
//    flight without holding registers.  The first D - 1 steps are issued
//    before griddepcontrol.wait: under programmatic dependent launch the
//    weight fetch overlaps the previous kernel's tail and this kernel's
//    activation prologue.
//  * INT4 / INT8: the activation vector is turned, once per CTA, into 22-bit
//    fixed point split into three byte planes laid out to match the nibble /
//    byte order of a weight word.  A weight word then costs dp4a per plane:
//    exact integer products, 3 dp4a per 4 INT8 weights, 6 dp4a + 3 integer
//    ops per 8 INT4 weights.
//    INT8 (signed, no zero point) uses one power-of-two scale per token,
//    accumulates the whole row exactly in int32 per plane and applies the row
//    scale once.  INT4 uses one power-of-two scale per 32-column chunk (found
//    by the four lanes that convert the chunk, so staging is a single pass
//    with no block-wide reduction), folds its zero point (8) through per-chunk
//    sums of x_int and applies group scale x chunk scale per chunk.
//  * RMSNorm (INT4 / FP16): x * (1 + gamma') is staged and the per-token
//    1 / rms, a scalar, multiplies the folded dot product in the epilogue;
//    the sum of squares is reduced alongside the conversion.
//  * FP16 (lm_head): fp32 activations in smem, packed fma.rn.f32x2.
//  * Each finished row group is folded with warp shuffles and its epilogue is
//    run by the owning lanes.
#pragma once

#include "common.cuh"

namespace du {

constexpr int GV_THREADS = 256;
constexpr int GV_WARPS = GV_THREADS / 32;
constexpr int GV_WARPS_WIDE = 16;   // one CTA per SM (decode token tile 1, large K)

enum GemvMap { MAP_IDENT = 0, MAP_ROPE_PAIR = 1, MAP_GATEUP = 2 };
// EPI_TP_RESID: resid += the sum over the tensor-parallel ranks' outputs, through
// peer memory (tp_fuse.cuh); y is not written.  The launch must fit in one wave.
enum GemvEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_GATEUP = 3, EPI_LOGITS = 4, EPI_TP_RESID = 5 };

struct GemvParams {
    // activations in: x fp32 [M][ldx]; optional RMSNorm with gamma' = gamma - 1 (fp16)
    const float *x;
    int ldx;
    const __half *gamma;
    float eps;
    // weights: physical row r starts at w + r * row_bytes
    const uint8_t *w;
    const void *scales;
    int scale_f32;          // INT8 only: scales are fp32 instead of fp16
    int64_t row_bytes;
    int K, N, M, group;
    int map, map_hd, map_I;
    int64_t row_off;        // added to the mapped physical row
    int grid;               // CTAs (0 = as many as fit); also the number of argmax partials
    // epilogue
    int epi;
    float *y;
    int ldy;
    // EPI_QKV
    float *q_out;           // [M][hq*hd]
    __half *k_cache, *v_cache;   // [seq][cap][hkv][hd]
    const int *pos;         // [M] cache slot / RoPE position per token
    const int *seq_of;      // [M] sequence per token (nullptr: token m -> sequence seq_off + m)
    int seq_off;
    int hq, hkv, hd, cap;
    const __half *rope_cos, *rope_sin;  // [cap][hd/2]
    float *kv_stage;        // optional (INT8 KV): K / V rows as fp32 [M][2][hkv][hd] instead of the
                            // fp16 cache; the next kernel quantizes them into the cache
    int act;                // EPI_GATEUP: 0 SiLU(g) * u, 1 gelu(g) * u (tanh form)
    // EPI_LOGITS: logits[m][row] of this rank's vocab shard (optional) + per-CTA
    // (max, argmax) with the global vocab index vocab_off + row
    float *logits;
    int ldl;
    float *am_val;          // [M][gridDim.x]
    int *am_idx;
    int vocab_off;
    // EPI_TP_RESID: peer handles (device memory) and the residual
    const TpFuse *tp;
    float *resid;
};

// COLS: weight columns per 16-byte chunk; XU4: uint4s of staged activations per chunk
template <int QT> struct GvTraits;
template <> struct GvTraits<Q_I4> { static constexpr int COLS = 32, XU4 = 7; };   // 6 used + 1 pad (banks)
template <> struct GvTraits<Q_I8> { static constexpr int COLS = 16, XU4 = 3; };
template <> struct GvTraits<Q_F16> { static constexpr int COLS = 8, XU4 = 2; };   // fp32 x, swizzled

__device__ __forceinline__ int64_t gv_map_row(const GemvParams &p, int lr)
{
    int64_t r;
    if (p.map == MAP_ROPE_PAIR) {
        const int h = lr / p.map_hd, w = lr - h * p.map_hd;
        r = (int64_t)h * p.map_hd + (w >> 1) + (w & 1) * (p.map_hd >> 1);
    } else if (p.map == MAP_GATEUP) {
        r = (lr & 1) ? (int64_t)p.map_I + (lr >> 1) : (int64_t)(lr >> 1);
    } else {
        r = lr;
    }
    return r + p.row_off;
}

// dp4a with explicit operand signedness (a: weights, b: activation plane)
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// exact int -> float for |v| < 2^22 without the conversion unit
__device__ __forceinline__ float gv_i2f_small(int v)
{
    return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

// acc += a * b on two fp32 lanes with one packed FFMA2 (sm_100 fma.rn.f32x2)
__device__ __forceinline__ void ffma2(float2 &acc, float a0, float a1, float b0, float b1)
{
    asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%0, %1};\n\t"
        "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rc;\n\t}"
        : "+f"(acc.x), "+f"(acc.y)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ void gv_dot_f16(uint32_t w, float a, float b, float2 &acc)
{
    __half2 h = *reinterpret_cast<__half2 *>(&w);
    const float2 f = __half22float2(h);
    ffma2(acc, f.x, f.y, a, b);
}

// L2 policy for data read once per step (weights): evicted first, so the
// streamed gigabytes do not push kernel code, activations and the KV rows
// written this step out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void cp_async16_cg_ef(void *smem, const void *gmem, bool valid, uint64_t pol)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(s), "l"(gmem), "r"(n), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async4_ca_ef(void *smem, const void *gmem, bool valid, uint64_t pol)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 4, %2, %3;" ::"r"(s), "l"(gmem), "r"(n), "l"(pol)
                 : "memory");
}

__device__ __forceinline__ void cp_async16_cg(void *smem, const void *gmem, bool valid)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async4_ca(void *smem, const void *gmem, bool valid)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
// Round-to-nearest-even of v * sc for |v * sc| <= 2^22, sc a power of two:
// the single rounding of v * sc + 1.5 * 2^23 leaves the integer in the low
// mantissa bits (the same result as __float2int_rn(v * sc)).
__device__ __forceinline__ int gv_rint_small(float v, float sc)
{
    return __float_as_int(fmaf(v, sc, 12582912.0f)) - 0x4B400000;
}

__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

}  // namespace du
