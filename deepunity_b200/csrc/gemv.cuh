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
//  * The grid is 2 CTAs per SM; each CTA owns a contiguous range of row
//    groups (RW = 4 rows at M <= 2, else 2) so every SM streams the same
//    number of bytes.  Warps take the CTA's groups round-robin and never
//    synchronise with each other after the prologue.
//  * A warp streams a row group 512 bytes per row per step (one 128-bit
//    L1-bypassing load per lane and row) through a 4-deep register ring: the
//    loads of the next 3 steps are in flight while one step computes.  The
//    first 3 steps are issued before griddepcontrol.wait, so under
//    programmatic dependent launch the weight fetch overlaps the previous
//    kernel's tail and this kernel's own activation prologue.
//  * The activation vector is staged once per CTA in shared memory, already
//    multiplied by a per-column power of two (bank-conflict-free swizzle).
//    Each weight nibble / byte is then turned into an fp32 operand with ONE
//    bitwise AND: a masked nibble (or byte, xor 0x80 so it is unsigned) read
//    as a float is the exact subnormal n * 2^(p - 149), p = its bit position,
//    so x' * that = x * n * 2^-50, rounded once, with two columns per packed
//    fma.rn.f32x2.  The zero points (8 for INT4, 128 for INT8) come back out
//    through per-chunk / per-token sums of x.  Cost per INT4 weight: ~1.1
//    integer op + 0.5 FFMA2.
//  * Each finished row group is folded with warp shuffles and its epilogue is
//    run by the owning lanes.
#pragma once

#include "common.cuh"

namespace du {

constexpr int GV_THREADS = 256;
constexpr float GV_TWO50 = 1125899906842624.0f;   // 2^50

enum GemvMap { MAP_IDENT = 0, MAP_ROPE_PAIR = 1, MAP_GATEUP = 2 };
enum GemvEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_GATEUP = 3, EPI_LOGITS = 4 };

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
    int grid;               // CTAs (0 = 2 per SM); also the number of argmax partials
    // epilogue
    int epi;
    float *y;
    int ldy;
    // EPI_QKV
    float *q_out;           // [M][hq*hd]
    __half *k_cache, *v_cache;   // [seq][cap][hkv][hd]
    const int *pos;         // [M] cache slot / RoPE position per token
    const int *seq_of;      // [M] sequence per token (nullptr: token m -> sequence m)
    int hq, hkv, hd, cap;
    const __half *rope_cos, *rope_sin;  // [cap][hd/2]
    // EPI_LOGITS: logits[m][vocab_off + row] (optional) + per-CTA (max, argmax)
    float *logits;
    int ldl;
    float *am_val;          // [M][gridDim.x]
    int *am_idx;
    int vocab_off;
};

template <int QT> struct GvTraits;
template <> struct GvTraits<Q_I4> { static constexpr int COLS = 32, F4 = 8; };   // cols per 16 B chunk
template <> struct GvTraits<Q_I8> { static constexpr int COLS = 16, F4 = 4; };
template <> struct GvTraits<Q_F16> { static constexpr int COLS = 8, F4 = 2; };

// 2^e as an exact fp32 constant, e in [-126, 127]
__device__ __forceinline__ float gv_pow2(int e) { return __int_as_float((127 + e) << 23); }

// power-of-two exponent applied to x at column position k (see header note)
template <int QT>
__device__ __forceinline__ int gv_xexp(int k)
{
    if (QT == Q_I4) {
        const int p = k & 7;
        const int e = p < 5 ? 4 * p : 4 * (p - 3);
        return 99 - e;
    } else if (QT == Q_I8) {
        return (k & 1) ? 91 : 99;
    }
    return 0;
}

// physical float4 slot of logical float4 f of a token row (bank-conflict-free
// for the lane-block reads of the main loop)
template <int QT>
__device__ __forceinline__ int gv_swz(int f)
{
    return f ^ ((f >> 3) & (GvTraits<QT>::F4 - 1));
}

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

// 8 INT4 weights (one 32-bit word, nibble j = column k0 + j) against x'[0..7]
__device__ __forceinline__ void gv_dot_i4(uint32_t w, float4 a, float4 b, float2 &acc)
{
    const uint32_t w12 = w >> 12;
    ffma2(acc, __uint_as_float(w & 0x0000000Fu), __uint_as_float(w & 0x000000F0u), a.x, a.y);
    ffma2(acc, __uint_as_float(w & 0x00000F00u), __uint_as_float(w & 0x0000F000u), a.z, a.w);
    ffma2(acc, __uint_as_float(w & 0x000F0000u), __uint_as_float(w12 & 0x00000F00u), b.x, b.y);
    ffma2(acc, __uint_as_float(w12 & 0x0000F000u), __uint_as_float(w12 & 0x000F0000u), b.z, b.w);
}

// 4 INT8 weights (byte j = column k0 + j), offset to unsigned (q + 128)
__device__ __forceinline__ void gv_dot_i8(uint32_t w, float4 a, float2 &acc)
{
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t u16 = u >> 16;
    ffma2(acc, __uint_as_float(u & 0x000000FFu), __uint_as_float(u & 0x0000FF00u), a.x, a.y);
    ffma2(acc, __uint_as_float(u16 & 0x000000FFu), __uint_as_float(u16 & 0x0000FF00u), a.z, a.w);
}

__device__ __forceinline__ void gv_dot_f16(uint32_t w, float a, float b, float2 &acc)
{
    __half2 h = *reinterpret_cast<__half2 *>(&w);
    const float2 f = __half22float2(h);
    ffma2(acc, f.x, f.y, a, b);
}

}  // namespace du
