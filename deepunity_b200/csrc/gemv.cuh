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
//  * 256-thread CTA = 4 K-split warps x 2 row groups; each warp owns 4 rows
//    per pass and streams 512 contiguous weight bytes per row per step with
//    one 128-bit L1-bypassing load per lane; the next step's loads are in
//    flight while the current step computes.
//  * The activation vector is staged once per CTA in shared memory, already
//    multiplied by a per-column power of two (bank-conflict-free swizzle).
//    Each weight nibble / byte is then turned into an fp32 operand with ONE
//    bitwise AND: a masked nibble (or byte, xor 0x80 so it is unsigned) read
//    as a float is the exact subnormal n * 2^(p - 149), p = its bit position,
//    so x' * that = x * n * 2^-50 exactly-rounded in one FFMA.  The zero
//    points (8 for INT4, 128 for INT8) come back out through per-chunk /
//    per-token sums of x.  Cost: ~1.1 integer op + 1 FFMA per weight.
//  * Partial sums are folded with a shuffle reduce-scatter (4 rows in 6
//    shuffles instead of 20), then across the 4 K-warps through smem.
#pragma once

#include "common.cuh"

namespace du {

constexpr int GV_THREADS = 256;
constexpr int GV_KW = 4;                  // warps that split K
constexpr int GV_RG = 2;                  // row groups
constexpr int GV_RW = 4;                  // rows per warp per pass
constexpr int GV_PASS = GV_RG * GV_RW;    // logical rows per pass
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
    int rows_per_cta;       // logical rows per CTA (even)
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

// 8 INT4 weights (one 32-bit word, nibble j = column k0 + j) against x'[0..7]
__device__ __forceinline__ float gv_dot_i4(uint32_t w, float4 a, float4 b, float acc)
{
    const uint32_t w12 = w >> 12;
    acc = fmaf(__uint_as_float(w & 0x0000000Fu), a.x, acc);
    acc = fmaf(__uint_as_float(w & 0x000000F0u), a.y, acc);
    acc = fmaf(__uint_as_float(w & 0x00000F00u), a.z, acc);
    acc = fmaf(__uint_as_float(w & 0x0000F000u), a.w, acc);
    acc = fmaf(__uint_as_float(w & 0x000F0000u), b.x, acc);
    acc = fmaf(__uint_as_float(w12 & 0x00000F00u), b.y, acc);
    acc = fmaf(__uint_as_float(w12 & 0x0000F000u), b.z, acc);
    acc = fmaf(__uint_as_float(w12 & 0x000F0000u), b.w, acc);
    return acc;
}

// 4 INT8 weights (byte j = column k0 + j), offset to unsigned (q + 128)
__device__ __forceinline__ float gv_dot_i8(uint32_t w, float4 a, float acc)
{
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t u16 = u >> 16;
    acc = fmaf(__uint_as_float(u & 0x000000FFu), a.x, acc);
    acc = fmaf(__uint_as_float(u & 0x0000FF00u), a.y, acc);
    acc = fmaf(__uint_as_float(u16 & 0x000000FFu), a.z, acc);
    acc = fmaf(__uint_as_float(u16 & 0x0000FF00u), a.w, acc);
    return acc;
}

__device__ __forceinline__ float gv_dot_f16(uint32_t w, float a, float b, float acc)
{
    __half2 h = *reinterpret_cast<__half2 *>(&w);
    float2 f = __half22float2(h);
    acc = fmaf(f.x, a, acc);
    acc = fmaf(f.y, b, acc);
    return acc;
}

// Reduce-scatter of V values over the 32 lanes: afterwards lane l holds the
// full sum of value index (l >> (5 - log2 V)) in v[0].
template <int V>
__device__ __forceinline__ float gv_reduce_scatter(float (&v)[V], int lane)
{
    if constexpr (V == 1) {
        return warp_sum(v[0]);
    } else {
        constexpr int H = V / 2;
        constexpr int OFF = 16 >> 0;
        float nv[H];
        const bool up = lane & OFF;
#pragma unroll
        for (int i = 0; i < H; i++) {
            float send = up ? v[i] : v[i + H];
            float keep = up ? v[i + H] : v[i];
            nv[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
        }
        // continue with V/2 values and offsets 8, 4, ...
        if constexpr (H == 1) {
            float r = nv[0];
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
            return r;
        } else {
            // second level (offset 8)
            constexpr int H2 = H / 2;
            float n2[H2 > 0 ? H2 : 1];
            const bool up2 = lane & 8;
#pragma unroll
            for (int i = 0; i < H2; i++) {
                float send = up2 ? nv[i] : nv[i + H2];
                float keep = up2 ? nv[i + H2] : nv[i];
                n2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
            }
            static_assert(H2 == 1, "reduce-scatter implemented for V <= 4");
            float r = n2[0];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
            return r;
        }
    }
}

// value index that lane l holds after gv_reduce_scatter<V>
template <int V>
__device__ __forceinline__ int gv_rs_index(int lane)
{
    if constexpr (V == 1) return 0;
    else if constexpr (V == 2) return (lane >> 4) & 1;
    else return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
}

}  // namespace du
