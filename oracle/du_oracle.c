/*
 * du_oracle.c -- CPU restatement of DeepUnity's quantized llama decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library in
 * deepunity_b200/csrc: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The product path never links or calls it.
 *
 * Every function restates one piece of the reference (paths relative to the
 * DeepUnity project root):
 *   IMP  = Assets/DeepUnity/InferenceEngine/import_params.py
 *   G3CS = Assets/Resources/ComputeShaders/Gemma3CS.compute
 *   KVH  = Assets/Resources/ComputeShaders/KVCache.hlsl
 *   M5M  = Assets/DeepUnity/InferenceEngine/LLM/MiniCPM5/MiniCPM5Model.cs
 *   MOD  = Assets/DeepUnity/Modules/
 *
 * Arithmetic is plain IEEE fp32, compiled with -ffp-contract=off so that every
 * product and sum is rounded separately, in the order the HLSL source writes
 * them.  (FXC may contract a*b+c into a mad; that choice is not observable from
 * the source, so bit-exactness with the D3D shaders is not claimed -- the
 * reference's own GEMV parity probe says the same.)  Integer work (quantize,
 * pack, unpack, argmax) is exact and is pinned bit-for-bit against the
 * reference's Python quantizers by tests/test_oracle_golden.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ fp16 */

/* float32 -> float16, round to nearest even.  Restates the managed converter
 * F32ToF16 (M5M:205-234); numpy's astype(float16) (IMP:233,248) rounds the
 * same way for every finite input. */
ORC_EXPORT uint16_t orc_f32_to_f16(float value)
{
    int32_t i;
    memcpy(&i, &value, 4);
    int32_t s = (i >> 16) & 0x00008000;
    int32_t e = ((i >> 23) & 0x000000ff) - (127 - 15);
    int32_t m = i & 0x007fffff;
    if (e <= 0) {
        if (e < -10) return (uint16_t)s;
        m |= 0x00800000;
        int32_t t = 14 - e;
        int32_t a = (1 << (t - 1)) - 1;
        int32_t b = (m >> t) & 1;
        m = (m + a + b) >> t;
        return (uint16_t)(s | m);
    } else if (e == 0xff - (127 - 15)) {
        if (m == 0) return (uint16_t)(s | 0x7c00);
        m >>= 13;
        return (uint16_t)(s | 0x7c00 | m | (m == 0 ? 1 : 0));
    } else {
        m = m + 0x00000fff + ((m >> 13) & 1);
        if ((m & 0x00800000) != 0) { m = 0; e += 1; }
        if (e > 30) return (uint16_t)(s | 0x7c00);
        return (uint16_t)(s | (e << 10) | (m >> 13));
    }
}

/* float16 -> float32 (exact).  HLSL f16tof32 as used by readH (G3CS:49-54). */
ORC_EXPORT float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* -------------------------------------------------------------- quantizers */

/* quantize_int8 (IMP:229-233): scale_r = max(max|w_r| / 127, 1e-8) in fp32,
 * q = clip(rint(w / scale_r), -127, 127); the scale is stored as fp16 but the
 * division uses the fp32 scale. */
ORC_EXPORT void orc_quantize_int8(const float *w, int64_t rows, int64_t cols,
                                  int8_t *q, uint16_t *scales)
{
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float *wr = w + r * cols;
        float mx = 0.0f;
        for (int64_t c = 0; c < cols; c++) {
            float a = fabsf(wr[c]);
            if (a > mx) mx = a;
        }
        float s = mx / 127.0f;
        if (!(s >= 1e-8f)) s = 1e-8f;
        for (int64_t c = 0; c < cols; c++) {
            float v = rintf(wr[c] / s);
            if (v < -127.0f) v = -127.0f;
            if (v > 127.0f) v = 127.0f;
            q[r * cols + c] = (int8_t)v;
        }
        scales[r] = orc_f32_to_f16(s);
    }
}

/* quantize_int4 (IMP:236-248) with the group size as a parameter (the
 * reference fixes G4 = 32 at IMP:78).  Per group: the element of largest
 * magnitude (first one on ties, numpy argmax) gives d = w_max / -8 (signed),
 * |d| < 1e-10 -> 1e-10, q = clip(rint(w / d) + 8, 0, 15); nibbles are packed
 * low = even column, high = odd column; d is stored fp16 as [rows, cols/G]. */
ORC_EXPORT void orc_quantize_int4(const float *w, int64_t rows, int64_t cols, int group,
                                  uint8_t *packed, uint16_t *scales)
{
    int64_t ng = cols / group;
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t g = 0; g < ng; g++) {
            const float *gr = w + r * cols + g * group;
            int64_t best = 0;
            float bestabs = fabsf(gr[0]);
            for (int64_t k = 1; k < group; k++) {
                float a = fabsf(gr[k]);
                if (a > bestabs) { bestabs = a; best = k; }
            }
            float d = gr[best] / -8.0f;
            if (fabsf(d) < 1e-10f) d = 1e-10f;
            for (int64_t k = 0; k < group; k += 2) {
                float v0 = rintf(gr[k] / d) + 8.0f;
                float v1 = rintf(gr[k + 1] / d) + 8.0f;
                v0 = v0 < 0.0f ? 0.0f : (v0 > 15.0f ? 15.0f : v0);
                v1 = v1 < 0.0f ? 0.0f : (v1 > 15.0f ? 15.0f : v1);
                packed[(r * cols + g * group + k) >> 1] =
                    (uint8_t)((uint8_t)v0 | ((uint8_t)v1 << 4));
            }
            scales[r * ng + g] = orc_f32_to_f16(d);
        }
    }
}

/* ------------------------------------------------------------ unpack/read */

enum { ORC_FP16 = 0, ORC_INT8 = 1, ORC_INT4 = 2 };

/* readQ8 (G3CS:72-77): byte idx of the little-endian packed words, sign-extended. */
static inline float read_q8(const uint8_t *buf, uint64_t idx)
{
    return (float)(int8_t)buf[idx];
}

/* readQ4 (G3CS:84-87): nibble idx (low nibble = even index) minus 8. */
static inline float read_q4(const uint8_t *buf, uint64_t idx)
{
    uint8_t b = buf[idx >> 1];
    return (float)((idx & 1) ? (b >> 4) : (b & 0xF)) - 8.0f;
}

/* readH through a table of every fp16 value's orc_f16_to_f32 (filled once when
 * the library loads): the same values, without the per-element bit decoding. */
static float g_f16_table[65536];

__attribute__((constructor)) static void orc_fill_f16_table(void)
{
    for (uint32_t h = 0; h < 65536u; h++) g_f16_table[h] = orc_f16_to_f32((uint16_t)h);
}

static inline float read_h(const uint16_t *buf, uint64_t idx)
{
    return g_f16_table[buf[idx]];
}

/* A (possibly concatenated) matmul weight as the shader sees it. */
typedef struct {
    const void *w;          /* int8 bytes / packed nibbles / fp16 halves */
    const uint16_t *s;      /* fp16 scales: per row (INT8) or per group (INT4) */
    int quant;
    int group;              /* INT4 group size (reference: 32) */
} orc_w;

/* readW (G3CS:92-101): INT4 folds the per-group scale into every element
 * (group = flat index / G); INT8 and FP16 return the raw value. */
static inline float read_w(const orc_w *W, uint64_t idx)
{
    switch (W->quant) {
    case ORC_INT8: return read_q8((const uint8_t *)W->w, idx);
    case ORC_INT4: return read_q4((const uint8_t *)W->w, idx) * read_h(W->s, idx / (uint64_t)W->group);
    default:       return read_h((const uint16_t *)W->w, idx);
    }
}

/* wScale (G3CS:92-101): INT8 applies the row scale once after the dot. */
static inline float w_scale(const orc_w *W, uint64_t row)
{
    return W->quant == ORC_INT8 ? read_h(W->s, row) : 1.0f;
}

/* Dequantised weight values exactly as readW(idx) * wScale(row) produces them. */
ORC_EXPORT void orc_dequant(const void *w, const uint16_t *s, int quant, int group,
                            int64_t rows, int64_t cols, float *out)
{
    orc_w W = { w, s, quant, group };
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++)
            out[r * cols + c] = read_w(&W, (uint64_t)(r * cols + c)) * w_scale(&W, (uint64_t)r);
}

/* GVC_DOT + GVC_REDUCE (G3CS:1196-1212): lane l accumulates 4 consecutive
 * elements per step at stride 128, then a 5-level tree folds the 32 lanes.
 * `base` is the row's flat element offset in the (concatenated) weight. */
static float coal_dot(const float *x, int K, const orc_w *W, uint64_t base)
{
    float red[32];
    for (int lane = 0; lane < 32; lane++) {
        float acc = 0.0f;
        for (int hh = lane * 4; hh < K; hh += 128) {
            float t = x[hh] * read_w(W, base + hh);
            t = t + x[hh + 1] * read_w(W, base + hh + 1);
            t = t + x[hh + 2] * read_w(W, base + hh + 2);
            t = t + x[hh + 3] * read_w(W, base + hh + 3);
            acc = acc + t;
        }
        red[lane] = acc;
    }
    for (int ss = 16; ss > 0; ss >>= 1)
        for (int lane = 0; lane < ss; lane++)
            red[lane] = red[lane] + red[lane + ss];
    return red[0];
}

/* Generic y[m, row] = wScale(row_off+row) * coal_dot(x[m], W row (row_off+row))
 * for rows [0, N): the common core of QKVProj1VecCoal / OProj1VecCoal /
 * Down1VecCoal and their GemmCoal twins (G3CS:1217-1439; the GEMM kernels walk
 * the same per-lane column sequence, so one restatement covers both). */
ORC_EXPORT void orc_gemv(const float *x, int M, int K, const void *w, const uint16_t *s,
                         int quant, int group, int64_t row_off, int N, float *y)
{
    orc_w W = { w, s, quant, group };
    #pragma omp parallel for schedule(static) collapse(2)
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            uint64_t row = (uint64_t)(row_off + n);
            y[(int64_t)m * N + n] = coal_dot(x + (int64_t)m * K, K, &W, row * (uint64_t)K) * w_scale(&W, row);
        }
}

/* ------------------------------------------------------------ elementwise */

static float silu_ref(float x) { return x / (1.0f + expf(-x)); }   /* G3CS:173-176 */

/* gelu / safe_tanh (G3CS:162-172): tanh through exp(-2|x|), sign(0) = 0. */
static float gelu_ref(float x)
{
    const float t = 0.7978845608f * (x + 0.044715f * x * x * x);
    const float a = fabsf(t), e = expf(-2.0f * a);
    const float sg = t > 0.0f ? 1.0f : (t < 0.0f ? -1.0f : 0.0f);
    return 0.5f * x * (1.0f + sg * ((1.0f - e) / (1.0f + e)));
}

/* RmsNormHead (G3CS:227-245): every hd-vector of buf [n, hd] in place,
 * x * rms * (1 + gamma[i]). */
static void rmsnorm_heads(float *buf, int n, int hd, const uint16_t *gamma, float eps)
{
    for (int v = 0; v < n; v++) {
        float *x = buf + (int64_t)v * hd;
        float sum_sq = 0.0f;
        for (int i = 0; i < hd; i++) sum_sq = sum_sq + x[i] * x[i];
        const float rms = 1.0f / sqrtf(sum_sq / (float)hd + eps);
        for (int i = 0; i < hd; i++) x[i] = x[i] * rms * (1.0f + read_h(gamma, i));
    }
}

/* RmsNormHidden (G3CS:204-223): one row at a time, sequential sum of squares,
 * y = x * rsqrt(mean + eps) * (1 + gamma') with gamma' = gamma - 1 stored fp16
 * (IMP:314-315).  rsqrt is restated as 1/sqrt. */
ORC_EXPORT void orc_rmsnorm(const float *x, int rows, int H, const uint16_t *gamma_m1,
                            float eps, float *y)
{
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (int64_t)r * H;
        float sum_sq = 0.0f;
        for (int i = 0; i < H; i++) sum_sq = sum_sq + xr[i] * xr[i];
        float rms = 1.0f / sqrtf(sum_sq / (float)H + eps);
        for (int i = 0; i < H; i++)
            y[(int64_t)r * H + i] = xr[i] * rms * (1.0f + read_h(gamma_m1, i));
    }
}

/* RoPE tables (M5M:163-191): inv_freq_i = 1 / theta^(2i/hd) in fp32, cos/sin
 * of pos * inv_freq in fp32, each rounded to fp16; layout [pos, hd/2]. */
ORC_EXPORT void orc_rope_table(int max_seq, int head_dim, float theta,
                               uint16_t *cos_tab, uint16_t *sin_tab)
{
    int hd2 = head_dim / 2;
    for (int pos = 0; pos < max_seq; pos++)
        for (int i = 0; i < hd2; i++) {
            float f = 1.0f / powf(theta, 2.0f * (float)i / (float)head_dim);
            float ang = (float)pos * f;
            cos_tab[(int64_t)pos * hd2 + i] = orc_f32_to_f16(cosf(ang));
            sin_tab[(int64_t)pos * hd2 + i] = orc_f32_to_f16(sinf(ang));
        }
}

/* ApplyRopePartial (Qwen3_5CS.compute:367-393): pair (i, i + rot/2) for i < rot/2 of
 * every head, dims [rot, hd) untouched; tables [pos, rot/2] (Qwen3_5Model.cs:228-260:
 * inv_freq_i = 1 / theta^(2i/rot)). */
ORC_EXPORT void orc_rope_apply_partial(float *buf, int seq_len, int num_heads, int head_dim, int rot,
                                       int position_offset, const uint16_t *cos_tab, const uint16_t *sin_tab)
{
    int r2 = rot / 2;
    for (int l = 0; l < seq_len; l++)
        for (int h = 0; h < num_heads; h++) {
            float *b = buf + ((int64_t)l * num_heads + h) * head_dim;
            int64_t p = (int64_t)(position_offset + l) * r2;
            for (int i = 0; i < r2; i++) {
                float x1 = b[i], x2 = b[i + r2];
                float c = read_h(cos_tab, p + i), s = read_h(sin_tab, p + i);
                b[i] = x1 * c - x2 * s;
                b[i + r2] = x2 * c + x1 * s;
            }
        }
}

/* ApplyRopeSplitHalf (G3CS:271-297): pair (i, i + hd/2) of every head. */
ORC_EXPORT void orc_rope_apply(float *buf, int seq_len, int num_heads, int head_dim,
                               int position_offset, const uint16_t *cos_tab,
                               const uint16_t *sin_tab)
{
    int hd2 = head_dim / 2;
    for (int l = 0; l < seq_len; l++)
        for (int h = 0; h < num_heads; h++) {
            float *b = buf + ((int64_t)l * num_heads + h) * head_dim;
            int64_t p = (int64_t)(position_offset + l) * hd2;
            for (int i = 0; i < hd2; i++) {
                float x1 = b[i], x2 = b[i + hd2];
                float c = read_h(cos_tab, p + i), s = read_h(sin_tab, p + i);
                b[i] = x1 * c - x2 * s;
                b[i + hd2] = x2 * c + x1 * s;
            }
        }
}

/* WriteCacheFull, fp16 variant (G3CS:382-411 + KVH:33-43): element
 * ((cache_len + l) * Hkv + h) * hd + d of the [capacity, Hkv, hd] cache. */
ORC_EXPORT void orc_kv_write(const float *kv_new, int seq_len, int hkv, int head_dim,
                             int cache_len, uint16_t *cache)
{
    int64_t n = (int64_t)seq_len * hkv * head_dim;
    int64_t off = (int64_t)cache_len * hkv * head_dim;
    for (int64_t i = 0; i < n; i++) cache[off + i] = orc_f32_to_f16(kv_new[i]);
}

/* WriteCacheFull, INT8 variant (G3CS:300-380, KVH:46-82): one (token, kv head)
 * row of head_dim values at a time.  min / max over the row, scale = (max -
 * min) / 255 (floored at 1e-9), zp = round(-min / scale) clamped to [0, 255],
 * q = clamp(round(x * (1 / scale)) + zp, 0, 255); round() is round-half-even
 * (HLSL round); the row's fp16 (scale | zp << 16) word goes to sz[pos * hkv + h].
 * Divisions and the reciprocal are IEEE fp32. */
ORC_EXPORT void orc_kv_write_int8(const float *kv_new, int seq_len, int hkv, int head_dim,
                                  int cache_len, uint8_t *cache, uint32_t *sz)
{
    for (int l = 0; l < seq_len; l++)
        for (int h = 0; h < hkv; h++) {
            const float *x = kv_new + ((int64_t)l * hkv + h) * head_dim;
            float mn = 3.0e38f, mx = -3.0e38f;
            for (int d = 0; d < head_dim; d++) {
                mn = fminf(mn, x[d]);
                mx = fmaxf(mx, x[d]);
            }
            float scale = (mx - mn) / 255.0f;
            if (scale < 1e-9f) scale = 1e-9f;
            float zp = rintf(-mn / scale);
            zp = zp < 0.0f ? 0.0f : (zp > 255.0f ? 255.0f : zp);
            const float inv = 1.0f / scale;
            const int64_t row = ((int64_t)(cache_len + l) * hkv + h);
            for (int d = 0; d < head_dim; d++) {
                float v = rintf(x[d] * inv) + zp;
                v = v < 0.0f ? 0.0f : (v > 255.0f ? 255.0f : v);
                cache[row * head_dim + d] = (uint8_t)v;
            }
            sz[row] = (uint32_t)orc_f32_to_f16(scale) | ((uint32_t)orc_f32_to_f16(zp) << 16);
        }
}

/* kv_unpack8 (KVH:55-62): element d of cache row `row`. */
static inline float read_kv8(const uint8_t *cache, const uint32_t *sz, int64_t row, int hd, int d)
{
    const uint32_t w = sz[row];
    const float scale = orc_f16_to_f32((uint16_t)(w & 0xffffu)), zp = orc_f16_to_f32((uint16_t)(w >> 16));
    return ((float)cache[row * hd + d] - zp) * scale;
}

/* FlashAttention (G3CS:643-753): one (query position, q head) at a time, KV
 * tiles of 256, tree max / tree sum per tile, online rescale, causal
 * j_hi = abs_q, out = acc / max(l, 1e-12).  K/V are fp16 caches laid out
 * [pos, Hkv, hd]; Q and out are fp32 [seq_q, Hq, hd]. */
#define FA_T 256
static void flash_attention_any(const float *Q, const uint16_t *Kc, const uint16_t *Vc, const uint8_t *K8,
                                const uint32_t *Ksz, const uint8_t *V8, const uint32_t *Vsz,
                                int seq_q, int kv_len, int hq, int hkv, int hd, float scale, int window,
                                float *out);

ORC_EXPORT void orc_flash_attention(const float *Q, const uint16_t *Kc, const uint16_t *Vc,
                                    int seq_q, int kv_len, int hq, int hkv, int hd,
                                    float scale, float *out)
{
    flash_attention_any(Q, Kc, Vc, NULL, NULL, NULL, NULL, seq_q, kv_len, hq, hkv, hd, scale, 0, out);
}

/* The same over an INT8 cache (KV_READ_K / KV_READ_V of the KV_INT8 variant). */
ORC_EXPORT void orc_flash_attention_kv8(const float *Q, const uint8_t *K8, const uint32_t *Ksz,
                                        const uint8_t *V8, const uint32_t *Vsz, int seq_q, int kv_len,
                                        int hq, int hkv, int hd, float scale, float *out)
{
    flash_attention_any(Q, NULL, NULL, K8, Ksz, V8, Vsz, seq_q, kv_len, hq, hkv, hd, scale, 0, out);
}

/* Sliding-window FlashAttention (G3CS:673-686): query abs_q sees positions
 * j_lo .. abs_q, j_lo = abs_q - window when abs_q > window (else 0); the tile
 * walk starts at j_lo. */
ORC_EXPORT void orc_flash_attention_window(const float *Q, const uint16_t *Kc, const uint16_t *Vc,
                                           int seq_q, int kv_len, int hq, int hkv, int hd, float scale,
                                           int window, float *out)
{
    flash_attention_any(Q, Kc, Vc, NULL, NULL, NULL, NULL, seq_q, kv_len, hq, hkv, hd, scale, window, out);
}

static void flash_attention_any(const float *Q, const uint16_t *Kc, const uint16_t *Vc, const uint8_t *K8,
                                const uint32_t *Ksz, const uint8_t *V8, const uint32_t *Vsz,
                                int seq_q, int kv_len, int hq, int hkv, int hd, float scale, int window,
                                float *out)
{
    int grp = hq / (hkv > 0 ? hkv : 1);
    if (grp < 1) grp = 1;
    #pragma omp parallel for schedule(static) collapse(2)
    for (int qp = 0; qp < seq_q; qp++)
        for (int h = 0; h < hq; h++) {
            int kvh = h / grp;
            int kl = kv_len > 1 ? kv_len : 1;
            int abs_q = (kl - seq_q) + qp;
            int j_hi = abs_q < kl - 1 ? abs_q : kl - 1;
            int j_lo = (window > 0 && abs_q > window) ? abs_q - window : 0;
            float fq[512], acc[512], s[FA_T], p[FA_T], red[FA_T];
            const float *q = Q + ((int64_t)qp * hq + h) * hd;
            for (int d = 0; d < hd; d++) { fq[d] = q[d] * scale; acc[d] = 0.0f; }
            float m = -3.0e38f, l = 0.0f;
            for (int tile = j_lo; tile <= j_hi; tile += FA_T) {
                for (int t = 0; t < FA_T; t++) {
                    int j = tile + t;
                    s[t] = -3.0e38f;
                    if (j <= j_hi) {
                        float dot = 0.0f;
                        if (K8) {
                            for (int d = 0; d < hd; d++)
                                dot = dot + fq[d] * read_kv8(K8, Ksz, (int64_t)j * hkv + kvh, hd, d);
                        } else {
                            const uint16_t *kr = Kc + ((int64_t)j * hkv + kvh) * hd;
                            for (int d = 0; d < hd; d++) dot = dot + fq[d] * read_h(kr, d);
                        }
                        s[t] = dot;
                    }
                    red[t] = s[t];
                }
                for (int r = FA_T / 2; r > 0; r >>= 1)
                    for (int t = 0; t < r; t++) red[t] = fmaxf(red[t], red[t + r]);
                float m_new = fmaxf(m, red[0]);
                for (int t = 0; t < FA_T; t++) {
                    p[t] = (tile + t <= j_hi) ? expf(s[t] - m_new) : 0.0f;
                    red[t] = p[t];
                }
                for (int r = FA_T / 2; r > 0; r >>= 1)
                    for (int t = 0; t < r; t++) red[t] = red[t] + red[t + r];
                float tile_sum = red[0];
                float alpha = expf(m - m_new);
                l = l * alpha + tile_sum;
                int n_valid = j_hi - tile + 1;
                if (n_valid > FA_T) n_valid = FA_T;
                for (int d = 0; d < hd; d++) {
                    float a = acc[d] * alpha;
                    for (int jj = 0; jj < n_valid; jj++)
                        a = a + p[jj] * (V8 ? read_kv8(V8, Vsz, (int64_t)(tile + jj) * hkv + kvh, hd, d)
                                            : read_h(Vc, ((int64_t)(tile + jj) * hkv + kvh) * hd + d));
                    acc[d] = a;
                }
                m = m_new;
            }
            float *o = out + ((int64_t)qp * hq + h) * hd;
            float den = l > 1e-12f ? l : 1e-12f;
            for (int d = 0; d < hd; d++) o[d] = acc[d] / den;
        }
}

/* ArgMax (G3CS:911-928): 256 threads stride the vocab keeping the first
 * strict maximum, then a tree where ties keep the lower thread. */
ORC_EXPORT int orc_argmax(const float *logits, int vocab)
{
    float val[256];
    int idx[256];
    for (int t = 0; t < 256; t++) {
        float bv = -3.0e38f;
        int bi = 0;
        for (int i = t; i < vocab; i += 256)
            if (logits[i] > bv) { bv = logits[i]; bi = i; }
        val[t] = bv; idx[t] = bi;
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int t = 0; t < s; t++)
            if (val[t + s] > val[t]) { val[t] = val[t + s]; idx[t] = idx[t + s]; }
    return idx[0];
}

/* --------------------------------------------------------------- sampler */

/* runif (G3CS:177-186): the shader's hash on its signed int seed.  `>>` on the
 * signed seed is an arithmetic shift; the divisor 4294967295.0 is an fp32
 * literal (2^32 after rounding), so u = float(seed) * 2^-32 + 0.5 in [0, 1). */
ORC_EXPORT float orc_runif(int32_t *seed)
{
    uint32_t s = (uint32_t)*seed;
    s ^= 2747636419u;
    s *= 2654435769u;
    s ^= (uint32_t)((int32_t)s >> 16);
    s *= 2654435769u;
    s ^= (uint32_t)((int32_t)s >> 16);
    s *= 2654435769u;
    *seed = (int32_t)s;
    return (float)(int32_t)s / 4294967296.0f + 0.5f;
}

#define SMP_THREADS 256
#define SMP_MAXK 64

/* SampleToken (G3CS:1029-1132), the parallel path for 1 <= top_k <= 64: probabilities
 * normalised over the full vocabulary (256 strided partial sums + a tree, as the
 * shader reduces), the top_k largest scaled logits as candidates in descending order
 * (ties: the ArgMax tree order, orc_argmax), min-p and top-p cuts as a prefix walk,
 * then r = runif() * cum against the candidates' running sum.
 * SampleTokenSerial (G3CS:932-1019) for top_k outside 1..64, restricted here to
 * top_p >= 1 and top_k <= 0: min-p filter, full renormalisation, r = runif() and an
 * index-order walk of the cumulative distribution.  temperature <= 0: ArgMax.
 * Returns the sampled id, or -1 for an unsupported combination. */
ORC_EXPORT int orc_sample(const float *logits, int vocab, float temperature, int top_k, float top_p,
                          float min_p, int32_t seed, float *probs_scratch)
{
    if (!(temperature > 0.0f)) return orc_argmax(logits, vocab);
    const float inv_temp = 1.0f / temperature;
    if (top_k >= 1 && top_k <= SMP_MAXK) {
        float *sc = probs_scratch;
        float red[SMP_THREADS];
        for (int t = 0; t < SMP_THREADS; t++) {
            float bv = -3.0e38f;
            for (int i = t; i < vocab; i += SMP_THREADS) {
                const float v = logits[i] * inv_temp;
                sc[i] = v;
                bv = fmaxf(bv, v);
            }
            red[t] = bv;
        }
        for (int s1 = SMP_THREADS / 2; s1 > 0; s1 >>= 1)
            for (int t = 0; t < s1; t++) red[t] = fmaxf(red[t], red[t + s1]);
        const float gmax = red[0];
        for (int t = 0; t < SMP_THREADS; t++) {
            float acc = 0.0f;
            for (int i = t; i < vocab; i += SMP_THREADS) acc = acc + expf(sc[i] - gmax);
            red[t] = acc;
        }
        for (int s2 = SMP_THREADS / 2; s2 > 0; s2 >>= 1)
            for (int t = 0; t < s2; t++) red[t] = red[t] + red[t + s2];
        const float sum_exp = red[0] > 1e-12f ? red[0] : 1e-12f;
        float cand_p[SMP_MAXK];
        int cand_i[SMP_MAXK];
        for (int k = 0; k < top_k; k++) {
            const int wi = orc_argmax(sc, vocab);
            cand_i[k] = wi;
            cand_p[k] = expf(sc[wi] - gmax) / sum_exp;
            sc[wi] = -3.0e38f;
        }
        const float min_thresh = min_p > 0.0f ? cand_p[0] * min_p : 0.0f;
        float cum = 0.0f;
        int count = 0;
        for (int c = 0; c < top_k; c++) {
            const float pc = cand_p[c];
            if (min_p > 0.0f && pc < min_thresh) break;
            if (top_p < 1.0f && cum >= top_p) break;
            cum = cum + pc;
            count++;
        }
        if (count == 0) count = 1;
        int32_t sd = seed;
        const float r = orc_runif(&sd) * cum;
        float cdf = 0.0f;
        int sampled = cand_i[count - 1];
        for (int c = 0; c < count; c++) {
            cdf = cdf + cand_p[c];
            if (cdf >= r) { sampled = cand_i[c]; break; }
        }
        return sampled;
    }
    if (top_k > 0 && top_k < vocab) return -1;
    if (top_p < 1.0f) return -1;
    float *pr = probs_scratch;
    float max_l = logits[0];
    for (int i = 1; i < vocab; i++) max_l = fmaxf(max_l, logits[i]);
    float sum_exp = 0.0f;
    for (int i = 0; i < vocab; i++) {
        const float e = expf((logits[i] - max_l) * inv_temp);
        pr[i] = e;
        sum_exp = sum_exp + e;
    }
    const float inv_sum = 1.0f / (sum_exp > 1e-12f ? sum_exp : 1e-12f);
    for (int i = 0; i < vocab; i++) pr[i] = pr[i] * inv_sum;
    float max_prob = 0.0f;
    for (int i = 0; i < vocab; i++) max_prob = fmaxf(max_prob, pr[i]);
    int cand = 0;
    if (min_p > 0.0f) {
        const float th = max_prob * min_p;
        for (int i = 0; i < vocab; i++) {
            if (pr[i] >= th) cand++;
            else pr[i] = 0.0f;
        }
    } else {
        for (int i = 0; i < vocab; i++)
            if (pr[i] > 0.0f) cand++;
    }
    if (cand == 0) return orc_argmax(logits, vocab);
    float new_sum = 0.0f;
    for (int i = 0; i < vocab; i++) new_sum = new_sum + pr[i];
    if (new_sum <= 0.0f) return orc_argmax(logits, vocab);
    const float inv_new = 1.0f / new_sum;
    for (int i = 0; i < vocab; i++) pr[i] = pr[i] * inv_new;
    int32_t sd = seed;
    const float r = orc_runif(&sd);
    float cdf = 0.0f;
    for (int i = 0; i < vocab; i++) {
        cdf = cdf + pr[i];
        if (cdf >= r) return i;
    }
    return 0;
}

/* ----------------------------------------------------------- whole model */

/* Host-side view of one model (weights as the reference's loader concatenates
 * them, AddConcatW M5/MiniCPM5Weights.cs:139-191): W_QKV = q|k|v rows,
 * mlp = gate|up|down, scale buffers concatenated in the same row order. */
typedef struct {
    int32_t hidden, inter, layers, hq, hkv, hd, vocab;
    int32_t quant, group, capacity;
    float eps, theta, embed_scale;
    const void **w_qkv;  const uint16_t **s_qkv;
    const void **w_o;    const uint16_t **s_o;
    const void **w_mlp;  const uint16_t **s_mlp;
    const uint16_t **ln1; const uint16_t **ln2;
    const uint16_t *final_norm;
    const uint16_t *embed;
    const uint16_t *lm_head;
    const uint16_t *rope_cos; const uint16_t *rope_sin;
    uint16_t **k_cache; uint16_t **v_cache;     /* per layer [capacity, hkv, hd]; uint8 for kv_quant 2 */
    int32_t cache_len;
    int32_t kv_quant;                            /* 2: INT8 cache (k_sz / v_sz per layer [capacity, hkv]) */
    uint32_t **k_sz; uint32_t **v_sz;
    /* Gemma3 variants (Gemma3Model.cs:315-590): arch bits 1 qk-norm (q_norm / k_norm [hd]),
     * 2 sandwich norms (post_attn_ln / post_ffn_ln [H]; ln2 is then the pre-MLP norm),
     * 4 GELU GLU; sliding-window layers (window > 0: every layer except each pattern-th)
     * use the local RoPE tables; attn_scale 0 = hd^-0.5. */
    int32_t arch, window, pattern;
    float attn_scale;
    const uint16_t *rope_cos_local; const uint16_t *rope_sin_local;
    const uint16_t **q_norm; const uint16_t **k_norm;
    const uint16_t **post_attn_ln; const uint16_t **post_ffn_ln;
    /* Qwen3.5 full-attention layers (Qwen3_5Model.cs:397-574): arch bit 8 = gated q
     * (QProjGated, Qwen3_5CS.compute:306-330: head h's rows are hd q rows then hd gate rows;
     * ApplyAttnGate :706-714: attended *= sigmoid(gate)); rot_dim < hd = partial RoPE with
     * the rope_*_partial tables [pos, rot_dim/2]. */
    int32_t rot_dim;
    const uint16_t *rope_cos_partial; const uint16_t *rope_sin_partial;
} orc_model;

static int layer_is_sliding(const orc_model *md, int li)
{
    return md->window > 0 && (md->pattern <= 0 || (li + 1) % md->pattern != 0);
}

/* MiniCPM5Model.Forward(ids, useCache = true, lastPosOnly) (M5M:531-549) with
 * DispatchLayer (M5M:294-518) and DispatchFinalLast / DispatchFinalAll
 * (M5M:598-650).  logits: [V] if last_pos_only else [seq_len, V].
 * Returns 0, or -1 if the cache would overflow. */
ORC_EXPORT int orc_forward(orc_model *md, const int32_t *ids, int seq_len, int last_pos_only,
                           float *logits)
{
    const int H = md->hidden, I = md->inter, hq = md->hq, hkv = md->hkv, hd = md->hd;
    const int gated = (md->arch & 8) != 0;
    const int inner = hq * hd, qkvd = (gated ? 2 : 1) * inner + 2 * hkv * hd, S = seq_len;
    const int rot = md->rot_dim > 0 && md->rot_dim < hd ? md->rot_dim : hd;
    if (md->cache_len + S > md->capacity) return -1;
    const int cache_len = md->cache_len, kv_len = cache_len + S;
    const float scale = md->attn_scale > 0.0f ? md->attn_scale : powf((float)hd, -0.5f);

    float *hidden = malloc(sizeof(float) * S * H), *skip = malloc(sizeof(float) * S * H);
    float *norm = malloc(sizeof(float) * S * H), *qkv = malloc(sizeof(float) * S * qkvd);
    float *q = malloc(sizeof(float) * S * inner), *k = malloc(sizeof(float) * S * hkv * hd);
    float *v = malloc(sizeof(float) * S * hkv * hd), *att = malloc(sizeof(float) * S * inner);
    float *ao = malloc(sizeof(float) * S * H), *mid = malloc(sizeof(float) * S * I);
    float *g = malloc(sizeof(float) * S * I), *u = malloc(sizeof(float) * S * I);
    float *gate = malloc(sizeof(float) * S * inner);

    for (int l = 0; l < S; l++)                                   /* EmbeddingLookup G3CS:189-201 */
        for (int h = 0; h < H; h++)
            hidden[(int64_t)l * H + h] = read_h(md->embed, (uint64_t)ids[l] * H + h) * md->embed_scale;

    for (int li = 0; li < md->layers; li++) {
        memcpy(skip, hidden, sizeof(float) * S * H);
        orc_rmsnorm(hidden, S, H, md->ln1[li], md->eps, norm);
        orc_gemv(norm, S, H, md->w_qkv[li], md->s_qkv[li], md->quant, md->group, 0, qkvd, qkv);
        const int kv0 = (gated ? 2 : 1) * inner;                    /* first k row */
        for (int l = 0; l < S; l++) {                              /* SplitQKV G3CS:249-269 */
            if (gated)                                             /* QProjGated's split */
                for (int h = 0; h < hq; h++) {
                    memcpy(q + (int64_t)l * inner + h * hd, qkv + (int64_t)l * qkvd + h * 2 * hd, sizeof(float) * hd);
                    memcpy(gate + (int64_t)l * inner + h * hd, qkv + (int64_t)l * qkvd + h * 2 * hd + hd,
                           sizeof(float) * hd);
                }
            else
                memcpy(q + (int64_t)l * inner, qkv + (int64_t)l * qkvd, sizeof(float) * inner);
            memcpy(k + (int64_t)l * hkv * hd, qkv + (int64_t)l * qkvd + kv0, sizeof(float) * hkv * hd);
            memcpy(v + (int64_t)l * hkv * hd, qkv + (int64_t)l * qkvd + kv0 + hkv * hd, sizeof(float) * hkv * hd);
        }
        if (md->arch & 1) {                                        /* RmsNormHead on q and k */
            rmsnorm_heads(q, S * hq, hd, md->q_norm[li], md->eps);
            rmsnorm_heads(k, S * hkv, hd, md->k_norm[li], md->eps);
        }
        const int sw = layer_is_sliding(md, li);
        const uint16_t *rc = sw && md->rope_cos_local ? md->rope_cos_local : md->rope_cos;
        const uint16_t *rs = sw && md->rope_sin_local ? md->rope_sin_local : md->rope_sin;
        const int win = sw ? md->window : 0;
        if (rot < hd) {
            orc_rope_apply_partial(q, S, hq, hd, rot, cache_len, md->rope_cos_partial, md->rope_sin_partial);
            orc_rope_apply_partial(k, S, hkv, hd, rot, cache_len, md->rope_cos_partial, md->rope_sin_partial);
        } else {
            orc_rope_apply(q, S, hq, hd, cache_len, rc, rs);
            orc_rope_apply(k, S, hkv, hd, cache_len, rc, rs);
        }
        if (md->kv_quant == 2) {
            orc_kv_write_int8(k, S, hkv, hd, cache_len, (uint8_t *)md->k_cache[li], md->k_sz[li]);
            orc_kv_write_int8(v, S, hkv, hd, cache_len, (uint8_t *)md->v_cache[li], md->v_sz[li]);
            flash_attention_any(q, NULL, NULL, (const uint8_t *)md->k_cache[li], md->k_sz[li],
                                (const uint8_t *)md->v_cache[li], md->v_sz[li], S, kv_len, hq, hkv, hd, scale, win,
                                att);
        } else {
            orc_kv_write(k, S, hkv, hd, cache_len, md->k_cache[li]);
            orc_kv_write(v, S, hkv, hd, cache_len, md->v_cache[li]);
            flash_attention_any(q, md->k_cache[li], md->v_cache[li], NULL, NULL, NULL, NULL, S, kv_len, hq, hkv, hd,
                                scale, win, att);
        }
        if (gated)                                                 /* ApplyAttnGate */
            for (int64_t i = 0; i < (int64_t)S * inner; i++) att[i] = att[i] * (1.0f / (1.0f + expf(-gate[i])));
        orc_gemv(att, S, inner, md->w_o[li], md->s_o[li], md->quant, md->group, 0, H, ao);
        if (md->arch & 2) {                                        /* post-attention norm, then the residual */
            orc_rmsnorm(ao, S, H, md->post_attn_ln[li], md->eps, norm);
            memcpy(ao, norm, sizeof(float) * S * H);
        }
        for (int64_t i = 0; i < (int64_t)S * H; i++) ao[i] = ao[i] + skip[i];     /* AddResidual */
        memcpy(skip, ao, sizeof(float) * S * H);
        orc_rmsnorm(ao, S, H, md->ln2[li], md->eps, hidden);
        /* GateUp1VecCoal (G3CS:1244-1267): gate rows [0,I), up rows [I,2I) */
        orc_gemv(hidden, S, H, md->w_mlp[li], md->s_mlp[li], md->quant, md->group, 0, I, g);
        orc_gemv(hidden, S, H, md->w_mlp[li], md->s_mlp[li], md->quant, md->group, I, I, u);
        for (int64_t i = 0; i < (int64_t)S * I; i++)
            mid[i] = ((md->arch & 4) ? gelu_ref(g[i]) : silu_ref(g[i])) * u[i];
        /* Down1VecCoal (G3CS:1269-1282): rows [2I, 2I+H) of the concat, K = I */
        {
            orc_w W = { md->w_mlp[li], md->s_mlp[li], md->quant, md->group };
            #pragma omp parallel for schedule(static) collapse(2)
            for (int l = 0; l < S; l++)
                for (int n = 0; n < H; n++) {
                    uint64_t base = 2ull * H * I + (uint64_t)n * I;
                    hidden[(int64_t)l * H + n] = coal_dot(mid + (int64_t)l * I, I, &W, base) *
                                                 w_scale(&W, 2ull * I + n);
                }
        }
        if (md->arch & 2) {                                        /* post-FFN norm, then the residual */
            orc_rmsnorm(hidden, S, H, md->post_ffn_ln[li], md->eps, norm);
            memcpy(hidden, norm, sizeof(float) * S * H);
        }
        for (int64_t i = 0; i < (int64_t)S * H; i++) hidden[i] = hidden[i] + skip[i];
    }
    md->cache_len += S;

    int rows = last_pos_only ? 1 : S;
    const float *src = last_pos_only ? hidden + (int64_t)(S - 1) * H : hidden;
    orc_rmsnorm(src, rows, H, md->final_norm, md->eps, norm);
    orc_gemv(norm, rows, H, md->lm_head, NULL, ORC_FP16, 0, 0, md->vocab, logits);

    free(hidden); free(skip); free(norm); free(qkv); free(q); free(k); free(v);
    free(att); free(ao); free(mid); free(g); free(u); free(gate);
    return 0;
}

/* -------------------------------------------- CPU module path (baseline) */

/* Dense.Linear (MOD/Learnable/Dense.cs:261-303) on fp32 weights [H_out, H_in]:
 * 1-D input -> Parallel.For over output rows; 2-D input [B, H_in] ->
 * Parallel.For over the batch.  Sequential k sum starting from the bias.
 * `threads` <= 0 uses every available thread. */
ORC_EXPORT void orc_dense_linear(const float *x, int batch, int batched, int h_in, int h_out,
                                 const float *W, const float *bias, float *y, int threads)
{
#ifdef _OPENMP
    int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    (void)threads;
#endif
    if (batched) {
        #pragma omp parallel for schedule(static) num_threads(nt)
        for (int b = 0; b < batch; b++)
            for (int o = 0; o < h_out; o++) {
                float sum = bias ? bias[o] : 0.0f;
                const float *wr = W + (int64_t)o * h_in;
                const float *xb = x + (int64_t)b * h_in;
                for (int i = 0; i < h_in; i++) sum = sum + xb[i] * wr[i];
                y[(int64_t)b * h_out + o] = sum;
            }
    } else {
        #pragma omp parallel for schedule(static) num_threads(nt)
        for (int o = 0; o < h_out; o++) {
            float sum = bias ? bias[o] : 0.0f;
            const float *wr = W + (int64_t)o * h_in;
            for (int i = 0; i < h_in; i++) sum = sum + x[i] * wr[i];
            y[o] = sum;
        }
    }
}

/* One decode layer of the CPU module composition the reference runs on the
 * CPU (MOD: RMSNorm.Predict -> GroupedQueryAttention.Predict with RoPE and a
 * growing KV cache -> residual -> RMSNorm -> GatedLinearUnit("silu") ->
 * residual), on fp32 dequantised weights, one token.  Linears use the 1-D
 * Dense.Linear path (Parallel.For over output rows); attention scores and
 * values run Parallel.For over q heads (GroupedQueryAttention.cs:387-473);
 * RoPE uses fp32 tables (RotaryPositionalEmbeddings.cs:48-58).  The debug
 * string GatedLinearUnit.Predict builds each call is left out.
 * kcache/vcache: fp32 [capacity, hkv, hd]; pos = tokens already cached.
 * scratch needs 2*H + qkvd + 2*inner + 3*I + hq*(pos+1) floats. */
ORC_EXPORT void orc_module_layer_decode(float *x, int H, int I, int hq, int hkv, int hd,
                                        float eps, float theta,
                                        const float *ln1, const float *ln2,
                                        const float *Wqkv, const float *Wo,
                                        const float *Wg, const float *Wu, const float *Wd,
                                        float *kcache, float *vcache, int pos,
                                        float *scratch, int threads)
{
#ifdef _OPENMP
    int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    int nt = 1; (void)threads;
#endif
    const int inner = hq * hd, qkvd = inner + 2 * hkv * hd, L = pos + 1, grp = hq / hkv;
    float *xn = scratch, *qkv = xn + H, *att = qkv + qkvd, *o = att + inner;
    float *g = o + H, *u = g + I, *mid = u + I, *sc = mid + I;
    (void)inner;
    /* RMSNorm.Predict (MOD/Learnable/Norm/RMSNorm.cs:67-83): x * rsqrt(mean(x^2) + eps) * gamma */
    float ms = 0.0f;
    for (int i = 0; i < H; i++) ms = ms + x[i] * x[i];
    ms = ms / (float)H;
    float r = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < H; i++) xn[i] = x[i] * r * ln1[i];
    orc_dense_linear(xn, 1, 0, H, qkvd, Wqkv, NULL, qkv, nt);
    /* RoPE split-half with fp32 tables on q and k, then append k, v to the cache */
    for (int part = 0; part < 2; part++) {
        int nh = part == 0 ? hq : hkv;
        float *b = part == 0 ? qkv : qkv + inner;
        for (int h = 0; h < nh; h++)
            for (int i = 0; i < hd / 2; i++) {
                float f = 1.0f / powf(theta, (2.0f * (float)i) / (float)hd);
                float ang = (float)pos * f, c = cosf(ang), s = sinf(ang);
                float x1 = b[h * hd + i], x2 = b[h * hd + i + hd / 2];
                b[h * hd + i] = x1 * c - x2 * s;
                b[h * hd + i + hd / 2] = x2 * c + x1 * s;
            }
    }
    memcpy(kcache + (int64_t)pos * hkv * hd, qkv + inner, sizeof(float) * hkv * hd);
    memcpy(vcache + (int64_t)pos * hkv * hd, qkv + inner + hkv * hd, sizeof(float) * hkv * hd);
    const float scale = 1.0f / sqrtf((float)hd);
    #pragma omp parallel for schedule(static) num_threads(nt)
    for (int h = 0; h < hq; h++) {
        int kh = h / grp;
        float *srow = sc + (int64_t)h * L;
        float mx = -INFINITY;
        for (int j = 0; j < L; j++) {
            float dot = 0.0f;
            for (int d = 0; d < hd; d++) dot = dot + qkv[h * hd + d] * kcache[((int64_t)j * hkv + kh) * hd + d];
            srow[j] = dot * scale;
            if (srow[j] > mx) mx = srow[j];
        }
        float sum = 0.0f;
        for (int j = 0; j < L; j++) { srow[j] = expf(srow[j] - mx); sum = sum + srow[j]; }
        for (int j = 0; j < L; j++) srow[j] = srow[j] / sum;
        for (int d = 0; d < hd; d++) {
            float ws = 0.0f;
            for (int j = 0; j < L; j++) ws = ws + srow[j] * vcache[((int64_t)j * hkv + kh) * hd + d];
            att[h * hd + d] = ws;
        }
    }
    orc_dense_linear(att, 1, 0, hq * hd, H, Wo, NULL, o, nt);
    for (int i = 0; i < H; i++) x[i] = x[i] + o[i];
    ms = 0.0f;
    for (int i = 0; i < H; i++) ms = ms + x[i] * x[i];
    ms = ms / (float)H;
    r = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < H; i++) xn[i] = x[i] * r * ln2[i];
    orc_dense_linear(xn, 1, 0, H, I, Wu, NULL, u, nt);
    orc_dense_linear(xn, 1, 0, H, I, Wg, NULL, g, nt);
    for (int i = 0; i < I; i++) mid[i] = (g[i] / (expf(-g[i]) + 1.0f)) * u[i];   /* Silu.cs:27-43 */
    orc_dense_linear(mid, 1, 0, I, H, Wd, NULL, o, nt);
    for (int i = 0; i < H; i++) x[i] = x[i] + o[i];
}

ORC_EXPORT int orc_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
