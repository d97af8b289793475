// elementwise.cu -- the small kernels around the GEMVs: embedding gather,
// RMSNorm, argmax finalisation, IMP-exact quantizers and seeded synthetic
// weights.
#include "internal.h"

namespace du {

// EmbeddingLookup (Gemma3CS.compute:189-201): h[t, :] = fp16 embed[tok, :] * scale.
__global__ void embed_kernel(const int *ids, const __half *embed, float scale, int H, float *out)
{
    const int m = blockIdx.y;
    const size_t tok = (size_t)ids[m];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
        out[(size_t)m * H + i] = __half2float(embed[tok * H + i]) * scale;
}

int launch_embed(const int *ids, const __half *embed, float scale, int M, int H, float *out, cudaStream_t st)
{
    if (M <= 0) return DU_OK;
    dim3 grid((H + 255) / 256, M);
    embed_kernel<<<grid, 256, 0, st>>>(ids, embed, scale, H, out);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// RmsNormHidden (Gemma3CS.compute:204-223): one CTA per row.
__global__ void rmsnorm_kernel(const float *x, const __half *g, int H, float eps, float *y)
{
    __shared__ float part[32];
    const float *xr = x + (size_t)blockIdx.x * H;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += part[i];
    const float inv = 1.0f / sqrtf(tot / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        y[(size_t)blockIdx.x * H + i] = xr[i] * inv * (1.0f + __half2float(g[i]));
}

int launch_rmsnorm(const float *x, const __half *g, int rows, int H, float eps, float *y, cudaStream_t st)
{
    if (rows <= 0) return DU_OK;
    rmsnorm_kernel<<<rows, 256, 0, st>>>(x, g, H, eps, y);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// RmsNormHidden + AddResidual (Gemma3Model.cs:515-528, 575-585): the sandwich
// norm of a block output y, then the residual: x_res += y * rms(y) * (1 + gamma').
__global__ void norm_add_kernel(const float *y, const __half *g, int H, float eps, float *x_res)
{
    __shared__ float part[32];
    pdl_wait();
    const float *yr = y + (size_t)blockIdx.x * H;
    float *xr = x_res + (size_t)blockIdx.x * H;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss += yr[i] * yr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += part[i];
    const float inv = 1.0f / sqrtf(tot / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) xr[i] = yr[i] * inv * (1.0f + __half2float(g[i])) + xr[i];
}

int launch_norm_add(const float *y, const __half *g, int rows, int H, float eps, float *x_res, cudaStream_t st)
{
    if (rows <= 0) return DU_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, norm_add_kernel, y, g, H, eps, x_res));
    return DU_OK;
}

// After an EPI_STORE QKV GEMV of a qk-norm model: one warp per (token, head) of
// the fp32 rows [M][hq + 2 hkv][hd] (q heads, k heads, v heads).  q and k:
// RmsNormHead (Gemma3CS.compute:227-245) with their gammas, then split-half RoPE
// (ApplyRopeSplitHalf, :271-297) at the token's position; q goes to q_out, k and
// v to the fp16 cache, or through the INT8 quantization into the INT8 cache.
// A lane holds elements lane * epl .. lane * epl + epl - 1, so a RoPE pair
// (i, i + hd / 2) sits on lanes l and l + 16.
__global__ void __launch_bounds__(256) qkv_post_kernel(QkvPost a)
{
    pdl_wait();
    const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    const int nh = a.hq + 2 * a.hkv;
    if (w >= a.M * nh) return;
    const int m = w / nh, h = w - m * nh;
    const int epl = a.hd >> 5;
    // token row: q heads (each hd q rows, then hd gate rows when gated), k heads, v heads
    const int qw = a.gated ? 2 : 1;
    const float *row_m = a.qkv + (size_t)m * (a.hq * qw + 2 * a.hkv) * a.hd;
    const float *x = row_m + (h < a.hq ? (size_t)h * qw * a.hd : (size_t)(a.hq * (qw - 1) + h) * a.hd) + lane * epl;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = e < epl ? x[e] : 0.0f;
    const bool isq = h < a.hq, isk = !isq && h < a.hq + a.hkv;
    if (isq && a.gated) {            // the head's gate rows, as computed (QProjGated's split)
        float *g = a.gate_out + ((size_t)m * a.hq + h) * a.hd + lane * epl;
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (e < epl) g[e] = x[a.hd + e];
    }
    const __half *gam = isq ? a.q_norm : (isk ? a.k_norm : nullptr);
    if (gam != nullptr) {
        float ss = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++) ss += v[e] * v[e];
        ss = warp_sum(ss);
        const float rms = 1.0f / sqrtf(ss / (float)a.hd + a.eps);
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (e < epl) v[e] = v[e] * rms * (1.0f + __half2float(gam[lane * epl + e]));
    }
    const int pos = a.pos[m];
    if (isq || isk) {
        // split-half RoPE over the first rot dims (all of them: ApplyRopeSplitHalf; fewer:
        // ApplyRopePartial, Qwen3_5CS.compute:367-393): dim d < rot/2 pairs with d + rot/2,
        // which lives rot/2 / epl lanes away; dims >= rot are left as they are
        const int hd2 = a.hd >> 1, rot = a.rot > 0 ? a.rot : a.hd, r2 = rot >> 1, d0 = lane * epl;
        const int xs = r2 / epl;                         // a power of two <= 16 (checked on the host)
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const float o = __shfl_xor_sync(0xffffffffu, v[e], xs);
            if (e < epl && d0 < rot) {
                const bool first = d0 < r2;
                const int i = (first ? d0 : d0 - r2) + e;
                const float c = __half2float(a.rope_cos[(size_t)pos * hd2 + i]);
                const float s = __half2float(a.rope_sin[(size_t)pos * hd2 + i]);
                v[e] = first ? v[e] * c - o * s : v[e] * c + o * s;
            }
        }
    }
    if (isq) {
        float *dst = a.q_out + ((size_t)m * a.hq + h) * a.hd + lane * epl;
#pragma unroll
        for (int e = 0; e < 8; e++)
            if (e < epl) dst[e] = v[e];
        return;
    }
    const int kh = isk ? h - a.hq : h - a.hq - a.hkv;
    const int seq = a.seq_of ? a.seq_of[m] : a.seq_off + m;
    const size_t row = ((size_t)seq * a.cap + pos) * a.hkv + kh;
    if (a.kv8.k8 != nullptr) {
        kv8_store_row(v, epl, lane, (isk ? a.kv8.k8 : a.kv8.v8) + row * a.hd, (isk ? a.kv8.ksz : a.kv8.vsz) + row);
        return;
    }
    __half *dst = (isk ? a.k_cache : a.v_cache) + row * a.hd + lane * epl;
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (e < epl) dst[e] = __float2half_rn(v[e]);
}

// ApplyAttnGate (Qwen3_5CS.compute:706-714): att[i] *= 1 / (1 + exp(-gate[i])).
__global__ void __launch_bounds__(256) attn_gate_kernel(float *att, const float *gate, size_t n)
{
    pdl_wait();
    pdl_trigger();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) att[i] = att[i] * (1.0f / (1.0f + expf(-gate[i])));
}

int launch_attn_gate(float *att, const float *gate, size_t n, cudaStream_t st)
{
    if (n == 0) return DU_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_gate_kernel, att, gate, n));
    return DU_OK;
}

int launch_qkv_post(const QkvPost &a, cudaStream_t st)
{
    if (a.M <= 0) return DU_OK;
    if (a.hd % 64 != 0 || a.hd > 256) return fail(DU_EINVAL, "qkv_post: head_dim must be 64, 128, 192 or 256");
    const int warps = a.M * (a.hq + 2 * a.hkv);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((warps + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, qkv_post_kernel, a));
    return DU_OK;
}

// Final greedy pick from the per-CTA (max, argmax) partials of the lm_head
// GEMV: the largest value wins, ties follow the reference's ArgMax tree
// (am_better, common.cuh).  Writes the id (and optionally the next step's input
// id, for the device-resident loop) or, with `pairs`, the (value, index-bits)
// pair that tensor-parallel ranks exchange.

__global__ void argmax_final_kernel(const float *am_val, const int *am_idx, int nparts, int *out_ids,
                                    int *feed_ids, float *pairs, TokHist hist)
{
    const int m = blockIdx.x;
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
        const float v = am_val[(size_t)m * nparts + i];
        const int ix = am_idx[(size_t)m * nparts + i];
        if (am_better(v, ix, bv, bi)) { bv = v; bi = ix; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        bv = sv[0]; bi = si[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (am_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
        if (pairs) {
            pairs[2 * m] = bv;
            pairs[2 * m + 1] = __int_as_float(bi);
        } else {
            out_ids[m] = bi;
            if (feed_ids) feed_ids[m] = bi;
            if (hist.tok) hist.tok[(size_t)m * hist.cap + hist.cache_len[m]] = bi;
        }
    }
}

int launch_argmax_final(const float *am_val, const int *am_idx, int M, int nparts, int *out_ids, int *feed_ids,
                        TokHist hist, cudaStream_t st)
{
    if (M <= 0) return DU_OK;
    argmax_final_kernel<<<M, 256, 0, st>>>(am_val, am_idx, nparts, out_ids, feed_ids, nullptr, hist);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

int launch_argmax_final_pairs(const float *am_val, const int *am_idx, int M, int nparts, float *pairs,
                              cudaStream_t st)
{
    if (M <= 0) return DU_OK;
    argmax_final_kernel<<<M, 256, 0, st>>>(am_val, am_idx, nparts, nullptr, nullptr, pairs, TokHist{});
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// gpairs [tp][maxb][2]: best (value, index) of each rank's vocab shard
__global__ void argmax_pick_tp_kernel(const float *gpairs, int tp, int maxb, int M, int *out_ids, int *feed_ids,
                                      TokHist hist)
{
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < tp; r++) {
        const float v = gpairs[((size_t)r * maxb + m) * 2];
        const int i = __float_as_int(gpairs[((size_t)r * maxb + m) * 2 + 1]);
        if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    out_ids[m] = bi;
    if (feed_ids) feed_ids[m] = bi;
    if (hist.tok) hist.tok[(size_t)m * hist.cap + hist.cache_len[m]] = bi;
}

int launch_argmax_pick_tp(const float *gpairs, int tp, int maxb, int M, int *out_ids, int *feed_ids,
                          TokHist hist, cudaStream_t st)
{
    if (M <= 0) return DU_OK;
    argmax_pick_tp_kernel<<<(M + 127) / 128, 128, 0, st>>>(gpairs, tp, maxb, M, out_ids, feed_ids, hist);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

__global__ void add_inplace_kernel(float *y, const float *x, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] += x[i];
}

int launch_add_inplace(float *y, const float *x, size_t n, cudaStream_t st)
{
    if (n == 0) return DU_OK;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    add_inplace_kernel<<<grid, 256, 0, st>>>(y, x, n);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

__global__ void step_advance_kernel(int *cache_len, int M)
{
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m < M) cache_len[m] += 1;
}

int launch_step_advance(int *cache_len, int M, cudaStream_t st)
{
    step_advance_kernel<<<(M + 127) / 128, 128, 0, st>>>(cache_len, M);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// ---------------------------------------------------------------- quantizers

// quantize_int8 (import_params.py:229-233), one CTA per row: fp32 absmax,
// s = max(absmax / 127, 1e-8), q = clip(rint(w / s), -127, 127) with IEEE
// division and round-half-even, s stored as fp16 (RNE).  Bit-exact with numpy.
__global__ void quantize_int8_kernel(const float *w, int64_t cols, int8_t *q, __half *s)
{
    __shared__ float part[32];
    const float *wr = w + (size_t)blockIdx.x * cols;
    float mx = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) mx = fmaxf(mx, fabsf(wr[c]));
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = mx;
    __syncthreads();
    float m = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, part[i]);
    float sc = __fdiv_rn(m, 127.0f);
    if (!(sc >= 1e-8f)) sc = 1e-8f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        float v = rintf(__fdiv_rn(wr[c], sc));
        v = fminf(fmaxf(v, -127.0f), 127.0f);
        q[(size_t)blockIdx.x * cols + c] = (int8_t)v;
    }
    if (threadIdx.x == 0) s[blockIdx.x] = __float2half_rn(sc);
}

int launch_quantize_int8(const float *w, int64_t rows, int64_t cols, int8_t *q, __half *s, cudaStream_t st)
{
    if (rows <= 0) return DU_OK;
    if (rows > 0x7fffffff) return fail(DU_EINVAL, "quantize_int8: too many rows");
    quantize_int8_kernel<<<(unsigned)rows, 256, 0, st>>>(w, cols, q, s);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// quantize_int4 (import_params.py:236-248) with group size G: one warp per
// group; the element of largest |w| (lowest index on ties, numpy argmax)
// gives d = w / -8, |d| < 1e-10 -> 1e-10, q = clip(rint(w / d) + 8, 0, 15),
// low nibble = even column, d stored fp16 [rows, cols / G].
__global__ void quantize_int4_kernel(const float *w, int64_t rows, int64_t cols, int group, uint8_t *p,
                                     __half *s)
{
    const int64_t ng = cols / group;
    const int64_t gid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gid >= rows * ng) return;
    const int64_t r = gid / ng, g = gid - r * ng;
    const float *gr = w + r * cols + g * group;
    float ba = -1.0f;
    int bi = 0;
    for (int k = lane; k < group; k += 32) {
        const float a = fabsf(gr[k]);
        if (a > ba) { ba = a; bi = k; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, ba, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oa > ba || (oa == ba && oi < bi)) { ba = oa; bi = oi; }
    }
    float d = __fdiv_rn(gr[bi], -8.0f);
    if (fabsf(d) < 1e-10f) d = 1e-10f;
    uint8_t *pr = p + (r * cols + g * group) / 2;
    for (int k = 2 * lane; k < group; k += 64) {
        float v0 = rintf(__fdiv_rn(gr[k], d)) + 8.0f;
        float v1 = rintf(__fdiv_rn(gr[k + 1], d)) + 8.0f;
        v0 = fminf(fmaxf(v0, 0.0f), 15.0f);
        v1 = fminf(fmaxf(v1, 0.0f), 15.0f);
        pr[k >> 1] = (uint8_t)((unsigned)v0 | ((unsigned)v1 << 4));
    }
    if (lane == 0) s[r * ng + g] = __float2half_rn(d);
}

int launch_quantize_int4(const float *w, int64_t rows, int64_t cols, int group, uint8_t *p, __half *s,
                         cudaStream_t st)
{
    if (rows <= 0) return DU_OK;
    if (group <= 0 || group % 2 || cols % group) return fail(DU_EINVAL, "quantize_int4: cols % group != 0");
    const int64_t groups = rows * (cols / group);
    const int64_t blocks = (groups + 7) / 8;
    if (blocks > 0x7fffffff) return fail(DU_EINVAL, "quantize_int4: matrix too large");
    quantize_int4_kernel<<<(unsigned)blocks, 256, 0, st>>>(w, rows, cols, group, p, s);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// ------------------------------------------------------- synthetic weights
// Counter-based generator: a 64-bit mix (splitmix64 finaliser) of
// (seed, index) gives two uniforms, Box-Muller turns them into a normal.
// Only used to stand in for checkpoints; parity tests load host weights.
__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i)
{
    const uint64_t h = mix64(seed ^ mix64(i));
    const float u1 = ((float)(uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)(uint32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void random_normal_kernel(float *out, size_t n, uint64_t seed, uint64_t off, float std)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = std * normal_at(seed, off + i);
}

__global__ void random_normal_half_kernel(__half *out, size_t n, uint64_t seed, uint64_t off, float std)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(std * normal_at(seed, off + i));
}

int launch_random_normal(float *out, size_t n, uint64_t seed, uint64_t off, float std, cudaStream_t st)
{
    if (n == 0) return DU_OK;
    random_normal_kernel<<<num_sms() * 8, 256, 0, st>>>(out, n, seed, off, std);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

int launch_random_normal_half(__half *out, size_t n, uint64_t seed, uint64_t off, float std, cudaStream_t st)
{
    if (n == 0) return DU_OK;
    random_normal_half_kernel<<<num_sms() * 8, 256, 0, st>>>(out, n, seed, off, std);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

__global__ void fill_half_kernel(__half *out, size_t n, float v)
{
    const __half h = __float2half_rn(v);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = h;
}

int launch_fill_half(__half *out, size_t n, float v, cudaStream_t st)
{
    if (n == 0) return DU_OK;
    fill_half_kernel<<<num_sms() * 4, 256, 0, st>>>(out, n, v);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

__global__ void convert_kernel(const void *x, int dtype, size_t n, float *out)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v;
        if (dtype == DU_DTYPE_F16) v = __half2float(reinterpret_cast<const __half *>(x)[i]);
        else if (dtype == DU_DTYPE_BF16) {
            const uint16_t b = reinterpret_cast<const uint16_t *>(x)[i];
            v = __uint_as_float((uint32_t)b << 16);
        } else v = reinterpret_cast<const float *>(x)[i];
        out[i] = v;
    }
}

int launch_convert_to_f32(const void *x, int dtype, size_t n, float *out, cudaStream_t st)
{
    if (n == 0) return DU_OK;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    convert_kernel<<<grid, 256, 0, st>>>(x, dtype, n, out);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

}  // namespace du
