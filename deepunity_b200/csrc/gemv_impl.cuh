// gemv_impl.cuh -- device implementation of the decode GEMV (design notes in
// gemv.cuh), shared by the standalone kernel (gemv.cu) and the persistent
// decode-step kernel (decode_step.cu).
//
// A GEMV runs in two phases so that a persistent kernel can overlap them with a
// grid barrier:
//   prefetch(): compute this CTA / warp's share of the rows and issue the first
//               D - 1 ring stages of weight (and INT4 scale) loads;
//   run():      stage the activations (needs the producer's output), stream the
//               rest of the weights through the ring, run the epilogues.
#pragma once

#include "gemv.cuh"
#include "tp_fuse.cuh"

// Timing hook: GV_STAMP(event) marks the phases of a GEMV launch (entry,
// ring issued, dependency met, activations staged, stream done, exit) for a
// timing build; it compiles to nothing in the library.
#ifndef GV_STAMP
#define GV_STAMP(event)
#endif

namespace du {

// FP16 path: physical float4 slot of logical float4 f of a token row
// (conflict-free for the lane-chunk reads of the main loop).
__device__ __forceinline__ int gv_swz16(int f) { return f ^ ((f >> 3) & 1); }

// x_k (optionally RMSNorm'd: x * rms * (1 + gamma'_k)), computed identically
// wherever it is needed
__device__ __forceinline__ float gv_xval(const GemvParams &p, const float *xr, float inv, int k)
{
    float v = xr[k];
    if (p.gamma != nullptr) v = v * inv * (1.0f + __half2float(p.gamma[k]));
    return v;
}

// Residual rows a CTA of an EPI_RESID launch keeps in shared memory (more rows:
// the epilogue reads the residual from global memory instead).
constexpr int GV_YRES_ROWS = 32;

// Shared-memory scratch a GEMV run needs besides the ring and activation stage.
template <int MT, int NW = GV_WARPS>
struct __align__(16) GemvShared {
    float yres[GV_YRES_ROWS * MT];   // EPI_RESID: this CTA's residual rows, [row - first row][token]
    float red[2 * NW];
    float ssq[NW][MT];   // per-warp sums of squares (RMSNorm)
    float xscale[MT];          // per-token factor of the folded dot product
    float amv[NW][MT];
    int ami[NW][MT];
    float pbuf[NW][2][16];     // partial row groups split between warps (first / last); rows x tokens <= 16
};

// Stages the activations of the MT tokens in shared memory.
//  INT4: one pass; per 32-column chunk 6 plane words x 4 word groups, then
//        (128 * sum x_int, 2^-(s + 4)) in the pad words 24, 25 (the factor 16 of
//        the odd-nibble sums, gv_unit_math); xscale = 1 / rms (or 1)
//  INT8: per-token power-of-two scale over the normalised x; xscale = 2^-s
//  FP16: x * (1 + gamma') in fp32, swizzled; xscale = 1 / rms (or 1)
template <int QT, int MT, int NW>
__device__ __forceinline__ void gv_stage_x(const GemvParams &p, uint4 *xq, GemvShared<MT, NW> &sh, int nchunk)
{
    constexpr int NT = NW * 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (QT == Q_I8) {
        for (int m = 0; m < MT; m++) {
            const float *xr = p.x + (size_t)m * p.ldx;
            const bool live = m < p.M;
            // sum of squares (RMSNorm) and max |x * (1 + gamma')| (fixed-point range)
            float ss = 0.0f, mx = 0.0f;
            if (live) {
                for (int k4 = tid; k4 < (p.K >> 2); k4 += NT) {
                    const float4 v = reinterpret_cast<const float4 *>(xr)[k4];
                    float g0 = 1.0f, g1 = 1.0f, g2 = 1.0f, g3 = 1.0f;
                    if (p.gamma != nullptr) {
                        const __half2 *g2p = reinterpret_cast<const __half2 *>(p.gamma) + 2 * k4;
                        const float2 a = __half22float2(g2p[0]), b = __half22float2(g2p[1]);
                        g0 = 1.0f + a.x; g1 = 1.0f + a.y; g2 = 1.0f + b.x; g3 = 1.0f + b.y;
                    }
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * g0), fabsf(v.y * g1)), fmaxf(fabsf(v.z * g2), fabsf(v.w * g3))));
                }
            }
            ss = warp_sum(ss);
            mx = warp_max(mx);
            __syncthreads();
            if (lane == 0) { sh.red[warp] = ss; sh.red[NW + warp] = mx; }
            __syncthreads();
            ss = 0.0f; mx = 0.0f;
#pragma unroll
            for (int i = 0; i < NW; i++) { ss += sh.red[i]; mx = fmaxf(mx, sh.red[NW + i]); }
            float inv = 1.0f;
            if (p.gamma != nullptr) {
                inv = 1.0f / sqrtf(ss / (float)p.K + p.eps);
                mx *= inv * 1.0000002f;     // bound on max |normalised x| (rounding of the product order)
            }
            // per-token power-of-two scale: max |x| * 2^s < 2^22
            const int s = mx > 0.0f ? 21 - ilogbf(mx) : 0;
            const float sc = ldexpf(1.0f, s);
            if (tid == 0) sh.xscale[m] = ldexpf(1.0f, -s);
            uint32_t *xw = reinterpret_cast<uint32_t *>(xq) + (size_t)m * nchunk * GvTraits<QT>::XU4 * 4;
            // word-group g = 4 columns; chunk c = g / 4, slot wd = g % 4; words [P0, P1, P2]
            for (int g = tid; g < nchunk * 4; g += NT) {
                uint32_t pw[3] = {0, 0, 0};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int v = live ? __float2int_rn(gv_xval(p, xr, inv, 4 * g + j) * sc) : 0;
                    pw[0] |= (uint32_t)(v & 0xFF) << (8 * j);
                    pw[1] |= (uint32_t)((v >> 8) & 0xFF) << (8 * j);
                    pw[2] |= (uint32_t)((v >> 16) & 0xFF) << (8 * j);
                }
                const int c = g >> 2, wd = g & 3;
                uint32_t *o = xw + (size_t)c * GvTraits<QT>::XU4 * 4 + wd * 3;
                o[0] = pw[0]; o[1] = pw[1]; o[2] = pw[2];
            }
        }
        __syncthreads();
        return;
    }

    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) {
        ss[m] = 0.0f;
        const float *xr = p.x + (size_t)m * p.ldx;
        const bool live = m < p.M;
        if (QT == Q_F16) {
            float4 *xs = reinterpret_cast<float4 *>(xq) + (size_t)m * nchunk * 2;
#pragma unroll 4
            for (int f = tid; f < nchunk * 2; f += NT) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (live) {
                    v = reinterpret_cast<const float4 *>(xr)[f];
                    ss[m] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    if (p.gamma != nullptr) {
                        const __half2 *g2p = reinterpret_cast<const __half2 *>(p.gamma) + 2 * f;
                        const float2 a = __half22float2(g2p[0]), b = __half22float2(g2p[1]);
                        v.x *= 1.0f + a.x; v.y *= 1.0f + a.y; v.z *= 1.0f + b.x; v.w *= 1.0f + b.y;
                    }
                }
                xs[gv_swz16(f)] = v;
            }
            continue;
        }
        // INT4: word-group g = 8 columns, 4 consecutive lanes convert one 32-column chunk.
        // The loads of up to SB groups per thread are issued together (one round trip).
        uint32_t *xw = reinterpret_cast<uint32_t *>(xq) + (size_t)m * nchunk * GvTraits<QT>::XU4 * 4;
        const int ngroups = nchunk * 4;
        constexpr int SB = 4;
        for (int g0 = 0; g0 < ngroups; g0 += SB * NT) {
            float4 xa[SB], xb[SB];
            uint4 gw[SB];
#pragma unroll
            for (int b = 0; b < SB; b++) {
                const int g = g0 + b * NT + tid;
                xa[b] = xb[b] = make_float4(0.f, 0.f, 0.f, 0.f);
                gw[b] = make_uint4(0u, 0u, 0u, 0u);     // gamma' = 0
                if (live && g < ngroups) {
                    xa[b] = reinterpret_cast<const float4 *>(xr)[2 * g];
                    xb[b] = reinterpret_cast<const float4 *>(xr)[2 * g + 1];
                    if (p.gamma != nullptr) gw[b] = reinterpret_cast<const uint4 *>(p.gamma)[g];
                }
            }
#pragma unroll
            for (int b = 0; b < SB; b++) {
                const int g = g0 + b * NT + tid;
                if (g0 + b * NT >= ngroups) break;      // uniform across the CTA
                float v[8] = {xa[b].x, xa[b].y, xa[b].z, xa[b].w, xb[b].x, xb[b].y, xb[b].z, xb[b].w};
#pragma unroll
                for (int j = 0; j < 8; j++) ss[m] += v[j] * v[j];
                if (p.gamma != nullptr) {
                    const uint32_t gv4[4] = {gw[b].x, gw[b].y, gw[b].z, gw[b].w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float2 gg = __half22float2(*reinterpret_cast<const __half2 *>(&gv4[j]));
                        v[2 * j] *= 1.0f + gg.x;
                        v[2 * j + 1] *= 1.0f + gg.y;
                    }
                }
                float mx = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; j++) mx = fmaxf(mx, fabsf(v[j]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                // chunk scale 2^s with max |v| * 2^s < 2^22 (s capped so 2^s and 2^-(s + 4) stay normal)
                int s = mx > 0.0f ? 21 - ilogbf(mx) : 0;
                if (s > 122) s = 122;
                const float sc = __int_as_float((127 + s) << 23);
                int n[8], part = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    n[j] = gv_rint_small(v[j], sc);
                    part += n[j];
                }
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                if (g < ngroups) {
                    // byte planes of the even (0,2,4,6) and odd (1,3,5,7) columns
                    const uint32_t e01 = __byte_perm(n[0], n[2], 0x5140), e23 = __byte_perm(n[4], n[6], 0x5140);
                    const uint32_t o01 = __byte_perm(n[1], n[3], 0x5140), o23 = __byte_perm(n[5], n[7], 0x5140);
                    const uint32_t e2 = __byte_perm(__byte_perm(n[0], n[2], 0x0062), __byte_perm(n[4], n[6], 0x0062), 0x5410);
                    const uint32_t o2 = __byte_perm(__byte_perm(n[1], n[3], 0x0062), __byte_perm(n[5], n[7], 0x0062), 0x5410);
                    const int c = g >> 2, wd = g & 3;
                    uint32_t *o = xw + (size_t)c * GvTraits<QT>::XU4 * 4 + wd * 6;
                    o[0] = __byte_perm(e01, e23, 0x5410);
                    o[1] = __byte_perm(o01, o23, 0x5410);
                    o[2] = __byte_perm(e01, e23, 0x7632);
                    o[3] = __byte_perm(o01, o23, 0x7632);
                    o[4] = e2;
                    o[5] = o2;
                    if (wd == 0) {
                        uint32_t *pad = xw + (size_t)c * GvTraits<QT>::XU4 * 4 + 24;
                        pad[0] = __float_as_uint(128.0f * (float)part);
                        pad[1] = __float_as_uint(__int_as_float((127 - s - 4) << 23));
                    }
                }
            }
        }
    }
    // 1 / rms per token for the epilogue
#pragma unroll
    for (int m = 0; m < MT; m++) {
        const float w = warp_sum(ss[m]);
        if (lane == 0) sh.ssq[warp][m] = w;
    }
    __syncthreads();
    if (tid < MT) {
        float t = 0.0f;
#pragma unroll
        for (int i = 0; i < NW; i++) t += sh.ssq[i][tid];
        sh.xscale[tid] = p.gamma != nullptr ? 1.0f / sqrtf(t / (float)p.K + p.eps) : 1.0f;
    }
    __syncthreads();
}

// Inputs of a lane's epilogue that live in global memory, read when the warp
// starts the row group (gv_epi_fetch) so that the loads complete under the
// group's weight stream instead of stalling the epilogue (at the end of the
// launch, a stalled epilogue delays the exit of the CTA and the next kernel).
struct GvEpiPre {
    float sa, sb;       // INT8 row scales of the lane's row(s)
    float c, s;         // EPI_QKV: RoPE cos / sin of the lane's pair
};

// Per-token inputs of EPI_QKV: cache slot / RoPE position and sequence of token m.
struct GvTok {
    int pos, seq;
};

__device__ __forceinline__ GvTok gv_tok(const GemvParams &p, int m)
{
    GvTok t = {0, 0};
    if (p.epi == EPI_QKV && m < p.M) {
        t.pos = p.pos[m];
        t.seq = p.seq_of ? p.seq_of[m] : p.seq_off + m;
    }
    return t;
}

__device__ __forceinline__ void gv_epi_pair(const GemvParams &p, int lr0, int m, float x1, float x2, const GvEpiPre &e,
                                            const GvTok &tk)
{
    if (p.epi == EPI_GATEUP) {
        p.y[(size_t)m * p.ldy + (lr0 >> 1)] = (p.act == 1 ? gelu_tanh(x1) : x1 / (1.0f + expf(-x1))) * x2;
        return;
    }
    // EPI_QKV: rows (lr0, lr0 + 1) are the RoPE pair (i, i + hd/2) of one head
    const int hd = p.hd, head = lr0 / hd, i = (lr0 - head * hd) >> 1;
    const int pos = tk.pos;
    const int seq = tk.seq;
    if (head < p.hq + p.hkv) {
        const float c = e.c;
        const float s = e.s;
        const float r1 = x1 * c - x2 * s;
        const float r2 = x2 * c + x1 * s;
        x1 = r1;
        x2 = r2;
    }
    if (head < p.hq) {
        float *qo = p.q_out + (size_t)m * p.hq * hd + (size_t)head * hd;
        qo[i] = x1;
        qo[i + (hd >> 1)] = x2;
    } else {
        const bool isk = head < p.hq + p.hkv;
        const int kh = isk ? head - p.hq : head - p.hq - p.hkv;
        if (p.kv_stage != nullptr) {
            float *dst = p.kv_stage + (((size_t)m * 2 + (isk ? 0 : 1)) * p.hkv + kh) * hd;
            dst[i] = x1;
            dst[i + (hd >> 1)] = x2;
            return;
        }
        __half *dst = (isk ? p.k_cache : p.v_cache) + (((size_t)seq * p.cap + pos) * p.hkv + kh) * hd;
        dst[i] = __float2half_rn(x1);
        dst[i + (hd >> 1)] = __float2half_rn(x2);
    }
}

// The same, reading its inputs here (callers without a prefetch: the tensor-core
// GEMM and GEMV epilogues).
__device__ __forceinline__ void gv_epi_pair(const GemvParams &p, int lr0, int m, float x1, float x2)
{
    GvEpiPre e = {1.0f, 1.0f, 1.0f, 0.0f};
    const GvTok tk = gv_tok(p, m);
    if (p.epi == EPI_QKV) {
        const int hd = p.hd, head = lr0 / hd, i = (lr0 - head * hd) >> 1;
        if (head < p.hq + p.hkv) {
            e.c = __half2float(p.rope_cos[(size_t)tk.pos * (hd >> 1) + i]);
            e.s = __half2float(p.rope_sin[(size_t)tk.pos * (hd >> 1) + i]);
        }
    }
    gv_epi_pair(p, lr0, m, x1, x2, e, tk);
}

template <int QT>
__device__ __forceinline__ float gv_row_scale(const GemvParams &p, int lr)
{
    const int64_t pr = gv_map_row(p, lr);
    return p.scale_f32 ? reinterpret_cast<const float *>(p.scales)[pr]
                       : __half2float(reinterpret_cast<const __half *>(p.scales)[pr]);
}



// Bytes of the per-CTA weight ring (all warps) for depth D.
template <int QT, int RW, int D, int NW = GV_WARPS>
__host__ __device__ constexpr size_t gemv_ring_bytes()
{
    return (size_t)NW * D * RW * 32 * 16 + (QT == Q_I4 ? (size_t)NW * D * RW * 32 * 4 : 0);
}

// Epilogue of the finished row group starting at logical row lr0 (v: every lane
// holds every value); lane j * MT + m owns output (row j, token m).
// TPR: the EPI_TP_RESID kernels (a separate instantiation, so that the other
// epilogues compile exactly as without it): each output goes to every rank.
// The global inputs of lane `lane`'s share of the epilogue of the row group at
// logical row lr0 (the lane's rows as gv_epilogue assigns them).
template <int QT, int MT, int RW, bool TPR = false>
__device__ __forceinline__ GvEpiPre gv_epi_fetch(const GemvParams &p, int lr0, int lane, const GvTok &tk)
{
    GvEpiPre e = {1.0f, 1.0f, 1.0f, 0.0f};
    if (!TPR && (p.epi == EPI_QKV || p.epi == EPI_GATEUP)) {
        const int pair = lane / MT, jp = 2 * pair;
        if (pair < RW / 2 && lr0 + jp + 1 < p.N) {
            if (QT == Q_I8) {
                e.sa = gv_row_scale<QT>(p, lr0 + jp);
                e.sb = gv_row_scale<QT>(p, lr0 + jp + 1);
            }
            if (p.epi == EPI_QKV && lane - pair * MT < p.M) {
                const int hd = p.hd, head = (lr0 + jp) / hd, i = (lr0 + jp - head * hd) >> 1;
                if (head < p.hq + p.hkv) {
                    e.c = __half2float(p.rope_cos[(size_t)tk.pos * (hd >> 1) + i]);
                    e.s = __half2float(p.rope_sin[(size_t)tk.pos * (hd >> 1) + i]);
                }
            }
        }
    } else if (QT == Q_I8 && p.epi != EPI_LOGITS) {
        const int j = lane / MT;
        if (j < RW && lr0 + j < p.N) e.sa = gv_row_scale<QT>(p, lr0 + j);
    }
    return e;
}

// yres (EPI_RESID, may be null): the residual of rows yr0.. staged in shared memory
// before the stream, so that the epilogue only stores.  e / tk: the lane's
// prefetched inputs (gv_epi_fetch, gv_tok).
template <int QT, int MT, int RW, bool TPR = false>
__device__ __forceinline__ void gv_epilogue(const GemvParams &p, int lr0, const float (&v)[RW][MT], float *am_v,
                                        int *am_i, int lane, unsigned tp_s, const float *yres, int yr0,
                                        const GvEpiPre &e, const GvTok &tk)
{
    if constexpr (TPR) {
#pragma unroll
        for (int j = 0; j < RW; j++)
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const int lr = lr0 + j;
                if (lane == j * MT + m && m < p.M && lr < p.N) {
                    float f = v[j][m];
                    if (QT == Q_I8) f *= e.sa;
                    tp_push(*p.tp, tp_s, (size_t)m * p.N + lr, f);
                }
            }
        return;
    }
    if (p.epi == EPI_QKV || p.epi == EPI_GATEUP) {
#pragma unroll
        for (int jp = 0; jp < RW; jp += 2)
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (lane == (jp / 2) * MT + m && m < p.M && lr0 + jp + 1 < p.N) {
                    float x1 = v[jp][m], x2 = v[jp + 1][m];
                    if (QT == Q_I8) {
                        x1 *= e.sa;
                        x2 *= e.sb;
                    }
                    gv_epi_pair(p, lr0 + jp, m, x1, x2, e, tk);
                }
    } else {
#pragma unroll
        for (int j = 0; j < RW; j++)
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const int lr = lr0 + j;
                if (m < p.M && lr < p.N) {
                    if (p.epi == EPI_LOGITS) {
                        const float f = v[j][m];
                        const int ix = p.vocab_off + lr;    // global index; the shard write is local
                        if (am_better(f, ix, am_v[m], am_i[m])) { am_v[m] = f; am_i[m] = ix; }
                        if (lane == j * MT + m && p.logits) p.logits[(size_t)m * p.ldl + lr] = f;
                    } else if (lane == j * MT + m) {
                        float f = v[j][m];
                        if (QT == Q_I8) f *= e.sa;
                        if (p.epi == EPI_STORE) p.y[(size_t)m * p.ldy + lr] = f;
                        else if (yres != nullptr) p.y[(size_t)m * p.ldy + lr] = yres[(lr - yr0) * MT + m] + f;
                        else p.y[(size_t)m * p.ldy + lr] += f;      // EPI_RESID
                    }
                }
            }
    }
}


// One unit: this lane's 16-byte chunk c (of nchunk per row) of the RW rows held
// in ring slot `stage`, accumulated into acc (INT4 / FP16, fp32) or s8 (INT8,
// exact int32 sums per activation plane).
template <int QT, int MT, int RW>
__device__ __forceinline__ void gv_unit_math(const uint4 *ring, const uint32_t *sring, int stage, int c, int nchunk,
                                             int gshift, const uint4 *xq, float (&acc)[RW][MT], int (&s8)[RW][MT][3])
{
    using T = GvTraits<QT>;
    uint4 wv[RW];
#pragma unroll
    for (int j = 0; j < RW; j++) wv[j] = ring[(stage * RW + j) * 32];
    if (c < nchunk) {
        if (QT == Q_I4) {
            float d[RW];
            const int hsel = (((c * 32) >> gshift) & 1) * 16;
#pragma unroll
            for (int j = 0; j < RW; j++)
                d[j] = __half2float(__ushort_as_half((unsigned short)(sring[(stage * RW + j) * 32] >> hsel)));
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const uint4 *xp = xq + ((size_t)m * nchunk + c) * T::XU4;
                uint32_t xw[24];
#pragma unroll
                for (int q = 0; q < 6; q++) {
                    const uint4 t = xp[q];
                    xw[4 * q] = t.x; xw[4 * q + 1] = t.y; xw[4 * q + 2] = t.z; xw[4 * q + 3] = t.w;
                }
                const uint2 pad = *reinterpret_cast<const uint2 *>(xp + 6);
                const float xs8 = __uint_as_float(pad.x), xcs = __uint_as_float(pad.y);
#pragma unroll
                for (int j = 0; j < RW; j++) {
                    // even / odd nibble streams accumulate separately (shorter dependency chains);
                    // the odd nibbles stay in the high half of their bytes (16 n, one AND
                    // instead of a shift and an AND), so the b sums are 16 x their values
                    int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
                    for (int wd = 0; wd < 4; wd++) {
                        const uint32_t w = wd == 0 ? wv[j].x : wd == 1 ? wv[j].y : wd == 2 ? wv[j].z : wv[j].w;
                        const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
                        a0 = dp4a_uu(lo, xw[wd * 6 + 0], a0);
                        b0 = dp4a_uu(hi, xw[wd * 6 + 1], b0);
                        a1 = dp4a_uu(lo, xw[wd * 6 + 2], a1);
                        b1 = dp4a_uu(hi, xw[wd * 6 + 3], b1);
                        a2 = dp4a_us(lo, xw[wd * 6 + 4], a2);
                        b2 = dp4a_us(hi, xw[wd * 6 + 5], b2);
                    }
                    // 16 x (sum n * x_int - 8 * sum x_int): planes 0 and 1 join exactly in
                    // int32 (< 2^29), plane 2 (< 2^20 in magnitude) is exact in fp32; the
                    // staged xs8 = 128 * sum x_int and xcs = 2^-s / 16 carry the factor 16
                    const int p01 = (a0 * 16 + b0) + ((a1 * 16 + b1) << 8);
                    const float f = fmaf((float)(a2 * 16 + b2), 65536.0f, (float)p01) - xs8;
                    acc[j][m] = fmaf(d[j], f * xcs, acc[j][m]);
                }
            }
        } else if (QT == Q_I8) {
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const uint4 *xp = xq + ((size_t)m * nchunk + c) * T::XU4;
                const uint4 t0 = xp[0], t1 = xp[1], t2 = xp[2];
                const uint32_t xw[12] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w, t2.x, t2.y, t2.z, t2.w};
#pragma unroll
                for (int j = 0; j < RW; j++)
#pragma unroll
                    for (int wd = 0; wd < 4; wd++) {
                        const uint32_t w = wd == 0 ? wv[j].x : wd == 1 ? wv[j].y : wd == 2 ? wv[j].z : wv[j].w;
                        s8[j][m][0] = dp4a_su(w, xw[wd * 3 + 0], s8[j][m][0]);
                        s8[j][m][1] = dp4a_su(w, xw[wd * 3 + 1], s8[j][m][1]);
                        s8[j][m][2] = dp4a_ss(w, xw[wd * 3 + 2], s8[j][m][2]);
                    }
            }
        } else {
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const float4 *xm = reinterpret_cast<const float4 *>(xq) + (size_t)m * nchunk * 2;
                const float4 a = xm[gv_swz16(c * 2)];
                const float4 b = xm[gv_swz16(c * 2 + 1)];
#pragma unroll
                for (int j = 0; j < RW; j++) {
                    float2 part = make_float2(0.f, 0.f);
                    gv_dot_f16(wv[j].x, a.x, a.y, part);
                    gv_dot_f16(wv[j].y, a.z, a.w, part);
                    gv_dot_f16(wv[j].z, b.x, b.y, part);
                    gv_dot_f16(wv[j].w, b.z, b.w, part);
                    acc[j][m] += part.x + part.y;
                }
            }
        }
    }
}

// Folds the lanes' accumulators of a finished run of units into v (every lane
// holds every value) and resets them.
template <int QT, int MT, int RW>
__device__ __forceinline__ void gv_fold(float (&acc)[RW][MT], int (&s8)[RW][MT][3], const float *xscale,
                                        float (&v)[RW][MT])
{
#pragma unroll
    for (int j = 0; j < RW; j++)
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (QT == Q_I8) {
                long long t0 = s8[j][m][0], t1 = s8[j][m][1], t2 = s8[j][m][2];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    t0 += __shfl_xor_sync(0xffffffffu, t0, o);
                    t1 += __shfl_xor_sync(0xffffffffu, t1, o);
                    t2 += __shfl_xor_sync(0xffffffffu, t2, o);
                }
                const long long tot = t0 + (t1 << 8) + (t2 << 16);   // exact sum q * x_int
                v[j][m] = (float)tot * xscale[m];
                s8[j][m][0] = s8[j][m][1] = s8[j][m][2] = 0;
            } else {
                v[j][m] = warp_sum(acc[j][m]) * xscale[m];
                acc[j][m] = 0.0f;
            }
        }
}

// Work split: a CTA owns a contiguous range of row groups; their (group,
// 512-byte segment) units, group-major, are cut into NW contiguous, equal
// ranges, one per warp (split-K inside the CTA).  A group whose units fall to
// several warps leaves per-warp partial sums in shared memory; the warp that
// holds its last unit adds them in warp order (deterministic) and runs the
// epilogue.
template <int QT, int MT, int RW, int D, int NW = GV_WARPS, bool TPR = false>
struct GemvStream {
    using T = GvTraits<QT>;
    int lane, warp, nchunk, S, gshift;
    int row_bytes, srow_bytes;
    const uint8_t *wbase;  // this lane's 16 bytes of physical row 0
    const uint8_t *sbase;  // INT4 scales
    uint4 *ring;          // this lane's slot 0 (weights)
    uint32_t *sring;      // this lane's slot 0 (INT4 scales)
    int g_begin, U;       // the CTA's first row group and its number of units
    int u0, u1;           // this warp's units
    // issue side: (group, segment, ring slot) of the next unit to fetch, units left,
    // and the physical rows of that group (-1 past the last row)
    int is_g, is_s, is_stage, is_left;
    int ipr[RW];
    uint64_t pol;         // L2 evict-first policy of the weight stream
    unsigned tp_s;        // TPR: sequence number of this launch's reduction
    const float *yres;    // EPI_RESID: residual rows in shared memory (null: read y in the epilogue)
    int yr0;              // first row of yres

    __device__ __forceinline__ int unit_lo(int w) const { return (int)(((int64_t)w * U) / NW); }

    __device__ __forceinline__ void set_issue_rows(const GemvParams &p)
    {
#pragma unroll
        for (int j = 0; j < RW; j++) {
            const int lr = is_g * RW + j;
            ipr[j] = lr < p.N ? (int)gv_map_row(p, lr) : -1;
        }
    }

    __device__ __forceinline__ void issue(const GemvParams &p)
    {
        if (is_left > 0) {
            const int c = is_s * 32 + lane;
            const bool cv = c < nchunk;
            // 4-byte word holding the fp16 scale of group (c * 32) >> gshift
            const int sw_off = (((c * 32) >> gshift) * 2) & ~3;
#pragma unroll
            for (int j = 0; j < RW; j++) {
                const int64_t r = ipr[j] < 0 ? 0 : ipr[j];
                cp_async16_cg_ef(ring + (is_stage * RW + j) * 32, wbase + r * row_bytes + is_s * 512, cv && ipr[j] >= 0,
                                 pol);
                if (QT == Q_I4)
                    cp_async4_ca_ef(sring + (is_stage * RW + j) * 32, sbase + r * srow_bytes + sw_off,
                                    cv && ipr[j] >= 0, pol);
            }
            is_left--;
            if (++is_stage == D) is_stage = 0;
            if (++is_s == S) {
                is_s = 0;
                is_g++;
                if (is_left > 0) set_issue_rows(p);
            }
        }
        cp_async_commit_group();
    }

    // Phase 1: work split (CTA `cta` of `ncta`) and the first D - 1 ring stages.
    __device__ __forceinline__ void prefetch(const GemvParams &p, unsigned char *ring_smem, int cta, int ncta)
    {
        lane = threadIdx.x & 31;
        warp = threadIdx.x >> 5;
        nchunk = (int)(p.row_bytes >> 4);
        S = (nchunk + 31) >> 5;                         // 512-byte segments per row
        ring = reinterpret_cast<uint4 *>(ring_smem) + (size_t)warp * D * RW * 32 + lane;
        sring = reinterpret_cast<uint32_t *>(reinterpret_cast<uint4 *>(ring_smem) + (size_t)NW * D * RW * 32) +
                (size_t)warp * D * RW * 32 + lane;
        gshift = QT == Q_I4 ? __ffs(p.group) - 1 : 0;   // group is a power of two
        row_bytes = (int)p.row_bytes;
        srow_bytes = QT == Q_I4 ? (p.K >> gshift) * 2 : 0;
        wbase = p.w + lane * 16;
        sbase = reinterpret_cast<const uint8_t *>(p.scales);
        pol = l2_evict_first_policy();
        const int NG = (p.N + RW - 1) / RW;
        g_begin = (int)(((int64_t)cta * NG) / ncta);
        const int g_end = (int)(((int64_t)(cta + 1) * NG) / ncta);
        U = (g_end - g_begin) * S;
        u0 = unit_lo(warp);
        u1 = unit_lo(warp + 1);
        is_g = g_begin + u0 / S;
        is_s = u0 % S;
        is_left = u1 - u0;
        is_stage = 0;
        if (is_left > 0) set_issue_rows(p);
#pragma unroll
        for (int j = 0; j < D - 1; j++) issue(p);
    }

    __device__ __forceinline__ void epilogue(const GemvParams &p, int lr0, const float (&v)[RW][MT], float *am_v,
                                             int *am_i, const GvEpiPre &e, const GvTok &tk) const
    {
        gv_epilogue<QT, MT, RW, TPR>(p, lr0, v, am_v, am_i, lane, tp_s, yres, yr0, e, tk);
    }

    // Phase 2: activations -> smem, stream, epilogue.  All threads of the CTA call it.
    // `after_stage` runs once the activations are staged (PDL trigger in the standalone kernel).
    template <typename AfterStage>
    __device__ __forceinline__ void run(const GemvParams &p, unsigned char *x_smem, GemvShared<MT, NW> &sh, int cta,
                                        int ncta, AfterStage after_stage)
    {
        uint4 *xq = reinterpret_cast<uint4 *>(x_smem);
        // EPI_RESID: the residual of this CTA's rows, loaded now (the previous kernels are
        // complete) so that the loads overlap the activation staging and the epilogues
        // do not wait on a read of y
        yres = nullptr;
        yr0 = g_begin * RW;
        const int yrows = min((g_begin + U / S) * RW, p.N) - yr0;
        const bool ystage = !TPR && p.epi == EPI_RESID && yrows > 0 && yrows <= GV_YRES_ROWS;
        float yv = 0.0f;
        if (ystage && (int)threadIdx.x < yrows * MT) {
            const int r = threadIdx.x / MT, m = threadIdx.x - r * MT;
            if (m < p.M) yv = p.y[(size_t)m * p.ldy + yr0 + r];
        }
        const GvTok tk = gv_tok(p, lane % MT);       // the lane's token in gv_epilogue
        gv_stage_x<QT, MT, NW>(p, xq, sh, nchunk);
        if (ystage) {
            if ((int)threadIdx.x < yrows * MT) sh.yres[threadIdx.x] = yv;
            __syncthreads();
            yres = sh.yres;
        }
        GV_STAMP(3);
        after_stage();
        if constexpr (TPR) tp_s = tp_next_seq(*p.tp);

        // accumulators: INT8 exact int32 plane sums; INT4 / FP16 fp32
        int s8[RW][MT][3];
        float acc[RW][MT];
#pragma unroll
        for (int j = 0; j < RW; j++)
#pragma unroll
            for (int m = 0; m < MT; m++) {
                acc[j][m] = 0.0f;
                s8[j][m][0] = s8[j][m][1] = s8[j][m][2] = 0;
            }
        float am_v[MT];
        int am_i[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) { am_v[m] = -INFINITY; am_i[m] = 0x7fffffff; }

        // compute side (group, segment, ring slot)
        int cs_g = g_begin + u0 / S, cs_s = u0 % S, cs_stage = 0;
        const int first_g = cs_g;
        const bool first_whole = cs_s == 0;       // this warp starts its first group at segment 0
        const int n = u1 - u0;
        // epilogue inputs of the current group, and of the first group (whose epilogue,
        // if the group is split between warps, runs after the stream)
        const GvEpiPre e_first = n > 0 ? gv_epi_fetch<QT, MT, RW, TPR>(p, first_g * RW, lane, tk) : GvEpiPre{};
        GvEpiPre e_cur = e_first;
        for (int i = 0; i < n; i++) {
            issue(p);
            cp_async_wait_group<D - 1>();
            const int stage = cs_stage;
            if (++cs_stage == D) cs_stage = 0;
            gv_unit_math<QT, MT, RW>(ring, sring, stage, cs_s * 32 + lane, nchunk, gshift, xq, acc, s8);
            const bool end_g = ++cs_s == S;
            if (end_g || i == n - 1) {
                // ---- this warp's part of row group cs_g is done: fold the lanes, reset
                float v[RW][MT];
                gv_fold<QT, MT, RW>(acc, s8, sh.xscale, v);
                if (end_g && (cs_g != first_g || first_whole)) {
                    epilogue(p, cs_g * RW, v, am_v, am_i, e_cur, tk);   // the whole group was this warp's
                } else if (lane == 0) {
                    float *pb = sh.pbuf[warp][cs_g == first_g ? 0 : 1];
#pragma unroll
                    for (int j = 0; j < RW; j++)
#pragma unroll
                        for (int m = 0; m < MT; m++) pb[j * MT + m] = v[j][m];
                }
                if (end_g) {
                    cs_s = 0;
                    cs_g++;
                    if (i + 1 < n) e_cur = gv_epi_fetch<QT, MT, RW, TPR>(p, cs_g * RW, lane, tk);
                }
            }
        }
        cp_async_wait_group<0>();
        GV_STAMP(4);

        // groups split between warps: the holder of a group's last unit (which started the
        // group past segment 0) adds the parts of every contributing warp in warp order
        __syncthreads();
        if (n > 0 && !first_whole && u1 > (u0 / S) * S + S - 1) {
            const int gl = u0 / S;
            float v[RW][MT];
#pragma unroll
            for (int j = 0; j < RW; j++)
#pragma unroll
                for (int m = 0; m < MT; m++) v[j][m] = 0.0f;
            for (int w = 0; w <= warp; w++) {
                const int lo = unit_lo(w), hi = unit_lo(w + 1);
                if (hi <= lo || hi <= gl * S || lo >= gl * S + S) continue;    // empty, or not in this group
                const float *pb = sh.pbuf[w][lo / S == gl ? 0 : 1];
#pragma unroll
                for (int j = 0; j < RW; j++)
#pragma unroll
                    for (int m = 0; m < MT; m++) v[j][m] += pb[j * MT + m];
            }
            epilogue(p, (g_begin + gl) * RW, v, am_v, am_i, e_first, tk);
        }

        if constexpr (TPR) {
            // every rank's values of this CTA's rows (the same rows on every rank),
            // added to the residual in rank order
            const TpFuse &t = *p.tp;
            const int r0 = g_begin * RW, r1 = min((g_begin + U / S) * RW, p.N), nr = r1 - r0;
            for (int e = threadIdx.x; e < nr * p.M; e += NW * 32) {
                const int m = e / nr, lr = r0 + (e - m * nr);
                float sum;
                if (!tp_wait_sum(t, tp_s, (size_t)m * p.N + lr, sum)) break;
                p.resid[(size_t)m * p.ldy + lr] += sum;
            }
            tp_launch_done(t, tp_s);
        }

        if (p.epi == EPI_LOGITS) {
            // per-CTA (max, argmax); ties follow the reference's ArgMax tree (am_better)
            if (lane == 0)
#pragma unroll
                for (int m = 0; m < MT; m++) { sh.amv[warp][m] = am_v[m]; sh.ami[warp][m] = am_i[m]; }
            __syncthreads();
            const int tid = threadIdx.x;
            if (tid < p.M && tid < MT) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int w = 0; w < NW; w++) {
                    const float vv = sh.amv[w][tid];
                    const int ix = sh.ami[w][tid];
                    if (am_better(vv, ix, bv, bi)) { bv = vv; bi = ix; }
                }
                p.am_val[(size_t)tid * ncta + cta] = bv;
                p.am_idx[(size_t)tid * ncta + cta] = bi;
            }
            __syncthreads();
        }
    }
};

}  // namespace du
