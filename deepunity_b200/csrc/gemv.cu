// gemv.cu -- decode GEMV kernel (see gemv.cuh) and its launchers.
#include "gemv.cuh"
#include "internal.h"

namespace du {

template <int QT, int MT>
__global__ void __launch_bounds__(GV_THREADS) qgemv_kernel(const GemvParams p)
{
    using T = GvTraits<QT>;
    extern __shared__ __align__(16) float gv_smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kw = warp % GV_KW, rg = warp / GV_KW;
    const int K = p.K;
    const int nchunk = (int)(p.row_bytes >> 4);          // 16-byte chunks per row
    const int k4 = nchunk * T::F4;                       // float4 slots per token (K / 4)
    float4 *xs = reinterpret_cast<float4 *>(gv_smem);    // [MT][k4] swizzled, pre-scaled x'
    float *xsum = gv_smem + (size_t)MT * k4 * 4;         // INT4: [MT][nchunk] 8*sum(x); INT8: [MT] 128*sum(x)
    float *red = xsum + (QT == Q_I4 ? MT * nchunk : MT); // [KW][PASS][MT]
    __shared__ float s_stat[MT][GV_THREADS / 32];

    const int r_begin = blockIdx.x * p.rows_per_cta;
    const int r_end = min(r_begin + p.rows_per_cta, p.N);

    // ---------------- prologue: x (optionally RMSNorm'd) -> smem, scaled by 2^e(k)
    for (int m = 0; m < MT; m++) {
        float inv = 1.0f;
        if (p.gamma != nullptr && m < p.M) {
            float ss = 0.0f;
            const float4 *xr = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.ldx);
            for (int f = tid; f < k4; f += GV_THREADS) {
                float4 v = xr[f];
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
            ss = warp_sum(ss);
            if (lane == 0) s_stat[m][warp] = ss;
            __syncthreads();
            float tot = 0.0f;
#pragma unroll
            for (int i = 0; i < GV_THREADS / 32; i++) tot += s_stat[m][i];
            inv = 1.0f / sqrtf(tot / (float)K + p.eps);
            __syncthreads();
        }
        const float4 *xr = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.ldx);
        for (int f = tid; f < k4; f += GV_THREADS) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < p.M) {
                v = xr[f];
                if (p.gamma != nullptr) {
                    const __half2 *g2 = reinterpret_cast<const __half2 *>(p.gamma) + 2 * f;
                    float2 g01 = __half22float2(g2[0]), g23 = __half22float2(g2[1]);
                    v.x = v.x * inv * (1.0f + g01.x);
                    v.y = v.y * inv * (1.0f + g01.y);
                    v.z = v.z * inv * (1.0f + g23.x);
                    v.w = v.w * inv * (1.0f + g23.y);
                }
            }
            if (QT != Q_F16) {
                const int k0 = 4 * f;
                v.x = ldexpf(v.x, gv_xexp<QT>(k0));
                v.y = ldexpf(v.y, gv_xexp<QT>(k0 + 1));
                v.z = ldexpf(v.z, gv_xexp<QT>(k0 + 2));
                v.w = ldexpf(v.w, gv_xexp<QT>(k0 + 3));
            }
            xs[(size_t)m * k4 + gv_swz<QT>(f)] = v;
        }
    }
    __syncthreads();
    if (QT == Q_I4) {
        // 8 * sum of x over each 32-column chunk (unscaled back exactly)
        for (int i = tid; i < MT * nchunk; i += GV_THREADS) {
            const int m = i / nchunk, c = i - m * nchunk;
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 v = xs[(size_t)m * k4 + gv_swz<QT>(c * 8 + j)];
                const int k0 = c * 32 + 4 * j;
                s += ldexpf(v.x, -gv_xexp<QT>(k0)) + ldexpf(v.y, -gv_xexp<QT>(k0 + 1)) +
                     ldexpf(v.z, -gv_xexp<QT>(k0 + 2)) + ldexpf(v.w, -gv_xexp<QT>(k0 + 3));
            }
            xsum[i] = 8.0f * s;
        }
    } else if (QT == Q_I8) {
        for (int m = 0; m < MT; m++) {
            float s = 0.0f;
            for (int f = tid; f < k4; f += GV_THREADS) {
                float4 v = xs[(size_t)m * k4 + gv_swz<QT>(f)];
                s += ldexpf(v.x, -99) + ldexpf(v.y, -91) + ldexpf(v.z, -99) + ldexpf(v.w, -91);
            }
            s = warp_sum(s);
            if (lane == 0) s_stat[m][warp] = s;
        }
        __syncthreads();
        if (tid < MT) {
            float t = 0.0f;
            for (int i = 0; i < GV_THREADS / 32; i++) t += s_stat[tid][i];
            xsum[tid] = 128.0f * t;
        }
    }
    __syncthreads();

    // ---------------- main loop over passes of GV_PASS logical rows
    const int nseg = (nchunk + 31) >> 5;
    const int64_t spr = (QT == Q_I4) ? (int64_t)K / p.group : 0;   // INT4 scales per row
    for (int pass0 = r_begin; pass0 < r_end; pass0 += GV_PASS) {
        const uint8_t *wrow[GV_RW];
        int64_t prow[GV_RW];
        bool rvalid[GV_RW];
#pragma unroll
        for (int j = 0; j < GV_RW; j++) {
            const int lr = pass0 + rg * GV_RW + j;
            rvalid[j] = lr < r_end;
            prow[j] = rvalid[j] ? gv_map_row(p, lr) : 0;
            wrow[j] = p.w + prow[j] * p.row_bytes;
        }
        float acc[GV_RW][MT];
#pragma unroll
        for (int j = 0; j < GV_RW; j++)
#pragma unroll
            for (int m = 0; m < MT; m++) acc[j][m] = 0.0f;

        uint4 cur[GV_RW];
        int seg = kw;
        {
            const int c = seg * 32 + lane;
#pragma unroll
            for (int j = 0; j < GV_RW; j++)
                cur[j] = (seg < nseg && c < nchunk && rvalid[j]) ? ldg_stream(wrow[j] + (int64_t)c * 16)
                                                                  : make_uint4(0, 0, 0, 0);
        }
        for (; seg < nseg; seg += GV_KW) {
            const int c = seg * 32 + lane;
            const int cn = c + 32 * GV_KW;
            uint4 nxt[GV_RW];
#pragma unroll
            for (int j = 0; j < GV_RW; j++)
                nxt[j] = (cn < nchunk && rvalid[j]) ? ldg_stream(wrow[j] + (int64_t)cn * 16)
                                                    : make_uint4(0, 0, 0, 0);
            if (c < nchunk) {
                float dsc[GV_RW];
                if (QT == Q_I4) {
                    const __half *sc = reinterpret_cast<const __half *>(p.scales);
                    const int g = (c * 32) / p.group;
#pragma unroll
                    for (int j = 0; j < GV_RW; j++)
                        dsc[j] = rvalid[j] ? __half2float(sc[prow[j] * spr + g]) : 0.0f;
                }
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    const float4 *xm = xs + (size_t)m * k4;
                    if (QT == Q_I4) {
                        float part[GV_RW];
#pragma unroll
                        for (int j = 0; j < GV_RW; j++) part[j] = 0.0f;
#pragma unroll
                        for (int wd = 0; wd < 4; wd++) {
                            const float4 a = xm[gv_swz<QT>(c * 8 + 2 * wd)];
                            const float4 b = xm[gv_swz<QT>(c * 8 + 2 * wd + 1)];
#pragma unroll
                            for (int j = 0; j < GV_RW; j++) {
                                const uint32_t wv = wd == 0 ? cur[j].x : wd == 1 ? cur[j].y : wd == 2 ? cur[j].z : cur[j].w;
                                part[j] = gv_dot_i4(wv, a, b, part[j]);
                            }
                        }
                        const float xs8 = xsum[m * nchunk + c];
#pragma unroll
                        for (int j = 0; j < GV_RW; j++)
                            acc[j][m] = fmaf(dsc[j], fmaf(part[j], GV_TWO50, -xs8), acc[j][m]);
                    } else if (QT == Q_I8) {
#pragma unroll
                        for (int wd = 0; wd < 4; wd++) {
                            const float4 a = xm[gv_swz<QT>(c * 4 + wd)];
#pragma unroll
                            for (int j = 0; j < GV_RW; j++) {
                                const uint32_t wv = wd == 0 ? cur[j].x : wd == 1 ? cur[j].y : wd == 2 ? cur[j].z : cur[j].w;
                                acc[j][m] = gv_dot_i8(wv, a, acc[j][m]);
                            }
                        }
                    } else {
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const float4 a = xm[gv_swz<QT>(c * 2 + h)];
#pragma unroll
                            for (int j = 0; j < GV_RW; j++) {
                                const uint32_t w0 = h == 0 ? cur[j].x : cur[j].z;
                                const uint32_t w1 = h == 0 ? cur[j].y : cur[j].w;
                                acc[j][m] = gv_dot_f16(w0, a.x, a.y, acc[j][m]);
                                acc[j][m] = gv_dot_f16(w1, a.z, a.w, acc[j][m]);
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < GV_RW; j++) cur[j] = nxt[j];
        }

        // fold lanes: reduce-scatter over the 4 rows, one token at a time
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float v[GV_RW];
#pragma unroll
            for (int j = 0; j < GV_RW; j++) v[j] = acc[j][m];
            const float r = gv_reduce_scatter<GV_RW>(v, lane);
            if ((lane & 7) == 0)
                red[((size_t)kw * GV_PASS + rg * GV_RW + gv_rs_index<GV_RW>(lane)) * MT + m] = r;
        }
        __syncthreads();

        // ---------------- epilogue: one thread per (row, token) of this pass
        const int prs = min(GV_PASS, r_end - pass0);
        if (p.epi == EPI_QKV || p.epi == EPI_GATEUP) {
            // pairs of logical rows (2i, 2i+1)
            for (int t = tid; t < (prs >> 1) * p.M; t += GV_THREADS) {
                const int pr = t / p.M, m = t - pr * p.M;
                float v2[2];
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int lrow = 2 * pr + e;
                    float s = 0.0f;
#pragma unroll
                    for (int q = 0; q < GV_KW; q++) s += red[((size_t)q * GV_PASS + lrow) * MT + m];
                    if (QT == Q_I8) {
                        const int64_t pr_ = gv_map_row(p, pass0 + lrow);
                        const float sc = p.scale_f32 ? reinterpret_cast<const float *>(p.scales)[pr_]
                                                     : __half2float(reinterpret_cast<const __half *>(p.scales)[pr_]);
                        s = sc * fmaf(s, GV_TWO50, -xsum[m]);
                    }
                    v2[e] = s;
                }
                const int lr0 = pass0 + 2 * pr;
                if (p.epi == EPI_GATEUP) {
                    const float g = v2[0], u = v2[1];
                    p.y[(size_t)m * p.ldy + (lr0 >> 1)] = (g / (1.0f + expf(-g))) * u;
                } else {
                    const int hd = p.hd, head = lr0 / hd, i = (lr0 - head * hd) >> 1;
                    const int pos = p.pos[m];
                    const int seq = p.seq_of ? p.seq_of[m] : m;
                    float x1 = v2[0], x2 = v2[1];
                    if (head < p.hq + p.hkv) {
                        const float c = __half2float(p.rope_cos[(size_t)pos * (hd >> 1) + i]);
                        const float s = __half2float(p.rope_sin[(size_t)pos * (hd >> 1) + i]);
                        const float r1 = x1 * c - x2 * s;
                        const float r2 = x2 * c + x1 * s;
                        x1 = r1; x2 = r2;
                    }
                    if (head < p.hq) {
                        float *qo = p.q_out + (size_t)m * p.hq * hd + (size_t)head * hd;
                        qo[i] = x1;
                        qo[i + (hd >> 1)] = x2;
                    } else {
                        const bool isk = head < p.hq + p.hkv;
                        const int kh = isk ? head - p.hq : head - p.hq - p.hkv;
                        __half *cache = isk ? p.k_cache : p.v_cache;
                        __half *dst = cache + (((size_t)seq * p.cap + pos) * p.hkv + kh) * hd;
                        dst[i] = __float2half_rn(x1);
                        dst[i + (hd >> 1)] = __float2half_rn(x2);
                    }
                }
            }
        } else {
            for (int t = tid; t < prs * p.M; t += GV_THREADS) {
                const int lrow = t / p.M, m = t - lrow * p.M;
                float s = 0.0f;
#pragma unroll
                for (int q = 0; q < GV_KW; q++) s += red[((size_t)q * GV_PASS + lrow) * MT + m];
                const int lr = pass0 + lrow;
                if (QT == Q_I8) {
                    const int64_t pr_ = gv_map_row(p, lr);
                    const float sc = p.scale_f32 ? reinterpret_cast<const float *>(p.scales)[pr_]
                                                 : __half2float(reinterpret_cast<const __half *>(p.scales)[pr_]);
                    s = sc * fmaf(s, GV_TWO50, -xsum[m]);
                }
                if (p.epi == EPI_STORE) {
                    p.y[(size_t)m * p.ldy + lr] = s;
                } else if (p.epi == EPI_RESID) {
                    p.y[(size_t)m * p.ldy + lr] += s;
                } else {  // EPI_LOGITS: keep the value in red for the CTA argmax below
                    if (p.logits) p.logits[(size_t)m * p.ldl + p.vocab_off + lr] = s;
                    red[((size_t)GV_KW * GV_PASS + lrow) * MT + m] = s;
                }
            }
            if (p.epi == EPI_LOGITS) {
                __syncthreads();
                if (tid < p.M) {
                    const int m = tid;
                    float bv = (pass0 == r_begin) ? -INFINITY : p.am_val[(size_t)m * gridDim.x + blockIdx.x];
                    int bi = (pass0 == r_begin) ? 0 : p.am_idx[(size_t)m * gridDim.x + blockIdx.x];
                    for (int lrow = 0; lrow < prs; lrow++) {
                        const float v = red[((size_t)GV_KW * GV_PASS + lrow) * MT + m];
                        if (v > bv) { bv = v; bi = p.vocab_off + pass0 + lrow; }
                    }
                    p.am_val[(size_t)m * gridDim.x + blockIdx.x] = bv;
                    p.am_idx[(size_t)m * gridDim.x + blockIdx.x] = bi;
                }
            }
        }
        __syncthreads();
    }
}

size_t gemv_smem_bytes(int qt, int mt, int64_t row_bytes)
{
    const int nchunk = (int)(row_bytes >> 4);
    const int f4 = qt == Q_I4 ? 8 : qt == Q_I8 ? 4 : 2;
    size_t b = (size_t)mt * nchunk * f4 * 16;
    b += (qt == Q_I4 ? (size_t)mt * nchunk : (size_t)mt) * 4;
    b += (size_t)(GV_KW + 1) * GV_PASS * mt * 4;
    return b;
}

template <int QT, int MT>
static int launch_mt(const GemvParams &p, int grid, size_t smem, cudaStream_t st)
{
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        DU_CUDA_TRY(cudaFuncSetAttribute(qgemv_kernel<QT, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         220 * 1024));
        attr_set[dev & 63] = true;
    }
    qgemv_kernel<QT, MT><<<grid, GV_THREADS, smem, st>>>(p);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

int gemv_grid(const GemvParams &p0, int target_ctas)
{
    const int N = p0.N;
    int rpc = (N + target_ctas - 1) / target_ctas;
    rpc = (rpc + 1) & ~1;           // even: RoPE / gate-up pairs stay in one CTA
    if (rpc < 2) rpc = 2;
    return rpc;
}

int launch_gemv(int qt, GemvParams p, cudaStream_t st)
{
    if (p.M <= 0 || p.N <= 0) return DU_OK;
    if (p.M > 8) return fail(DU_EINVAL, "gemv: M > 8 must be split by the caller");
    const int mt = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
    const size_t smem = gemv_smem_bytes(qt, mt, p.row_bytes);
    if (smem > 220 * 1024) return fail(DU_EINVAL, "gemv: M*K too large for the shared-memory stage");
    if (p.rows_per_cta <= 0) p.rows_per_cta = gemv_grid(p, 2 * num_sms());
    const int grid = (p.N + p.rows_per_cta - 1) / p.rows_per_cta;
#define DU_GV_CASE(Q, M_)                                        \
    if (qt == Q && mt == M_) return launch_mt<Q, M_>(p, grid, smem, st);
    DU_GV_CASE(Q_I4, 1) DU_GV_CASE(Q_I4, 2) DU_GV_CASE(Q_I4, 4) DU_GV_CASE(Q_I4, 8)
    DU_GV_CASE(Q_I8, 1) DU_GV_CASE(Q_I8, 2) DU_GV_CASE(Q_I8, 4) DU_GV_CASE(Q_I8, 8)
    DU_GV_CASE(Q_F16, 1) DU_GV_CASE(Q_F16, 2) DU_GV_CASE(Q_F16, 4) DU_GV_CASE(Q_F16, 8)
#undef DU_GV_CASE
    return fail(DU_EINVAL, "gemv: unsupported quant kind");
}

}  // namespace du
