// gemv.cu -- decode GEMV kernel (see gemv.cuh) and its launcher.
#include "gemv.cuh"
#include "internal.h"

namespace du {

constexpr int GV_WARPS = GV_THREADS / 32;

// x' = x * 2^e(k), staged in smem (swizzled), plus the zero-point sums.
template <int QT, int MT>
__device__ __forceinline__ void gv_stage_x(const GemvParams &p, float4 *xs, float *xsum, int k4, int nchunk,
                                           float (*s_stat)[GV_WARPS])
{
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int m = 0; m < MT; m++) {
        float inv = 1.0f;
        if (p.gamma != nullptr && m < p.M) {
            float ss = 0.0f;
            const float4 *xr = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.ldx);
            for (int f = tid; f < k4; f += GV_THREADS) {
                const float4 v = xr[f];
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
            ss = warp_sum(ss);
            if (lane == 0) s_stat[m][warp] = ss;
            __syncthreads();
            float tot = 0.0f;
#pragma unroll
            for (int i = 0; i < GV_WARPS; i++) tot += s_stat[m][i];
            inv = 1.0f / sqrtf(tot / (float)p.K + p.eps);
            __syncthreads();
        }
        const float4 *xr = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.ldx);
        for (int f = tid; f < k4; f += GV_THREADS) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < p.M) {
                v = xr[f];
                if (p.gamma != nullptr) {
                    const __half2 *g2 = reinterpret_cast<const __half2 *>(p.gamma) + 2 * f;
                    const float2 g01 = __half22float2(g2[0]), g23 = __half22float2(g2[1]);
                    v.x = v.x * inv * (1.0f + g01.x);
                    v.y = v.y * inv * (1.0f + g01.y);
                    v.z = v.z * inv * (1.0f + g23.x);
                    v.w = v.w * inv * (1.0f + g23.y);
                }
            }
            if (QT != Q_F16) {
                const int k0 = 4 * f;
                v.x *= gv_pow2(gv_xexp<QT>(k0));
                v.y *= gv_pow2(gv_xexp<QT>(k0 + 1));
                v.z *= gv_pow2(gv_xexp<QT>(k0 + 2));
                v.w *= gv_pow2(gv_xexp<QT>(k0 + 3));
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
                const float4 v = xs[(size_t)m * k4 + gv_swz<QT>(c * 8 + j)];
                const int k0 = 4 * j;   // column position within the 8-column word only matters mod 8
                s += v.x * gv_pow2(-gv_xexp<QT>(k0)) + v.y * gv_pow2(-gv_xexp<QT>(k0 + 1)) +
                     v.z * gv_pow2(-gv_xexp<QT>(k0 + 2)) + v.w * gv_pow2(-gv_xexp<QT>(k0 + 3));
            }
            xsum[i] = 8.0f * s;
        }
    } else if (QT == Q_I8) {
        for (int m = 0; m < MT; m++) {
            float s = 0.0f;
            for (int f = tid; f < k4; f += GV_THREADS) {
                const float4 v = xs[(size_t)m * k4 + gv_swz<QT>(f)];
                s += v.x * gv_pow2(-99) + v.y * gv_pow2(-91) + v.z * gv_pow2(-99) + v.w * gv_pow2(-91);
            }
            s = warp_sum(s);
            if (lane == 0) s_stat[m][warp] = s;
        }
        __syncthreads();
        if (tid < MT) {
            float t = 0.0f;
            for (int i = 0; i < GV_WARPS; i++) t += s_stat[tid][i];
            xsum[tid] = 128.0f * t;
        }
    }
    __syncthreads();
}

// Epilogue for one finished value pair / value.  v: full sums (scaled for INT4).
template <int QT>
__device__ __forceinline__ float gv_finish(const GemvParams &p, const float *xsum, int lr, int m, float v)
{
    if (QT == Q_I8) {
        const int64_t pr = gv_map_row(p, lr);
        const float sc = p.scale_f32 ? reinterpret_cast<const float *>(p.scales)[pr]
                                     : __half2float(reinterpret_cast<const __half *>(p.scales)[pr]);
        v = sc * fmaf(v, GV_TWO50, -xsum[m]);
    }
    return v;
}

__device__ __forceinline__ void gv_epi_pair(const GemvParams &p, int lr0, int m, float x1, float x2)
{
    if (p.epi == EPI_GATEUP) {
        p.y[(size_t)m * p.ldy + (lr0 >> 1)] = (x1 / (1.0f + expf(-x1))) * x2;
        return;
    }
    // EPI_QKV: rows (lr0, lr0 + 1) are the RoPE pair (i, i + hd/2) of one head
    const int hd = p.hd, head = lr0 / hd, i = (lr0 - head * hd) >> 1;
    const int pos = p.pos[m];
    const int seq = p.seq_of ? p.seq_of[m] : m;
    if (head < p.hq + p.hkv) {
        const float c = __half2float(p.rope_cos[(size_t)pos * (hd >> 1) + i]);
        const float s = __half2float(p.rope_sin[(size_t)pos * (hd >> 1) + i]);
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
        __half *dst = (isk ? p.k_cache : p.v_cache) + (((size_t)seq * p.cap + pos) * p.hkv + kh) * hd;
        dst[i] = __float2half_rn(x1);
        dst[i + (hd >> 1)] = __float2half_rn(x2);
    }
}

// Streaming GEMV.  Template: weight kind, token tile MT, rows per warp group RW
// (even, so RoPE / gate-up pairs stay in one warp), ring depth D.
template <int QT, int MT, int RW, int D>
__global__ void __launch_bounds__(GV_THREADS, 2) qgemv_kernel(const GemvParams p)
{
    using T = GvTraits<QT>;
    extern __shared__ __align__(16) float gv_smem[];
    __shared__ float s_stat[MT][GV_WARPS];
    __shared__ float s_amv[GV_WARPS][MT];
    __shared__ int s_ami[GV_WARPS][MT];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nchunk = (int)(p.row_bytes >> 4);
    const int S = (nchunk + 31) >> 5;                    // 512-byte segments per row
    const int k4 = nchunk * T::F4;
    float4 *xs = reinterpret_cast<float4 *>(gv_smem);
    float *xsum = gv_smem + (size_t)MT * k4 * 4;

    // contiguous range of row groups for this CTA, round-robin over its warps
    const int NG = (p.N + RW - 1) / RW;
    const int g_begin = (int)(((int64_t)blockIdx.x * NG) / gridDim.x);
    const int g_end = (int)(((int64_t)(blockIdx.x + 1) * NG) / gridDim.x);
    const int my_groups = g_end - g_begin > warp ? (g_end - g_begin - warp + GV_WARPS - 1) / GV_WARPS : 0;
    const int nsteps = my_groups * S;
    const int64_t spr = QT == Q_I4 ? (int64_t)p.K / p.group : 0;
    const __half *sc4 = reinterpret_cast<const __half *>(p.scales);

    // ---- issue side state: (group, segment) of the next step to load
    int is_g = g_begin + warp, is_s = 0;
    const uint8_t *iw[RW];
    const __half *isc[RW];
    bool iv[RW];
    auto set_issue_rows = [&]() {
#pragma unroll
        for (int j = 0; j < RW; j++) {
            const int lr = is_g * RW + j;
            iv[j] = lr < p.N;
            const int64_t pr = iv[j] ? gv_map_row(p, lr) : 0;
            iw[j] = p.w + pr * p.row_bytes + lane * 16;
            if (QT == Q_I4) isc[j] = sc4 + pr * spr;
        }
    };
    uint4 buf[D][RW];
    __half dsc[D][RW];          // INT4 group scales travel with their weights (fp16, packed in pairs)
    auto issue = [&](uint4 (&b)[RW], __half (&d)[RW], int i) {
        if (i < nsteps) {
            const int c = is_s * 32 + lane;
            const bool cv = c < nchunk;
#pragma unroll
            for (int j = 0; j < RW; j++) {
                const bool ok = cv && iv[j];
                b[j] = ok ? ldg_stream(iw[j] + (int64_t)is_s * 512) : make_uint4(0, 0, 0, 0);
                if (QT == Q_I4) d[j] = ok ? isc[j][(c * 32) / p.group] : __float2half_rn(0.0f);
            }
            if (++is_s == S) {
                is_s = 0;
                is_g += GV_WARPS;
                set_issue_rows();
            }
        }
    };
    set_issue_rows();
#pragma unroll
    for (int j = 0; j < D - 1; j++) issue(buf[j], dsc[j], j);

    // activations of the previous kernel are complete from here on
    pdl_wait();
    gv_stage_x<QT, MT>(p, xs, xsum, k4, nchunk, s_stat);
    pdl_trigger();

    float acc[RW][MT];
#pragma unroll
    for (int j = 0; j < RW; j++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[j][m] = 0.0f;
    float am_v[MT];
    int am_i[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) { am_v[m] = -INFINITY; am_i[m] = 0x7fffffff; }

    int cs_g = g_begin + warp, cs_s = 0;     // compute side (group, segment)
    for (int base = 0; base < nsteps; base += D) {
#pragma unroll
        for (int jj = 0; jj < D; jj++) {
            const int i = base + jj;
            if (i >= nsteps) break;
            issue(buf[(jj + D - 1) % D], dsc[(jj + D - 1) % D], i + D - 1);
            const int c = cs_s * 32 + lane;
            if (c < nchunk) {
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    const float4 *xm = xs + (size_t)m * k4;
                    if (QT == Q_I4) {
                        float2 part[RW];
#pragma unroll
                        for (int j = 0; j < RW; j++) part[j] = make_float2(0.f, 0.f);
#pragma unroll
                        for (int wd = 0; wd < 4; wd++) {
                            const float4 a = xm[gv_swz<QT>(c * 8 + 2 * wd)];
                            const float4 b = xm[gv_swz<QT>(c * 8 + 2 * wd + 1)];
#pragma unroll
                            for (int j = 0; j < RW; j++) {
                                const uint4 &w4 = buf[jj][j];
                                const uint32_t wv = wd == 0 ? w4.x : wd == 1 ? w4.y : wd == 2 ? w4.z : w4.w;
                                gv_dot_i4(wv, a, b, part[j]);
                            }
                        }
                        const float xs8 = xsum[m * nchunk + c];
#pragma unroll
                        for (int j = 0; j < RW; j++)
                            acc[j][m] = fmaf(__half2float(dsc[jj][j]), fmaf(part[j].x + part[j].y, GV_TWO50, -xs8),
                                             acc[j][m]);
                    } else if (QT == Q_I8) {
                        float2 part[RW];
#pragma unroll
                        for (int j = 0; j < RW; j++) part[j] = make_float2(0.f, 0.f);
#pragma unroll
                        for (int wd = 0; wd < 4; wd++) {
                            const float4 a = xm[gv_swz<QT>(c * 4 + wd)];
#pragma unroll
                            for (int j = 0; j < RW; j++) {
                                const uint4 &w4 = buf[jj][j];
                                const uint32_t wv = wd == 0 ? w4.x : wd == 1 ? w4.y : wd == 2 ? w4.z : w4.w;
                                gv_dot_i8(wv, a, part[j]);
                            }
                        }
#pragma unroll
                        for (int j = 0; j < RW; j++) acc[j][m] += part[j].x + part[j].y;
                    } else {
                        float2 part[RW];
#pragma unroll
                        for (int j = 0; j < RW; j++) part[j] = make_float2(0.f, 0.f);
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const float4 a = xm[gv_swz<QT>(c * 2 + h)];
#pragma unroll
                            for (int j = 0; j < RW; j++) {
                                const uint4 &w4 = buf[jj][j];
                                gv_dot_f16(h == 0 ? w4.x : w4.z, a.x, a.y, part[j]);
                                gv_dot_f16(h == 0 ? w4.y : w4.w, a.z, a.w, part[j]);
                            }
                        }
#pragma unroll
                        for (int j = 0; j < RW; j++) acc[j][m] += part[j].x + part[j].y;
                    }
                }
            }
            if (++cs_s == S) {
                // ---- row group done: fold the lanes, epilogue, reset
                float v[RW][MT];
#pragma unroll
                for (int j = 0; j < RW; j++)
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        v[j][m] = warp_sum(acc[j][m]);
                        acc[j][m] = 0.0f;
                    }
                const int lr0 = cs_g * RW;
                if (p.epi == EPI_QKV || p.epi == EPI_GATEUP) {
#pragma unroll
                    for (int jp = 0; jp < RW; jp += 2)
#pragma unroll
                        for (int m = 0; m < MT; m++)
                            if (lane == (jp / 2) * MT + m && m < p.M && lr0 + jp + 1 < p.N) {
                                const float x1 = gv_finish<QT>(p, xsum, lr0 + jp, m, v[jp][m]);
                                const float x2 = gv_finish<QT>(p, xsum, lr0 + jp + 1, m, v[jp + 1][m]);
                                gv_epi_pair(p, lr0 + jp, m, x1, x2);
                            }
                } else {
#pragma unroll
                    for (int j = 0; j < RW; j++)
#pragma unroll
                        for (int m = 0; m < MT; m++) {
                            const int lr = lr0 + j;
                            if (m < p.M && lr < p.N) {
                                if (p.epi == EPI_LOGITS) {
                                    const float f = gv_finish<QT>(p, xsum, lr, m, v[j][m]);
                                    if (f > am_v[m]) { am_v[m] = f; am_i[m] = p.vocab_off + lr; }
                                    if (lane == j * MT + m && p.logits) p.logits[(size_t)m * p.ldl + p.vocab_off + lr] = f;
                                } else if (lane == j * MT + m) {
                                    const float f = gv_finish<QT>(p, xsum, lr, m, v[j][m]);
                                    if (p.epi == EPI_STORE) p.y[(size_t)m * p.ldy + lr] = f;
                                    else p.y[(size_t)m * p.ldy + lr] += f;      // EPI_RESID
                                }
                            }
                        }
                }
                cs_s = 0;
                cs_g += GV_WARPS;
            }
        }
    }

    if (p.epi == EPI_LOGITS) {
        // per-CTA (max, argmax): rows ascend within a warp, so '>' keeps the lowest index on ties
        if (lane == 0)
#pragma unroll
            for (int m = 0; m < MT; m++) { s_amv[warp][m] = am_v[m]; s_ami[warp][m] = am_i[m]; }
        __syncthreads();
        if (tid < p.M && tid < MT) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int w = 0; w < GV_WARPS; w++) {
                const float v = s_amv[w][tid];
                const int ix = s_ami[w][tid];
                if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
            }
            p.am_val[(size_t)tid * gridDim.x + blockIdx.x] = bv;
            p.am_idx[(size_t)tid * gridDim.x + blockIdx.x] = bi;
        }
    }
}

size_t gemv_smem_bytes(int qt, int mt, int64_t row_bytes)
{
    const int nchunk = (int)(row_bytes >> 4);
    const int f4 = qt == Q_I4 ? 8 : qt == Q_I8 ? 4 : 2;
    size_t b = (size_t)mt * nchunk * f4 * 16;
    b += (qt == Q_I4 ? (size_t)mt * nchunk : (size_t)mt) * 4;
    return b;
}

static bool g_pdl = true;
void gemv_set_pdl(bool on) { g_pdl = on; }
bool pdl_enabled() { return g_pdl; }

template <int QT, int MT>
static int launch_mt(const GemvParams &p, int grid, size_t smem, cudaStream_t st)
{
    constexpr int RW = MT == 1 ? 4 : 2;
    constexpr int D = MT >= 2 ? 3 : 4;
    auto kern = qgemv_kernel<QT, MT, RW, D>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        DU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_set[dev & 63] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
    return DU_OK;
}

int gemv_rows_per_group(int M) { return M == 1 ? 4 : 2; }

int launch_gemv(int qt, GemvParams p, cudaStream_t st)
{
    if (p.M <= 0 || p.N <= 0) return DU_OK;
    if (p.M > 8) return fail(DU_EINVAL, "gemv: M > 8 must be split by the caller");
    const int mt = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
    const size_t smem = gemv_smem_bytes(qt, mt, p.row_bytes);
    if (smem > 200 * 1024) return fail(DU_EINVAL, "gemv: M*K too large for the shared-memory stage");
    const int grid = gemv_grid_for(p.N, mt, p.grid);
#define DU_GV_CASE(Q, M_)                                        \
    if (qt == Q && mt == M_) return launch_mt<Q, M_>(p, grid, smem, st);
    DU_GV_CASE(Q_I4, 1) DU_GV_CASE(Q_I4, 2) DU_GV_CASE(Q_I4, 4) DU_GV_CASE(Q_I4, 8)
    DU_GV_CASE(Q_I8, 1) DU_GV_CASE(Q_I8, 2) DU_GV_CASE(Q_I8, 4) DU_GV_CASE(Q_I8, 8)
    DU_GV_CASE(Q_F16, 1) DU_GV_CASE(Q_F16, 2) DU_GV_CASE(Q_F16, 4) DU_GV_CASE(Q_F16, 8)
#undef DU_GV_CASE
    return fail(DU_EINVAL, "gemv: unsupported quant kind");
}

// CTAs for N rows at token tile M: `want` (0 = 2 per SM), at most one per row group
int gemv_grid_for(int N, int M, int want)
{
    const int RW = gemv_rows_per_group(M);
    const int ng = (N + RW - 1) / RW;
    const int grid = want > 0 ? want : 2 * num_sms();
    return grid > ng ? ng : grid;
}

}  // namespace du
