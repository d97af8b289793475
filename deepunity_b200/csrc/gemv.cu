// gemv.cu -- decode GEMV kernel (see gemv.cuh) and its launcher.
#include "gemv.cuh"
#include "internal.h"

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

// Stages the activations of the MT tokens in shared memory.
//  INT4 / INT8: 22-bit fixed-point byte planes + zero-point sums, per-token shift
//  FP16: fp32, swizzled
template <int QT, int MT>
__device__ void gv_stage_x(const GemvParams &p, uint4 *xq, float *xsumf, long long *xsum64, float *xscale,
                           int nchunk, float *red)
{
    const int tid = threadIdx.x;
    for (int m = 0; m < MT; m++) {
        const float *xr = p.x + (size_t)m * p.ldx;
        const bool live = m < p.M;
        // one pass: sum of squares (RMSNorm) and max |x * (1 + gamma')| (fixed-point range)
        float ss = 0.0f, mx = 0.0f;
        if (live) {
            for (int k4 = tid; k4 < (p.K >> 2); k4 += GV_THREADS) {
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
        {
            const int lane = tid & 31, warp = tid >> 5;
            ss = warp_sum(ss);
            mx = warp_max(mx);
            __syncthreads();
            if (lane == 0) { red[warp] = ss; red[GV_WARPS + warp] = mx; }
            __syncthreads();
            ss = 0.0f; mx = 0.0f;
#pragma unroll
            for (int i = 0; i < GV_WARPS; i++) { ss += red[i]; mx = fmaxf(mx, red[GV_WARPS + i]); }
        }
        float inv = 1.0f;
        if (p.gamma != nullptr) {
            inv = 1.0f / sqrtf(ss / (float)p.K + p.eps);
            mx *= inv * 1.0000002f;     // bound on max |normalised x| (rounding of the product order)
        }
        if (QT == Q_F16) {
            float4 *xs = reinterpret_cast<float4 *>(xq) + (size_t)m * nchunk * 2;
            for (int f = tid; f < nchunk * 2; f += GV_THREADS) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (live) {
                    v.x = gv_xval(p, xr, inv, 4 * f);
                    v.y = gv_xval(p, xr, inv, 4 * f + 1);
                    v.z = gv_xval(p, xr, inv, 4 * f + 2);
                    v.w = gv_xval(p, xr, inv, 4 * f + 3);
                }
                xs[gv_swz16(f)] = v;
            }
            continue;
        }
        // per-token power-of-two scale: max |x| * 2^s < 2^22 (so |x_int| < 2^23 always)
        const int s = mx > 0.0f ? 21 - ilogbf(mx) : 0;
        const float sc = ldexpf(1.0f, s);
        if (tid == 0) xscale[m] = ldexpf(1.0f, -s);
        uint32_t *xw = reinterpret_cast<uint32_t *>(xq) + (size_t)m * nchunk * GvTraits<QT>::XU4 * 4;
        if (QT == Q_I4) {
            // word-group g = 8 columns; chunk c = g / 4, slot wd = g % 4; words
            // [P0 even, P0 odd, P1 even, P1 odd, P2 even, P2 odd] (even = columns 0,2,4,6)
            const int ngroups = nchunk * 4;
            for (int g0 = 0; g0 < ngroups; g0 += GV_THREADS) {
                const int g = g0 + tid;
                int part = 0;
                if (g < ngroups) {
                    uint32_t pe[3] = {0, 0, 0}, po[3] = {0, 0, 0};
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int v = live ? __float2int_rn(gv_xval(p, xr, inv, 8 * g + j) * sc) : 0;
                        part += v;
                        const int sh = 8 * (j >> 1);
                        uint32_t *dst = (j & 1) ? po : pe;
                        dst[0] |= (uint32_t)(v & 0xFF) << sh;
                        dst[1] |= (uint32_t)((v >> 8) & 0xFF) << sh;
                        dst[2] |= (uint32_t)((v >> 16) & 0xFF) << sh;
                    }
                    const int c = g >> 2, wd = g & 3;
                    uint32_t *o = xw + (size_t)c * GvTraits<QT>::XU4 * 4 + wd * 6;
                    o[0] = pe[0]; o[1] = po[0]; o[2] = pe[1]; o[3] = po[1]; o[4] = pe[2]; o[5] = po[2];
                }
                // chunk sum over the 4 word-groups held by 4 consecutive lanes
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                if (g < ngroups && (g & 3) == 0) xsumf[(size_t)m * nchunk + (g >> 2)] = 8.0f * (float)part;
            }
        } else {
            // word-group g = 4 columns; chunk c = g / 4, slot wd = g % 4; words [P0, P1, P2]
            const int ngroups = nchunk * 4;
            long long tot = 0;
            for (int g = tid; g < ngroups; g += GV_THREADS) {
                uint32_t pw[3] = {0, 0, 0};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int v = live ? __float2int_rn(gv_xval(p, xr, inv, 4 * g + j) * sc) : 0;
                    tot += v;
                    pw[0] |= (uint32_t)(v & 0xFF) << (8 * j);
                    pw[1] |= (uint32_t)((v >> 8) & 0xFF) << (8 * j);
                    pw[2] |= (uint32_t)((v >> 16) & 0xFF) << (8 * j);
                }
                const int c = g >> 2, wd = g & 3;
                uint32_t *o = xw + (size_t)c * GvTraits<QT>::XU4 * 4 + wd * 3;
                o[0] = pw[0]; o[1] = pw[1]; o[2] = pw[2];
            }
            // exact block sum of the int64 totals (two 32-bit halves through fp-free shuffles)
            for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
            __syncthreads();
            long long *r64 = reinterpret_cast<long long *>(red);
            if ((tid & 31) == 0) r64[tid >> 5] = tot;
            __syncthreads();
            if (tid == 0) {
                long long t = 0;
                for (int i = 0; i < GV_WARPS; i++) t += r64[i];
                xsum64[m] = t;
            }
        }
    }
    __syncthreads();
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

template <int QT>
__device__ __forceinline__ float gv_row_scale(const GemvParams &p, int lr)
{
    const int64_t pr = gv_map_row(p, lr);
    return p.scale_f32 ? reinterpret_cast<const float *>(p.scales)[pr]
                       : __half2float(reinterpret_cast<const __half *>(p.scales)[pr]);
}

template <int QT, int MT, int RW, int D>
__global__ void __launch_bounds__(GV_THREADS) qgemv_kernel(const GemvParams p)
{
    using T = GvTraits<QT>;
    extern __shared__ __align__(16) unsigned char gv_smem[];
    __shared__ float s_red[2 * GV_WARPS];
    __shared__ float s_xscale[MT];
    __shared__ long long s_xsum64[MT];
    __shared__ float s_amv[GV_WARPS][MT];
    __shared__ int s_ami[GV_WARPS][MT];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nchunk = (int)(p.row_bytes >> 4);
    const int S = (nchunk + 31) >> 5;                    // 512-byte segments per row

    // ring: [warp][stage][row][lane] 16-byte weight slots; INT4 also [warp][stage][row][lane]
    // 4-byte slots holding the fp16 pair that contains the lane's group scale; then the
    // staged activations
    uint4 *ring = reinterpret_cast<uint4 *>(gv_smem) + (size_t)warp * D * RW * 32 + lane;
    uint32_t *sring = reinterpret_cast<uint32_t *>(reinterpret_cast<uint4 *>(gv_smem) + (size_t)GV_WARPS * D * RW * 32) +
                      (size_t)warp * D * RW * 32 + lane;
    uint4 *xq = reinterpret_cast<uint4 *>(gv_smem) + (size_t)GV_WARPS * D * RW * 32 +
                (QT == Q_I4 ? (size_t)GV_WARPS * D * RW * 32 / 4 : 0);
    float *xsumf = reinterpret_cast<float *>(xq + (size_t)MT * nchunk * T::XU4);
    const uint8_t *sbase = reinterpret_cast<const uint8_t *>(p.scales);
    const int gshift = QT == Q_I4 ? __ffs(p.group) - 1 : 0;        // group is a power of two
    const int64_t srow_bytes = QT == Q_I4 ? ((int64_t)p.K >> gshift) * 2 : 0;

    // contiguous range of row groups for this CTA, round-robin over its warps
    const int NG = (p.N + RW - 1) / RW;
    const int g_begin = (int)(((int64_t)blockIdx.x * NG) / gridDim.x);
    const int g_end = (int)(((int64_t)(blockIdx.x + 1) * NG) / gridDim.x);
    const int my_groups = g_end - g_begin > warp ? (g_end - g_begin - warp + GV_WARPS - 1) / GV_WARPS : 0;
    const int nsteps = my_groups * S;

    // ---- issue side: (group, segment) of the next step to fetch
    int is_g = g_begin + warp, is_s = 0, is_stage = 0;
    const uint8_t *iw[RW];
    const uint8_t *isw[RW];
    bool iv[RW];
    auto set_issue_rows = [&]() {
#pragma unroll
        for (int j = 0; j < RW; j++) {
            const int lr = is_g * RW + j;
            iv[j] = lr < p.N;
            const int64_t pr = iv[j] ? gv_map_row(p, lr) : 0;
            iw[j] = p.w + pr * p.row_bytes + lane * 16;
            if (QT == Q_I4) isw[j] = sbase + pr * srow_bytes;
        }
    };
    auto issue = [&](int i) {
        if (i < nsteps) {
            const int c = is_s * 32 + lane;
            const bool cv = c < nchunk;
            // 4-byte word holding the fp16 scale of group (c * 32) >> gshift
            const int sw_off = (((c * 32) >> gshift) * 2) & ~3;
#pragma unroll
            for (int j = 0; j < RW; j++) {
                cp_async16_cg(ring + (is_stage * RW + j) * 32, iw[j] + (int64_t)is_s * 512, cv && iv[j]);
                if (QT == Q_I4) cp_async4_ca(sring + (is_stage * RW + j) * 32, isw[j] + sw_off, cv && iv[j]);
            }
            if (++is_stage == D) is_stage = 0;
            if (++is_s == S) {
                is_s = 0;
                is_g += GV_WARPS;
                set_issue_rows();
            }
        }
        cp_async_commit_group();
    };
    set_issue_rows();
#pragma unroll
    for (int j = 0; j < D - 1; j++) issue(j);

    // activations of the previous kernel are complete from here on
    pdl_wait();
    gv_stage_x<QT, MT>(p, xq, xsumf, s_xsum64, s_xscale, nchunk, s_red);
    pdl_trigger();

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

    int cs_g = g_begin + warp, cs_s = 0, cs_stage = 0;     // compute side (group, segment, ring slot)

    for (int i = 0; i < nsteps; i++) {
        issue(i + D - 1);
        cp_async_wait_group<D - 1>();
        const int stage = cs_stage;
        if (++cs_stage == D) cs_stage = 0;
        uint4 wv[RW];
#pragma unroll
        for (int j = 0; j < RW; j++) wv[j] = ring[(stage * RW + j) * 32];
        const int c = cs_s * 32 + lane;
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
                    const float xs8 = xsumf[(size_t)m * nchunk + c];
#pragma unroll
                    for (int j = 0; j < RW; j++) {
                        // even / odd nibble streams accumulate separately (shorter dependency chains)
                        int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
                        for (int wd = 0; wd < 4; wd++) {
                            const uint32_t w = wd == 0 ? wv[j].x : wd == 1 ? wv[j].y : wd == 2 ? wv[j].z : wv[j].w;
                            const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
                            a0 = dp4a_uu(lo, xw[wd * 6 + 0], a0);
                            b0 = dp4a_uu(hi, xw[wd * 6 + 1], b0);
                            a1 = dp4a_uu(lo, xw[wd * 6 + 2], a1);
                            b1 = dp4a_uu(hi, xw[wd * 6 + 3], b1);
                            a2 = dp4a_us(lo, xw[wd * 6 + 4], a2);
                            b2 = dp4a_us(hi, xw[wd * 6 + 5], b2);
                        }
                        // sum n * x_int - 8 * sum x_int: planes 0 and 1 join exactly in int32
                        // (< 2^25), plane 2 (< 2^19 in magnitude) is exact in fp32
                        const int p01 = (a0 + b0) + ((a1 + b1) << 8);
                        const float f = fmaf((float)(a2 + b2), 65536.0f, (float)p01) - xs8;
                        acc[j][m] = fmaf(d[j], f, acc[j][m]);
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
        if (++cs_s == S) {
            // ---- row group done: fold the lanes, epilogue, reset
            float v[RW][MT];
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
                        v[j][m] = (float)tot * s_xscale[m];
                        s8[j][m][0] = s8[j][m][1] = s8[j][m][2] = 0;
                    } else {
                        v[j][m] = warp_sum(acc[j][m]) * (QT == Q_I4 ? s_xscale[m] : 1.0f);
                        acc[j][m] = 0.0f;
                    }
                }
            const int lr0 = cs_g * RW;
            if (p.epi == EPI_QKV || p.epi == EPI_GATEUP) {
#pragma unroll
                for (int jp = 0; jp < RW; jp += 2)
#pragma unroll
                    for (int m = 0; m < MT; m++)
                        if (lane == (jp / 2) * MT + m && m < p.M && lr0 + jp + 1 < p.N) {
                            float x1 = v[jp][m], x2 = v[jp + 1][m];
                            if (QT == Q_I8) {
                                x1 *= gv_row_scale<QT>(p, lr0 + jp);
                                x2 *= gv_row_scale<QT>(p, lr0 + jp + 1);
                            }
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
                                const float f = v[j][m];
                                if (f > am_v[m]) { am_v[m] = f; am_i[m] = p.vocab_off + lr; }
                                if (lane == j * MT + m && p.logits)   // local shard; the index carries the offset
                                    p.logits[(size_t)m * p.ldl + lr] = f;
                            } else if (lane == j * MT + m) {
                                float f = v[j][m];
                                if (QT == Q_I8) f *= gv_row_scale<QT>(p, lr);
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
    cp_async_wait_group<0>();

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
                const float vv = s_amv[w][tid];
                const int ix = s_ami[w][tid];
                if (vv > bv || (vv == bv && ix < bi)) { bv = vv; bi = ix; }
            }
            p.am_val[(size_t)tid * gridDim.x + blockIdx.x] = bv;
            p.am_idx[(size_t)tid * gridDim.x + blockIdx.x] = bi;
        }
    }
}

// ------------------------------------------------------------------ launch

// Ring depth D: 4 when two CTAs per SM fit in shared memory, else 3 if that
// makes two fit (large K), else 4 with one CTA per SM.
static constexpr int rw_of(int mt) { return mt == 1 ? 4 : 2; }
static constexpr size_t SMEM_PER_SM = 227 * 1024;

static size_t ring_bytes(int qt, int mt, int d)
{
    const size_t slots = (size_t)GV_WARPS * d * rw_of(mt) * 32;
    return slots * 16 + (qt == Q_I4 ? slots * 4 : 0);
}

static size_t x_bytes(int qt, int mt, int64_t row_bytes)
{
    const int nchunk = (int)(row_bytes >> 4);
    const int xu4 = qt == Q_I4 ? 7 : qt == Q_I8 ? 3 : 2;
    return (size_t)mt * nchunk * xu4 * 16 + (qt == Q_I4 ? (size_t)mt * nchunk * 4 : 0);
}

static int choose_depth(int qt, int mt, int64_t row_bytes, int *cps)
{
    const size_t x = x_bytes(qt, mt, row_bytes);
    for (int d = 4; d >= 3; d--)
        if (2 * (ring_bytes(qt, mt, d) + x + 1024) <= SMEM_PER_SM) { *cps = 2; return d; }
    *cps = 1;
    return 4;
}

size_t gemv_smem_bytes(int qt, int mt, int64_t row_bytes)
{
    int cps = 1;
    const int d = choose_depth(qt, mt, row_bytes, &cps);
    return ring_bytes(qt, mt, d) + x_bytes(qt, mt, row_bytes);
}

static bool g_pdl = true;
void gemv_set_pdl(bool on) { g_pdl = on; }
bool pdl_enabled() { return g_pdl; }

int gemv_rows_per_group(int M) { return rw_of(M <= 1 ? 1 : 2); }

template <int QT, int MT, int D>
static int launch_kernel(const GemvParams &p, int grid, size_t smem, cudaStream_t st)
{
    auto kern = qgemv_kernel<QT, MT, rw_of(MT), D>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        DU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
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

template <int QT, int MT>
static int launch_mt(const GemvParams &p, int grid, int depth, size_t smem, cudaStream_t st)
{
    return depth == 3 ? launch_kernel<QT, MT, 3>(p, grid, smem, st) : launch_kernel<QT, MT, 4>(p, grid, smem, st);
}

// CTAs for N rows at token tile M: `want` (0 = 2 per SM), never more than one per row group
int gemv_grid_for(int N, int M, int want)
{
    const int RW = gemv_rows_per_group(M);
    const int ng = (N + RW - 1) / RW;
    const int grid = want > 0 ? want : 2 * num_sms();
    return grid > ng ? ng : grid;
}

int launch_gemv(int qt, GemvParams p, cudaStream_t st)
{
    if (p.M <= 0 || p.N <= 0) return DU_OK;
    if (p.M > 8) return fail(DU_EINVAL, "gemv: M > 8 must be split by the caller");
    if (qt == Q_I4 && (p.group < 32 || (p.group & (p.group - 1)) || ((p.K / p.group) & 1)))
        return fail(DU_EINVAL, "gemv: int4 group must be a power of two >= 32 with an even number of groups per row");
    const int mt = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
    int cps = 1;
    const int depth = choose_depth(qt, mt, p.row_bytes, &cps);
    const size_t smem = ring_bytes(qt, mt, depth) + x_bytes(qt, mt, p.row_bytes);
    if (smem > 220 * 1024) return fail(DU_EINVAL, "gemv: M*K too large for the shared-memory stage");
    const int grid = gemv_grid_for(p.N, mt, p.grid > 0 ? p.grid : cps * num_sms());
#define DU_GV_CASE(Q, M_)                                        \
    if (qt == Q && mt == M_) return launch_mt<Q, M_>(p, grid, depth, smem, st);
    DU_GV_CASE(Q_I4, 1) DU_GV_CASE(Q_I4, 2) DU_GV_CASE(Q_I4, 4) DU_GV_CASE(Q_I4, 8)
    DU_GV_CASE(Q_I8, 1) DU_GV_CASE(Q_I8, 2) DU_GV_CASE(Q_I8, 4) DU_GV_CASE(Q_I8, 8)
    DU_GV_CASE(Q_F16, 1) DU_GV_CASE(Q_F16, 2) DU_GV_CASE(Q_F16, 4) DU_GV_CASE(Q_F16, 8)
#undef DU_GV_CASE
    return fail(DU_EINVAL, "gemv: unsupported quant kind");
}

}  // namespace du
