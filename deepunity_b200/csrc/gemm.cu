// gemm.cu -- tensor-core dequant GEMM (tcgen05 + TMA) for prefill chunks and
// large decode batches.
//
// Replaces the coalesced GEMMs of Gemma3CS.compute (QKVProjGemmCoal ..
// DownGemmCoal, G3CS:1304-1439: 8 output rows x 8 tokens per thread group,
// weights re-read per group) for M > 8 token rows.  The decode GEMV
// (gemv.cu) streams each weight once per 8 tokens; this kernel streams it once
// per 128 (or more) tokens and multiplies on the 5th-generation tensor cores.
//
// One CTA computes a tile of 128 weight rows x TN tokens, looping over K in
// blocks of 64 columns.  Eight warps with fixed roles, connected by mbarriers:
//   warp 0  raw-weight producer: TMA tile loads of the packed INT4 / INT8 / fp16
//           rows into a ring of RS raw stages (no swizzle); runs ahead of the
//           previous kernel (before griddepcontrol.wait), since weights are
//           never written by the decode step;
//   warp 1  activation producer: TMA loads (128-byte swizzle) of the staged fp16
//           hi / lo activation tiles into the operand ring;
//   warp 2  TMEM owner and MMA issuer: one thread issues tcgen05.mma into a
//           128 x TN fp32 accumulator in tensor memory and commits each
//           operand stage back to the producers;
//   warps 4-7  dequant, then epilogue: thread j unpacks weight row j of each raw
//           stage into the exact fp16 hi (+ lo) operand rows (gemm_impl.cuh) in
//           the swizzled layout; after the last K block it reads its TMEM lane
//           (= weight row j) with tcgen05.ld and runs the fused epilogue of the
//           decode GEMV (store, residual add, split + RoPE + fp16 KV write,
//           SiLU(g) * u) for every token of the tile.
// Rows are visited in the decode GEMV's logical order (RoPE pairs and gate|up
// interleaved), so each epilogue pair sits in adjacent lanes (one shuffle).
//
// Every mbarrier wait is bounded; a wait that runs out sets a device error word,
// the CTA drains its in-flight copies, frees its tensor memory and returns.
// No load uses cluster multicast (the library runs tensor-parallel across GPUs).
#include <cstdlib>
#include <mutex>

#include "gemm_impl.cuh"
#include "gemv_impl.cuh"
#include "internal.h"

namespace du {

constexpr int GM_ROWS = 128;            // weight rows per tile (MMA M)
constexpr int GM_KB = 64;               // K columns per block: one 128-byte row of fp16
constexpr int GM_THREADS = 256;
constexpr uint64_t GM_SPIN_LIMIT = 2000000000ull;    // ns a bounded wait polls before giving up
constexpr size_t GM_SMEM_BUDGET = 225 * 1024;

struct GemmArgs {
    GemvParams p;           // weights, row map, epilogue (as the decode GEMV)
    const float *xscale;    // [M] per-token factor of the staged activations
    int tn;                 // tokens per tile (MMA N)
    int op_stages, raw_stages;
    int raw_bytes;          // one raw stage
    int kb_bytes;           // raw bytes of one row per K block
    int tmem_cols;
    int *err;               // device error word (bounded waits)
    // split-K: gridDim.z CTAs share a (row tile, token tile); each leaves its partial
    // accumulators in `partials`, the last to finish (per `counters`) sums them in
    // split order and runs the epilogue
    int ksplit;
    float *partials;        // [tiles][ksplit][TN][128]
    unsigned *counters;     // [tiles], zero between launches
};

// ------------------------------------------------------------ staging kernel

// Activations -> exact fp16 pairs: v = x (optionally RMSNorm'd, x * rsqrt(mean(x^2)
// + eps) * (1 + gamma'), RmsNormHidden G3CS:204-223), scaled by 2^s per token so
// that max |v| * 2^s < 2^15; hi = fp16(v * 2^s), lo = fp16(v * 2^s - hi);
// xscale[m] = 2^-s.  One CTA per token row.
__global__ void __launch_bounds__(256) gemm_stage_kernel(const float *x, int ldx, const __half *gamma, float eps,
                                                         int K, __half *xh, __half *xl, float *xscale)
{
    __shared__ float red[2][8];
    pdl_wait();
    const int m = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (size_t)m * ldx;
    float ss = 0.0f;
    if (gamma != nullptr)
        for (int k = tid; k < K; k += 256) ss += xr[k] * xr[k];
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[0][tid >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += red[0][i];
    const float inv = gamma != nullptr ? 1.0f / sqrtf(tot / (float)K + eps) : 1.0f;
    float mx = 0.0f;
    for (int k = tid; k < K; k += 256) {
        float v = xr[k];
        if (gamma != nullptr) v = v * inv * (1.0f + __half2float(gamma[k]));
        mx = fmaxf(mx, fabsf(v));
    }
    mx = warp_max(mx);
    if ((tid & 31) == 0) red[1][tid >> 5] = mx;
    __syncthreads();
    mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) mx = fmaxf(mx, red[1][i]);
    int s = mx > 0.0f ? 14 - ilogbf(mx) : 0;
    s = s > 100 ? 100 : (s < -100 ? -100 : s);
    const float sc = ldexpf(1.0f, s);
    if (tid == 0) xscale[m] = ldexpf(1.0f, -s);
    __half *oh = xh + (size_t)m * K, *ol = xl + (size_t)m * K;
    for (int k = tid; k < K; k += 256) {
        float v = xr[k];
        if (gamma != nullptr) v = v * inv * (1.0f + __half2float(gamma[k]));
        v *= sc;
        const __half h = __float2half_rn(v);
        oh[k] = h;
        ol[k] = __float2half_rn(v - __half2float(h));
    }
    pdl_trigger();
}

// ------------------------------------------------------------------ kernel

// Physical row (within the tile's raw stage) holding logical tile row j.
__device__ __forceinline__ int gm_raw_row(const GemvParams &p, int j)
{
    if (p.map == MAP_GATEUP) return (j & 1) ? 64 + (j >> 1) : (j >> 1);
    if (p.map == MAP_ROPE_PAIR) {
        const int hd = p.map_hd, h = j / hd, w = j - h * hd;
        return h * hd + (w >> 1) + (w & 1) * (hd >> 1);
    }
    return j;
}

// Global physical row of logical row lr (the decode GEMV's map plus row_off).
__device__ __forceinline__ int64_t gm_phys_row(const GemvParams &p, int lr) { return gv_map_row(p, lr); }

template <int QT>
__global__ void __launch_bounds__(GM_THREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xh,
                 const __grid_constant__ CUtensorMap tm_xl, const GemmArgs a)
{
    constexpr int NA = QT == Q_I4 ? 2 : 1;           // weight operands: hi (+ lo)
    extern __shared__ unsigned char gm_smem_raw[];
    const GemvParams &p = a.p;
    unsigned char *base = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(gm_smem_raw) + 1023) & ~(uintptr_t)1023);
    const int S = a.op_stages, RS = a.raw_stages, TN = a.tn;
    const int a_bytes = GM_ROWS * 128, b_bytes = TN * 128;
    const int op_bytes = NA * a_bytes + 2 * b_bytes;
    unsigned char *ops = base;
    unsigned char *raw = ops + (size_t)S * op_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(raw + (size_t)RS * a.raw_bytes);
    uint64_t *raw_full = bars, *raw_empty = bars + RS, *b_full = bars + 2 * RS, *a_full = b_full + S;
    uint64_t *op_empty = a_full + S, *acc_full = op_empty + S;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *abort_f = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_f = reinterpret_cast<volatile int *>(tmem_slot + 2);
    float *am_v = reinterpret_cast<float *>(tmem_slot + 4);          // [4 warps][32 tokens] (EPI_LOGITS)
    int *am_i = reinterpret_cast<int *>(am_v + 4 * 32);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row_tile = blockIdx.x, tok0 = blockIdx.y * TN;
    // this CTA's K blocks [kb0, kb0 + KB) (split-K part blockIdx.z of a.ksplit)
    const int KB_all = p.K / GM_KB, ks = blockIdx.z;
    const int kb0 = (int)(((int64_t)ks * KB_all) / a.ksplit);
    const int KB = (int)(((int64_t)(ks + 1) * KB_all) / a.ksplit) - kb0;
    auto A_hi = [&](int s) { return ops + (size_t)s * op_bytes; };
    auto A_lo = [&](int s) { return ops + (size_t)s * op_bytes + a_bytes; };
    auto B_hi = [&](int s) { return ops + (size_t)s * op_bytes + NA * a_bytes; };
    auto B_lo = [&](int s) { return ops + (size_t)s * op_bytes + NA * a_bytes + b_bytes; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < RS; i++) {
            mbar_init(smem_u32(raw_full + i), 1);
            mbar_init(smem_u32(raw_empty + i), 4);
        }
        for (int i = 0; i < S; i++) {
            mbar_init(smem_u32(b_full + i), 1);
            mbar_init(smem_u32(a_full + i), 4);
            mbar_init(smem_u32(op_empty + i), 1);
        }
        mbar_init(smem_u32(acc_full), 1);
        *abort_f = 0;
        mbar_fence_init();
    }
    if (warp == 2) {
        tmem_alloc(smem_u32(tmem_slot), (uint32_t)a.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- raw weights (independent of the previous kernel)
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            const int rows_box = p.map == MAP_GATEUP ? 64 : 128;
            int issued = 0;
            for (int kb = 0; kb < KB; kb++) {
                const int rs = kb % RS;
                if (!mbar_wait(smem_u32(raw_empty + rs), ((kb / RS) & 1) ^ 1, abort_f, a.err, GM_SPIN_LIMIT)) break;
                const uint32_t bar = smem_u32(raw_full + rs);
                mbar_arrive_expect_tx(bar, (uint32_t)a.raw_bytes);
                const uint32_t dst = smem_u32(raw + (size_t)rs * a.raw_bytes);
                const int x = (kb0 + kb) * a.kb_bytes;
                if (p.map == MAP_GATEUP) {
                    const int g0 = (int)p.row_off + row_tile * 64;
                    tma_load_2d(dst, &tm_w, bar, x, g0, pol);
                    tma_load_2d(dst + rows_box * a.kb_bytes, &tm_w, bar, x, g0 + p.map_I, pol);
                } else {
                    tma_load_2d(dst, &tm_w, bar, x, (int)p.row_off + row_tile * GM_ROWS, pol);
                }
                issued = kb + 1;
            }
            if (*abort_f) {     // let every issued copy land before the CTA exits
                for (int kb = issued - RS > 0 ? issued - RS : 0; kb < issued; kb++)
                    mbar_wait(smem_u32(raw_full + kb % RS), (kb / RS) & 1, abort_f, nullptr, GM_SPIN_LIMIT);
            }
        }
    } else if (warp == 1) {
        // ---------------- activations (written by the staging kernel)
        if (lane == 0) {
            pdl_wait();
            const uint64_t pol = l2_policy_evict_last();
            int issued = 0;
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % S;
                if (!mbar_wait(smem_u32(op_empty + s), ((kb / S) & 1) ^ 1, abort_f, a.err, GM_SPIN_LIMIT)) break;
                const uint32_t bar = smem_u32(b_full + s);
                mbar_arrive_expect_tx(bar, (uint32_t)(2 * b_bytes));
                tma_load_2d(smem_u32(B_hi(s)), &tm_xh, bar, (kb0 + kb) * GM_KB, tok0, pol);
                tma_load_2d(smem_u32(B_lo(s)), &tm_xl, bar, (kb0 + kb) * GM_KB, tok0, pol);
                issued = kb + 1;
            }
            if (*abort_f) {
                for (int kb = issued - S > 0 ? issued - S : 0; kb < issued; kb++)
                    mbar_wait(smem_u32(b_full + kb % S), (kb / S) & 1, abort_f, nullptr, GM_SPIN_LIMIT);
            }
        }
    } else if (warp == 2) {
        // ---------------- MMA issue
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(TN);
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % S;
                const uint32_t ph = (kb / S) & 1;
                if (!mbar_wait(smem_u32(a_full + s), ph, abort_f, a.err, GM_SPIN_LIMIT)) break;
                if (!mbar_wait(smem_u32(b_full + s), ph, abort_f, a.err, GM_SPIN_LIMIT)) break;
                tc_fence_after();
                const uint32_t ah = smem_u32(A_hi(s)), al = smem_u32(A_lo(s));
                const uint32_t bh = smem_u32(B_hi(s)), bl = smem_u32(B_lo(s));
#pragma unroll
                for (int k = 0; k < GM_KB / 16; k++) {
                    const uint64_t dah = umma_desc_sw128(ah + 32 * k);
                    const uint64_t dbh = umma_desc_sw128(bh + 32 * k);
                    const uint64_t dbl = umma_desc_sw128(bl + 32 * k);
                    tc_mma_f16(tmem, dah, dbh, idesc, (kb | k) != 0);
                    tc_mma_f16(tmem, dah, dbl, idesc, 1u);
                    if (NA == 2) tc_mma_f16(tmem, umma_desc_sw128(al + 32 * k), dbh, idesc, 1u);
                }
                tc_commit(smem_u32(op_empty + s));      // operand stage s is free once these MMAs complete
            }
            tc_commit(smem_u32(acc_full));              // the accumulator is final (or the loop gave up)
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---------------- dequant
        const int j = threadIdx.x - 128;            // weight row of the tile = TMEM lane
        const int lr = row_tile * GM_ROWS + j;      // logical row
        const bool row_ok = lr < p.N;
        const int rr = gm_raw_row(p, j);
        const int64_t pr = row_ok ? gm_phys_row(p, lr) : 0;
        const int ng = QT == Q_I4 ? p.K / p.group : 0;
        const __half *sc = reinterpret_cast<const __half *>(p.scales);
        bool ok = true;
        for (int kb = 0; kb < KB && ok; kb++) {
            // INT4 group scales of this row's 64 columns (one group, or two of 32)
            __half2 d0 = __half2half2(__float2half(0.0f)), d1 = d0;
            if (QT == Q_I4 && row_ok) {
                const int g = ((kb0 + kb) * GM_KB) / p.group;
                d0 = __half2half2(sc[pr * ng + g]);
                d1 = p.group == 32 ? __half2half2(sc[pr * ng + g + 1]) : d0;
            }
            const int rs = kb % RS, s = kb % S;
            if (!mbar_wait(smem_u32(raw_full + rs), (kb / RS) & 1, abort_f, a.err, GM_SPIN_LIMIT)) { ok = false; break; }
            const unsigned char *src = raw + (size_t)rs * a.raw_bytes + (size_t)rr * a.kb_bytes;
            // the raw row into registers; the stage goes back to the producer only after
            // these values are in the operand stage (below)
            uint4 w[8];
            constexpr int NW16 = QT == Q_I4 ? 2 : QT == Q_I8 ? 4 : 8;
#pragma unroll
            for (int i = 0; i < NW16; i++) w[i] = lds128_volatile(src + 16 * i);
            if (!mbar_wait(smem_u32(op_empty + s), ((kb / S) & 1) ^ 1, abort_f, a.err, GM_SPIN_LIMIT)) { ok = false; break; }
            unsigned char *ah = A_hi(s), *al = A_lo(s);
            if (QT == Q_I4) {
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const uint4 &u = w[c >> 2];
                    const uint32_t word = (c & 3) == 0 ? u.x : (c & 3) == 1 ? u.y : (c & 3) == 2 ? u.z : u.w;
                    uint4 hi, lo;
                    dq_int4_word(row_ok ? word : 0x88888888u, c < 4 ? d0 : d1, hi, lo);
                    *reinterpret_cast<uint4 *>(ah + sw128_off(j, c)) = hi;
                    *reinterpret_cast<uint4 *>(al + sw128_off(j, c)) = lo;
                }
            } else if (QT == Q_I8) {
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const uint4 &u = w[c >> 1];
                    const uint4 q = (c & 1) ? dq_int8_2words(u.z, u.w) : dq_int8_2words(u.x, u.y);
                    *reinterpret_cast<uint4 *>(ah + sw128_off(j, c)) = row_ok ? q : make_uint4(0, 0, 0, 0);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 8; c++)
                    *reinterpret_cast<uint4 *>(ah + sw128_off(j, c)) = row_ok ? w[c] : make_uint4(0, 0, 0, 0);
            }
            // Order this thread's generic-proxy accesses before the async proxy's: the operand
            // stores before the tensor cores read them, and the raw-stage loads (whose values
            // the stores consumed) before the next TMA load overwrites that stage.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_u32(raw_empty + rs));
                mbar_arrive(smem_u32(a_full + s));
            }
        }

        // ---------------- epilogue: TMEM lane j = logical row lr, column t = token tok0 + t
        pdl_wait();        // residual / KV / positions come from earlier kernels
        const bool acc_ok = mbar_wait(smem_u32(acc_full), 0, abort_f, a.err, GM_SPIN_LIMIT);
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        bool run = acc_ok && !*abort_f;
        if (run && a.ksplit > 1) {
            // leave this part's accumulators; the last part of the tile to arrive finishes it
            float *mine = a.partials + ((size_t)tile * a.ksplit + ks) * TN * GM_ROWS;
            for (int c0 = 0; c0 < TN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(taddr + (uint32_t)c0, r);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++) __stcg(mine + (size_t)(c0 + i) * GM_ROWS + j, __uint_as_float(r[i]));
            }
            __threadfence();
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (j == 0) *last_f = atomicAdd(a.counters + tile, 1u) == (unsigned)(a.ksplit - 1);
            asm volatile("bar.sync 1, 128;" ::: "memory");
            run = *last_f != 0;
            if (run) __threadfence();
        }
        if (run) {
            const float rsc = (QT == Q_I8 && row_ok) ? (p.scale_f32 ? reinterpret_cast<const float *>(p.scales)[pr]
                                                                    : __half2float(sc[pr]))
                                                     : 1.0f;
            for (int c0 = 0; c0 < TN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(taddr + (uint32_t)c0, r);
                tmem_wait_ld();
                if (tok0 + c0 >= p.M) continue;       // uniform across the epilogue warps
                float v[32];
                if (a.ksplit > 1) {
                    // sum of the parts in split order (this part's own values from TMEM)
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = 0.0f;
                    for (int k = 0; k < a.ksplit; k++) {
                        const float *part = a.partials + ((size_t)tile * a.ksplit + k) * TN * GM_ROWS;
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            v[i] += k == ks ? __uint_as_float(r[i]) : __ldcg(part + (size_t)(c0 + i) * GM_ROWS + j);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
                }
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int t = tok0 + c0 + i;
                    const bool tok_ok = t < p.M;
                    const float val = v[i] * (tok_ok ? a.xscale[t] : 0.0f) * rsc;
                    if (p.epi == EPI_QKV || p.epi == EPI_GATEUP) {
                        const float o = __shfl_xor_sync(0xffffffffu, val, 1);
                        if (tok_ok && row_ok && (lr & 1) == 0) {
                            if (p.epi == EPI_GATEUP)
                                p.y[(size_t)t * p.ldy + (lr >> 1)] = (p.act == 1 ? gelu_tanh(val) : val / (1.0f + expf(-val))) * o;
                            else gv_epi_pair(p, lr, t, val, o);
                        }
                    } else if (p.epi == EPI_LOGITS) {
                        if (tok_ok && row_ok && p.logits) p.logits[(size_t)t * p.ldl + lr] = val;
                        // this tile's (max, argmax) for token t, the reference's tie-break
                        float bv = (tok_ok && row_ok) ? val : -INFINITY;
                        int bi = row_ok ? p.vocab_off + lr : 0x7fffffff;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                            if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                        }
                        if (lane == 0) { am_v[(warp & 3) * 32 + i] = bv; am_i[(warp & 3) * 32 + i] = bi; }
                    } else if (tok_ok && row_ok) {
                        float *dst = p.y + (size_t)t * p.ldy + lr;
                        if (p.epi == EPI_RESID) *dst += val;
                        else *dst = val;
                    }
                }
                if (p.epi == EPI_LOGITS) {
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    const int t = tok0 + c0 + j;
                    if (j < 32 && t < p.M) {
                        float bv = am_v[j];
                        int bi = am_i[j];
#pragma unroll
                        for (int w = 1; w < 4; w++)
                            if (am_better(am_v[w * 32 + j], am_i[w * 32 + j], bv, bi)) {
                                bv = am_v[w * 32 + j];
                                bi = am_i[w * 32 + j];
                            }
                        p.am_val[(size_t)t * gridDim.x + row_tile] = bv;
                        p.am_idx[(size_t)t * gridDim.x + row_tile] = bi;
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                }
            }
            if (a.ksplit > 1 && j == 0) a.counters[tile] = 0u;     // every part has arrived: ready for the next launch
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
    }
}

// -------------------------------------------------------------------- host

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// 2-D tensor map over a row-major [rows, inner] array (inner elements contiguous).
int make_tmap(CUtensorMap *tm, CUtensorMapDataType dt, int esize, const void *ptr, uint64_t inner, uint64_t rows,
              uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(DU_ECUDA, "gemm: cuTensorMapEncodeTiled is unavailable");
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || ((inner * esize) & 15))
        return fail(DU_EINVAL, "gemm: operand base or row pitch not 16-byte aligned");
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * (uint64_t)esize};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DU_ECUDA, "gemm: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return DU_OK;
}

struct GemmPlan {
    int tn, op_stages, raw_stages, raw_bytes, kb_bytes, tmem_cols;
    size_t smem;
};

// Token tile (MMA N).  One thread issues a tcgen05.mma about every 110 cycles; an
// M = 128, N = 256, K = 16 MMA carries about as much tensor work (128 cycles), an
// N = 128 one half of it.  So large M takes N = 256 when the tiles still fill the GPU.
static int gm_tn_for(int M, int N)
{
    const int row_tiles = (N + GM_ROWS - 1) / GM_ROWS;
    if (M > 128 && (int64_t)row_tiles * ((M + 255) / 256) >= num_sms()) return 256;
    if (M > 64) return 128;
    if (M > 32) return 64;
    return 32;
}

static GemmPlan gm_plan(int qt, int M, int N)
{
    GemmPlan g = {};
    g.tn = gm_tn_for(M, N);
    g.kb_bytes = qt == Q_I4 ? 32 : qt == Q_I8 ? 64 : 128;
    g.raw_bytes = GM_ROWS * g.kb_bytes;
    g.raw_stages = qt == Q_I4 ? 8 : qt == Q_I8 ? 6 : 4;
    if (g.tn == 256) g.raw_stages = qt == Q_I4 ? 4 : qt == Q_I8 ? 3 : 2;   // two operand stages must fit
    static const int env_rs = [] { const char *e = getenv("DU_GEMM_RAW_STAGES"); return e ? atoi(e) : 0; }();
    if (env_rs > 0 && env_rs < g.raw_stages) g.raw_stages = env_rs;  // tuning knob: fewer raw-weight stages
    const int na = qt == Q_I4 ? 2 : 1;
    const size_t op = (size_t)na * GM_ROWS * 128 + 2 * (size_t)g.tn * 128;
    // alignment slack, raw ring, barriers + TMEM slot + flags + argmax scratch
    const size_t fixed = 1024 + (size_t)g.raw_stages * g.raw_bytes + 256 + 1040;
    int s = (int)((GM_SMEM_BUDGET - fixed) / op);
    g.op_stages = s > 4 ? 4 : s;
    static const int env_s = [] { const char *e = getenv("DU_GEMM_OP_STAGES"); return e ? atoi(e) : 0; }();
    if (env_s > 0 && env_s < g.op_stages) g.op_stages = env_s;      // tuning knob: fewer operand stages
    g.smem = fixed + (size_t)g.op_stages * op;
    g.tmem_cols = g.tn < 32 ? 32 : g.tn;
    return g;
}

bool gemm_supported(int qt, const GemvParams &p)
{
    if (p.M <= 0 || p.N <= 0 || p.K <= 0 || (p.K % GM_KB) != 0) return false;
    if (qt == Q_I4 && (p.group < 32 || (p.group & (p.group - 1)) != 0)) return false;
    if (p.epi != EPI_STORE && p.epi != EPI_RESID && p.epi != EPI_QKV && p.epi != EPI_GATEUP && p.epi != EPI_LOGITS)
        return false;
    if (p.map == MAP_GATEUP && (p.N != 2 * p.map_I || (p.map_I % 64) != 0)) return false;
    if (p.map == MAP_ROPE_PAIR && ((p.map_hd != 64 && p.map_hd != 128) || (p.N % GM_ROWS) != 0)) return false;
    return true;
}

int gemm_min_tokens()
{
    static const int v = [] {
        const char *e = getenv("DU_GEMM_MIN_M");
        const int x = e ? atoi(e) : 0;
        return x > 0 ? x : 16;
    }();
    return v;
}

template <int QT>
static int gm_launch(const CUtensorMap &tw, const CUtensorMap &th, const CUtensorMap &tl, const GemmArgs &a,
                     dim3 grid, size_t smem, cudaStream_t st)
{
    auto kern = qgemm_kernel<QT>;
    int rc = ensure_func_attrs((const void *)kern, (int)smem);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(GM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tw, th, tl, a));
    return DU_OK;
}

int launch_gemm(int qt, const GemvParams &p, const GemmScratch &scr, cudaStream_t st)
{
    if (p.M <= 0 || p.N <= 0) return DU_OK;
    if (!gemm_supported(qt, p)) return fail(DU_EINVAL, "gemm: unsupported shape, map or epilogue");
    if (!scr.xh || !scr.xl || !scr.xscale || (size_t)p.M * p.K > scr.elems || (size_t)p.M > scr.rows)
        return fail(DU_EINVAL, "gemm: activation scratch too small");
    // 1. activations -> exact fp16 pairs (RMSNorm folded in when gamma is set)
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(p.M);
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl_enabled() ? 1 : 0;
        DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_stage_kernel, p.x, p.ldx, p.gamma, p.eps, p.K, scr.xh, scr.xl,
                                       scr.xscale));
    }
    // 2. tensor maps
    const GemmPlan g = gm_plan(qt, p.M, p.N);
    const int64_t w_rows = p.row_off + (p.map == MAP_GATEUP ? 2 * (int64_t)p.map_I : (int64_t)p.N);
    CUtensorMap tw, th, tl;
    int rc = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.w, (uint64_t)p.row_bytes, (uint64_t)w_rows,
                       (uint32_t)g.kb_bytes, p.map == MAP_GATEUP ? 64u : (uint32_t)GM_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!rc) rc = make_tmap(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, scr.xh, (uint64_t)p.K, (uint64_t)p.M, GM_KB,
                            (uint32_t)g.tn, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc) rc = make_tmap(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, scr.xl, (uint64_t)p.K, (uint64_t)p.M, GM_KB,
                            (uint32_t)g.tn, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    // 3. the GEMM
    GemmArgs a = {};
    a.p = p;
    a.xscale = scr.xscale;
    a.tn = g.tn;
    a.op_stages = g.op_stages;
    a.raw_stages = g.raw_stages;
    a.raw_bytes = g.raw_bytes;
    a.kb_bytes = g.kb_bytes;
    a.tmem_cols = g.tmem_cols;
    a.err = scr.err;
    // split K when the tiles alone leave SMs idle: aim at two CTAs per SM in flight,
    // at least 4 K blocks per part, within the partial-sum scratch
    const int row_tiles = (p.N + GM_ROWS - 1) / GM_ROWS, tok_tiles = (p.M + g.tn - 1) / g.tn;
    const int tiles = row_tiles * tok_tiles, KB = p.K / GM_KB;
    int ks = 1;
    if (p.epi != EPI_LOGITS && tiles < num_sms()) {
        ks = (2 * num_sms() + tiles - 1) / tiles;
        if (ks > KB / 4) ks = KB / 4;
        while (ks > 1 && ((size_t)tiles * ks * g.tn * GM_ROWS > scr.partial_floats || (size_t)tiles > scr.counter_n))
            ks--;
        if (ks < 1) ks = 1;
    }
    static const int env_ks = [] { const char *e = getenv("DU_GEMM_KSPLIT"); return e ? atoi(e) : 0; }();
    if (env_ks > 0 && env_ks <= KB && (size_t)tiles * env_ks * g.tn * GM_ROWS <= scr.partial_floats &&
        (size_t)tiles <= scr.counter_n && p.epi != EPI_LOGITS)
        ks = env_ks;                                              // tuning knob: force a split count
    a.ksplit = ks;
    a.partials = scr.partials;
    a.counters = scr.counters;
    const dim3 grid(row_tiles, tok_tiles, ks);
    if (qt == Q_I4) return gm_launch<Q_I4>(tw, th, tl, a, grid, g.smem, st);
    if (qt == Q_I8) return gm_launch<Q_I8>(tw, th, tl, a, grid, g.smem, st);
    return gm_launch<Q_F16>(tw, th, tl, a, grid, g.smem, st);
}

// ---------------------------------------------------- dequant check kernel

// Writes the weight values the GEMM's unpack feeds the tensor cores, as fp32:
// INT4 hi + lo (= (n - 8) * d exactly), INT8 q * row scale, fp16 as is.
template <int QT>
__global__ void dequant_rows_kernel(const uint8_t *w, const void *scales, int scale_f32, int group, int64_t row0,
                                    int nrows, int K, float *out)
{
    const int r = blockIdx.y;
    const int64_t pr = row0 + r;
    const int nchunk = K / 8;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < nchunk; c += gridDim.x * blockDim.x) {
        float v[8];
        if (QT == Q_I4) {
            const uint32_t word = reinterpret_cast<const uint32_t *>(w + pr * (K / 2))[c];
            const __half d = reinterpret_cast<const __half *>(scales)[pr * (K / group) + (c * 8) / group];
            uint4 hi, lo;
            dq_int4_word(word, __half2half2(d), hi, lo);
            const uint32_t hh[4] = {hi.x, hi.y, hi.z, hi.w}, ll[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 a = __half22float2(u2h(hh[i])), b = __half22float2(u2h(ll[i]));
                v[2 * i] = a.x + b.x;
                v[2 * i + 1] = a.y + b.y;
            }
        } else if (QT == Q_I8) {
            const uint2 ww = reinterpret_cast<const uint2 *>(w + pr * K)[c];
            const uint4 q = dq_int8_2words(ww.x, ww.y);
            const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
            const float s = scale_f32 ? reinterpret_cast<const float *>(scales)[pr]
                                      : __half2float(reinterpret_cast<const __half *>(scales)[pr]);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 a = __half22float2(u2h(qq[i]));
                v[2 * i] = a.x * s;
                v[2 * i + 1] = a.y * s;
            }
        } else {
            const uint4 h = reinterpret_cast<const uint4 *>(w + pr * K * 2)[c];
            const uint32_t hh[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 a = __half22float2(u2h(hh[i]));
                v[2 * i] = a.x;
                v[2 * i + 1] = a.y;
            }
        }
        float *o = out + (size_t)r * K + (size_t)c * 8;
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = v[i];
    }
}

int launch_dequant_rows(int qt, const void *w, const void *scales, int scale_f32, int group, int64_t row0, int nrows,
                        int K, float *out, cudaStream_t st)
{
    if (nrows <= 0) return DU_OK;
    dim3 grid((K / 8 + 255) / 256, nrows);
    const uint8_t *wb = static_cast<const uint8_t *>(w);
    if (qt == Q_I4) dequant_rows_kernel<Q_I4><<<grid, 256, 0, st>>>(wb, scales, 0, group, row0, nrows, K, out);
    else if (qt == Q_I8) dequant_rows_kernel<Q_I8><<<grid, 256, 0, st>>>(wb, scales, scale_f32, 0, row0, nrows, K, out);
    else dequant_rows_kernel<Q_F16><<<grid, 256, 0, st>>>(wb, nullptr, 0, 0, row0, nrows, K, out);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

}  // namespace du
