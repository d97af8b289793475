// tgemv.cu -- the decode GEMV (one or two token rows) on the 5th-generation tensor
// cores: tcgen05.mma kind::i8, TMA weight streaming, TMEM accumulators.
//
// Replaces the coalesced decode GEMVs of Gemma3CS.compute (QKVProj1VecCoal ..
// Down1VecCoal, G3CS:1217-1282, with readQ4 / wScale of G3CS:84-101) for INT4
// weights, with the same fused prologue (RMSNorm) and epilogues (store, residual
// add, split + RoPE + fp16 KV write, SiLU(g) * u) as the dp4a GEMV (gemv.cu).
//
// Exact integer products.  A weight row is used as its unsigned nibbles n in
// 0..15 (u8); the activations of a token become 22-bit fixed point x_int =
// round(x * (1 + gamma') * 2^s) (one power-of-two scale per token) split into
// three signed byte planes, x_int = p0 + 256 p1 + 65536 p2.  One MMA per 32
// columns multiplies 128 weight rows by 8 B rows (3 planes x up to 2 tokens, 2
// zero rows) into int32 accumulators: sum n * p exactly.  Per quantization
// group the accumulators are read from tensor memory and folded in fp32:
//   d_g * (c0 + 256 c1 + 65536 c2 - 8 * sum_g x_int) * 2^-s,
// which is the reference's sum of (n - 8) * d * x to ~2^-22 of the token's
// largest |x|; 1 / rms (RMSNorm) multiplies the finished dot product.
// Within each 8-column word the weight bytes are stored as the low nibbles
// (columns 0, 2, 4, 6) then the high ones (1, 3, 5, 7); the activation planes
// use the same K order, so the unpack is two logical operations per word.
//
// Work split: units are (128-row tile, 128-column K block) pairs, tile-major;
// CTA c of C (one per SM) takes the contiguous range [c U / C, (c + 1) U / C), so
// every CTA streams the same number of bytes.  A tile whose blocks span several
// CTAs is finished by the last of them to arrive (per-tile counter): it adds
// the parts' partial sums in CTA order (deterministic) and runs the epilogue.
// No CTA waits for another.
//
// Roles (256 threads): warp 0 lane 0 issues the TMA loads of the raw weight
// tiles (the first stages before griddepcontrol.wait: weights never depend on
// the previous kernel); warp 1 owns the tensor memory and one of its threads
// issues the MMAs; warps 4-7 unpack weight row j of each tile into the MMA's
// A layout and, a few units later, read row j's accumulators (TMEM lane j) and
// fold them.  All warps stage the activation planes once.  Every mbarrier wait is
// bounded in time.  Shared memory stays under half an SM so that the next
// kernel's CTA (launched early under programmatic dependent launch) can be
// resident and stream its own weights while this kernel finishes.
#include <cstdlib>
#include <cstring>

#include "gemm_impl.cuh"
#include "gemv_impl.cuh"
#include "internal.h"

// Event hook for timing studies of the pipeline; expands to nothing in the library.
#ifndef TG_STAMP
#define TG_STAMP(event, unit)
#endif

namespace du {

constexpr int TG_ROWS = 128;           // weight rows per tile = MMA M = TMEM lanes
constexpr int TG_KB = 128;             // K columns per unit
constexpr int TG_THREADS = 256;
constexpr int TG_NBUF = 16;            // group-scale prefetch ring (units)
constexpr int TG_TMEM_COLS = 128;      // accumulator ring in tensor memory: 128 / (8 * GPB) units
constexpr int TG_MAX_AS = 8;           // unpacked-weight (A operand) stages, at most
constexpr int TG_PF = 4;               // slots of the scale ring the readout keeps clear of the unpack
constexpr int TG_RAW_STAGE = 8192 + 2048;   // a unit's packed weights (128 rows x 64 B) + its scale box (128 x 16 B)
constexpr uint64_t TG_WAIT_NS = 2000000000ull;

struct TgArgs {
    GemvParams p;
    int C;                 // CTAs
    int64_t U;             // units: tiles * NB
    int NB;                // K blocks per row
    int gpb;               // quantization groups per K block (1, 2 or 4)
    int rs;                // raw-weight ring depth
    int nb_max;            // activation blocks staged per CTA
    int max_parts;         // partial-sum slots per tile
    int as;                // unpacked-weight (A operand) stages
    int lag;               // accumulator readout trails the unpack by this many units (< TG_NBUF - TG_PF)
    int tmem_cols;
    float *partials;       // [tiles][max_parts][2 tokens][128 rows]
    unsigned *counters;    // [tiles], zero between launches
    int *err;
};

__device__ __forceinline__ int64_t tg_lo(int64_t c, int64_t U, int C) { return (c * U) / C; }

// CTA that owns unit u
__device__ __forceinline__ int tg_owner(int64_t u, int64_t U, int C)
{
    int c = (int)((u * C) / U);
    while (c + 1 < C && tg_lo(c + 1, U, C) <= u) c++;
    while (c > 0 && tg_lo(c, U, C) > u) c--;
    return c;
}

__device__ __forceinline__ void tc_mma_i8(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// kind::i8: int32 accumulators, A unsigned (nibbles), B signed (planes), both K-major, M = 128, N = 8
__host__ __device__ constexpr uint32_t tg_idesc() { return (2u << 4) | (0u << 7) | (1u << 10) | ((8u >> 3) << 17) | ((128u >> 4) << 24); }

template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, int (&c)[NC])
{
    static_assert(NC == 8 || NC == 16 || NC == 32, "8, 16 or 32 columns");
    uint32_t r[32];
    if (NC == 32) {
        tmem_ld32(taddr, r);
    } else if (NC == 16) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                     "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                       "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                       "=r"(r[14]), "=r"(r[15])
                     : "r"(taddr));
    } else {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                       "=r"(r[7])
                     : "r"(taddr));
    }
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < NC; i++) c[i] = (int)r[i];
}

// final epilogue of logical row lr for tokens 0..M-1 (y[m] = finished dot product);
// every lane of the warp calls it (pair epilogues exchange with the neighbour lane)
__device__ __forceinline__ void tg_epilogue(const GemvParams &p, int lr, bool row_ok, const float (&y)[2])
{
#pragma unroll
    for (int m = 0; m < 2; m++) {
        const float v = y[m];
        if (p.epi == EPI_QKV || p.epi == EPI_GATEUP) {
            const float o = __shfl_xor_sync(0xffffffffu, v, 1);
            if (m < p.M && row_ok && (lr & 1) == 0) {
                if (p.epi == EPI_GATEUP)
                    p.y[(size_t)m * p.ldy + (lr >> 1)] = (p.act == 1 ? gelu_tanh(v) : v / (1.0f + expf(-v))) * o;
                else gv_epi_pair(p, lr, m, v, o);
            }
        } else if (m < p.M && row_ok) {
            float *dst = p.y + (size_t)m * p.ldy + lr;
            if (p.epi == EPI_RESID) *dst += v;
            else *dst = v;
        }
    }
}

template <int GPB>
__global__ void __launch_bounds__(TG_THREADS, 2)
    tgemv_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s, const TgArgs a)
{
    constexpr int CPA = GPB * 8;                 // TMEM columns of one unit's accumulators
    constexpr int NBT = TG_TMEM_COLS / CPA;      // units in the accumulator ring
    constexpr int KPG = 4 / GPB;                 // 32-column MMA steps per quantization group
    extern __shared__ unsigned char tg_smem_raw[];
    const GemvParams &p = a.p;
    unsigned char *base = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(tg_smem_raw) + 1023) & ~(uintptr_t)1023);
    const int RS = a.rs, NB = a.NB, TG_AS = a.as, TG_LAG = a.lag;
    unsigned char *A = base;                                         // [TG_AS][128 rows][128 B], swizzled
    unsigned char *B = A + TG_AS * 16384;                            // [nb_max][8 rows][128 B], swizzled
    unsigned char *raw = B + (size_t)a.nb_max * 1024;                // [RS][128 rows][64 B] + [128 rows][16 B] scales
    // raw fp16 group-scale words of each unit's rows, fetched TG_PF units ahead with cp.async:
    // [TG_NBUF][128 rows][SW] 32-bit words (the aligned word(s) holding the unit's GPB scales)
    uint32_t *sring = reinterpret_cast<uint32_t *>(raw + (size_t)RS * TG_RAW_STAGE);
    int *zsum = reinterpret_cast<int *>(sring + TG_NBUF * 128 * 2);      // [nb_max][GPB][2]
    float *tok = reinterpret_cast<float *>(zsum + a.nb_max * GPB * 2);   // [0..1] 2^-s, [2..3] 1/rms, [4..35] red
    uint64_t *bars = reinterpret_cast<uint64_t *>(tok + 40);
    uint64_t *raw_full = bars, *raw_empty = bars + RS, *a_full = bars + 2 * RS, *a_empty = a_full + TG_AS;
    uint64_t *acc_full = a_empty + TG_AS, *acc_empty = acc_full + NBT;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + NBT);
    volatile int *abort_f = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_f = reinterpret_cast<volatile int *>(tmem_slot + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = a.C, c = blockIdx.x;
    const int64_t U = a.U, u0 = tg_lo(c, U, C), u1 = tg_lo(c + 1, U, C);
    const int n = (int)(u1 - u0);
    const int b_first = (int)(u0 % NB), nbs = n < NB ? n : NB;      // activation blocks this CTA uses
    auto slot_of = [&](int b) { return (b - b_first + NB) % NB; };

    if (tid == 0) {
        for (int i = 0; i < RS; i++) {
            mbar_init(smem_u32(raw_full + i), 1);
            mbar_init(smem_u32(raw_empty + i), 4);
        }
        for (int i = 0; i < TG_AS; i++) {
            mbar_init(smem_u32(a_full + i), 4);
            mbar_init(smem_u32(a_empty + i), 1);
        }
        for (int i = 0; i < NBT; i++) {
            mbar_init(smem_u32(acc_full + i), 1);
            mbar_init(smem_u32(acc_empty + i), 4);
        }
        *abort_f = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), (uint32_t)a.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // ---- raw weight tiles of unit i into stage i % RS
    const uint64_t pol = l2_policy_evict_first();
    // the aligned window of 8 group scales holding this unit's GPB groups
    auto scale_x = [&](int b) { return ((b * TG_KB) / p.group) & ~7; };
    auto issue = [&](int i) {
        const int64_t u = u0 + i;
        const int t = (int)(u / NB), b = (int)(u % NB);
        const uint32_t bar = smem_u32(raw_full + i % RS);
        mbar_arrive_expect_tx(bar, (uint32_t)TG_RAW_STAGE);
        const uint32_t dst = smem_u32(raw + (size_t)(i % RS) * TG_RAW_STAGE);
        const int sx = scale_x(b);
        if (p.map == MAP_GATEUP) {
            const int g0 = (int)p.row_off + t * 64;
            tma_load_2d(dst, &tm_w, bar, b * 64, g0, pol);
            tma_load_2d(dst + 64 * 64, &tm_w, bar, b * 64, g0 + p.map_I, pol);
            tma_load_2d(dst + 8192, &tm_s, bar, sx, g0, pol);
            tma_load_2d(dst + 8192 + 64 * 16, &tm_s, bar, sx, g0 + p.map_I, pol);
        } else {
            tma_load_2d(dst, &tm_w, bar, b * 64, (int)p.row_off + t * TG_ROWS, pol);
            tma_load_2d(dst + 8192, &tm_s, bar, sx, (int)p.row_off + t * TG_ROWS, pol);
        }
    };
    const int pre = n < RS ? n : RS;
    if (warp == 0 && lane == 0)
        for (int i = 0; i < pre; i++) {
            issue(i);
            TG_STAMP(0, i);
        }

    // ---- activations (written by the previous kernel) -> signed byte planes
    pdl_wait();
    pdl_trigger();        // the next kernel may become resident and start streaming its weights
    {
        uint4 *bz = reinterpret_cast<uint4 *>(B);
        for (int i = tid; i < nbs * 64; i += TG_THREADS) bz[i] = make_uint4(0u, 0u, 0u, 0u);
        for (int i = tid; i < nbs * GPB * 2; i += TG_THREADS) zsum[i] = 0;
        float *red = tok + 4;
        for (int m = 0; m < p.M; m++) {
            const float *xr = p.x + (size_t)m * p.ldx;
            float ss = 0.0f, mx = 0.0f;
            for (int k8 = tid; k8 < (p.K >> 3); k8 += TG_THREADS) {
                const float4 xa = reinterpret_cast<const float4 *>(xr)[2 * k8];
                const float4 xb = reinterpret_cast<const float4 *>(xr)[2 * k8 + 1];
                float v[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                float g[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
                if (p.gamma != nullptr) {
                    const uint4 gw = reinterpret_cast<const uint4 *>(p.gamma)[k8];
                    const uint32_t gg[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float2 f = __half22float2(u2h(gg[q]));
                        g[2 * q] = 1.0f + f.x;
                        g[2 * q + 1] = 1.0f + f.y;
                    }
                }
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    ss += v[q] * v[q];
                    mx = fmaxf(mx, fabsf(v[q] * g[q]));
                }
            }
            ss = warp_sum(ss);
            mx = warp_max(mx);
            if (lane == 0) { red[warp] = ss; red[8 + warp] = mx; }
            __syncthreads();
            if (tid == 0) {
                float s2 = 0.0f, m2 = 0.0f;
                for (int w = 0; w < 8; w++) { s2 += red[w]; m2 = fmaxf(m2, red[8 + w]); }
                int e = m2 > 0.0f ? 21 - ilogbf(m2) : 0;
                e = e > 120 ? 120 : e;
                tok[m] = ldexpf(1.0f, -e);                   // 2^-s
                tok[2 + m] = p.gamma != nullptr ? 1.0f / sqrtf(s2 / (float)p.K + p.eps) : 1.0f;
                red[16 + m] = ldexpf(1.0f, e);               // 2^s
            }
            __syncthreads();
        }
        __syncthreads();
        // planes of the blocks this CTA uses: one 8-column word group per work item
        const int G = p.group;
        for (int it = tid; it < nbs * 16 * p.M; it += TG_THREADS) {
            const int m = it % p.M, rest = it / p.M, q = rest & 15, sl = rest >> 4;
            const int b = (b_first + sl) % NB;
            const int col0 = b * TG_KB + q * 8;
            const float *xr = p.x + (size_t)m * p.ldx + col0;
            const float4 xa = reinterpret_cast<const float4 *>(xr)[0];
            const float4 xb = reinterpret_cast<const float4 *>(xr)[1];
            float v[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            if (p.gamma != nullptr) {
                const uint4 gw = reinterpret_cast<const uint4 *>(p.gamma + col0)[0];
                const uint32_t gg[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
                for (int qq = 0; qq < 4; qq++) {
                    const float2 f = __half22float2(u2h(gg[qq]));
                    v[2 * qq] *= 1.0f + f.x;
                    v[2 * qq + 1] *= 1.0f + f.y;
                }
            }
            const float sc = tok[4 + 16 + m];
            int xi[8], part = 0;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                xi[e] = __float2int_rn(v[e] * sc);
                part += xi[e];
            }
            // balanced base-256 digits; K order within the word: columns 0,2,4,6,1,3,5,7
            uint32_t pl[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int x = xi[e];
                const int d0 = ((x + 128) & 255) - 128;
                const int x1 = (x - d0) >> 8;
                const int d1 = ((x1 + 128) & 255) - 128;
                const int d2 = (x1 - d1) >> 8;
                const int kp = (e & 1) ? 4 + (e >> 1) : (e >> 1);
                pl[0][kp >> 2] |= (uint32_t)(d0 & 255) << (8 * (kp & 3));
                pl[1][kp >> 2] |= (uint32_t)(d1 & 255) << (8 * (kp & 3));
                pl[2][kp >> 2] |= (uint32_t)(d2 & 255) << (8 * (kp & 3));
            }
#pragma unroll
            for (int pp = 0; pp < 3; pp++) {
                const int r = 3 * m + pp;
                *reinterpret_cast<uint2 *>(B + (size_t)sl * 1024 + r * 128 + ((((q >> 1) ^ r) & 7) << 4) + ((q & 1) << 3)) =
                    make_uint2(pl[pp][0], pl[pp][1]);
            }
            const int gi = G >= TG_KB ? 0 : (q * 8) / G;
            atomicAdd(zsum + (sl * GPB + gi) * 2 + m, part);
        }
        fence_proxy_async_smem();
        __syncthreads();
    }
    if (tid == 0) TG_STAMP(9, 0);

    if (warp == 0) {
        // ---------------- raw weight producer (the rest of the units)
        if (lane == 0) {
            int issued = pre;
            for (int i = pre; i < n; i++) {
                if (!mbar_wait(smem_u32(raw_empty + i % RS), ((i / RS) & 1) ^ 1, abort_f, a.err, TG_WAIT_NS)) break;
                issue(i);
                TG_STAMP(0, i);
                issued = i + 1;
            }
            if (*abort_f)
                for (int i = issued - RS > 0 ? issued - RS : 0; i < issued; i++)
                    mbar_wait(smem_u32(raw_full + i % RS), (i / RS) & 1, abort_f, nullptr, TG_WAIT_NS);
        }
    } else if (warp == 1) {
        // ---------------- MMA issue
        if (lane == 0) {
            const uint32_t idesc = tg_idesc();
            for (int i = 0; i < n; i++) {
                const int as = i % TG_AS, ab = i % NBT;
                if (!mbar_wait(smem_u32(a_full + as), (i / TG_AS) & 1, abort_f, a.err, TG_WAIT_NS)) break;
                TG_STAMP(4, i);
                if (!mbar_wait(smem_u32(acc_empty + ab), ((i / NBT) & 1) ^ 1, abort_f, a.err, TG_WAIT_NS)) break;
                TG_STAMP(5, i);
                tc_fence_after();
                const int b = (int)((u0 + i) % NB);
                const uint32_t aa = smem_u32(A + as * 16384), bb = smem_u32(B + (size_t)slot_of(b) * 1024);
#pragma unroll
                for (int k = 0; k < 4; k++)
                    tc_mma_i8(tmem + (uint32_t)(ab * CPA + (k / KPG) * 8), umma_desc_sw128(aa + 32 * k),
                              umma_desc_sw128(bb + 32 * k), idesc, (uint32_t)(k % KPG));
                tc_commit(smem_u32(a_empty + as));
                tc_commit(smem_u32(acc_full + ab));
                TG_STAMP(6, i);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---------------- unpack (unit it) and accumulator readout (unit it - TG_LAG)
        const int j = tid - 128;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        float acc[2] = {0.0f, 0.0f};
        bool ok = true;
        for (int it = 0; it < n + TG_LAG && ok; it++) {
            if (it < n) {
                const int64_t u = u0 + it;
                const int t = (int)(u / NB);
                const int lr = t * TG_ROWS + j;
                const bool row_ok = lr < p.N;
                const int rs = it % RS, as = it % TG_AS;
                if (!mbar_wait(smem_u32(raw_full + rs), (it / RS) & 1, abort_f, a.err, TG_WAIT_NS)) { ok = false; break; }
                if (j == 0) TG_STAMP(1, it);
                int rr = j;
                if (p.map == MAP_GATEUP) rr = (j & 1) ? 64 + (j >> 1) : (j >> 1);
                else if (p.map == MAP_ROPE_PAIR) {
                    const int hd = p.map_hd, h = j / hd, w = j - h * hd;
                    rr = h * hd + (w >> 1) + (w & 1) * (hd >> 1);
                }
                const unsigned char *src = raw + (size_t)rs * TG_RAW_STAGE + (size_t)rr * 64;
                uint4 w4[4];
#pragma unroll
                for (int q = 0; q < 4; q++) w4[q] = lds128_volatile(src + 16 * q);
                // this row's GPB scales (halves first .. first + GPB - 1 of its 8-scale window) into
                // the scale ring, where the readout finds them TG_LAG units later
                {
                    const uint4 sv = lds128_volatile(raw + (size_t)rs * TG_RAW_STAGE + 8192 + (size_t)rr * 16);
                    const int b = (int)(u % NB), first = ((b * TG_KB) / p.group) - scale_x(b);
                    uint32_t *dst = sring + ((it % TG_NBUF) * 128 + j) * 2;
                    uint32_t o0 = 0u, o1 = 0u;
#pragma unroll
                    for (int gi = 0; gi < GPB; gi++) {
                        const int hx = first + gi;
                        const int wq = hx >> 1;
                        const uint32_t wsel = wq == 0 ? sv.x : wq == 1 ? sv.y : wq == 2 ? sv.z : sv.w;
                        const uint32_t h = (wsel >> ((hx & 1) * 16)) & 0xFFFFu;
                        if (gi < 2) o0 |= h << (16 * gi);
                        else o1 |= h << (16 * (gi - 2));
                    }
                    dst[0] = row_ok ? o0 : 0u;
                    dst[1] = row_ok ? o1 : 0u;
                }
                if (!mbar_wait(smem_u32(a_empty + as), ((it / TG_AS) & 1) ^ 1, abort_f, a.err, TG_WAIT_NS)) { ok = false; break; }
                if (j == 0) TG_STAMP(2, it);
                unsigned char *arow = A + as * 16384;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const uint32_t ww[4] = {w4[q].x, w4[q].y, w4[q].z, w4[q].w};
                    uint32_t o[8];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const uint32_t wv = row_ok ? ww[e] : 0u;
                        o[2 * e] = wv & 0x0F0F0F0Fu;            // columns 0, 2, 4, 6 of the word
                        o[2 * e + 1] = (wv >> 4) & 0x0F0F0F0Fu; // columns 1, 3, 5, 7
                    }
                    *reinterpret_cast<uint4 *>(arow + sw128_off(j, 2 * q)) = make_uint4(o[0], o[1], o[2], o[3]);
                    *reinterpret_cast<uint4 *>(arow + sw128_off(j, 2 * q + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(raw_empty + rs));
                    mbar_arrive(smem_u32(a_full + as));
                }
                if (j == 0) TG_STAMP(3, it);
            }
            if (it >= TG_LAG) {
                const int ro = it - TG_LAG, ab = ro % NBT;
                if (!mbar_wait(smem_u32(acc_full + ab), (ro / NBT) & 1, abort_f, a.err, TG_WAIT_NS)) { ok = false; break; }
                if (j == 0) TG_STAMP(7, ro);
                tc_fence_after();
                int cc[CPA];
                tmem_ld_cols<CPA>(tmem + lane_base + (uint32_t)(ab * CPA), cc);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(acc_empty + ab));
                if (j == 0) TG_STAMP(8, ro);
                const int64_t u = u0 + ro;
                const int t = (int)(u / NB), b = (int)(u % NB), sl = slot_of(b);
                const uint32_t *sw = sring + ((ro % TG_NBUF) * 128 + j) * 2;
#pragma unroll
                for (int gi = 0; gi < GPB; gi++) {
                    const uint32_t word = sw[gi >> 1];
                    const float d = __half2float(__ushort_as_half((unsigned short)(word >> ((gi & 1) * 16))));
#pragma unroll
                    for (int m = 0; m < 2; m++) {
                        const int s01 = cc[gi * 8 + 3 * m] + (cc[gi * 8 + 3 * m + 1] << 8);
                        const float f = fmaf((float)cc[gi * 8 + 3 * m + 2], 65536.0f, (float)s01) -
                                        8.0f * (float)zsum[(sl * GPB + gi) * 2 + m];
                        acc[m] = fmaf(d, f, acc[m]);
                    }
                }
                if (b == NB - 1 || ro == n - 1) {
                    // ---- this CTA's part of tile t is complete
                    const int lr = t * TG_ROWS + j;
                    const bool row_ok = lr < p.N;
                    const int64_t tu0 = (int64_t)t * NB, tu1 = tu0 + NB;
                    float y[2];
                    if (tu0 >= u0 && tu1 <= u1) {
#pragma unroll
                        for (int m = 0; m < 2; m++) y[m] = acc[m] * tok[m] * tok[2 + m];
                        tg_epilogue(p, lr, row_ok, y);
                    } else {
                        const int cf = tg_owner(tu0, U, C), parts = tg_owner(tu1 - 1, U, C) - cf + 1;
                        float *pbase = a.partials + (size_t)t * a.max_parts * 256;
                        float *mine = pbase + (size_t)(c - cf) * 256;
                        mine[j] = acc[0];
                        mine[128 + j] = acc[1];
                        __threadfence();
                        asm volatile("bar.sync 1, 128;" ::: "memory");
                        if (j == 0) *last_f = atomicAdd(a.counters + t, 1u) == (unsigned)(parts - 1);
                        asm volatile("bar.sync 1, 128;" ::: "memory");
                        if (*last_f) {
                            __threadfence();
                            float s[2] = {0.0f, 0.0f};
                            for (int k = 0; k < parts; k++) {
                                const float *pp = pbase + (size_t)k * 256;
                                s[0] += k == c - cf ? acc[0] : __ldcg(pp + j);
                                s[1] += k == c - cf ? acc[1] : __ldcg(pp + 128 + j);
                            }
#pragma unroll
                            for (int m = 0; m < 2; m++) y[m] = s[m] * tok[m] * tok[2 + m];
                            tg_epilogue(p, lr, row_ok, y);
                            if (j == 0) a.counters[t] = 0u;
                        }
                    }
                    acc[0] = acc[1] = 0.0f;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
    }
}

// -------------------------------------------------------------------- host

struct TgPlan {
    int gpb, rs, nb_max, max_parts, tmem_cols, as, lag;
    int64_t U;
    int NB, C;
    size_t smem;
};

static int tg_env(const char *name, int dflt)
{
    const char *e = getenv(name);
    const int v = e ? atoi(e) : 0;
    return v > 0 ? v : dflt;
}

static bool tg_plan(const GemvParams &p, TgPlan *g)
{
    // tuning knobs (read once): A stages, readout lag, shared-memory budget in KB
    static const int env_as = tg_env("DU_TG_AS", 2), env_lag = tg_env("DU_TG_LAG", 3),
                     env_budget = tg_env("DU_TG_SMEM_KB", 112);
    g->as = env_as > TG_MAX_AS ? TG_MAX_AS : env_as;
    g->lag = env_lag > TG_NBUF - TG_PF - 1 ? TG_NBUF - TG_PF - 1 : env_lag;
    const size_t budget = (size_t)(env_budget > 225 ? 225 : env_budget) * 1024;
    if (p.group < 32 || (p.group & (p.group - 1)) != 0) return false;
    g->gpb = p.group >= TG_KB ? 1 : TG_KB / p.group;
    g->NB = p.K / TG_KB;
    const int tiles = (p.N + TG_ROWS - 1) / TG_ROWS;
    g->U = (int64_t)tiles * g->NB;
    g->C = num_sms();
    if (g->U < g->C) g->C = (int)g->U;
    const int64_t per = (g->U + g->C - 1) / g->C;
    g->nb_max = (int)(per < g->NB ? per : g->NB);
    // parts per tile: CTAs whose ranges meet one tile
    int mp = 1;
    for (int t = 0; t < tiles; t++) {
        const int64_t a0 = (int64_t)t * g->NB, a1 = a0 + g->NB - 1;
        const int c0 = (int)((a0 * g->C) / g->U), c1 = (int)((a1 * g->C) / g->U);
        if (c1 - c0 + 2 > mp) mp = c1 - c0 + 2;     // +1: floor rounding of the owner estimate
    }
    g->max_parts = mp;
    const size_t fixed = 1024 + (size_t)g->as * 16384 + (size_t)g->nb_max * 1024 + (size_t)TG_NBUF * 128 * 2 * 4 +
                         (size_t)g->nb_max * g->gpb * 2 * 4 + 40 * 4 + (size_t)(2 * g->as + 2 * 16) * 8 + 64;
    if (fixed + 2 * TG_RAW_STAGE > budget) return false;
    int rs = (int)((budget - fixed) / TG_RAW_STAGE);
    g->rs = rs > 12 ? 12 : rs;
    g->smem = fixed + (size_t)g->rs * TG_RAW_STAGE + (size_t)2 * g->rs * 8;
    // the unpack may run at most (A stages + accumulator units - 1) ahead of the readout
    const int nbt = TG_TMEM_COLS / (8 * g->gpb);
    if (g->lag > g->as + nbt - 1) g->lag = g->as + nbt - 1;
    g->tmem_cols = TG_TMEM_COLS;
    return true;
}

// Opt-in (DU_DECODE_GEMV=tcgen05): measured slower than the dp4a GEMV.  One thread
// issues a tcgen05.mma about every 110 cycles whatever its shape, and an N = 8 MMA
// carries only a few cycles of tensor work, so a batch-1 GEMV of this form is bound
// by MMA issue (gate|up of the 8B model: ~194 MMAs per SM, >= 11 us) before HBM.
bool tgemv_enabled()
{
    static const bool on = [] {
        const char *e = getenv("DU_DECODE_GEMV");
        return e != nullptr && strcmp(e, "tcgen05") == 0;
    }();
    return on;
}

bool tgemv_supported(int qt, const GemvParams &p)
{
    if (!tgemv_enabled() || qt != Q_I4 || p.M < 1 || p.M > 2 || p.N <= 0 || (p.K % TG_KB) != 0) return false;
    if (p.epi != EPI_STORE && p.epi != EPI_RESID && p.epi != EPI_QKV && p.epi != EPI_GATEUP) return false;
    if (p.map == MAP_GATEUP && (p.N != 2 * p.map_I || (p.map_I % 64) != 0)) return false;
    if (p.map == MAP_ROPE_PAIR && ((p.map_hd != 64 && p.map_hd != 128) || (p.N % TG_ROWS) != 0)) return false;
    if ((p.ldx & 3) != 0 || (reinterpret_cast<uintptr_t>(p.x) & 15) != 0) return false;
    // the scale rows are fetched by TMA: a 16-byte multiple per row, 16-byte aligned base
    if (p.group < 32 || ((p.K / p.group) % 8) != 0 || (reinterpret_cast<uintptr_t>(p.scales) & 15) != 0)
        return false;
    if (p.gamma != nullptr && (reinterpret_cast<uintptr_t>(p.gamma) & 15) != 0) return false;
    TgPlan g;
    return tg_plan(p, &g);
}

size_t tgemv_partial_floats(const GemvParams &p)
{
    TgPlan g;
    if (!tg_plan(p, &g)) return 0;
    return (size_t)((p.N + TG_ROWS - 1) / TG_ROWS) * g.max_parts * 256;
}

typedef CUresult (*TgEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                               const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int launch_tgemv(int qt, const GemvParams &p, const GemmScratch &scr, cudaStream_t st)
{
    if (p.M <= 0 || p.N <= 0) return DU_OK;
    TgPlan g;
    if (!tgemv_supported(qt, p) || !tg_plan(p, &g)) return fail(DU_EINVAL, "tgemv: unsupported shape");
    const int tiles = (p.N + TG_ROWS - 1) / TG_ROWS;
    if ((size_t)tiles * g.max_parts * 256 > scr.partial_floats || (size_t)tiles > scr.counter_n || !scr.partials ||
        !scr.counters)
        return fail(DU_EINVAL, "tgemv: partial-sum scratch too small");
    static TgEncodeFn enc = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<TgEncodeFn>(f);
    }();
    if (!enc) return fail(DU_ECUDA, "tgemv: cuTensorMapEncodeTiled is unavailable");
    const int64_t w_rows = p.row_off + (p.map == MAP_GATEUP ? 2 * (int64_t)p.map_I : (int64_t)p.N);
    if ((reinterpret_cast<uintptr_t>(p.w) & 15) || (p.row_bytes & 15)) return fail(DU_EINVAL, "tgemv: weight alignment");
    CUtensorMap tw;
    const cuuint64_t dims[2] = {(cuuint64_t)p.row_bytes, (cuuint64_t)w_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)p.row_bytes};
    const cuuint32_t box[2] = {64u, p.map == MAP_GATEUP ? 64u : (cuuint32_t)TG_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(p.w), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DU_ECUDA, "tgemv: cuTensorMapEncodeTiled failed");
    CUtensorMap ts;       // fp16 group scales [w_rows][K / group]: boxes of 8 scales x 128 (or 64) rows
    const int NG = p.K / p.group;
    const cuuint64_t sdims[2] = {(cuuint64_t)NG, (cuuint64_t)w_rows};
    const cuuint64_t sstrides[1] = {(cuuint64_t)NG * 2};
    const cuuint32_t sbox[2] = {8u, box[1]};
    r = enc(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(p.scales), sdims, sstrides, sbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DU_ECUDA, "tgemv: cuTensorMapEncodeTiled (scales) failed");
    TgArgs a = {};
    a.p = p;
    a.C = g.C;
    a.U = g.U;
    a.NB = g.NB;
    a.gpb = g.gpb;
    a.rs = g.rs;
    a.nb_max = g.nb_max;
    a.max_parts = g.max_parts;
    a.as = g.as;
    a.lag = g.lag;
    a.tmem_cols = g.tmem_cols;
    a.partials = scr.partials;
    a.counters = scr.counters;
    a.err = scr.err;
    const void *kern = g.gpb == 1 ? (const void *)tgemv_kernel<1>
                                  : g.gpb == 2 ? (const void *)tgemv_kernel<2> : (const void *)tgemv_kernel<4>;
    int rc = ensure_func_attrs(kern, (int)g.smem);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g.C);
    cfg.blockDim = dim3(TG_THREADS);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    if (g.gpb == 1) DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, tgemv_kernel<1>, tw, ts, a));
    else if (g.gpb == 2) DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, tgemv_kernel<2>, tw, ts, a));
    else DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, tgemv_kernel<4>, tw, ts, a));
    return DU_OK;
}

}  // namespace du
