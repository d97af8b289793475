// attn_impl.cuh -- one split-K flash-decode work unit (query row, kv head, KV
// split) processed by all NT threads of a CTA; shared by the standalone
// kernel (attention.cu, NT = 128) and the persistent decode-step kernel
// (decode_step.cu, NT = 256).  Design notes in attention.cu.
#pragma once

#include "common.cuh"

namespace du {

constexpr int FD_TILE = 64;
constexpr float FD_NEG = -3.0e38f;
constexpr int FD_MAXSPLIT = 128;          // gridDim.x upper bound (combine weights live in smem)
constexpr int FD_MAXG = 8;                // GQA group upper bound

struct FdParams {
    const float *q;              // [nq][hq][HD] fp32 (roped, unscaled)
    const __half *k_cache;       // [nseq][cap][hkv][HD]
    const __half *v_cache;
    const int *seq_of;           // [nq] sequence of each query row (nullptr: row -> row)
    const int *kv_len;           // [nq] valid positions for each query row
    int kv_len_add;              // added to kv_len[row] (decode passes cache_len, +1)
    int hq, hkv, cap;
    float scale;
    float *out;                  // [nq][hq][HD]
    float *part_o;               // [nq][hkv][nsplit][G][HD]
    float *part_ml;              // [nq][hkv][nsplit][G][2]
    unsigned *counters;          // [nq][hkv], zero between launches
    // INT8 cache (the KV8 instantiations): uint8 [nseq][cap][hkv][HD] and per-(position,
    // kv head) words (fp16 scale | fp16 zero point << 16) [nseq][cap][hkv]
    const uint8_t *k8, *v8;
    const uint32_t *ksz, *vsz;
    int window;                  // > 0: a query at position kv_len - 1 sees positions >= kv_len - 1 - window
    // O projection fused after the cluster combine (the OF instantiations; one query row):
    // resid[n] += sum over kv heads of W_o[n][kvh's G*HD columns] . att(kvh)
    const uint8_t *wo;           // INT4 nibbles or INT8 bytes, row-major [H][hq * HD]
    const __half *wo_scales;     // INT4 [H][hq * HD / group], INT8 [H]
    int wo_quant, wo_group, H;
    float *resid;                // [H]
    float *opart;                // [hkv][H] per-kv-head partial sums
    unsigned *ocnt;              // [C] arrivals per row slice, zero between launches
    int *err;                    // a bounded wait that gave up
};

// Shared memory of one unit: K/V tiles (dynamic, 4 * FD_TILE * (HD + 8) halves) + these.
template <int HD>
struct __align__(16) FdShared {     // qs is read as float4
    float qs[FD_MAXG][HD];
    float ps[FD_TILE][FD_MAXG];              // scores, then probabilities
    float m[FD_MAXG], l[FD_MAXG], alpha[FD_MAXG];
    float w[FD_MAXG][FD_MAXSPLIT], inv[FD_MAXG];
    unsigned last;
    // INT8 cache, per tile: K scales, V scales / the tile's largest V scale, that largest scale
    float kv8_ks[FD_TILE], kv8_vs[FD_TILE], kv8_vm;
};

// 8 INT8 cache bytes -> 8 halves (q - zp), exact: 0x64 as the high byte makes
// the half 1024 + q, and 1024 + zp (an integer <= 1279) is exact too.
__device__ __forceinline__ uint4 fd_q8_to_h8(uint2 r, __half2 base)
{
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t w = i < 2 ? r.x : r.y;
        const uint32_t u = __byte_perm(w, 0x64646464u, (i & 1) ? 0x4342u : 0x4140u);
        __half2 h = __hsub2(*reinterpret_cast<const __half2 *>(&u), base);
        o[i] = *reinterpret_cast<uint32_t *>(&h);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void fd_cp_async16(void *smem, const void *gmem, bool valid)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void fd_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void fd_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// warp-wide 8x8 b16 matrix loads (rows 16-byte aligned) and the f16 tensor-core MMA
__device__ __forceinline__ void fd_ldsm_x4(uint32_t (&r)[4], const void *p)
{
    const unsigned a = (unsigned)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void fd_ldsm_x2(uint32_t &r0, uint32_t &r1, const void *p)
{
    const unsigned a = (unsigned)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(a));
}
__device__ __forceinline__ void fd_ldsm_x4_t(uint32_t (&r)[4], const void *p)
{
    const unsigned a = (unsigned)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void fd_ldsm_x2_t(uint32_t &r0, uint32_t &r1, const void *p)
{
    const unsigned a = (unsigned)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(a));
}
// c += a (16x16, row) * b (16x8, col), f16 inputs, f32 accumulators
__device__ __forceinline__ void fd_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Bytes after the K/V tiles that the tensor-core unit (TO_SMEM, 256 threads) also
// uses: q and P as fp16 hi + lo parts, [2][16][HD + 8] and [2][16][FD_TILE + 8],
// and the scores head-major, [FD_MAXG][FD_TILE + 4] fp32.
template <int HD>
__host__ __device__ constexpr size_t fd_mma_extra_bytes()
{
    return (size_t)2 * 16 * (HD + 8) * 2 + (size_t)2 * 16 * (FD_TILE + 8) * 2 + (size_t)FD_MAXG * (FD_TILE + 4) * 4;
}

// INT8 cache: raw rows and their scale / zero-point words, two tile buffers each,
// after the tensor-core scratch: K [2][FD_TILE][HD] bytes, V the same, then the
// K and V words [2][FD_TILE] each.
template <int HD>
__host__ __device__ constexpr size_t fd_kv8_off()
{
    return (size_t)4 * FD_TILE * (HD + 8) * 2 + fd_mma_extra_bytes<HD>();
}
template <int HD>
__host__ __device__ constexpr size_t fd_kv8_bytes()
{
    return (size_t)4 * FD_TILE * HD + (size_t)4 * FD_TILE * 4;
}

// Positions of unit (row, kv head, split).
struct FdGeom {
    int kv_len, ns_act, start, end, ntiles;
    const __half *kbase, *vbase;
    const uint8_t *k8base, *v8base;       // INT8 cache
    const uint32_t *kzbase, *vzbase;
};

// EVEN: the kv_len's tiles are dealt evenly over the nsplit splits (cluster
// combine); otherwise each active split takes the same whole number of tiles and
// the active splits are counted in ns_act (global combine).
template <int HD, bool EVEN = false>
__device__ __forceinline__ FdGeom fd_geom(const FdParams &p, int row, int kvh, int split, int nsplit)
{
    FdGeom g;
    const int seq = p.seq_of ? p.seq_of[row] : row;
    g.kv_len = p.kv_len[row] + p.kv_len_add;
    // sliding window (G3CS:673-686): the query (position kv_len - 1) sees lo .. kv_len - 1
    const int lo = (p.window > 0 && g.kv_len - 1 > p.window) ? g.kv_len - 1 - p.window : 0;
    const int T = (g.kv_len - lo + FD_TILE - 1) / FD_TILE;
    if (EVEN) {
        g.ns_act = nsplit;
        g.start = lo + (int)(((int64_t)split * T) / nsplit) * FD_TILE;
        g.end = min(lo + (int)(((int64_t)(split + 1) * T) / nsplit) * FD_TILE, g.kv_len);
        if (g.end < g.start) g.end = g.start;
    } else {
        // splits actually used for this length: at least one tile each
        g.ns_act = max(1, min(nsplit, T));
        int chunk = (g.kv_len - lo + g.ns_act - 1) / g.ns_act;
        chunk = (chunk + FD_TILE - 1) & ~(FD_TILE - 1);
        g.start = lo + split * chunk;
        g.end = split < g.ns_act ? min(g.start + chunk, g.kv_len) : g.start;
    }
    g.ntiles = g.end > g.start ? (g.end - g.start + FD_TILE - 1) / FD_TILE : 0;
    const size_t row0 = (size_t)seq * p.cap * p.hkv + kvh;
    g.kbase = p.k_cache + row0 * HD;
    g.vbase = p.v_cache + row0 * HD;
    g.k8base = p.k8 + row0 * HD;
    g.v8base = p.v8 + row0 * HD;
    g.kzbase = p.ksz + row0;
    g.vzbase = p.vsz + row0;
    return g;
}

__device__ __forceinline__ void fd_cp_async4(void *smem, const void *gmem, bool valid)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}

// cp.async of the K/V rows of tile t at positions [lo, hi) into buffer buf
// (rows past the unit's end are zero-filled); one commit group.  KV8: the raw
// bytes and the scale / zero-point words into the INT8 staging buffers.
template <int HD, int NT, bool KV8 = false>
__device__ __forceinline__ void fd_load_rows(const FdParams &p, const FdGeom &g, int t, int buf, int lo, int hi,
                                             unsigned char *tiles)
{
    constexpr int LDS = HD + 8;
    constexpr int CPR = HD / 8;
    auto Ks = reinterpret_cast<__half (*)[FD_TILE][LDS]>(tiles);
    auto Vs = reinterpret_cast<__half (*)[FD_TILE][LDS]>(tiles + 2 * FD_TILE * LDS * 2);
    const size_t pos_stride = (size_t)p.hkv * HD;
    const int p0 = g.start + t * FD_TILE;
    lo = max(lo, p0);
    hi = min(hi, p0 + FD_TILE);
    if constexpr (KV8) {
        unsigned char *raw = tiles + fd_kv8_off<HD>();
        auto Kr = reinterpret_cast<uint8_t (*)[FD_TILE][HD]>(raw);
        auto Vr = reinterpret_cast<uint8_t (*)[FD_TILE][HD]>(raw + 2 * FD_TILE * HD);
        auto Kz = reinterpret_cast<uint32_t (*)[FD_TILE]>(raw + 4 * FD_TILE * HD);
        auto Vz = reinterpret_cast<uint32_t (*)[FD_TILE]>(raw + 4 * FD_TILE * HD + 2 * FD_TILE * 4);
        constexpr int CB = HD / 16;            // 16-byte chunks per INT8 row
        for (int i = threadIdx.x; i < (hi - lo) * CB; i += NT) {
            const int j = lo - p0 + i / CB, c = i % CB;
            const int pos = p0 + j;
            const bool ok = pos < g.end;
            const size_t off = (size_t)(ok ? pos : 0) * pos_stride + c * 16;
            fd_cp_async16(&Kr[buf][j][c * 16], g.k8base + off, ok);
            fd_cp_async16(&Vr[buf][j][c * 16], g.v8base + off, ok);
        }
        for (int i = threadIdx.x; i < hi - lo; i += NT) {
            const int j = lo - p0 + i, pos = p0 + j;
            const bool ok = pos < g.end;
            const size_t off = (size_t)(ok ? pos : 0) * p.hkv;
            fd_cp_async4(&Kz[buf][j], g.kzbase + off, ok);
            fd_cp_async4(&Vz[buf][j], g.vzbase + off, ok);
        }
        fd_cp_commit();
        return;
    }
    for (int i = threadIdx.x; i < (hi - lo) * CPR; i += NT) {
        const int j = lo - p0 + i / CPR, c = i % CPR;
        const int pos = p0 + j;
        const bool ok = pos < g.end;
        const size_t off = (size_t)(ok ? pos : 0) * pos_stride + c * 8;
        fd_cp_async16(&Ks[buf][j][c * 8], g.kbase + off, ok);
        fd_cp_async16(&Vs[buf][j][c * 8], g.vbase + off, ok);
    }
    fd_cp_commit();
}

// Loads, ahead of the producer of this step's K/V rows, the rows of tiles 0 and
// 1 (the two tile buffers) that earlier steps wrote: positions below kv_len -
// new_rows; two commit groups.  The unit is then run with pre_new = new_rows.
template <int HD, int NT, bool EVEN = false, bool KV8 = false>
__device__ __forceinline__ void fd_prefetch(const FdParams &p, int row, int kvh, int split, int nsplit, int new_rows,
                                            unsigned char *tiles)
{
    const FdGeom g = fd_geom<HD, EVEN>(p, row, kvh, split, nsplit);
    if (g.ntiles > 0) fd_load_rows<HD, NT, KV8>(p, g, 0, 0, g.start, g.kv_len - new_rows, tiles);
    if (g.ntiles > 1) fd_load_rows<HD, NT, KV8>(p, g, 1, 1, g.start, g.kv_len - new_rows, tiles);
}

// Processes unit (row, kvh, split) of a launch with `nsplit` splits per
// (row, kv head).  The CTA that finishes the last split of a (row, kv head)
// merges all splits into p.out.  All NT threads must call it.  pre_new < 0:
// nothing was prefetched; else fd_prefetch(..., new_rows = pre_new) ran and
// only the rows of tiles 0 and 1 from kv_len - pre_new on are loaded here.
//
// TO_SMEM: instead of publishing to p.part_o / p.part_ml and combining through
// global memory, leave this split's unnormalised state in shared memory --
// acc as float [G][HD] at `tiles`, (m, l) in sh.m / sh.l -- for a cluster
// combine (flash_decode_cluster_kernel).
//
// With TO_SMEM and 256 threads the tile math runs on tensor cores
// (mma.sync m16n8k16, fp32 accumulators): q and the probabilities are split
// into fp16 hi + lo parts (x = hi + lo to ~22 bits) and multiplied against the
// exact fp16 K / V, one MMA per part; rows g >= G of the 16-row A operands are
// zero.  Needs fd_mma_extra_bytes<HD>() of shared memory after the tiles.
//
// KV8 (INT8 cache; tensor-core path only): each tile's raw bytes become (q - zp)
// halves in the tile buffers, exact.  Scores are q . (k_q - zp) times the row's
// K scale.  The probabilities enter P.V times (V scale / largest V scale of the
// tile); the accumulator is kept in units of that largest scale and rescaled
// with the softmax factor from tile to tile.
template <int HD, int NT, bool TO_SMEM = false, bool KV8 = false>
__device__ __forceinline__ void fd_unit(const FdParams &p, int G, int row, int kvh, int split, int nsplit, unsigned char *tiles,
                        FdShared<HD> &sh, int pre_new = -1)
{
    static_assert(!KV8 || (TO_SMEM && NT == 256), "the INT8 cache runs on the tensor-core path");
    static_assert(FD_TILE == 64, "two positions per lane of one warp");
    constexpr int LDS = HD + 8;               // padded row (halves): conflict-free 16 B reads
    constexpr int NW = NT / 32;
    constexpr size_t TILE_BYTES = 4 * FD_TILE * LDS * 2;
    constexpr bool MMA = TO_SMEM && NT == 256;
    constexpr int QLD = HD + 8, PLD = FD_TILE + 8;
    auto qh = reinterpret_cast<__half (*)[16][QLD]>(tiles + TILE_BYTES);                     // [2][16][QLD]
    auto ph = reinterpret_cast<__half (*)[16][PLD]>(tiles + TILE_BYTES + (size_t)2 * 16 * QLD * 2);   // [2][16][PLD]
    auto pst = reinterpret_cast<float (*)[FD_TILE + 4]>(tiles + TILE_BYTES + (size_t)2 * 16 * QLD * 2 +
                                                        (size_t)2 * 16 * PLD * 2);              // [FD_MAXG][FD_TILE + 4]
    auto Ks = reinterpret_cast<__half (*)[FD_TILE][LDS]>(tiles);
    auto Vs = reinterpret_cast<__half (*)[FD_TILE][LDS]>(tiles + 2 * FD_TILE * LDS * 2);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const FdGeom geo = fd_geom<HD, TO_SMEM>(p, row, kvh, split, nsplit);
    const int ns_act = geo.ns_act, start = geo.start, end = geo.end, ntiles = geo.ntiles;

    if (ntiles > 0)
        fd_load_rows<HD, NT, KV8>(p, geo, 0, 0, pre_new < 0 ? start : geo.kv_len - pre_new, 0x7fffffff, tiles);
    float vm_prev = 1.0f;        // KV8: the accumulator's unit (largest V scale of the previous tile)
    if (MMA) {
        // q rows g < G as hi + lo halves (rows G..15 zero); all loads issued before the stores
        constexpr int QV = (16 * HD / 4 + NT - 1) / NT;     // float4 per thread
        float4 qv[QV];
#pragma unroll
        for (int k = 0; k < QV; k++) {
            const int i4 = tid + k * NT, g = i4 * 4 / HD, d = i4 * 4 - g * HD;
            qv[k] = g < G && i4 < 16 * HD / 4
                        ? *reinterpret_cast<const float4 *>(p.q + ((size_t)row * p.hq + kvh * G + g) * HD + d)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < QV; k++) {
            const int i4 = tid + k * NT, g = i4 * 4 / HD, d = i4 * 4 - g * HD;
            if (i4 >= 16 * HD / 4) break;
            const float q[4] = {qv[k].x * p.scale, qv[k].y * p.scale, qv[k].z * p.scale, qv[k].w * p.scale};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const __half h = __float2half_rn(q[e]);
                qh[0][g][d + e] = h;
                qh[1][g][d + e] = __float2half_rn(q[e] - __half2float(h));
            }
        }
        for (int i = tid; i < 2 * 16 * PLD / 8; i += NT) reinterpret_cast<uint4 *>(&ph[0][0][0])[i] = make_uint4(0u, 0u, 0u, 0u);
    } else {
        for (int i = tid; i < G * HD; i += NT) {
            const int g = i / HD, d = i - g * HD;
            sh.qs[g][d] = p.q[((size_t)row * p.hq + kvh * G + g) * HD + d] * p.scale;
        }
    }
    if (tid < G) { sh.m[tid] = FD_NEG; sh.l[tid] = 0.0f; }

    // QK ownership: position qj, dim slice qsl (16-byte chunks qsl, qsl + DQ, ...),
    // every head; the DQ slices of a position sit on consecutive lanes.
    constexpr int DQ = NT / FD_TILE;
    constexpr int CH = HD / 8;                 // 16-byte chunks per K row
    const int qj = tid / DQ, qsl = tid % DQ;
    // PV ownership: dim pair dp, every head, positions pq, pq + PQ, ...; the PQ
    // partial sums are added once after the last tile.
    constexpr int NDP = HD / 2;
    constexpr int PQ = NT / NDP;
    const int dp = tid % NDP, pq = tid / NDP;
    float acc[FD_MAXG][2];
#pragma unroll
    for (int g = 0; g < FD_MAXG; g++) acc[g][0] = acc[g][1] = 0.0f;
    // MMA ownership: scores, positions [8 warp, 8 warp + 8); P.V, dims [warp HD/8, (warp + 1) HD/8)
    constexpr int NTL = HD / 64;               // 8-dim n-tiles per warp in P.V
    float oc[NTL][4];
#pragma unroll
    for (int n = 0; n < NTL; n++) oc[n][0] = oc[n][1] = oc[n][2] = oc[n][3] = 0.0f;
    __syncthreads();

    for (int t = 0; t < ntiles; t++) {
        const int buf = t & 1;
        if (t + 1 < ntiles) {
            // tile 1's older rows came with the prefetch
            fd_load_rows<HD, NT, KV8>(p, geo, t + 1, buf ^ 1, (t == 0 && pre_new >= 0) ? geo.kv_len - pre_new : 0,
                                      0x7fffffff, tiles);
            fd_cp_wait<1>();
        } else {
            fd_cp_wait<0>();
        }
        __syncthreads();
        float vm_ratio = 1.0f;
        if constexpr (KV8) {
            unsigned char *raw = tiles + fd_kv8_off<HD>();
            auto Kr = reinterpret_cast<const uint8_t (*)[FD_TILE][HD]>(raw);
            auto Vr = reinterpret_cast<const uint8_t (*)[FD_TILE][HD]>(raw + 2 * FD_TILE * HD);
            auto Kz = reinterpret_cast<const uint32_t (*)[FD_TILE]>(raw + 4 * FD_TILE * HD);
            auto Vz = reinterpret_cast<const uint32_t (*)[FD_TILE]>(raw + 4 * FD_TILE * HD + 2 * FD_TILE * 4);
            for (int i = tid; i < FD_TILE * HD / 8; i += NT) {
                const int j = i / (HD / 8), c = i - j * (HD / 8);
                const float kz = __half2float(__ushort_as_half((unsigned short)(Kz[buf][j] >> 16)));
                const float vz = __half2float(__ushort_as_half((unsigned short)(Vz[buf][j] >> 16)));
                *reinterpret_cast<uint4 *>(&Ks[buf][j][c * 8]) =
                    fd_q8_to_h8(*reinterpret_cast<const uint2 *>(&Kr[buf][j][c * 8]), __float2half2_rn(1024.0f + kz));
                *reinterpret_cast<uint4 *>(&Vs[buf][j][c * 8]) =
                    fd_q8_to_h8(*reinterpret_cast<const uint2 *>(&Vr[buf][j][c * 8]), __float2half2_rn(1024.0f + vz));
            }
            if (warp == 0) {
                const float va = __half2float(__ushort_as_half((unsigned short)(Vz[buf][lane] & 0xFFFFu)));
                const float vb = __half2float(__ushort_as_half((unsigned short)(Vz[buf][lane + 32] & 0xFFFFu)));
                float vm = warp_max(fmaxf(va, vb));
                if (!(vm > 0.0f)) vm = 1.0f;     // no V scale above zero: every V value of the tile is 0
                sh.kv8_ks[lane] = __half2float(__ushort_as_half((unsigned short)(Kz[buf][lane] & 0xFFFFu)));
                sh.kv8_ks[lane + 32] = __half2float(__ushort_as_half((unsigned short)(Kz[buf][lane + 32] & 0xFFFFu)));
                sh.kv8_vs[lane] = va / vm;
                sh.kv8_vs[lane + 32] = vb / vm;
                if (lane == 0) sh.kv8_vm = vm;
            }
            __syncthreads();
            const float vm = sh.kv8_vm;
            vm_ratio = vm_prev / vm;
            vm_prev = vm;
        }

        // ---- scores: each K chunk is read once and used for every head
        if (MMA) {
            const int n0 = warp * 8;
            float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int ks = 0; ks < HD / 16; ks++) {
                uint32_t b0, b1;
                fd_ldsm_x2(b0, b1, &Ks[buf][n0 + (lane & 7)][ks * 16 + ((lane >> 3) & 1) * 8]);
#pragma unroll
                for (int hl = 0; hl < 2; hl++) {
                    uint32_t a[4];
                    fd_ldsm_x4(a, &qh[hl][lane & 15][ks * 16 + (lane >> 4) * 8]);
                    fd_mma(c, a, b0, b1);
                }
            }
            const int g = lane >> 2, j = n0 + (lane & 3) * 2;
            if (KV8) {
                c[0] *= sh.kv8_ks[j];
                c[1] *= sh.kv8_ks[j + 1];
            }
            if (g < G) {
                const int pos = start + t * FD_TILE + j;
                *reinterpret_cast<float2 *>(&pst[g][j]) = make_float2(pos < end ? c[0] : FD_NEG, pos + 1 < end ? c[1] : FD_NEG);
            }
        } else {
            float s[FD_MAXG];
#pragma unroll
            for (int g = 0; g < FD_MAXG; g++) s[g] = 0.0f;
            const __half *kr = &Ks[buf][qj][0];
#pragma unroll
            for (int c = qsl; c < CH; c += DQ) {
                const uint4 raw = *reinterpret_cast<const uint4 *>(kr + c * 8);
                const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
                const float2 k0 = __half22float2(h[0]), k1 = __half22float2(h[1]);
                const float2 k2 = __half22float2(h[2]), k3 = __half22float2(h[3]);
#pragma unroll
                for (int g = 0; g < FD_MAXG; g++) {
                    if (g < G) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&sh.qs[g][c * 8]);
                        const float4 qc = *reinterpret_cast<const float4 *>(&sh.qs[g][c * 8 + 4]);
                        float a = s[g];
                        a = fmaf(qa.x, k0.x, a); a = fmaf(qa.y, k0.y, a);
                        a = fmaf(qa.z, k1.x, a); a = fmaf(qa.w, k1.y, a);
                        a = fmaf(qc.x, k2.x, a); a = fmaf(qc.y, k2.y, a);
                        a = fmaf(qc.z, k3.x, a); a = fmaf(qc.w, k3.y, a);
                        s[g] = a;
                    }
                }
            }
#pragma unroll
            for (int o = 1; o < DQ; o <<= 1)
#pragma unroll
                for (int g = 0; g < FD_MAXG; g++)
                    if (g < G) s[g] += __shfl_xor_sync(0xffffffffu, s[g], o);
            if (qsl == 0) {
                const bool valid = start + t * FD_TILE + qj < end;
#pragma unroll
                for (int g = 0; g < FD_MAXG; g++)
                    if (g < G) sh.ps[qj][g] = valid ? s[g] : FD_NEG;
            }
        }
        __syncthreads();

        // ---- online softmax, one warp per head
        for (int g = warp; g < G; g += NW) {
            float a, b;
            if (MMA) {              // head-major scores: one conflict-free 8-byte read per lane
                const float2 ab = *reinterpret_cast<const float2 *>(&pst[g][2 * lane]);
                a = ab.x;
                b = ab.y;
            } else {
                a = sh.ps[2 * lane][g];
                b = sh.ps[2 * lane + 1][g];
            }
            const float mt = warp_max(fmaxf(a, b));
            const float m_old = sh.m[g];
            const float m_new = fmaxf(m_old, mt);
            const float pa = expf(a - m_new), pb = expf(b - m_new);
            if (MMA) {
                const float qa = KV8 ? pa * sh.kv8_vs[2 * lane] : pa, qb = KV8 ? pb * sh.kv8_vs[2 * lane + 1] : pb;
                const __half ha = __float2half_rn(qa), hb = __float2half_rn(qb);
                *reinterpret_cast<__half2 *>(&ph[0][g][2 * lane]) = __halves2half2(ha, hb);
                *reinterpret_cast<__half2 *>(&ph[1][g][2 * lane]) =
                    __halves2half2(__float2half_rn(qa - __half2float(ha)), __float2half_rn(qb - __half2float(hb)));
            } else {
                sh.ps[2 * lane][g] = pa;
                sh.ps[2 * lane + 1][g] = pb;
            }
            const float ts = warp_sum(pa + pb);
            if (lane == 0) {
                const float alpha = expf(m_old - m_new);
                sh.alpha[g] = alpha;
                sh.l[g] = sh.l[g] * alpha + ts;
                sh.m[g] = m_new;
            }
        }
        __syncthreads();

        // ---- P.V over this thread's positions, every head
        if (MMA) {
            const int g = lane >> 2;
            const float al = (g < G ? sh.alpha[g] : 1.0f) * vm_ratio;
#pragma unroll
            for (int n = 0; n < NTL; n++) { oc[n][0] *= al; oc[n][1] *= al; }
            const int d0 = warp * (HD / 8);
#pragma unroll
            for (int ks = 0; ks < FD_TILE / 16; ks++) {
                const int pos = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                uint32_t b[2 * NTL > 4 ? 2 * NTL : 4];
                if (NTL == 1) {
                    fd_ldsm_x2_t(b[0], b[1], &Vs[buf][pos][d0]);
                } else {
#pragma unroll
                    for (int n2 = 0; n2 < NTL / 2; n2++) {     // two 8-dim n-tiles per transposed x4 load
                        uint32_t r[4];
                        fd_ldsm_x4_t(r, &Vs[buf][pos][d0 + n2 * 16 + (lane >> 4) * 8]);
                        b[4 * n2] = r[0]; b[4 * n2 + 1] = r[1]; b[4 * n2 + 2] = r[2]; b[4 * n2 + 3] = r[3];
                    }
                }
#pragma unroll
                for (int hl = 0; hl < 2; hl++) {
                    uint32_t a[4];
                    fd_ldsm_x4(a, &ph[hl][lane & 15][ks * 16 + (lane >> 4) * 8]);
#pragma unroll
                    for (int n = 0; n < NTL; n++) fd_mma(oc[n], a, b[2 * n], b[2 * n + 1]);
                }
            }
            __syncthreads();   // ps / buffers are rewritten next tile
            continue;
        }
#pragma unroll
        for (int g = 0; g < FD_MAXG; g++) {
            if (g < G) {
                const float al = sh.alpha[g];
                acc[g][0] *= al;
                acc[g][1] *= al;
            }
        }
#pragma unroll 4
        for (int j = pq; j < FD_TILE; j += PQ) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&Vs[buf][j][2 * dp]));
            const float4 p0 = *reinterpret_cast<const float4 *>(&sh.ps[j][0]);
            const float4 p1 = *reinterpret_cast<const float4 *>(&sh.ps[j][4]);
            const float pj[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
            for (int g = 0; g < FD_MAXG; g++) {
                if (g < G) {
                    acc[g][0] = fmaf(pj[g], v.x, acc[g][0]);
                    acc[g][1] = fmaf(pj[g], v.y, acc[g][1]);
                }
            }
        }
        __syncthreads();   // ps / buffers are rewritten next tile
    }

    // ---- this split's partial state: add the PQ position groups (fixed order)
    float *so = reinterpret_cast<float *>(tiles);           // [G][HD]; the tiles are free now
    if (MMA) {
        const int g = lane >> 2, d0 = warp * (HD / 8);
        const float unit = KV8 ? vm_prev : 1.0f;    // KV8: back from units of the last tile's V scale
        if (g < G)
#pragma unroll
            for (int n = 0; n < NTL; n++) {
                so[g * HD + d0 + n * 8 + (lane & 3) * 2] = oc[n][0] * unit;
                so[g * HD + d0 + n * 8 + (lane & 3) * 2 + 1] = oc[n][1] * unit;
            }
        __syncthreads();
        return;
    }
    float *sred = so + FD_MAXG * HD;                         // [PQ][G][HD]
#pragma unroll
    for (int g = 0; g < FD_MAXG; g++) {
        if (g < G) {
            sred[(pq * G + g) * HD + 2 * dp] = acc[g][0];
            sred[(pq * G + g) * HD + 2 * dp + 1] = acc[g][1];
        }
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += NT) {
        float v = 0.0f;
#pragma unroll
        for (int q = 0; q < PQ; q++) v += sred[q * G * HD + i];
        so[i] = v;
    }
    if (TO_SMEM) {
        __syncthreads();
        return;
    }
    const size_t rk = (size_t)row * p.hkv + kvh;
    float *po = p.part_o + (rk * nsplit + split) * G * HD;
    __syncthreads();
    for (int i = tid; i < G * HD; i += NT) po[i] = so[i];
    if (tid < G) {
        float *pm = p.part_ml + ((rk * nsplit + split) * G + tid) * 2;
        pm[0] = sh.m[tid];
        pm[1] = sh.l[tid];
    }
    // publish: the CTA's stores are ordered before thread 0's acq_rel add (bar.sync
    // then atom.acq_rel.gpu); the last CTA's add also acquires the other splits' stores
    __syncthreads();
    if (tid == 0) {
        unsigned prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&p.counters[rk]) : "memory");
        sh.last = (prev == (unsigned)nsplit - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!sh.last) return;

    // ---- last CTA of this (row, kv head): log-sum-exp combine, fixed split order
    const float *pmb = p.part_ml + rk * nsplit * G * 2;
    const float *pob = p.part_o + rk * nsplit * G * HD;
    const int per = G * HD;
    if ((size_t)ns_act * (per + 2 * G) * 4 <= TILE_BYTES) {
        // every split's (o, m, l) in one round of copies (the tiles are free now)
        float *so = reinterpret_cast<float *>(tiles);
        float *sml = so + (size_t)ns_act * per;
        for (int i = tid; i < ns_act * per / 4; i += NT) fd_cp_async16(so + 4 * i, pob + 4 * i, true);
        for (int i = tid; i < ns_act * G * 2; i += NT) sml[i] = __ldcg(pmb + i);
        fd_cp_commit();
        fd_cp_wait<0>();
        __syncthreads();
        pmb = sml;
        pob = so;
    }
    for (int g = warp; g < G; g += NW) {
        float M = FD_NEG;
        for (int s = lane; s < ns_act; s += 32) M = fmaxf(M, pmb[(s * G + g) * 2]);
        M = warp_max(M);
        float L = 0.0f;
        for (int s = lane; s < ns_act; s += 32) {
            const float w = expf(pmb[(s * G + g) * 2] - M);
            sh.w[g][s] = w;
            L = fmaf(pmb[(s * G + g) * 2 + 1], w, L);
        }
        L = warp_sum(L);
        if (lane == 0) sh.inv[g] = 1.0f / fmaxf(L, 1e-12f);
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += NT) {
        const int g = i / HD, d = i - g * HD;
        const float *po_gd = pob + g * HD + d;
        float O = 0.0f;
#pragma unroll 4
        for (int s = 0; s < ns_act; s++) O = fmaf(po_gd[(size_t)s * per], sh.w[g][s], O);
        p.out[((size_t)row * p.hq + kvh * G + g) * HD + d] = O * sh.inv[g];
    }
    if (tid == 0) p.counters[rk] = 0u;   // ready for the next launch / graph replay
    __syncthreads();
}

}  // namespace du
