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
};

// Shared memory of one unit: K/V tiles (dynamic, 4 * FD_TILE * (HD + 8) halves) + these.
template <int HD>
struct __align__(16) FdShared {     // qs is read as float4
    float qs[FD_MAXG][HD];
    float ps[FD_TILE][FD_MAXG];              // scores, then probabilities
    float m[FD_MAXG], l[FD_MAXG], alpha[FD_MAXG];
    float w[FD_MAXG][FD_MAXSPLIT], inv[FD_MAXG];
    unsigned last;
};

__device__ __forceinline__ void fd_cp_async16(void *smem, const void *gmem, bool valid)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void fd_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void fd_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Positions of unit (row, kv head, split).
struct FdGeom {
    int kv_len, ns_act, start, end, ntiles;
    const __half *kbase, *vbase;
};

template <int HD>
__device__ __forceinline__ FdGeom fd_geom(const FdParams &p, int row, int kvh, int split, int nsplit)
{
    FdGeom g;
    const int seq = p.seq_of ? p.seq_of[row] : row;
    g.kv_len = p.kv_len[row] + p.kv_len_add;
    // splits actually used for this length: at least one tile each
    g.ns_act = max(1, min(nsplit, (g.kv_len + FD_TILE - 1) / FD_TILE));
    int chunk = (g.kv_len + g.ns_act - 1) / g.ns_act;
    chunk = (chunk + FD_TILE - 1) & ~(FD_TILE - 1);
    g.start = split * chunk;
    g.end = split < g.ns_act ? min(g.start + chunk, g.kv_len) : g.start;
    g.ntiles = g.end > g.start ? (g.end - g.start + FD_TILE - 1) / FD_TILE : 0;
    g.kbase = p.k_cache + ((size_t)seq * p.cap * p.hkv + kvh) * HD;
    g.vbase = p.v_cache + ((size_t)seq * p.cap * p.hkv + kvh) * HD;
    return g;
}

// cp.async of the K/V rows of tile t at positions [lo, hi) into buffer buf
// (rows past the unit's end are zero-filled); one commit group.
template <int HD, int NT>
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

// Loads, ahead of the producer of this step's K/V rows, the rows of tile 0 that
// earlier steps wrote (positions below kv_len - new_rows).  The unit is then
// run with pre_new = new_rows.
template <int HD, int NT>
__device__ __forceinline__ void fd_prefetch(const FdParams &p, int row, int kvh, int split, int nsplit, int new_rows,
                                            unsigned char *tiles)
{
    const FdGeom g = fd_geom<HD>(p, row, kvh, split, nsplit);
    if (g.ntiles > 0) fd_load_rows<HD, NT>(p, g, 0, 0, g.start, g.kv_len - new_rows, tiles);
}

// Processes unit (row, kvh, split) of a launch with `nsplit` splits per
// (row, kv head).  The CTA that finishes the last split of a (row, kv head)
// merges all splits into p.out.  All NT threads must call it.  pre_new < 0:
// nothing was prefetched; else fd_prefetch(..., new_rows = pre_new) ran and
// only tile 0's rows from kv_len - pre_new on are loaded here.
template <int HD, int NT>
__device__ void fd_unit(const FdParams &p, int G, int row, int kvh, int split, int nsplit, unsigned char *tiles,
                        FdShared<HD> &sh, int pre_new = -1)
{
    constexpr int LDS = HD + 8;               // padded row (halves): conflict-free 16 B reads
    constexpr int NW = NT / 32;
    constexpr size_t TILE_BYTES = 4 * FD_TILE * LDS * 2;
    auto Ks = reinterpret_cast<__half (*)[FD_TILE][LDS]>(tiles);
    auto Vs = reinterpret_cast<__half (*)[FD_TILE][LDS]>(tiles + 2 * FD_TILE * LDS * 2);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const FdGeom geo = fd_geom<HD>(p, row, kvh, split, nsplit);
    const int ns_act = geo.ns_act, start = geo.start, end = geo.end, ntiles = geo.ntiles;

    if (ntiles > 0)
        fd_load_rows<HD, NT>(p, geo, 0, 0, pre_new < 0 ? start : geo.kv_len - pre_new, 0x7fffffff, tiles);
    for (int i = tid; i < G * HD; i += NT) {
        const int g = i / HD, d = i - g * HD;
        sh.qs[g][d] = p.q[((size_t)row * p.hq + kvh * G + g) * HD + d] * p.scale;
    }
    if (tid < G) { sh.m[tid] = FD_NEG; sh.l[tid] = 0.0f; }

    // PV ownership: dim pair dp, heads g = hb, hb + HSTEP, ...
    constexpr int NDP = HD / 2;
    constexpr int HSTEP = NT / NDP;
    constexpr int HPT = (FD_MAXG + HSTEP - 1) / HSTEP;
    const int dp = tid % NDP, hb = tid / NDP;
    float acc[HPT][2];
#pragma unroll
    for (int i = 0; i < HPT; i++) acc[i][0] = acc[i][1] = 0.0f;

    // QK ownership: position j = tid % 64, heads g = qb, qb + QSTEP, ...
    constexpr int QSTEP = NT / FD_TILE;
    constexpr int QHPT = (FD_MAXG + QSTEP - 1) / QSTEP;
    const int qj = tid % FD_TILE, qb = tid / FD_TILE;
    __syncthreads();

    for (int t = 0; t < ntiles; t++) {
        const int buf = t & 1;
        if (t + 1 < ntiles) { fd_load_rows<HD, NT>(p, geo, t + 1, buf ^ 1, 0, 0x7fffffff, tiles); fd_cp_wait<1>(); }
        else { fd_cp_wait<0>(); }
        __syncthreads();

        // ---- scores
        {
            float s[QHPT];
#pragma unroll
            for (int i = 0; i < QHPT; i++) s[i] = 0.0f;
            const __half *kr = &Ks[buf][qj][0];
#pragma unroll 4
            for (int d = 0; d < HD; d += 8) {
                const uint4 raw = *reinterpret_cast<const uint4 *>(kr + d);
                const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
                const float2 k0 = __half22float2(h[0]), k1 = __half22float2(h[1]);
                const float2 k2 = __half22float2(h[2]), k3 = __half22float2(h[3]);
#pragma unroll
                for (int i = 0; i < QHPT; i++) {
                    const int g = qb + QSTEP * i;
                    if (g < G) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&sh.qs[g][d]);
                        const float4 qc = *reinterpret_cast<const float4 *>(&sh.qs[g][d + 4]);
                        float a = s[i];
                        a = fmaf(qa.x, k0.x, a); a = fmaf(qa.y, k0.y, a);
                        a = fmaf(qa.z, k1.x, a); a = fmaf(qa.w, k1.y, a);
                        a = fmaf(qc.x, k2.x, a); a = fmaf(qc.y, k2.y, a);
                        a = fmaf(qc.z, k3.x, a); a = fmaf(qc.w, k3.y, a);
                        s[i] = a;
                    }
                }
            }
            const bool valid = start + t * FD_TILE + qj < end;
#pragma unroll
            for (int i = 0; i < QHPT; i++) {
                const int g = qb + QSTEP * i;
                if (g < G) sh.ps[qj][g] = valid ? s[i] : FD_NEG;
            }
        }
        __syncthreads();

        // ---- online softmax, one warp per head
        for (int g = warp; g < G; g += NW) {
            const float a = sh.ps[2 * lane][g], b = sh.ps[2 * lane + 1][g];
            const float mt = warp_max(fmaxf(a, b));
            const float m_old = sh.m[g];
            const float m_new = fmaxf(m_old, mt);
            const float pa = expf(a - m_new), pb = expf(b - m_new);
            sh.ps[2 * lane][g] = pa;
            sh.ps[2 * lane + 1][g] = pb;
            const float ts = warp_sum(pa + pb);
            if (lane == 0) {
                const float alpha = expf(m_old - m_new);
                sh.alpha[g] = alpha;
                sh.l[g] = sh.l[g] * alpha + ts;
                sh.m[g] = m_new;
            }
        }
        __syncthreads();

        // ---- P.V
#pragma unroll
        for (int i = 0; i < HPT; i++) {
            const int g = hb + i * HSTEP;
            if (g < G) {
                const float al = sh.alpha[g];
                acc[i][0] *= al;
                acc[i][1] *= al;
            }
        }
#pragma unroll 8
        for (int j = 0; j < FD_TILE; j++) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&Vs[buf][j][2 * dp]));
#pragma unroll
            for (int i = 0; i < HPT; i++) {
                const int g = hb + i * HSTEP;
                if (g < G) {
                    const float pj = sh.ps[j][g];
                    acc[i][0] = fmaf(pj, v.x, acc[i][0]);
                    acc[i][1] = fmaf(pj, v.y, acc[i][1]);
                }
            }
        }
        __syncthreads();   // ps / buffers are rewritten next tile
    }

    // ---- this split's partial state
    const size_t rk = (size_t)row * p.hkv + kvh;
    float *po = p.part_o + (rk * nsplit + split) * G * HD;
#pragma unroll
    for (int i = 0; i < HPT; i++) {
        const int g = hb + i * HSTEP;
        if (g < G) {
            po[g * HD + 2 * dp] = acc[i][0];
            po[g * HD + 2 * dp + 1] = acc[i][1];
        }
    }
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
