// attention.cu -- split-K flash-decode over the fp16 KV cache with GQA.
//
// Replaces FlashAttention (Gemma3CS.compute:643-753).  The reference runs one
// 256-thread group per (query, q head) and re-reads every K/V row once per q
// head of a GQA group.  Here one CTA owns a (query row, kv head, KV split):
//  * the whole GQA group (G q heads) is served from one pass over K/V, so
//    each cache byte is read from HBM once;
//  * K/V tiles of 64 positions are staged in shared memory with cp.async
//    (16 B per thread, zero-filled past kv_len), double-buffered so the next
//    tile streams in while the current one is consumed;
//  * online softmax per head with the reference's rescaling recurrence
//    (m, l, alpha = exp(m_old - m_new)); the -3e38 sentinel of the reference
//    marks empty state;
//  * the KV length is split across gridDim.x CTAs so that batch-1 decode
//    fills all 148 SMs; the last CTA of each (row, kv head) to finish merges
//    the partial (m, l, acc) triples (log-sum-exp combine, fixed split order,
//    so the result does not depend on which CTA finishes last).
// kv_len is read from device memory, so one captured CUDA graph serves every
// decode step.
#include "internal.h"

namespace du {

constexpr int FD_THREADS = 128;
constexpr int FD_TILE = 64;
constexpr float FD_NEG = -3.0e38f;
constexpr int FD_MAXSPLIT = 128;          // gridDim.x upper bound (combine weights live in smem)

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

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int HD, int G>
__global__ void __launch_bounds__(FD_THREADS) flash_decode_kernel(const FdParams p)
{
    constexpr int LDS = HD + 8;                       // padded row (halves): conflict-free 16 B reads
    constexpr int CPR = HD / 8;                       // 16 B chunks per row
    extern __shared__ __align__(16) unsigned char fd_smem[];
    auto Ks = reinterpret_cast<__half (*)[FD_TILE][LDS]>(fd_smem);                       // [2][TILE][LDS]
    auto Vs = reinterpret_cast<__half (*)[FD_TILE][LDS]>(fd_smem + 2 * FD_TILE * LDS * 2);
    __shared__ __align__(16) float qs[G][HD];
    __shared__ float ps[FD_TILE][G];                  // scores, then probabilities
    __shared__ float s_m[G], s_l[G], s_alpha[G];
    __shared__ float s_w[G][FD_MAXSPLIT], s_inv[G];
    __shared__ unsigned s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
    pdl_wait();      // q (and this step's K/V row) come from the previous kernel
    pdl_trigger();
    const int nsplit = gridDim.x;
    const int seq = p.seq_of ? p.seq_of[row] : row;
    const int kv_len = p.kv_len[row] + p.kv_len_add;
    // splits actually used for this length: at least one tile each
    const int ns_act = max(1, min(nsplit, (kv_len + FD_TILE - 1) / FD_TILE));
    int chunk = (kv_len + ns_act - 1) / ns_act;
    chunk = (chunk + FD_TILE - 1) & ~(FD_TILE - 1);
    const int start = split * chunk;
    const int end = split < ns_act ? min(start + chunk, kv_len) : start;
    const int ntiles = end > start ? (end - start + FD_TILE - 1) / FD_TILE : 0;

    const size_t pos_stride = (size_t)p.hkv * HD;    // halves between consecutive positions
    const __half *kbase = p.k_cache + ((size_t)seq * p.cap * p.hkv + kvh) * HD;
    const __half *vbase = p.v_cache + ((size_t)seq * p.cap * p.hkv + kvh) * HD;

    auto load_tile = [&](int t, int buf) {
        const int p0 = start + t * FD_TILE;
        for (int i = tid; i < FD_TILE * CPR; i += FD_THREADS) {
            const int j = i / CPR, c = i - j * CPR;
            const int pos = p0 + j;
            const bool ok = pos < end;
            const size_t off = (size_t)(ok ? pos : 0) * pos_stride + c * 8;
            cp_async16(&Ks[buf][j][c * 8], kbase + off, ok);
            cp_async16(&Vs[buf][j][c * 8], vbase + off, ok);
        }
        cp_async_commit();
    };

    if (ntiles > 0) load_tile(0, 0);
    for (int i = tid; i < G * HD; i += FD_THREADS) {
        const int g = i / HD, d = i - g * HD;
        qs[g][d] = p.q[((size_t)row * p.hq + kvh * G + g) * HD + d] * p.scale;
    }
    if (tid < G) { s_m[tid] = FD_NEG; s_l[tid] = 0.0f; }

    // PV ownership: dim pair dp, heads g = hb, hb + HSTEP, ...
    constexpr int NDP = HD / 2;                       // dim pairs
    constexpr int HSTEP = FD_THREADS / NDP;           // 2 (HD=128) or 4 (HD=64)
    constexpr int HPT = (G + HSTEP - 1) / HSTEP;      // heads per thread
    const int dp = tid % NDP, hb = tid / NDP;
    float acc[HPT][2];
#pragma unroll
    for (int i = 0; i < HPT; i++) acc[i][0] = acc[i][1] = 0.0f;

    // QK ownership: position j = tid % 64, heads g = qb, qb + 2, ...
    constexpr int QHPT = (G + 1) / 2;
    const int qj = tid % FD_TILE, qb = tid / FD_TILE;

    for (int t = 0; t < ntiles; t++) {
        const int buf = t & 1;
        if (t + 1 < ntiles) { load_tile(t + 1, buf ^ 1); cp_async_wait<1>(); }
        else { cp_async_wait<0>(); }
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
                    const int g = qb + 2 * i;
                    if (g < G) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&qs[g][d]);
                        const float4 qc = *reinterpret_cast<const float4 *>(&qs[g][d + 4]);
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
                const int g = qb + 2 * i;
                if (g < G) ps[qj][g] = valid ? s[i] : FD_NEG;
            }
        }
        __syncthreads();

        // ---- online softmax, one warp per head (heads w, w+4, ...)
        for (int g = warp; g < G; g += FD_THREADS / 32) {
            const float a = ps[2 * lane][g], b = ps[2 * lane + 1][g];
            const float mt = warp_max(fmaxf(a, b));
            const float m_old = s_m[g];
            const float m_new = fmaxf(m_old, mt);
            const float pa = expf(a - m_new), pb = expf(b - m_new);
            ps[2 * lane][g] = pa;
            ps[2 * lane + 1][g] = pb;
            const float ts = warp_sum(pa + pb);
            if (lane == 0) {
                const float alpha = expf(m_old - m_new);
                s_alpha[g] = alpha;
                s_l[g] = s_l[g] * alpha + ts;
                s_m[g] = m_new;
            }
        }
        __syncthreads();

        // ---- P.V
        {
#pragma unroll
            for (int i = 0; i < HPT; i++) {
                const int g = hb + i * HSTEP;
                if (g < G) {
                    const float al = s_alpha[g];
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
                        const float pj = ps[j][g];
                        acc[i][0] = fmaf(pj, v.x, acc[i][0]);
                        acc[i][1] = fmaf(pj, v.y, acc[i][1]);
                    }
                }
            }
        }
        __syncthreads();   // ps / buffers are rewritten next tile
    }

    // ---- write this split's partial state
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
        pm[0] = s_m[tid];
        pm[1] = s_l[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(&p.counters[rk], 1u);
        s_last = (prev == (unsigned)nsplit - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // ---- last CTA: log-sum-exp combine over the active splits, fixed order.
    // One warp per head computes M = max m_s, the weights w_s = exp(m_s - M)
    // and 1 / sum(l_s w_s) into smem; then every output element is an
    // independent weighted sum over the splits.
    const float *pmb = p.part_ml + rk * nsplit * G * 2;
    const float *pob = p.part_o + rk * nsplit * G * HD;
    for (int g = warp; g < G; g += FD_THREADS / 32) {
        float M = FD_NEG;
        for (int s = lane; s < ns_act; s += 32) M = fmaxf(M, __ldcg(&pmb[(s * G + g) * 2]));
        M = warp_max(M);
        float L = 0.0f;
        for (int s = lane; s < ns_act; s += 32) {
            const float w = expf(__ldcg(&pmb[(s * G + g) * 2]) - M);
            s_w[g][s] = w;
            L = fmaf(__ldcg(&pmb[(s * G + g) * 2 + 1]), w, L);
        }
        L = warp_sum(L);
        if (lane == 0) s_inv[g] = 1.0f / fmaxf(L, 1e-12f);
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += FD_THREADS) {
        const int g = i / HD, d = i - g * HD;
        const float *po_gd = pob + g * HD + d;
        float O = 0.0f;
#pragma unroll 4
        for (int s = 0; s < ns_act; s++) O = fmaf(__ldcg(po_gd + (size_t)s * G * HD), s_w[g][s], O);
        p.out[((size_t)row * p.hq + kvh * G + g) * HD + d] = O * s_inv[g];
    }
    if (tid == 0) p.counters[rk] = 0u;   // ready for the next launch / graph replay
}

template <int HD, int G>
static int fd_launch(const FdParams &p, int nsplit, int nq, cudaStream_t st)
{
    dim3 grid(nsplit, p.hkv, nq);
    const size_t smem = 4 * FD_TILE * (HD + 8) * sizeof(__half);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        DU_CUDA_TRY(cudaFuncSetAttribute(flash_decode_kernel<HD, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set[dev & 63] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(FD_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, flash_decode_kernel<HD, G>, p));
    return DU_OK;
}

int fd_choose_splits(int nq, int hkv, int max_kv)
{
    const int target = 3 * num_sms();
    int ns = (target + nq * hkv - 1) / (nq * hkv);
    const int max_by_len = (max_kv + FD_TILE - 1) / FD_TILE;
    if (ns > max_by_len) ns = max_by_len;
    if (ns > FD_MAXSPLIT) ns = FD_MAXSPLIT;
    if (ns < 1) ns = 1;
    return ns;
}

size_t fd_scratch_floats(int nq, int hkv, int G, int hd, int nsplit)
{
    return (size_t)nq * hkv * nsplit * G * (hd + 2);
}

int launch_flash_decode(const float *q, const __half *kc, const __half *vc, const int *seq_of,
                        const int *kv_len, int kv_len_add, int nq, int hq, int hkv, int hd, int cap,
                        float scale, float *out, float *scratch, unsigned *counters, int nsplit,
                        cudaStream_t st)
{
    if (nq <= 0) return DU_OK;
    if (hkv <= 0 || hq % hkv != 0) return fail(DU_EINVAL, "flash_decode: hq must be a multiple of hkv");
    const int G = hq / hkv;
    FdParams p;
    p.q = q; p.k_cache = kc; p.v_cache = vc; p.seq_of = seq_of; p.kv_len = kv_len;
    p.kv_len_add = kv_len_add;
    p.hq = hq; p.hkv = hkv; p.cap = cap; p.scale = scale; p.out = out;
    p.part_o = scratch;
    p.part_ml = scratch + (size_t)nq * hkv * nsplit * G * hd;
    p.counters = counters;
#define DU_FD_CASE(HD_, G_) \
    if (hd == HD_ && G == G_) return fd_launch<HD_, G_>(p, nsplit, nq, st);
    DU_FD_CASE(128, 1) DU_FD_CASE(128, 2) DU_FD_CASE(128, 4) DU_FD_CASE(128, 8)
    DU_FD_CASE(64, 1) DU_FD_CASE(64, 2) DU_FD_CASE(64, 4) DU_FD_CASE(64, 8)
#undef DU_FD_CASE
    return fail(DU_EINVAL, "flash_decode: supported head_dim 64/128 and GQA group 1/2/4/8");
}

}  // namespace du
