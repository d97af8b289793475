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
// decode step.  The unit itself lives in attn_impl.cuh (shared with the
// persistent decode-step kernel).
//
// flash_decode_cluster_kernel (the model's decode and prefill path): the C
// splits of one (row, kv head) form one thread-block cluster.  Each CTA leaves
// its split's (m, l, acc) in shared memory and pushes each output element's
// value, and every head's (m, l), into the shared memory of the CTA that merges
// it (distributed shared-memory stores): CTA r merges output elements
// [r * G*HD/C, (r + 1) * G*HD/C).  One cluster barrier later every CTA reads
// only its own shared memory and merges in split order, so there are no global
// partials, atomics or remote-read round trips.
#include <cooperative_groups.h>

#include <cstring>
#include <mutex>

#include "attn_impl.cuh"
#include "gemm_impl.cuh"
#include "internal.h"

namespace du {

constexpr int FD_THREADS = 128;
constexpr int FDC_THREADS = 256;     // cluster kernel: fewer positions per CTA, more threads per tile

// new_rows >= 0: each query row's last new_rows K/V rows come from the previous
// kernel (decode: 1); the unit's older rows of its first tile are loaded before
// griddepcontrol.wait, overlapping the QKV kernel's tail.  kv_len itself was
// written by kernels that completed before the QKV kernel passed its own wait.
template <int HD>
__global__ void __launch_bounds__(FD_THREADS) flash_decode_kernel(const FdParams p, int G, int new_rows)
{
    extern __shared__ __align__(16) unsigned char fd_smem[];
    __shared__ FdShared<HD> sh;
    if (new_rows >= 0) fd_prefetch<HD, FD_THREADS>(p, blockIdx.z, blockIdx.y, blockIdx.x, gridDim.x, new_rows, fd_smem);
    pdl_wait();      // q (and this step's K/V rows) come from the previous kernel
    pdl_trigger();
    fd_unit<HD, FD_THREADS>(p, G, blockIdx.z, blockIdx.y, blockIdx.x, gridDim.x, fd_smem, sh, new_rows);
}

template <int HD>
static int fd_launch(const FdParams &p, int G, int nsplit, int nq, cudaStream_t st, int new_rows)
{
    dim3 grid(nsplit, p.hkv, nq);
    const size_t smem = 4 * FD_TILE * (HD + 8) * sizeof(__half);
    int rc = ensure_func_attrs((const void *)flash_decode_kernel<HD>, (int)smem);
    if (rc) return rc;
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
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, flash_decode_kernel<HD>, p, G, new_rows));
    return DU_OK;
}

namespace cg = cooperative_groups;

// Shared memory of the cluster kernel after the tiles and the tensor-core
// operands: where the other splits push their state for this CTA's outputs.
template <int HD, int C>
__host__ __device__ constexpr size_t fdc_recv_bytes()
{
    return sizeof(float) * ((size_t)C * (FD_MAXG * HD / C) + (size_t)C * FD_MAXG * 2);
}

// Dynamic shared memory of the cluster kernel before the receive buffers: tiles,
// tensor-core operands and (INT8 cache) the raw staging buffers.
template <int HD, bool KV8>
__host__ __device__ constexpr size_t fdc_work_bytes()
{
    return (size_t)4 * FD_TILE * (HD + 8) * sizeof(__half) + fd_mma_extra_bytes<HD>() + (KV8 ? fd_kv8_bytes<HD>() : 0);
}

// Fused O projection (OF): after the combine, the C CTAs of a (row, kv head)
// cluster hold that kv head's G * HD attention outputs; each CTA multiplies them
// with its slice of W_o rows (rows [split * R, split * R + R), R = ceil(H / C),
// this kv head's G * HD columns), copied into shared memory by the bulk-copy unit
// at kernel start, while attention runs.  The hkv clusters' partial sums meet in
// global scratch; the cluster that arrives last for a row slice adds them in kv
// head order to the residual (no cluster waits for another).
constexpr int FDC_OF_MAX_BYTES = 96 * 1024;         // W_o slice per CTA
constexpr int FDC_OF_MAX_SCALES = 4096;             // its scales (halves)
template <int HD>
__host__ __device__ constexpr size_t fdc_of_bytes()
{
    // attention outputs, W_o slice (128-byte aligned: 128 bytes of slack), its scales, mbarrier
    return (size_t)FD_MAXG * HD * 4 + 128 + FDC_OF_MAX_BYTES + FDC_OF_MAX_SCALES * 2 + 16;
}

template <int HD, int C, bool KV8, bool OF>
__global__ void __launch_bounds__(FDC_THREADS)
    flash_decode_cluster_kernel(const FdParams p, int G, int new_rows, const __grid_constant__ CUtensorMap tm_wo)
{
    constexpr int PER_MAX = FD_MAXG * HD / C;        // outputs merged per CTA, at most
    extern __shared__ __align__(16) unsigned char fd_smem[];
    __shared__ FdShared<HD> sh;
    __shared__ int of_abort;
    cg::cluster_group cluster = cg::this_cluster();
    const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;     // gridDim.x == C == cluster size
    float *rcv_o = reinterpret_cast<float *>(fd_smem + fdc_work_bytes<HD, KV8>());
    float *rcv_ml = rcv_o + C * PER_MAX;             // [C][FD_MAXG][2]
    unsigned char *of_base = fd_smem + fdc_work_bytes<HD, KV8>() + fdc_recv_bytes<HD, C>();
    float *att_s = reinterpret_cast<float *>(of_base);                         // [G * HD]
    // W_o slice: TMA boxes of 256 columns x R rows, [box][row][256 bytes]
    uint8_t *wo_s = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(of_base + (size_t)FD_MAXG * HD * 4) + 127) & ~(uintptr_t)127);
    __half *sc_s = reinterpret_cast<__half *>(wo_s + FDC_OF_MAX_BYTES);         // the slice's scales
    uint64_t *of_bar = reinterpret_cast<uint64_t *>(wo_s + FDC_OF_MAX_BYTES + FDC_OF_MAX_SCALES * 2);
    const int ghd = G * HD;
    const int of_rows = (p.H + C - 1) / C, of_n0 = split * of_rows;
    const int of_nr = OF ? max(0, min(of_rows, p.H - of_n0)) : 0;
    const int of_rb = p.wo_quant == Q_I4 ? ghd / 2 : ghd;                       // bytes of a slice row
    const int of_spr = p.wo_quant == Q_I4 ? ghd / p.wo_group : 1;              // scales per slice row
    if constexpr (OF) {
        // W_o rows of this CTA (weights, so issued before the dependency wait): one TMA
        // box per 256 columns; rows past H arrive zero-filled and are not used
        const uint32_t bar = smem_u32(of_bar);
        if (threadIdx.x == 0) {
            of_abort = 0;
            mbar_init(bar, 1);
            mbar_fence_init();
            const int nb = of_rb / 256;
            mbar_arrive_expect_tx(bar, (uint32_t)(nb * of_rows * 256));
            const uint64_t pol = l2_policy_evict_first();
            for (int b = 0; b < nb; b++)
                tma_load_2d(smem_u32(wo_s + (size_t)b * of_rows * 256), &tm_wo, bar, kvh * of_rb + b * 256, of_n0, pol);
        }
        // the slice's scales with plain loads, all of a thread's loads issued before its stores
        const size_t spr_all = p.wo_quant == Q_I4 ? (size_t)p.hq * HD / p.wo_group : 1;
        constexpr int SPT = FDC_OF_MAX_SCALES / FDC_THREADS;
        __half sv[SPT];
#pragma unroll
        for (int k = 0; k < SPT; k++) {
            const int i = threadIdx.x + k * FDC_THREADS, r = i / of_spr, g = i - r * of_spr;
            sv[k] = i < of_nr * of_spr
                        ? p.wo_scales[(size_t)(of_n0 + r) * spr_all + (p.wo_quant == Q_I4 ? (size_t)kvh * of_spr + g : 0)]
                        : __float2half(0.0f);
        }
#pragma unroll
        for (int k = 0; k < SPT; k++)
            if (threadIdx.x + k * FDC_THREADS < of_nr * of_spr) sc_s[threadIdx.x + k * FDC_THREADS] = sv[k];
    }
    // first phase of the cluster barrier: every CTA of the cluster has started before
    // any CTA stores into a peer's shared memory (waited on just before the push)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    if (new_rows >= 0) fd_prefetch<HD, FDC_THREADS, true, KV8>(p, row, kvh, split, C, new_rows, fd_smem);
    pdl_wait();      // q (and this step's K/V rows) come from the previous kernel
    pdl_trigger();
    fd_unit<HD, FDC_THREADS, true, KV8>(p, G, row, kvh, split, C, fd_smem, sh, new_rows);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");

    // push: output o of this split's acc goes to CTA o / per, slot [split][o % per];
    // (m, l) of every head to every CTA
    const int n_out = G * HD, per = (n_out + C - 1) / C;
    const float *so = reinterpret_cast<const float *>(fd_smem);
    for (int o = threadIdx.x; o < n_out; o += FDC_THREADS) {
        const int j = o / per;
        cluster.map_shared_rank(rcv_o, j)[split * PER_MAX + (o - j * per)] = so[o];
    }
    if (threadIdx.x < C * G) {
        const int j = threadIdx.x / G, g = threadIdx.x - j * G;
        float *d = cluster.map_shared_rank(rcv_ml, j) + (split * FD_MAXG + g) * 2;
        d[0] = sh.m[g];
        d[1] = sh.l[g];
    }
    cluster.sync();  // every split's state for this CTA's outputs is in its own shared memory

    // merge outputs [split * per, (split + 1) * per) in split order
    for (int i = threadIdx.x; i < per; i += FDC_THREADS) {
        const int o = split * per + i;
        if (o >= n_out) break;
        const int g = o / HD;
        float M = FD_NEG;
#pragma unroll
        for (int r = 0; r < C; r++) M = fmaxf(M, rcv_ml[(r * FD_MAXG + g) * 2]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int r = 0; r < C; r++) {
            const float w = expf(rcv_ml[(r * FD_MAXG + g) * 2] - M);
            L = fmaf(rcv_ml[(r * FD_MAXG + g) * 2 + 1], w, L);
            O = fmaf(rcv_o[r * PER_MAX + i], w, O);
        }
        const float v = O * (1.0f / fmaxf(L, 1e-12f));
        p.out[((size_t)row * p.hq + kvh * G) * HD + o] = v;
        if (OF)     // every CTA of the cluster gets this kv head's outputs for its W_o rows
#pragma unroll 4
            for (int j = 0; j < C; j++) cluster.map_shared_rank(att_s, j)[o] = v;
    }
    if constexpr (OF) {
        cluster.sync();      // att_s complete in every CTA; no peer stores after this point
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        const int cpl = ghd >> 5;                     // columns per lane: 8 or 16
        float xa[16];
#pragma unroll
        for (int j = 0; j < 16; j++) xa[j] = j < cpl ? att_s[lane * cpl + j] : 0.0f;
        const bool ok = mbar_wait(smem_u32(of_bar), 0, &of_abort, p.err, 2000000000ull);
        if (ok) {
            for (int r = warp; r < of_nr; r += FDC_THREADS / 32) {
                const int n = of_n0 + r;
                // byte c of slice row r: box c / 256, [r][c % 256]
                auto wr = [&](int c) { return wo_s + ((size_t)(c >> 8) * of_rows + r) * 256 + (c & 255); };
                float a = 0.0f, d;
                if (p.wo_quant == Q_I4) {
                    // low nibble = even column; nibble j of word w is column lane * cpl + 8 w + j
                    const uint2 w2 = cpl == 16 ? *reinterpret_cast<const uint2 *>(wr(lane * 8))
                                               : make_uint2(*reinterpret_cast<const uint32_t *>(wr(lane * 4)), 0u);
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < cpl) {
                            const uint32_t w = j < 8 ? w2.x : w2.y;
                            a = fmaf((float)((int)((w >> (4 * (j & 7))) & 15u) - 8), xa[j], a);
                        }
                    d = __half2float(sc_s[r * of_spr + (lane * cpl) / p.wo_group]);
                } else {
                    const uint4 w4 = cpl == 16 ? *reinterpret_cast<const uint4 *>(wr(lane * 16))
                                               : make_uint4(*reinterpret_cast<const uint32_t *>(wr(lane * 8)),
                                                            *reinterpret_cast<const uint32_t *>(wr(lane * 8 + 4)), 0u, 0u);
                    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < cpl) a = fmaf((float)(int8_t)((ww[j >> 2] >> (8 * (j & 3))) & 0xFFu), xa[j], a);
                    d = __half2float(sc_s[r]);
                }
                const float v = warp_sum(a * d);
                if (lane == 0) p.opart[(size_t)kvh * p.H + n] = v;
            }
        }
        __syncthreads();
        // this kv head's part of rows [of_n0, of_n0 + of_nr) is out; the last kv head to
        // arrive adds all parts in kv head order to the residual
        if (threadIdx.x == 0) {
            __threadfence();
            sh.last = atomicAdd(&p.ocnt[split], 1u) == (unsigned)(p.hkv - 1) ? 1u : 0u;
        }
        __syncthreads();
        if (sh.last) {
            __threadfence();
            for (int r = threadIdx.x; r < of_nr; r += FDC_THREADS) {
                const int n = of_n0 + r;
                float part[FD_MAXG * 2];                // every kv head's part, loads issued together
#pragma unroll
                for (int k = 0; k < FD_MAXG * 2; k++)
                    part[k] = k < p.hkv ? __ldcg(p.opart + (size_t)k * p.H + n) : 0.0f;
                float sum = 0.0f;
#pragma unroll
                for (int k = 0; k < FD_MAXG * 2; k++)
                    if (k < p.hkv) sum += part[k];
                p.resid[n] += sum;
            }
            if (threadIdx.x == 0) p.ocnt[split] = 0u;     // ready for the next launch
        }
    }
}

template <int HD, int C, bool KV8, bool OF = false>
static int fdc_launch(const FdParams &p, int G, int nq, cudaStream_t st, int new_rows, bool probe, int *fits,
                      const CUtensorMap *tm = nullptr)
{
    auto kern = flash_decode_cluster_kernel<HD, C, KV8, OF>;
    const size_t smem = fdc_work_bytes<HD, KV8>() + fdc_recv_bytes<HD, C>() + (OF ? fdc_of_bytes<HD>() : 0);
    int rc = ensure_func_attrs((const void *)kern, (int)smem, C > 8);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C, p.hkv, nq);
    cfg.blockDim = dim3(FDC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    // Load-balanced cluster scheduling lets the hardware place CTAs of one cluster on
    // an SM that already holds another (two fit per SM with the fp16 cache): batched
    // fp16 attention 15-22 % faster at batch 8 (8B shapes, ctx 512..32768), 2-6 % at
    // batch 32; unchanged at batch 1 and with the INT8 cache.
    cudaLaunchAttribute attr[3];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
    attr[1].val.clusterSchedulingPolicyPreference = cudaClusterSchedulingPolicyLoadBalancing;
    attr[2].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[2].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 3 : 2;
    if (probe) {
        int n = 0;
        DU_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
        *fits = n;
        return DU_OK;
    }
    CUtensorMap none;
    memset(&none, 0, sizeof none);
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p, G, new_rows, tm ? *tm : none));
    return DU_OK;
}

// Cluster size per device (and cache format): 16 splits when such clusters can be
// resident, else 8.
template <int HD, bool KV8>
static int fdc_cluster_size(const FdParams &p, int G, cudaStream_t st)
{
    static std::mutex mu;
    static int chosen[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (chosen[dev & 63] == 0) {
        int n16 = 0;
        const int rc = fdc_launch<HD, 16, KV8>(p, G, 1, st, -1, true, &n16);
        if (rc != DU_OK) cudaGetLastError();    // the probe's own failure: 16-CTA clusters unavailable
        chosen[dev & 63] = (rc == DU_OK && n16 > 0) ? 16 : 8;
        const char *e = getenv("DU_FD_CLUSTER");   // tuning knob: 8 forces 8-CTA clusters
        if (e != nullptr && atoi(e) == 8) chosen[dev & 63] = 8;
    }
    return chosen[dev & 63];
}

// Cluster size per launch.  16 splits only when there are few clusters (query rows x
// kv heads <= 8) and the cache is fp16: 16-CTA clusters hold a whole SM each and at
// most 7 are resident on a B200, so with more clusters the 8-CTA form (about twice
// as many resident) wins despite twice the positions per CTA.  Measured on the
// 8B shapes (32 / 8 heads of 128, CUDA-graph timed): batch 8, ctx 512 24.9 -> 13.2 us,
// batch 32, ctx 2048 134.8 -> 96.1 us, INT8 cache batch 1, ctx 512 9.1 -> 4.9 us;
// batch 1, ctx 8192 stays on 16 (19.2 vs 26.0 us).
template <int HD, bool KV8>
static int fdc_dispatch(const FdParams &p, int G, int nq, cudaStream_t st, int new_rows)
{
    int dummy = 0;
    const bool few = !KV8 && (int64_t)nq * p.hkv <= 8;
    return few && fdc_cluster_size<HD, KV8>(p, G, st) == 16
               ? fdc_launch<HD, 16, KV8>(p, G, nq, st, new_rows, false, &dummy)
               : fdc_launch<HD, 8, KV8>(p, G, nq, st, new_rows, false, &dummy);
}

// Whether flash-decode with the fused O projection can run: one query row, 16-CTA
// clusters, fp16 cache, G * HD of 256 or 512, INT4 / INT8 W_o, a slice that fits.
bool flash_decode_fuse_o_supported(int nq, int hq, int hkv, int hd, int H, int quant, int group)
{
    if (nq != 1 || hkv <= 0 || hq % hkv != 0 || (hd != 64 && hd != 128)) return false;
    const int ghd = hq / hkv * hd;
    if (ghd != 256 && ghd != 512) return false;
    if (quant != Q_I4 && quant != Q_I8) return false;
    if (quant == Q_I4 && (group < 16 || (ghd / 32) % 8 != 0 || group % (ghd / 32) != 0)) return false;
    const int rb = quant == Q_I4 ? ghd / 2 : ghd;
    if ((size_t)((H + 15) / 16) * rb > (size_t)FDC_OF_MAX_BYTES || rb % 256 != 0 || (H + 15) / 16 > 256) return false;
    if ((size_t)((H + 15) / 16) * (quant == Q_I4 ? ghd / group : 1) > (size_t)FDC_OF_MAX_SCALES) return false;
    if (hkv > FD_MAXG * 2) return false;
    FdParams p = {};
    p.hq = hq; p.hkv = hkv;
    if (hd == 128 ? fdc_cluster_size<128, false>(p, hq / hkv, 0) != 16 : fdc_cluster_size<64, false>(p, hq / hkv, 0) != 16)
        return false;
    // every kv head's cluster must be resident at once: a second wave of 16-CTA clusters
    // costs more than the separate O GEMV saves (8B shapes: 8 clusters, 7 resident,
    // 41 vs 8 + 10.5 us serialised)
    int fits = 0;
    const int rc = hd == 128 ? fdc_launch<128, 16, false, true>(p, hq / hkv, 1, 0, -1, true, &fits)
                             : fdc_launch<64, 16, false, true>(p, hq / hkv, 1, 0, -1, true, &fits);
    if (rc != DU_OK) cudaGetLastError();      // the probe's own failure
    return rc == DU_OK && fits >= hkv;
}

int launch_flash_decode_fuse_o(const float *q, const __half *kc, const __half *vc, const int *seq_of, const int *kv_len,
                               int kv_len_add, int hq, int hkv, int hd, int cap, float scale, float *att, cudaStream_t st,
                               int new_rows, const FuseO &o)
{
    FdParams p = {};
    p.q = q; p.k_cache = kc; p.v_cache = vc; p.seq_of = seq_of; p.kv_len = kv_len; p.kv_len_add = kv_len_add;
    p.hq = hq; p.hkv = hkv; p.cap = cap; p.scale = scale; p.out = att;
    p.wo = o.w; p.wo_scales = o.scales; p.wo_quant = o.quant; p.wo_group = o.group; p.H = o.H;
    p.resid = o.resid; p.opart = o.part; p.ocnt = o.cnt; p.err = o.err;
    int dummy = 0;
    const int G = hq / hkv, rb = o.quant == Q_I4 ? G * hd / 2 : G * hd;
    // W_o as bytes [H][row bytes]; box 256 bytes x ceil(H / 16) rows
    CUtensorMap tm;
    const uint64_t row_bytes = o.quant == Q_I4 ? (uint64_t)hq * hd / 2 : (uint64_t)hq * hd;
    int rc = make_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, o.w, row_bytes, (uint64_t)o.H, 256u,
                       (uint32_t)((o.H + 15) / 16), CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    if (rb % 256 != 0) return fail(DU_EINVAL, "flash_decode_fuse_o: W_o slice rows must be multiples of 256 bytes");
    if (hd == 128) return fdc_launch<128, 16, false, true>(p, G, 1, st, new_rows, false, &dummy, &tm);
    if (hd == 64) return fdc_launch<64, 16, false, true>(p, G, 1, st, new_rows, false, &dummy, &tm);
    return fail(DU_EINVAL, "flash_decode_fuse_o: head_dim 64/128");
}

int launch_flash_decode_cluster(const float *q, const __half *kc, const __half *vc, const int *seq_of,
                                const int *kv_len, int kv_len_add, int nq, int hq, int hkv, int hd, int cap,
                                float scale, float *out, cudaStream_t st, int new_rows, const Kv8Cache *kv8,
                                int window)
{
    if (nq <= 0) return DU_OK;
    if (hkv <= 0 || hq % hkv != 0) return fail(DU_EINVAL, "flash_decode: hq must be a multiple of hkv");
    const int G = hq / hkv;
    if (G < 1 || G > FD_MAXG) return fail(DU_EINVAL, "flash_decode: GQA group must be 1..8");
    FdParams p = {};
    p.q = q; p.k_cache = kc; p.v_cache = vc; p.seq_of = seq_of; p.kv_len = kv_len;
    p.kv_len_add = kv_len_add;
    p.hq = hq; p.hkv = hkv; p.cap = cap; p.scale = scale; p.out = out;
    p.window = window;
    if (kv8 != nullptr) {
        p.k8 = kv8->k8; p.v8 = kv8->v8; p.ksz = kv8->ksz; p.vsz = kv8->vsz;
        if (hd == 128) return fdc_dispatch<128, true>(p, G, nq, st, new_rows);
        if (hd == 64) return fdc_dispatch<64, true>(p, G, nq, st, new_rows);
        return fail(DU_EINVAL, "flash_decode: the INT8 cache supports head_dim 64/128");
    }
    if (hd == 128) return fdc_dispatch<128, false>(p, G, nq, st, new_rows);
    if (hd == 64) return fdc_dispatch<64, false>(p, G, nq, st, new_rows);
    if (hd == 256) return fdc_dispatch<256, false>(p, G, nq, st, new_rows);
    return fail(DU_EINVAL, "flash_decode: supported head_dim 64/128/256");
}

// WriteCacheFull, INT8 variant (Gemma3CS.compute:300-380; layout KVCache.hlsl:46-82):
// one warp per (token, K|V, kv head) row of hd fp32 values from the QKV epilogue's
// staging buffer [M][nkv][hkv][hd] (nkv = 2: K and V rows; 1: K rows only).  min / max (exact in any order), scale = (max -
// min) / 255 floored at 1e-9, zp = round(-min / scale) clamped to [0, 255], q =
// clamp(round(x * (1 / scale)) + zp, 0, 255), round half to even, IEEE division
// and reciprocal; the row's word (fp16 scale | fp16 zp << 16).
__global__ void __launch_bounds__(256) kv_quant_int8_kernel(const float *stage, int M, int nkv, int hkv, int hd,
                                                            const int *pos, int pos_base, const int *seq_of,
                                                            int seq_off, int cap, Kv8Cache kv)
{
    pdl_wait();
    const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (w >= M * nkv * hkv) return;
    const int h = w % hkv, isv = (w / hkv) % nkv, m = w / (nkv * hkv);
    const int epl = hd >> 5;                         // values per lane (hd = 32 .. 256)
    const float *x = stage + (size_t)w * hd + lane * epl;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = e < epl ? x[e] : 0.0f;
    const int seq = seq_of ? seq_of[m] : seq_off + m;
    const size_t row = ((size_t)seq * cap + (pos ? pos[m] : pos_base + m)) * hkv + h;
    kv8_store_row(v, epl, lane, (isv ? kv.v8 : kv.k8) + row * hd, (isv ? kv.vsz : kv.ksz) + row);
}

int launch_kv_quant_int8(const float *stage, int M, int nkv, int hkv, int hd, const int *pos, int pos_base,
                         const int *seq_of, int seq_off, int cap, const Kv8Cache &kv, cudaStream_t st)
{
    if (M <= 0) return DU_OK;
    if (hd % 32 != 0 || hd > 256) return fail(DU_EINVAL, "kv_quant_int8: head_dim must be a multiple of 32, <= 256");
    if (nkv != 1 && nkv != 2) return fail(DU_EINVAL, "kv_quant_int8: nkv must be 1 or 2");
    const int warps = M * nkv * hkv;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((warps + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kv_quant_int8_kernel, stage, M, nkv, hkv, hd, pos, pos_base, seq_of, seq_off,
                                   cap, kv));
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
                        cudaStream_t st, int new_rows)
{
    if (nq <= 0) return DU_OK;
    if (hkv <= 0 || hq % hkv != 0) return fail(DU_EINVAL, "flash_decode: hq must be a multiple of hkv");
    const int G = hq / hkv;
    FdParams p = {};
    p.q = q; p.k_cache = kc; p.v_cache = vc; p.seq_of = seq_of; p.kv_len = kv_len;
    p.kv_len_add = kv_len_add;
    p.hq = hq; p.hkv = hkv; p.cap = cap; p.scale = scale; p.out = out;
    p.part_o = scratch;
    p.part_ml = scratch + (size_t)nq * hkv * nsplit * G * hd;
    p.counters = counters;
    if (G < 1 || G > FD_MAXG) return fail(DU_EINVAL, "flash_decode: GQA group must be 1..8");
    if (nsplit < 1 || nsplit > FD_MAXSPLIT) return fail(DU_EINVAL, "flash_decode: split count out of range");
    if (hd == 128) return fd_launch<128>(p, G, nsplit, nq, st, new_rows);
    if (hd == 64) return fd_launch<64>(p, G, nsplit, nq, st, new_rows);
    return fail(DU_EINVAL, "flash_decode: supported head_dim 64/128");
}

}  // namespace du
