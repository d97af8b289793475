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

#include <mutex>

#include "attn_impl.cuh"
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

template <int HD, int C, bool KV8>
__global__ void __launch_bounds__(FDC_THREADS) flash_decode_cluster_kernel(const FdParams p, int G, int new_rows)
{
    constexpr int PER_MAX = FD_MAXG * HD / C;        // outputs merged per CTA, at most
    extern __shared__ __align__(16) unsigned char fd_smem[];
    __shared__ FdShared<HD> sh;
    cg::cluster_group cluster = cg::this_cluster();
    const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;     // gridDim.x == C == cluster size
    float *rcv_o = reinterpret_cast<float *>(fd_smem + fdc_work_bytes<HD, KV8>());
    float *rcv_ml = rcv_o + C * PER_MAX;             // [C][FD_MAXG][2]
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
        p.out[((size_t)row * p.hq + kvh * G) * HD + o] = O * (1.0f / fmaxf(L, 1e-12f));
    }
}

template <int HD, int C, bool KV8>
static int fdc_launch(const FdParams &p, int G, int nq, cudaStream_t st, int new_rows, bool probe, int *fits)
{
    auto kern = flash_decode_cluster_kernel<HD, C, KV8>;
    const size_t smem = fdc_work_bytes<HD, KV8>() + fdc_recv_bytes<HD, C>();
    int rc = ensure_func_attrs((const void *)kern, (int)smem, C > 8);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C, p.hkv, nq);
    cfg.blockDim = dim3(FDC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    if (probe) {
        int n = 0;
        DU_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
        *fits = n;
        return DU_OK;
    }
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p, G, new_rows));
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
    }
    return chosen[dev & 63];
}

template <int HD, bool KV8>
static int fdc_dispatch(const FdParams &p, int G, int nq, cudaStream_t st, int new_rows)
{
    int dummy = 0;
    return fdc_cluster_size<HD, KV8>(p, G, st) == 16 ? fdc_launch<HD, 16, KV8>(p, G, nq, st, new_rows, false, &dummy)
                                                     : fdc_launch<HD, 8, KV8>(p, G, nq, st, new_rows, false, &dummy);
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
