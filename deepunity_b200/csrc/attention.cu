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
#include "attn_impl.cuh"
#include "internal.h"

namespace du {

constexpr int FD_THREADS = 128;

template <int HD>
__global__ void __launch_bounds__(FD_THREADS) flash_decode_kernel(const FdParams p, int G)
{
    extern __shared__ __align__(16) unsigned char fd_smem[];
    __shared__ FdShared<HD> sh;
    pdl_wait();      // q (and this step's K/V row) come from the previous kernel
    pdl_trigger();
    fd_unit<HD, FD_THREADS>(p, G, blockIdx.z, blockIdx.y, blockIdx.x, gridDim.x, fd_smem, sh);
}

template <int HD>
static int fd_launch(const FdParams &p, int G, int nsplit, int nq, cudaStream_t st)
{
    dim3 grid(nsplit, p.hkv, nq);
    const size_t smem = 4 * FD_TILE * (HD + 8) * sizeof(__half);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        DU_CUDA_TRY(cudaFuncSetAttribute(flash_decode_kernel<HD>,
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
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, flash_decode_kernel<HD>, p, G));
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
    if (G < 1 || G > FD_MAXG) return fail(DU_EINVAL, "flash_decode: GQA group must be 1..8");
    if (nsplit < 1 || nsplit > FD_MAXSPLIT) return fail(DU_EINVAL, "flash_decode: split count out of range");
    if (hd == 128) return fd_launch<128>(p, G, nsplit, nq, st);
    if (hd == 64) return fd_launch<64>(p, G, nsplit, nq, st);
    return fail(DU_EINVAL, "flash_decode: supported head_dim 64/128");
}

}  // namespace du
