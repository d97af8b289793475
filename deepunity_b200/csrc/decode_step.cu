// decode_step.cu -- persistent decode-step kernel.
//
// One cooperative launch runs a whole decode step (the reference dispatches
// ~389 shader dispatches per token, MiniCPM5Model.cs:294-674): one CTA per SM
// walks the stage list
//     embed, L x [QKV, attention, O, gate|up, down], lm_head, argmax
// with a grid barrier between stages.  Every GEMV stage is the same device
// code as the standalone GEMV kernel (gemv_impl.cuh), split into prefetch and
// run.  One 512-thread CTA (16 warps) per SM: enough warps to hide the
// latency of the dequant / dp4a chain, with one activation stage per SM.
// Weights and old K/V rows never wait for a barrier: once a CTA has arrived
// at the barrier that ends stage s, it issues the first ring stages of its
// rows of stage s + 1 (GEMV), or, before attention, the K/V rows of its first
// attention unit that earlier steps wrote (only the row this step's QKV
// epilogue wrote is loaded after the barrier).  Attention K/V tiles live in
// the ring region, which attention does not otherwise use.
// Attention units are the shared flash-decode unit (attn_impl.cuh) processed
// by the whole CTA.
//
// Barrier: a step-local counter (zeroed by a memset node before the kernel in
// the captured graph); thread 0 of each CTA adds 1 with release semantics and,
// after the CTA has issued its prefetches, spins with acquire loads until the
// counter reaches (barrier index + 1) * gridDim.x.  The spin is bounded: after
// a few seconds it sets the error word, and every CTA then waits for its own
// cp.async copies and returns; the host reports DU_ECUDA.  Co-residency of all
// CTAs is guaranteed by the cooperative launch.
#include "attn_impl.cuh"
#include "gemv_impl.cuh"
#include "internal.h"
#include "step_plan.h"

namespace du {

constexpr int DS_WARPS = 16;              // one 512-thread CTA per SM
constexpr int DS_THREADS = DS_WARPS * 32;
constexpr unsigned DS_SPIN_LIMIT = 1u << 22;     // a few seconds of polling before giving up

__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Grid barrier, split so that a CTA can issue prefetches between its arrival
// and its wait.  Arrival: the CTA's writes are ordered before thread 0's
// release add (bar.sync, then red.release.gpu).  Wait: thread 0 polls with
// acquire loads, then bar.sync releases the CTA.
__device__ __forceinline__ void ds_arrive(unsigned *ctr)
{
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

__device__ __forceinline__ bool ds_wait(unsigned *ctr, unsigned target, int *err)
{
    if (threadIdx.x == 0) {
        unsigned n = 0;
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
            if (v >= target) break;
            if (++n > DS_SPIN_LIMIT) {
                atomicExch(err, 1);
                break;
            }
            if ((n & 255) == 0 && *(volatile int *)err) break;
        }
    }
    __syncthreads();
    return *(volatile int *)err == 0;
}

template <int QT, int MT, int HD>
__global__ void __launch_bounds__(DS_THREADS, 1) decode_step_kernel(const StepPlan plan)
{
    constexpr int RW = MT == 1 ? 4 : 2;
    constexpr int DS_D = ds_depth(MT);
    constexpr int HEAD_D = ds_head_depth(MT);
    extern __shared__ __align__(16) unsigned char ds_smem[];
    __shared__ GemvShared<MT, DS_WARPS> gsh;
    __shared__ FdShared<HD> fsh;
    const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
    unsigned char *ring = ds_smem;                         // weight rings / attention K/V tiles
    unsigned char *xreg = ds_smem + plan.ring_bytes;       // activation stage

    GemvStream<QT, MT, RW, DS_D, DS_WARPS> gq;       // weight stream of the model's linears
    GemvStream<Q_F16, MT, RW, HEAD_D, DS_WARPS> gf;  // weight stream of an fp16 lm_head
    bool gq_ready = false, gf_ready = false;   // the ring holds the next stage's first steps
    unsigned nbar = 0;
    if (cta == 0 && tid == 0 && plan.stamps) plan.stamps[0] = globaltimer_ns();

    for (int s = 0; s < plan.nstages; s++) {
        const StepStage &st = plan.stages[s];
        const int type = st.type;
        const bool next_gq = s + 1 < plan.nstages && plan.stages[s + 1].type == SG_GEMV && plan.stages[s + 1].qt == QT;
        if (type == SG_EMBED) {
            const size_t n = (size_t)plan.M * plan.H;
            for (size_t i = (size_t)cta * DS_THREADS + tid; i < n; i += (size_t)ncta * DS_THREADS) {
                const int m = (int)(i / plan.H), k = (int)(i - (size_t)m * plan.H);
                plan.x_res[i] = __half2float(plan.embed[(size_t)plan.ids[m] * plan.H + k]) * plan.embed_scale;
            }
        } else if (type == SG_GEMV) {
            const GemvParams &gp = st.g;
            if (st.qt == QT) {
                if (!gq_ready) gq.prefetch(gp, ring, cta, ncta);
                gq.run(gp, xreg, gsh, cta, ncta, [] {});
                gq_ready = false;
            } else {
                if (!gf_ready) gf.prefetch(gp, ring, cta, ncta);
                gf.run(gp, xreg, gsh, cta, ncta, [] {});
                gf_ready = false;
            }
        } else if (type == SG_ATTN) {
            const FdParams &ap = st.a;
            const int units = st.nq * ap.hkv * st.nsplit;
            for (int u = cta; u < units; u += ncta) {
                const int split = u % st.nsplit, rest = u / st.nsplit;
                const int kvh = rest % ap.hkv, row = rest / ap.hkv;
                // the first unit's old K/V rows were loaded during the previous barrier
                fd_unit<HD, DS_THREADS>(ap, st.G, row, kvh, split, st.nsplit, ring, fsh, u == cta ? st.a_new : -1);
            }
        } else if (type == SG_ARGMAX) {
            // single CTA: greedy pick per sequence from the lm_head CTA partials
            if (cta == 0) {
                for (int m = 0; m < plan.M; m++) {
                    float bv = -INFINITY;
                    int bi = 0x7fffffff;
                    for (int i = tid; i < plan.nparts; i += DS_THREADS) {
                        const float v = plan.am_val[(size_t)m * plan.nparts + i];
                        const int ix = plan.am_idx[(size_t)m * plan.nparts + i];
                        if (am_better(v, ix, bv, bi)) { bv = v; bi = ix; }
                    }
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                        if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                    }
                    if ((tid & 31) == 0) { gsh.amv[tid >> 5][0] = bv; gsh.ami[tid >> 5][0] = bi; }
                    __syncthreads();
                    if (tid == 0) {
                        bv = gsh.amv[0][0]; bi = gsh.ami[0][0];
                        for (int w = 1; w < DS_WARPS; w++)
                            if (am_better(gsh.amv[w][0], gsh.ami[w][0], bv, bi)) {
                                bv = gsh.amv[w][0]; bi = gsh.ami[w][0];
                            }
                        plan.next_out[m] = bi;
                        if (plan.feed) plan.feed[m] = bi;
                        if (plan.hist) plan.hist[(size_t)m * plan.cap + plan.cache_len[m]] = bi;
                        if (plan.advance) plan.cache_len[m] += 1;
                    }
                    __syncthreads();
                }
            }
        }
        if (s + 1 < plan.nstages) {
            ds_arrive(plan.barrier);
            // only inputs that no stage writes from here to the wait (weights, old K/V rows)
            const StepStage &nx = plan.stages[s + 1];
            if (next_gq) {
                const GemvParams &np = nx.g;
                gq.prefetch(np, ring, cta, ncta);
                gq_ready = true;
            } else if (nx.type == SG_GEMV && nx.qt != QT) {
                // the fp16 stream's ring slots differ from gq's: only after the whole CTA is done
                const GemvParams &np = nx.g;
                gf.prefetch(np, ring, cta, ncta);
                gf_ready = true;
            } else if (nx.type == SG_ATTN && cta < nx.nq * nx.a.hkv * nx.nsplit) {
                // K/V rows that earlier steps wrote (this step's row comes from the stage
                // that is ending, so it is loaded after the barrier)
                const FdParams &ap = nx.a;
                const int split = cta % nx.nsplit, rest = cta / nx.nsplit;
                fd_prefetch<HD, DS_THREADS>(ap, rest / ap.hkv, rest % ap.hkv, split, nx.nsplit, nx.a_new, ring);
            }
            nbar++;
            if (!ds_wait(plan.barrier, nbar * (unsigned)ncta, plan.err)) break;
        }
        if (cta == 0 && tid == 0 && plan.stamps) plan.stamps[s + 1] = globaltimer_ns();
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// ------------------------------------------------------------------- host

template <int QT, int MT, int HD>
static int ds_launch(const StepPlan &plan, size_t smem, cudaStream_t st)
{
    auto kern = decode_step_kernel<QT, MT, HD>;
    int rc = ensure_func_attrs((const void *)kern, (int)smem);
    if (rc) return rc;
    int per_sm = 0;
    DU_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, DS_THREADS, smem));
    if (per_sm < 1) return fail(DU_EINVAL, "decode step kernel does not fit on an SM");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, plan));
    return DU_OK;
}

template <int QT, int MT, int HD>
static size_t ds_static_smem()
{
    cudaFuncAttributes a = {};
    if (cudaFuncGetAttributes(&a, decode_step_kernel<QT, MT, HD>) != cudaSuccess) return (size_t)-1;
    return a.sharedSizeBytes;
}

size_t step_ring_bytes(int qt, int mt, int depth)
{
    const int rw = mt == 1 ? 4 : 2;
    const size_t slots = (size_t)DS_WARPS * depth * rw * 32;
    return slots * 16 + (qt == Q_I4 ? slots * 4 : 0);
}

#define DU_DS_CASES(X)                                                \
    X(Q_I4, 1, 128) X(Q_I4, 2, 128) X(Q_I4, 4, 128) X(Q_I4, 8, 128)   \
    X(Q_I8, 1, 128) X(Q_I8, 2, 128) X(Q_I8, 4, 128) X(Q_I8, 8, 128)   \
    X(Q_F16, 1, 128) X(Q_F16, 2, 128) X(Q_F16, 4, 128) X(Q_F16, 8, 128) \
    X(Q_I4, 1, 64) X(Q_I4, 2, 64) X(Q_I4, 4, 64) X(Q_I4, 8, 64)       \
    X(Q_I8, 1, 64) X(Q_I8, 2, 64) X(Q_I8, 4, 64) X(Q_I8, 8, 64)       \
    X(Q_F16, 1, 64) X(Q_F16, 2, 64) X(Q_F16, 4, 64) X(Q_F16, 8, 64)

size_t step_smem_limit(int qt, int mt, int hd)
{
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
    size_t stat = (size_t)-1;
#define DU_DS_STAT(Q, M_, H_) \
    if (qt == Q && mt == M_ && hd == H_) stat = ds_static_smem<Q, M_, H_>();
    DU_DS_CASES(DU_DS_STAT)
#undef DU_DS_STAT
    return stat < (size_t)optin ? (size_t)optin - stat : 0;
}

int launch_decode_step(const StepPlan &plan, int qt, int mt, int hd, size_t smem, cudaStream_t st)
{
    if (smem > step_smem_limit(qt, mt, hd)) return fail(DU_EINVAL, "decode step kernel: shared memory budget exceeded");
#define DU_DS_CASE(Q, M_, H_) \
    if (qt == Q && mt == M_ && hd == H_) return ds_launch<Q, M_, H_>(plan, smem, st);
    DU_DS_CASES(DU_DS_CASE)
#undef DU_DS_CASE
    return fail(DU_EINVAL, "decode step kernel: unsupported configuration");
}

}  // namespace du
