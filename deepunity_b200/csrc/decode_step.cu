// decode_step.cu -- persistent decode-step kernel.
//
// One cooperative launch runs a whole decode step (the reference dispatches
// ~389 shader dispatches per token, MiniCPM5Model.cs:294-674): one CTA per SM
// walks the stage list
//     embed, L x [QKV, attention, O, gate|up, down], lm_head, argmax
// with a grid barrier between stages.  Every GEMV stage is the same device
// code as the standalone GEMV kernel (gemv_impl.cuh), split into prefetch and
// run: before a CTA arrives at the barrier that ends stage s, each warp has
// already issued the first ring stages of its rows of stage s + 1, so HBM keeps
// streaming weights across the barrier and there is no kernel launch, ramp-up
// or tail between stages.  Attention units are the shared flash-decode unit
// (attn_impl.cuh) processed by the whole CTA.
//
// Barrier: a step-local counter (zeroed by a memset node before the kernel in
// the captured graph); thread 0 of each CTA publishes its writes
// (__threadfence), adds 1, and spins with acquire loads until the counter
// reaches (barrier index + 1) * gridDim.x.  The spin is bounded: after about a
// second it sets the error word, and every CTA then waits for its own cp.async
// copies and returns; the host reports DU_ECUDA.  Co-residency of all CTAs is
// guaranteed by the cooperative launch.
#include "attn_impl.cuh"
#include "gemv_impl.cuh"
#include "internal.h"
#include "step_plan.h"

namespace du {

constexpr int DS_THREADS = GV_THREADS;    // 8 warps
constexpr int DS_D = 4;                   // ring depth
constexpr unsigned DS_SPIN_LIMIT = 1u << 22;     // ~1-2 s of polling before giving up

__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool ds_grid_sync(unsigned *ctr, unsigned target, int *err)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctr, 1u);
        unsigned n = 0;
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
            if (v >= target) break;
            if (++n > DS_SPIN_LIMIT) {
                atomicExch(err, 1);
                break;
            }
            if (*(volatile int *)err) break;
            __nanosleep(40);
        }
        __threadfence();
    }
    __syncthreads();
    return *(volatile int *)err == 0;
}

template <int QT, int MT, int HD>
__global__ void __launch_bounds__(DS_THREADS, 1) decode_step_kernel(const StepPlan plan)
{
    constexpr int RW = MT == 1 ? 4 : 2;
    extern __shared__ __align__(16) unsigned char ds_smem[];
    __shared__ GemvShared<MT> gsh;
    __shared__ FdShared<HD> fsh;
    const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
    unsigned char *ring = ds_smem;
    unsigned char *xreg = ds_smem + plan.ring_bytes;       // activation stage / attention tiles

    GemvStream<QT, MT, RW, DS_D> gq;       // weight stream of the model's linears
    bool gq_ready = false;                 // gq holds the prefetched next stage
    unsigned nbar = 0;
    if (cta == 0 && tid == 0 && plan.stamps) plan.stamps[0] = globaltimer_ns();

    for (int s = 0; s < plan.nstages; s++) {
        const StepStage &st = plan.stages[s];
        const int type = st.type;
        if (type == SG_EMBED) {
            const size_t n = (size_t)plan.M * plan.H;
            for (size_t i = (size_t)cta * DS_THREADS + tid; i < n; i += (size_t)ncta * DS_THREADS) {
                const int m = (int)(i / plan.H), k = (int)(i - (size_t)m * plan.H);
                plan.x_res[i] = __half2float(plan.embed[(size_t)plan.ids[m] * plan.H + k]) * plan.embed_scale;
            }
        } else if (type == SG_GEMV) {
            const GemvParams gp = st.g;
            if (st.qt == QT) {
                if (!gq_ready) gq.prefetch(gp, ring, cta, ncta);
                gq.run(gp, xreg, gsh, cta, ncta, [] {});
                gq_ready = false;
            } else {
                GemvStream<Q_F16, MT, RW, DS_D> gf;
                gf.prefetch(gp, ring, cta, ncta);
                gf.run(gp, xreg, gsh, cta, ncta, [] {});
            }
        } else if (type == SG_ATTN) {
            const FdParams ap = st.a;
            const int units = st.nq * ap.hkv * st.nsplit;
            for (int u = cta; u < units; u += ncta) {
                const int split = u % st.nsplit, rest = u / st.nsplit;
                const int kvh = rest % ap.hkv, row = rest / ap.hkv;
                fd_unit<HD, DS_THREADS>(ap, st.G, row, kvh, split, st.nsplit, xreg, fsh);
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
                        if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
                    }
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                    }
                    if ((tid & 31) == 0) { gsh.amv[tid >> 5][0] = bv; gsh.ami[tid >> 5][0] = bi; }
                    __syncthreads();
                    if (tid == 0) {
                        bv = gsh.amv[0][0]; bi = gsh.ami[0][0];
                        for (int w = 1; w < GV_WARPS; w++)
                            if (gsh.amv[w][0] > bv || (gsh.amv[w][0] == bv && gsh.ami[w][0] < bi)) {
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
            const StepStage &nx = plan.stages[s + 1];
            if (nx.type == SG_GEMV && nx.qt == QT) {
                const GemvParams np = nx.g;
                gq.prefetch(np, ring, cta, ncta);      // weights only: safe before the barrier
                gq_ready = true;
            }
            nbar++;
            if (!ds_grid_sync(plan.barrier, nbar * (unsigned)ncta, plan.err)) break;
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
    static size_t attr_set[64] = {};        // dynamic smem already allowed, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_set[dev & 63] < smem) {
        DU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set[dev & 63] = smem;
    }
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

size_t step_ring_bytes(int qt, int mt)
{
    const int rw = mt == 1 ? 4 : 2;
    const size_t slots = (size_t)GV_WARPS * DS_D * rw * 32;
    return slots * 16 + (qt == Q_I4 ? slots * 4 : 0);
}

int launch_decode_step(const StepPlan &plan, int qt, int mt, int hd, size_t smem, cudaStream_t st)
{
    if (smem > 220 * 1024) return fail(DU_EINVAL, "decode step kernel: shared memory budget exceeded");
#define DU_DS_CASE(Q, M_, H_) \
    if (qt == Q && mt == M_ && hd == H_) return ds_launch<Q, M_, H_>(plan, smem, st);
    DU_DS_CASE(Q_I4, 1, 128) DU_DS_CASE(Q_I4, 2, 128) DU_DS_CASE(Q_I4, 4, 128) DU_DS_CASE(Q_I4, 8, 128)
    DU_DS_CASE(Q_I8, 1, 128) DU_DS_CASE(Q_I8, 2, 128) DU_DS_CASE(Q_I8, 4, 128) DU_DS_CASE(Q_I8, 8, 128)
    DU_DS_CASE(Q_F16, 1, 128) DU_DS_CASE(Q_F16, 2, 128) DU_DS_CASE(Q_F16, 4, 128) DU_DS_CASE(Q_F16, 8, 128)
    DU_DS_CASE(Q_I4, 1, 64) DU_DS_CASE(Q_I4, 2, 64) DU_DS_CASE(Q_I4, 4, 64) DU_DS_CASE(Q_I4, 8, 64)
    DU_DS_CASE(Q_I8, 1, 64) DU_DS_CASE(Q_I8, 2, 64) DU_DS_CASE(Q_I8, 4, 64) DU_DS_CASE(Q_I8, 8, 64)
    DU_DS_CASE(Q_F16, 1, 64) DU_DS_CASE(Q_F16, 2, 64) DU_DS_CASE(Q_F16, 4, 64) DU_DS_CASE(Q_F16, 8, 64)
#undef DU_DS_CASE
    return fail(DU_EINVAL, "decode step kernel: unsupported configuration");
}

}  // namespace du
