// step_plan.h -- stage list of the persistent decode-step kernel (decode_step.cu).
#pragma once

#include "attn_impl.cuh"
#include "gemv.cuh"

namespace du {

enum StageType { SG_EMBED = 0, SG_GEMV = 1, SG_ATTN = 2, SG_ARGMAX = 3 };

struct StepStage {
    int type;
    int qt;              // SG_GEMV: Q_I4 / Q_I8 / Q_F16
    GemvParams g;        // SG_GEMV
    FdParams a;          // SG_ATTN
    int G, nsplit, nq;   // SG_ATTN
    int a_new;           // SG_ATTN: K/V rows per query row written by this step (loaded after the barrier)
};

struct StepPlan {
    int nstages;
    const StepStage *stages;     // device array
    size_t ring_bytes;           // bytes of the ring / attention-tile region (the activation stage follows)
    // SG_EMBED
    const int *ids;
    const __half *embed;
    float embed_scale;
    int M, H;
    float *x_res;
    // SG_ARGMAX
    const float *am_val;
    const int *am_idx;
    int nparts;
    int *next_out, *feed, *hist, *cache_len;
    int cap;
    int advance;
    // grid barrier
    unsigned *barrier;
    int *err;
    // globaltimer (ns) when CTA 0 leaves each barrier: [0] kernel start, [s + 1] end of stage s
    unsigned long long *stamps;
};

// weight-ring depths of the persistent kernel: the model's linears per token
// tile, and the fp16 lm_head
#ifndef DU_STEP_RING_DEPTH
#define DU_STEP_RING_DEPTH 4
#endif
#ifndef DU_STEP_HEAD_DEPTH
#define DU_STEP_HEAD_DEPTH 4
#endif
__host__ __device__ constexpr int ds_depth(int) { return DU_STEP_RING_DEPTH; }
__host__ __device__ constexpr int ds_head_depth(int) { return DU_STEP_HEAD_DEPTH; }

size_t step_ring_bytes(int qt, int mt, int depth);
// dynamic shared memory the persistent kernel of this configuration can be given
size_t step_smem_limit(int qt, int mt, int hd);
int launch_decode_step(const StepPlan &plan, int qt, int mt, int hd, size_t smem, cudaStream_t st);

}  // namespace du
