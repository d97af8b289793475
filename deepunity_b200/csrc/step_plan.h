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
};

struct StepPlan {
    int nstages;
    const StepStage *stages;     // device array
    size_t ring_bytes;           // offset of the activation / attention-tile region
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

size_t step_ring_bytes(int qt, int mt);
int launch_decode_step(const StepPlan &plan, int qt, int mt, int hd, size_t smem, cudaStream_t st);

}  // namespace du
