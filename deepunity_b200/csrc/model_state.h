// model_state.h -- the state of one model (weights, KV cache, scratch, captured
// graphs, tensor-parallel handles), shared by the executor (model.cu) and the
// KV snapshot / weight-folder I/O (snapshot.cu).
#pragma once

#include <atomic>
#include <map>
#include <vector>

#include "gemv.cuh"
#include "internal.h"
#include "nccl_shim.h"
#include "step_plan.h"
#include "tp_comm.h"

namespace du {

struct Layer {
    uint8_t *w_qkv = nullptr; __half *s_qkv = nullptr;    // [(hq+2hkv)*hd local rows, H]
    uint8_t *w_o = nullptr;   __half *s_o = nullptr;      // [H, hq_l*hd]
    uint8_t *w_gu = nullptr;  __half *s_gu = nullptr;     // gate|up [2*I_l, H]
    uint8_t *w_d = nullptr;   __half *s_d = nullptr;      // [H, I_l]
    __half *ln1 = nullptr, *ln2 = nullptr;                // gamma - 1, [H] (ln2: the pre-MLP norm)
    // Gemma3 variants: qk-norm gammas [hd]; sandwich norms after attention / the MLP [H]
    __half *q_norm = nullptr, *k_norm = nullptr;
    __half *post_attn = nullptr, *post_ffn = nullptr;
};

// Floats of sampler settings after the seeds: temperature, top_k, top_p, min_p,
// presence penalty, repetition penalty, two spare.
constexpr int SAMPLE_PARAMS = 8;

struct Graph {
    cudaGraph_t g = nullptr;
    cudaGraphExec_t exec = nullptr;
    StepStage *d_stages = nullptr;   // stage list of the persistent decode-step kernel (device)
    bool persistent = false;
};

}  // namespace du

struct du_model {
    du_model_config cfg;
    int device = 0;
    cudaStream_t stream = nullptr;
    int H, I, L, hq, hkv, hd, V, tp, rank;
    int hq_l, hkv_l, I_l, V_l, qkv_rows;
    int quant, group, cap, maxb;
    int max_tokens;                         // tokens per forward chunk (prefill)
    std::vector<du::Layer> layers;
    std::vector<void *> allocs;
    __half *final_norm = nullptr, *embed = nullptr, *lm_head = nullptr;
    __half *rope_cos = nullptr, *rope_sin = nullptr;
    __half *k_cache = nullptr, *v_cache = nullptr;      // [L][maxb][cap][hkv_l][hd]
    size_t kv_layer_elems = 0;
    bool kv8 = false;                                    // INT8 cache instead of the fp16 one:
    uint8_t *k8 = nullptr, *v8 = nullptr;                // [L][maxb][cap][hkv_l][hd]
    uint32_t *ksz = nullptr, *vsz = nullptr;             // [L][maxb][cap][hkv_l] scale | zp << 16
    float *kv_stage = nullptr;                           // QKV epilogue's fp32 K / V rows [T][2][hkv_l][hd]
    // Gemma3 variants (du_model_config.arch_flags / sliding_window)
    int arch = 0, window = 0, pattern = 0;
    float attn_scale = 0.0f;                             // softmax scale
    __half *rope_cos_local = nullptr, *rope_sin_local = nullptr;   // RoPE of the sliding-window layers
    float *qkv_buf = nullptr;                            // qk-norm models: QKV GEMV output [T][qkv_rows]
    float *gate_buf = nullptr;                           // DU_ARCH_ATTN_GATE: attention output gates [T][hq_l][hd]
    bool fuse_o = false;                                 // one-row decode: O projection inside flash-decode
    float *o_part = nullptr; unsigned *o_cnt = nullptr;  // its per-kv-head partial sums and arrival counters
    // device state
    int *d_cache_len = nullptr;             // [maxb]
    int *d_ids = nullptr;                   // [max_tokens] input ids
    int *d_next = nullptr;                  // [max_tokens] greedy ids
    int *d_hist = nullptr;                  // [maxb][cap] greedy id chosen at each input position
    int *d_pos = nullptr, *d_seq = nullptr, *d_kvlen = nullptr;   // per-token (prefill)
    float *x_res = nullptr;                 // [max_tokens][H]
    float *part = nullptr;                  // [max_tokens][H] TP partial sums
    float *q = nullptr;                     // [max_tokens][hq_l*hd]
    float *att = nullptr;                   // [max_tokens][hq_l*hd]
    float *inter = nullptr;                 // [max_tokens][I_l]
    float *logits = nullptr;                // [maxb][V_l] local shard
    float *logits_all = nullptr;            // [tp][maxb][V_l] (TP gather)
    float *am_val = nullptr; int *am_idx = nullptr;   // [maxb][am_parts]
    float *best_val = nullptr; int *best_idx = nullptr;  // TP: [maxb] local, [tp][maxb] gathered
    float *gbest_val = nullptr; int *gbest_idx = nullptr;
    int am_parts = 0;
    du::GemmScratch gm;                     // staged activations of the tensor-core GEMM (M >= 16 rows)
    float *fd_scratch = nullptr; unsigned *fd_counters = nullptr;
    int fd_nsplit_decode = 1;
    size_t fd_scratch_fl = 0;
    int *h_pin_ids = nullptr, *h_pin_next = nullptr;
    unsigned *d_barrier = nullptr;          // grid-barrier counter of the persistent step kernel
    int *d_err = nullptr;                   // its error word (barrier timeout)
    int *h_pin_err = nullptr;
    unsigned long long *d_stamps = nullptr; // per-stage timestamps of the last persistent step
    int stamp_stages = 0;                   // stages of the step that wrote them
    std::vector<int> h_cache_len;
    std::map<int, du::Graph> graphs;        // greedy decode step per batch size
    std::map<int, du::Graph> sgraphs;       // sampling decode step per batch size
    std::map<int, du::Graph> pgraphs;       // sampling decode step with repetition / presence penalty
    int32_t *d_seeds = nullptr;             // [maxb] sampler seeds of the next step
    float *d_sparams = nullptr;             // (temperature, top_k, top_p, min_p, presence, repetition) of the next
                                            // sampling step
    int32_t *h_pin_seeds = nullptr;         // pinned staging: [maxb] seeds then SAMPLE_PARAMS floats of settings
    unsigned *d_seen = nullptr;             // [maxb][V] ids seen per sequence since the last cache reset
                                            // (single GPU; the penalties' token_seen)
    int last_batch = 0, last_rows = 0;      // rows of logits written by the last call
    std::atomic<int> busy{0};
    // TP
    ncclComm_t comm = nullptr;
    bool tp_ready = false;
    du::TpComm tpc;                         // peer-memory allreduce of decode-sized reductions
    int nccl_timeout_ms = 60000;
    uint64_t weight_bytes = 0;
};

namespace du {

// One C-ABI call at a time per model (the reference's LLM.Busy guard); sets the
// model's device for the call.
struct CallGuard {
    du_model *m;
    bool ok;
    explicit CallGuard(du_model *mm) : m(mm), ok(false)
    {
        if (m && m->busy.exchange(1) == 0) {
            ok = true;
            cudaSetDevice(m->device);
        }
    }
    ~CallGuard()
    {
        if (ok) m->busy.store(0);
    }
};

#define DU_GUARD(m)                                                                   \
    if (!(m)) return fail(DU_EINVAL, "null model handle");                            \
    CallGuard _guard(m);                                                              \
    if (!_guard.ok) return fail(DU_EBUSY, "model is busy with another call")


// Copies the host cache lengths to the device (stream-ordered).
int sync_cache_len(du_model *m);

}  // namespace du
