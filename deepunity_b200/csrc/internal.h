// internal.h -- declarations shared by the library's translation units.
#pragma once

#include <cuda.h>

#include "../../include/deepunity_cuda.h"
#include "common.cuh"

namespace du {

struct GemvParams;

int num_sms();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device), thread-safe
int ensure_func_attrs(const void *kern, int smem_bytes, bool nonportable_cluster = false);

// gemv.cu
int launch_gemv(int qt, GemvParams p, cudaStream_t st);
size_t gemv_smem_bytes(int qt, int mt, int64_t row_bytes);
int gemv_ctas_per_sm(int qt, int mt, int64_t row_bytes);   // CTAs per SM of the launcher's layout
size_t gemv_x_bytes(int qt, int mt, int64_t row_bytes);     // activation stage of one CTA
int gemv_grid_for(int N, int M, int want);
void gemv_set_pdl(bool on);
bool pdl_enabled();

// gemm.cu: tensor-core dequant GEMM for M > 8 token rows (prefill chunks, large decode batches)
struct GemmScratch {
    __half *xh = nullptr, *xl = nullptr;   // [rows][K] staged activations (exact fp16 pairs)
    float *xscale = nullptr;               // [rows]
    size_t elems = 0, rows = 0;            // capacity: rows * K elements, rows
    int *err = nullptr;                    // device error word of the bounded waits (may be null)
    float *partials = nullptr;             // split-K partial tiles (may be null: no split)
    size_t partial_floats = 0;
    unsigned *counters = nullptr;          // one per (row tile, token tile), zero-initialised
    size_t counter_n = 0;
};
bool gemm_supported(int qt, const GemvParams &p);
int gemm_min_tokens();                      // smallest M routed to the GEMM (DU_GEMM_MIN_M, default 16)
// split-K scratch that serves every launch: two CTAs per SM of 128 x 128 partial tiles
constexpr size_t GEMM_PARTIAL_FLOATS_PER_SM = 2ull * 128 * 128;
int launch_gemm(int qt, const GemvParams &p, const GemmScratch &scr, cudaStream_t st);
// tgemv.cu: decode GEMV (M <= 2, INT4) on the tensor cores (tcgen05 kind::i8); shares the GEMM's
// split scratch (partials, counters)
bool tgemv_enabled();                        // DU_DECODE_GEMV=tcgen05 in the environment turns it on
bool tgemv_supported(int qt, const GemvParams &p);
int launch_tgemv(int qt, const GemvParams &p, const GemmScratch &scr, cudaStream_t st);
int launch_dequant_rows(int qt, const void *w, const void *scales, int scale_f32, int group, int64_t row0, int nrows,
                        int K, float *out, cudaStream_t st);

// attention.cu
int fd_choose_splits(int nq, int hkv, int max_kv);
size_t fd_scratch_floats(int nq, int hkv, int G, int hd, int nsplit);
int launch_flash_decode(const float *q, const __half *kc, const __half *vc, const int *seq_of,
                        const int *kv_len, int kv_len_add, int nq, int hq, int hkv, int hd, int cap,
                        float scale, float *out, float *scratch, unsigned *counters, int nsplit,
                        cudaStream_t st, int new_rows = -1);
// The model's path: splits of a (row, kv head) combined inside a thread-block cluster.
int launch_flash_decode_cluster(const float *q, const __half *kc, const __half *vc, const int *seq_of,
                                const int *kv_len, int kv_len_add, int nq, int hq, int hkv, int hd, int cap,
                                float scale, float *out, cudaStream_t st, int new_rows = -1,
                                const Kv8Cache *kv8 = nullptr, int window = 0);
// Flash-decode of one query row with the O projection fused after the cluster
// combine: resid += W_o . att (attention.cu).
struct FuseO {
    const uint8_t *w;            // W_o [H][hq * hd], INT4 or INT8
    const __half *scales;
    int quant, group, H;
    float *resid;                // [H]
    float *part;                 // [hkv][H] scratch
    unsigned *cnt;               // [16] arrivals, zero between launches
    int *err;
};
// 2-D tiled tensor map (row-major [rows][inner] elements of esize bytes; box
// [box_rows][box_inner]) through the driver's encoder (gemm.cu).
int make_tmap(CUtensorMap *tm, CUtensorMapDataType dt, int esize, const void *ptr, uint64_t inner, uint64_t rows,
              uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw);
bool flash_decode_fuse_o_supported(int nq, int hq, int hkv, int hd, int H, int quant, int group);
int launch_flash_decode_fuse_o(const float *q, const __half *kc, const __half *vc, const int *seq_of, const int *kv_len,
                               int kv_len_add, int hq, int hkv, int hd, int cap, float scale, float *att, cudaStream_t st,
                               int new_rows, const FuseO &o);
// INT8 KV: quantizes fp32 rows [M][nkv][hkv][hd] (nkv 2: K then V; 1: K only) into the
// cache at sequence seq_of[m] (or seq_off + m), position pos[m] (or pos_base + m).
int launch_kv_quant_int8(const float *stage, int M, int nkv, int hkv, int hd, const int *pos, int pos_base,
                         const int *seq_of, int seq_off, int cap, const Kv8Cache &kv, cudaStream_t st);

// elementwise.cu
// Gemma-style attention input: qk-norm + RoPE + cache write after an EPI_STORE QKV GEMV.
struct QkvPost {
    const float *qkv;                    // [M][hq + 2 hkv][hd], q heads then k heads then v heads
    int M, hq, hkv, hd;
    const __half *q_norm, *k_norm;       // gamma' [hd] (nullptr: no qk-norm)
    float eps;
    const int *pos, *seq_of;             // per token: cache slot / RoPE position, sequence (nullptr: seq_off + m)
    int seq_off, cap;
    const __half *rope_cos, *rope_sin;   // [cap][hd / 2]
    float *q_out;                        // [M][hq][hd]
    __half *k_cache, *v_cache;           // fp16 cache [seq][cap][hkv][hd], or
    Kv8Cache kv8;                        // the INT8 cache (kv8.k8 != nullptr)
    int gated;                           // q heads carry hd gate rows after their hd q rows
    float *gate_out;                     // gated: [M][hq][hd] gate values
    int rot;                             // rotated dims per head (0: hd)
};
int launch_qkv_post(const QkvPost &a, cudaStream_t st);
// att[i] *= sigmoid(gate[i]) (Qwen3.5 attention output gate)
int launch_attn_gate(float *att, const float *gate, size_t n, cudaStream_t st);
// x_res += y * rms(y) * (1 + gamma') per row (sandwich norm + residual)
int launch_norm_add(const float *y, const __half *gamma_m1, int rows, int H, float eps, float *x_res, cudaStream_t st);
int launch_embed(const int *ids, const __half *embed, float scale, int M, int H, float *out, cudaStream_t st);
int launch_rmsnorm(const float *x, const __half *gamma_m1, int rows, int H, float eps, float *y,
                   cudaStream_t st);
// Greedy-token history of the device-resident decode loop: the id chosen for
// sequence m is also written at tok[m * cap + cache_len[m]] (its input position).
struct TokHist {
    int *tok = nullptr;
    const int *cache_len = nullptr;
    int cap = 0;
};
int launch_argmax_final(const float *am_val, const int *am_idx, int M, int nparts, int *out_ids,
                        int *feed_ids, TokHist hist, cudaStream_t st);
int launch_argmax_final_pairs(const float *am_val, const int *am_idx, int M, int nparts, float *pairs,
                              cudaStream_t st);
int launch_argmax_pick_tp(const float *gpairs, int tp, int maxb, int M, int *out_ids, int *feed_ids,
                          TokHist hist, cudaStream_t st);
// sampler.cu: temperature / top-k / top-p / min-p sampling (or the greedy pick) per row of logits
bool sample_supported(float temperature, int top_k, float top_p, int V);
int launch_sample(const float *logits, int rows, int V, int ldl, float temperature, int top_k, float top_p,
                  float min_p, const int32_t *seeds, int32_t *out, int *feed, TokHist hist, int *err, cudaStream_t st,
                  const float *dparams);
// sampler.cu: repetition / presence penalty in place over rows of logits (in_ids: the step's
// input id per row counts as seen and is added to seen; dp: device (presence, repetition))
int launch_penalties(float *logits, int rows, int V, int ldl, unsigned *seen, int ld_seen, const int *in_ids,
                     const float *dp, float presence, float repetition, cudaStream_t st);
int launch_add_inplace(float *y, const float *x, size_t n, cudaStream_t st);
int launch_quantize_int8(const float *w, int64_t rows, int64_t cols, int8_t *q, __half *s, cudaStream_t st);
int launch_quantize_int4(const float *w, int64_t rows, int64_t cols, int group, uint8_t *p, __half *s,
                         cudaStream_t st);
int launch_random_normal(float *out, size_t n, uint64_t seed, uint64_t offset, float std, cudaStream_t st);
int launch_random_normal_half(__half *out, size_t n, uint64_t seed, uint64_t offset, float std,
                              cudaStream_t st);
int launch_fill_half(__half *out, size_t n, float v, cudaStream_t st);
int launch_convert_to_f32(const void *x, int dtype, size_t n, float *out, cudaStream_t st);
int launch_step_advance(int *cache_len, int M, cudaStream_t st);

// scratch owned by the library for kernel-level entry points (grow-only, per device)
void *device_scratch(size_t bytes, int slot);

}  // namespace du
