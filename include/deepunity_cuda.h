/*
 * deepunity_cuda.h -- C ABI of libdeepunity_cuda.so, the B200 (sm_100a)
 * library behind DeepUnity's quantized llama decode path.
 *
 * Every call returns an int status: 0 = OK, otherwise a DU_E* code, with a
 * message from du_last_error() (thread-local).  Opaque handles; the library
 * owns all device memory it allocates, the caller owns host buffers.  One CUDA
 * stream per model.  A handle is not re-entrant (the reference's Busy guard,
 * LLM.cs:393-406, becomes DU_EBUSY); different handles are independent.
 * Kernel-level entry points take device pointers and a cudaStream_t passed as
 * void* (NULL = the legacy default stream).
 *
 * Reference paths are relative to the DeepUnity project root:
 *   G3CS = Assets/Resources/ComputeShaders/Gemma3CS.compute
 *   M5M  = Assets/DeepUnity/InferenceEngine/LLM/MiniCPM5/MiniCPM5Model.cs
 *   M5W  = Assets/DeepUnity/InferenceEngine/LLM/MiniCPM5/MiniCPM5Weights.cs
 *   M5C  = Assets/DeepUnity/InferenceEngine/LLM/MiniCPM5/MiniCPM5Cache.cs
 *   LLMB = Assets/DeepUnity/InferenceEngine/LLM/Base/
 *   IMP  = Assets/DeepUnity/InferenceEngine/import_params.py
 */
#ifndef DEEPUNITY_CUDA_H
#define DEEPUNITY_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DU_API __attribute__((visibility("default")))

enum {
    DU_OK = 0,
    DU_EINVAL = 1,     /* bad argument (shape, id >= vocab, position >= capacity, ...) */
    DU_ECUDA = 2,      /* CUDA runtime error */
    DU_ENOMEM = 3,     /* device allocation failed */
    DU_EBUSY = 4,      /* handle already inside a call (reference Busy guard) */
    DU_ENCCL = 5,      /* NCCL error or collective timeout */
    DU_ENOTFOUND = 6,  /* unknown tensor name */
    DU_ESTATE = 7,     /* call not valid in the current state */
    DU_EIO = 8         /* file or directory error */
};

/* Weight formats of IMP (LLMQuant, LLMB/LLM.cs:15-59). */
enum { DU_QUANT_FP16 = 0, DU_QUANT_INT8 = 1, DU_QUANT_INT4 = 2 };
/* Element types for kernel-level activations. */
enum { DU_DTYPE_F32 = 0, DU_DTYPE_F16 = 1, DU_DTYPE_BF16 = 2 };

/* Architecture + runtime configuration; replaces the static MiniCPM5Config
 * constants (M5/MiniCPM5Config.cs:11-37) and the LLMQuant/KVQuant keywords. */
typedef struct du_model_config {
    int32_t hidden_size;
    int32_t intermediate_size;
    int32_t num_layers;
    int32_t num_heads_q;
    int32_t num_heads_kv;
    int32_t head_dim;
    int32_t vocab_size;
    float rms_eps;
    float rope_theta;
    float embed_scale;       /* 1.0 for llama (M5M:588) */
    int32_t quant;           /* DU_QUANT_* for the block linears */
    int32_t group_size;      /* INT4 group: 32 = reference Q4_0 (IMP:78), 128 = baseline */
    int32_t kv_capacity;     /* tokens per sequence (M5C ctor) */
    int32_t max_batch;       /* sequences decoded together */
    int32_t tp_rank;         /* tensor-parallel rank / size (1 = single GPU) */
    int32_t tp_size;
    int32_t tie_embedding;   /* 1: lm_head = embedding */
    int32_t flags;           /* DU_FLAG_* */
    int32_t kv_quant;        /* DU_KV_FP16 (0 or 1) or DU_KV_INT8 (KVQuant, LLM/Base/LLM.cs:15-87) */
    /* Gemma3 variants on the same kernels (Gemma3Model.cs:315-590); all 0 for llama */
    int32_t arch_flags;      /* DU_ARCH_* */
    int32_t sliding_window;  /* > 0: sliding-window layers see positions abs_q - window .. abs_q (G3CS:673-686) */
    int32_t sliding_pattern; /* every sliding_pattern-th layer (1-based) is full attention; <= 0: none */
    float rope_theta_local;  /* RoPE base of the sliding-window layers (0: rope_theta) */
    float attn_scale;        /* softmax scale (0: head_dim^-0.5; Gemma3: query_pre_attn_scalar^-0.5) */
    int32_t rope_rot_dim;    /* rotated dims per head (0: head_dim); < head_dim needs DU_ARCH_QK_NORM
                                (Qwen3.5 partial RoPE, Qwen3_5CS.compute:367-393) */
    int32_t reserved[1];
} du_model_config;

/* du_model_config.arch_flags */
enum {
    DU_ARCH_QK_NORM = 1,     /* RmsNormHead on q and k before RoPE (G3CS:227-245); tensors
                                layer_<i>/self_attn_q_norm.bin, self_attn_k_norm.bin [head_dim] */
    DU_ARCH_SANDWICH = 2,    /* post-attention and post-FFN RMSNorm before each residual add;
                                layer_<i>/post_attention_layernorm.bin is then the post-attention
                                norm, pre_feedforward_layernorm.bin the pre-MLP one and
                                post_feedforward_layernorm.bin the post-FFN one */
    DU_ARCH_GELU = 4,        /* GLU activation gelu (tanh form, G3CS:162-172) instead of SiLU */
    DU_ARCH_ATTN_GATE = 8    /* Qwen3.5 full-attention layers (Qwen3_5Model.cs:397-574): the q
                                projection holds, per head, head_dim q rows then head_dim gate rows
                                (QProjGated, Qwen3_5CS.compute:306-330), and the attention output
                                is multiplied by sigmoid(gate) before o_proj (ApplyAttnGate,
                                :706-714).  Needs DU_ARCH_QK_NORM and tp_size 1 */
};

/* du_model_config.kv_quant */
enum {
    DU_KV_FP16 = 1,   /* fp16 cache (0 selects it too) */
    DU_KV_INT8 = 2    /* asymmetric uint8 rows + per-(position, kv head) fp16 scale / zero point
                         (WriteCacheFull KV_INT8, G3CS:300-380); the per-stage decode graph */
};

/* du_model_config.flags */
enum {
    DU_FLAG_NO_PERSISTENT = 1,  /* decode steps as a graph of per-stage kernels (the default) */
    DU_FLAG_PERSISTENT = 2      /* decode steps as one persistent decode-step kernel (single GPU,
                                   batch <= 8, when its shared-memory plan fits; else per-stage) */
};

typedef struct du_model du_model;

/* ---------------------------------------------------------------- runtime */

/* Message for the last failing call on this thread. */
DU_API const char *du_last_error(void);
/* Library version string. */
DU_API const char *du_version(void);
/* Selects and initialises a device; replaces the shader-asset lookup
 * DeepUnityMeta.Gemma3CS (Assets/DeepUnity/Main/DeepUnityMeta.cs:25). */
DU_API int du_init(int device_ordinal);

/* ------------------------------------------------------------------ model */

/* Allocates weights, KV cache and scratch for one model (MiniCPM5Model ctor,
 * M5M:79-118, + MiniCPM5Cache ctor, M5C:34-72).  RoPE tables are built on the
 * host with the reference formula (M5M:163-191) and uploaded. */
DU_API int du_model_create(const du_model_config *cfg, du_model **out);

/* Copies one tensor of an IMP export from host memory into the model, in the
 * concatenated device layout of AddConcatW (M5W:139-191); with tp_size > 1
 * only this rank's shard is kept.  Names follow IMP's file layout (IMP:40-60,
 * 305-337): "norm.bin", "embed_tokens/part_<k>.bin", "lm_head/part_<k>.bin",
 * "layer_<i>/input_layernorm.bin", "layer_<i>/post_attention_layernorm.bin",
 * "layer_<i>/<self_attn_q_proj|..|mlp_down_proj>.<int8|int4>.bin",
 * "layer_<i>/<...>.scales.bin", fp16 linears as "layer_<i>/<...>.bin".
 * `bytes` must equal the file size.  Replaces MiniCPM5Weights' UploadPump
 * (M5W:315-380). */
DU_API int du_model_load_tensor(du_model *m, const char *name, const void *host, size_t bytes);

/* Fills every weight with seeded synthetic values on the device: linears
 * ~N(0, std) quantized with the IMP formulas, embedding / lm_head fp16
 * ~N(0, std), norm gammas 1 (stored as gamma - 1 = 0, IMP:314-315).  No
 * reference counterpart: stands in for a checkpoint when none exists. */
/* Loads every "*.bin" tensor of an import_params.py export folder (IMP's file
 * layout, see du_model_load_tensor), memory-mapped and placed by its path
 * relative to `folder`; replaces MiniCPM5Weights' upload pump (M5W:315-380).
 * n_files (optional) receives the number of tensors loaded. */
DU_API int du_model_load_folder(du_model *m, const char *folder, int *n_files);

DU_API int du_model_init_random(du_model *m, uint64_t seed, float std);

/* Writes a 128-byte NCCL unique id (call on rank 0, share with the others). */
DU_API int du_nccl_unique_id(void *out128);
/* Joins a tensor-parallel group of cfg.tp_size ranks (no reference
 * counterpart: the reference is single-GPU).  Non-blocking communicator
 * polled against timeout_ms. */
DU_API int du_tp_init(du_model *m, const void *nccl_unique_id, int timeout_ms);
/* Optional, after du_tp_init and before the first decode step (no reference
 * counterpart).  du_tp_comm_handle writes this rank's 64-byte CUDA IPC handle of
 * its peer-communication buffer; once every rank has every handle,
 * du_tp_comm_open(m, handles, tp_size) -- handles in rank order -- maps the
 * peers' buffers, and the decode graphs then reduce o_proj / down_proj partial
 * sums with a one-shot NVLink peer-memory allreduce instead of ncclAllReduce
 * (prefill keeps NCCL).  All ranks must open, or none. */
DU_API int du_tp_comm_handle(du_model *m, void *handle_out64);
DU_API int du_tp_comm_open(du_model *m, const void *handles, int nranks);
/* The peer-memory reduction waits for every rank's values with a bounded spin
 * (DU_TP_SPIN_LIMIT polls per value when set in the environment before
 * du_tp_comm_open, else about 2^24).  A wait that runs out sets the model's
 * error word, the kernels finish without the missing values, and the decode
 * call returns DU_ECUDA.  The ranks' residual streams and KV caches then
 * disagree for that step: destroy the models and build the group again.
 *
 * du_tp_wait_selftest (no reference counterpart) checks that bound on one GPU:
 * it runs the reduction kernel as rank 0 of a two-rank group in which no rank
 * 1 exists, with spin_limit polls per wait; *timed_out receives the error word
 * the host reads back (1 when the waits ran out, as they must). */
DU_API int du_tp_wait_selftest(unsigned spin_limit, int *timed_out);

/* Host-only (no device work): the slice of a global tensor that rank
 * cfg->tp_rank keeps.  tensor is a stem of IMP's file names
 * ("self_attn_q_proj", ..., "mlp_down_proj") or "lm_head"; out6 = {rows, cols,
 * r0, r1, c0, c1}: the global shape and the kept window [r0, r1) x [c0, c1).
 * No reference counterpart (the reference is single-GPU). */
DU_API int du_tp_shard_window(const du_model_config *cfg, const char *tensor, int64_t *out6);

/* MiniCPM5Model.Forward(ids, useCache, lastPosOnly) (M5M:531-549): runs
 * `seq_len` tokens of each of `batch` sequences (ids [batch, seq_len], host),
 * appending to the KV cache when use_cache != 0.  logits_out (host, may be
 * NULL): [batch, V] if last_pos_only else [batch, seq_len, V]; with TP each
 * rank receives the full vocab.  next_ids_out (host, may be NULL): greedy
 * argmax of the last position per sequence (ArgMax, G3CS:911-928). */
DU_API int du_forward(du_model *m, const int32_t *ids, int batch, int seq_len, int use_cache,
                      int last_pos_only, float *logits_out, int32_t *next_ids_out);

/* One greedy decode step for `batch` sequences (LLM.Generate inner loop:
 * M5/MiniCPM5.cs:152-166 -> ForwardYielding + SampleYielding, M5M:551-585,
 * 690-705): ids [batch] host in, next_ids [batch] host out.  The step is a
 * CUDA graph replay; the first call per batch size captures it. */
DU_API int du_decode_step(du_model *m, const int32_t *ids, int batch, int32_t *next_ids);

/* One sampled decode step: SampleYielding with temperature / top_k / top_p /
 * min_p (M5M:653-705 -> SampleToken / SampleTokenSerial, G3CS:932-1132).
 * seeds (host) [batch]: the sampler's signed 32-bit seed per sequence (the
 * reference draws one per step from UnityEngine.Random); the draw is
 * runif(seed) (G3CS:177-186).  temperature <= 0 is the greedy pick.  top_k in
 * 1..64 uses the reference's parallel sampler (probabilities over the full
 * vocabulary, candidates = the top_k logits); top_k <= 0 with top_p >= 1 the
 * full-vocabulary sampler with an index-order draw; top_p < 1 without a top_k
 * in 1..64 returns DU_EINVAL.  Single GPU (tp_size 1).  The step is a CUDA graph
 * (one per batch size) whose settings and seeds live in device memory. */
DU_API int du_decode_step_sample(du_model *m, const int32_t *ids, int batch, float temperature, int top_k,
                                 float top_p, float min_p, const int32_t *seeds, int32_t *next_ids);

/* du_decode_step_sample with the repetition and presence penalties of
 * DispatchSampleKernels (Qwen3_5/Qwen3_5Model.cs:1010-1058 ->
 * ApplyRepetitionPresencePenalty, MarkSampledTokenSeen, Qwen3_5CS.compute:1417-1441):
 * before the pick (greedy when temperature <= 0), every id already seen in the
 * sequence has its logit l replaced by (l > 0 ? l / repetition_penalty :
 * l * repetition_penalty) - presence_penalty, once per id whatever its count.
 * The ids seen are those fed to this entry point's steps since the last
 * du_reset_cache (ZeroTokenSeen), this step's ids included: each is the previous
 * step's pick, which the reference marks right after picking it.  (1, 0) are
 * no-ops.  repetition_penalty must be > 0.  Single GPU; its own captured graph
 * per batch size. */
DU_API int du_decode_step_sample_ex(du_model *m, const int32_t *ids, int batch, float temperature, int top_k,
                                    float top_p, float min_p, float presence_penalty, float repetition_penalty,
                                    const int32_t *seeds, int32_t *next_ids);

/* Device-resident greedy loop: n_steps decode steps, each feeding its argmax
 * into the next, without host round trips; tokens_out (host) [n_steps, batch].
 * ids (host) [batch] seeds the first step. */
DU_API int du_decode_loop(du_model *m, const int32_t *ids, int batch, int n_steps,
                          int32_t *tokens_out);

/* Logits of the last forward / decode step: [batch, V] fp32 (host). */
DU_API int du_read_logits(du_model *m, float *host_out, int batch);

/* MiniCPM5Model.ResetCache (M5M:714) / CachedTokenCount (M5C:16-22). */
DU_API int du_reset_cache(du_model *m);

/* KV snapshots of sequence `seq` (system-prompt / conversation reuse).
 * du_model_save_cache / du_model_load_cache: MiniCPM5Cache's "M5KV" version-1
 * folder (M5C:31-32, 78-200): meta.bin (int32 magic 0x4D354B56, version 1,
 * layers, kv heads, head_dim, tokens) and k_cache_layer_<i>.bin /
 * v_cache_layer_<i>.bin (tokens x kv heads x head_dim fp16, position-major).
 * Loading converts as the reference reader does (fp16 subnormals -> 0) and sets
 * the sequence's cache length; *loaded = 0 (not an error) on any mismatch, a
 * missing or short file, or with the INT8 cache (not kept in this format; its
 * save returns DU_ESTATE).  Nothing cached: the save writes nothing. */
DU_API int du_model_save_cache(du_model *m, int seq, const char *folder);
DU_API int du_model_load_cache(du_model *m, int seq, const char *folder, int *loaded);
/* One-file snapshot with the reference's version-2 prompt-cache layout
 * (Qwen3_5Cache.cs:149-170) for all-full-attention layers: magic 'LMKV',
 * version 2, uint64 context hash, uint8 kv format (DU_KV_*), tokens, layers,
 * caller bytes (`extra`), then per layer the K and V rows (+ the INT8 scale /
 * zero-point words).  Written to <path>.tmp and renamed.  The load checks hash,
 * format, layer count and every blob size before uploading; *loaded = 0 on any
 * mismatch.  du_kv_file_peek reads the header (and the caller bytes when
 * extra_cap suffices) without a model, so a caller can veto a restore first. */
DU_API int du_model_save_kv(du_model *m, int seq, const char *path, uint64_t context_hash, const void *extra,
                            int extra_len);
DU_API int du_model_load_kv(du_model *m, int seq, const char *path, uint64_t expected_hash, int *loaded);
DU_API int du_kv_file_peek(const char *path, int *valid, uint64_t *context_hash, int *kv_format, int *tokens,
                           int *layers, void *extra_out, int extra_cap, int *extra_len);
DU_API int du_cache_len(du_model *m, int seq, int *out);
/* Model stream (cudaStream_t) for callers that chain their own work. */
DU_API int du_model_stream(du_model *m, void **stream_out);
/* Bytes of weights resident on this rank (for roofline accounting). */
DU_API int du_model_weight_bytes(du_model *m, uint64_t *out);
/* Idempotent release (LLM.Release, LLMB/LLM.cs:654-655). */
DU_API int du_model_destroy(du_model *m);

/* Measurement hooks (the role of the reference's StageProfile,
 * LLM/Gemma3/Gemma3Model.cs:593-622, without its per-stage readbacks).
 * du_model_graph_info: kernel nodes / all nodes of the decode-step graph for
 * `batch` (captured on first use).  du_model_kernel_times: replays each of the
 * per-layer stages (0 QKV, 1 attention, 2 O proj, 3 gate|up, 4 down, 5 lm_head)
 * over every layer `reps` times on the model stream, timed with CUDA events;
 * ms_out[6] = average milliseconds per launch.  Valid after a prefill; it
 * rewrites the KV slot of the next position, which the next decode step
 * overwrites anyway. */
DU_API int du_model_graph_info(du_model *m, int batch, int *kernel_nodes, int *total_nodes);
/* Stage durations (microseconds, between consecutive grid-barrier exits of
 * CTA 0) of the most recent decode step that ran as the persistent decode-step
 * kernel: embed, then per layer QKV, attention, O, gate|up, down, then lm_head
 * and argmax.  n_out = stages written (0 if no persistent step ran). */
DU_API int du_model_stage_times(du_model *m, float *us_out, int max_stages, int *n_out);
DU_API int du_model_kernel_times(du_model *m, int batch, int reps, float *ms_out);

/* ------------------------------------------------ kernel-level entry points
 * Used by tests/benchmarks and by the secondary dispatch sites
 * (Dense.Predict's Device.GPU branch, Modules/Learnable/Dense.cs:88-132).
 * All pointers are device pointers. */

/* y[M, N] fp32 = x[M, K] (x_dtype) . W^T with W int8 [N, K] (row-major bytes,
 * IMP:229-233) and per-row scales (scale_dtype F16 as exported, or F32), the
 * scale applied once after the dot (QKVProj1VecCoal etc., G3CS:1217-1282). */
DU_API int du_gemv_q8(float *y, const void *x, int x_dtype, const int8_t *w, const void *scales,
                      int scale_dtype, int M, int N, int K, void *stream);
/* Same for INT4: packed nibbles [N, K/2] (low nibble = even column) and fp16
 * group scales [N, K/group] (IMP:236-248; readQ4, G3CS:84-101). */
DU_API int du_gemv_q4(float *y, const void *x, int x_dtype, const uint8_t *w,
                      const uint16_t *scales_f16, int group, int M, int N, int K, void *stream);
/* fp16 weights [N, K] (LmHeadPredict1VecCoal, G3CS:1284-1302). */
DU_API int du_gemv_f16(float *y, const void *x, int x_dtype, const uint16_t *w, int M, int N, int K,
                       void *stream);
/* The three entry points above run the decode GEMV for M < 16 token rows and
 * the tensor-core GEMM (tcgen05; the role of the *GemmCoal kernels,
 * G3CS:1304-1439) for M >= 16 when K is a multiple of 64 (DU_GEMM_MIN_M in the
 * environment moves the threshold).  The GEMM keeps fp32 accuracy: weights and
 * activations enter the tensor cores as exact fp16 hi + lo pairs. */

/* The weight values the tensor-core GEMM multiplies, as fp32, for rows
 * [row0, row0 + nrows) of a weight matrix [N, K] (readQ4 / readQ8 / readH and
 * wScale, G3CS:49-101): INT4 (n - 8) * d from the unpack's exact fp16 pair,
 * INT8 q * row scale (scale_dtype F16 or F32), fp16 as stored.  out [nrows, K]
 * fp32 (device).  quant: DU_QUANT_*; group: INT4 group size. */
DU_API int du_dequant(float *out, const void *w, const void *scales, int quant, int scale_dtype, int group,
                      int64_t row0, int nrows, int K, void *stream);

/* Split-K flash-decode (FlashAttention, G3CS:643-753) for one new query per
 * sequence: q fp32 [batch, hq, hd] (already roped, unscaled); caches fp16
 * [batch, capacity, hkv, hd] (position-major as KVCache.hlsl); kv_len int32
 * [batch] device; out fp32 [batch, hq, hd].  scale = 1/sqrt(hd) in the ref. */
DU_API int du_flash_decode(float *out, const float *q, const uint16_t *k_cache,
                           const uint16_t *v_cache, const int32_t *kv_len, int batch, int hq,
                           int hkv, int hd, int capacity, float scale, void *stream);

/* INT8 KV cache (KVQuant.INT8; WriteCacheFull's KV_INT8 variant, G3CS:300-380,
 * layout KVCache.hlsl:46-82): quantizes kv_new fp32 [seq_len, hkv, hd] (device)
 * into rows cache_len .. cache_len + seq_len - 1 of one sequence's cache: uint8
 * [capacity, hkv, hd] plus one word per (position, kv head), fp16 scale | fp16
 * zero point << 16, in sz [capacity, hkv].  Per row: scale = (max - min) / 255
 * (at least 1e-9), zp = round(-min / scale) clamped to [0, 255], q = clamp(round(
 * x / scale) + zp, 0, 255), round half to even.  hd a multiple of 32, <= 256. */
DU_API int du_kv_write_int8(const float *kv_new, int seq_len, int hkv, int hd, int cache_len, uint8_t *cache,
                            uint32_t *sz, void *stream);
/* du_flash_decode over INT8 caches: k8 / v8 uint8 [batch, capacity, hkv, hd],
 * ksz / vsz words [batch, capacity, hkv]; a cached value is (q - zp) * scale
 * (kv_unpack8, KVCache.hlsl:55-62).  hd 64 or 128. */
DU_API int du_flash_decode_kv8(float *out, const float *q, const uint8_t *k8, const uint32_t *ksz, const uint8_t *v8,
                               const uint32_t *vsz, const int32_t *kv_len, int batch, int hq, int hkv, int hd,
                               int capacity, float scale, void *stream);

/* du_flash_decode with a sliding window (Gemma3 sliding-window layers, G3CS:673-686):
 * the query of a sequence with kv_len positions sees positions kv_len - 1 - window
 * .. kv_len - 1 (all of them when window <= 0).  hd 64, 128 or 256. */
DU_API int du_flash_decode_window(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                  const int32_t *kv_len, int batch, int hq, int hkv, int hd, int capacity, float scale,
                                  int window, void *stream);

/* Same computation as du_flash_decode, but it allocates nothing: for callers
 * that must not call cudaMalloc / cudaFree, such as a game engine plugin
 * running on the engine's render or job thread (the engine owns the GPU memory
 * budget, and allocation can synchronise the whole device mid-frame).  No
 * counterpart in the reference.  Its scratch is a fixed device array of
 * 1048576 floats plus 8192 split counters (about 4 MiB), held by every GPU that
 * loads the library until exit; calls needing more (batch * num_heads_q *
 * (head_dim + 2) > 1048576, or batch * num_heads_kv > 8192) fail with DU_EINVAL.
 * The split count is reduced to fit the array.  The first call on a device
 * resolves the array's device address (cudaGetSymbolAddress) for that device;
 * make that first call before any stream capture.  The resolved address is
 * cached for the life of the process and does not survive cudaDeviceReset: do
 * not call this entry point on a device after resetting it.  Every call shares
 * the array and clears its counters first; calls whose kernels overlap on the
 * GPU race.  head_dim must be 64 or 128 and num_heads_q / num_heads_kv at most
 * 8 (DU_EINVAL otherwise). */
DU_API int du_flash_decode_noalloc(float *out, const float *q, const uint16_t *k_cache,
                                   const uint16_t *v_cache, const int32_t *kv_len, int batch, int hq,
                                   int hkv, int hd, int capacity, float scale, void *stream);

/* IMP quantizers on the device, bit-exact with quantize_int8 / quantize_int4
 * (IMP:229-248); group is a parameter (reference G4 = 32). */
DU_API int du_quantize_int8(const float *w, int64_t rows, int64_t cols, int8_t *q,
                            uint16_t *scales_f16, void *stream);
DU_API int du_quantize_int4(const float *w, int64_t rows, int64_t cols, int group,
                            uint8_t *packed, uint16_t *scales_f16, void *stream);

/* Sampler over rows of logits already on the device (SampleToken /
 * SampleTokenSerial, G3CS:932-1132; ArgMax when temperature <= 0): logits
 * [rows][ldl] fp32, seeds [rows] int32, out [rows] int32 (device).  Same
 * settings rules as du_decode_step_sample. */
DU_API int du_sample(int32_t *out, const float *logits, int rows, int vocab, int ldl, float temperature, int top_k,
                     float top_p, float min_p, const int32_t *seeds, void *stream);

/* ApplyRepetitionPresencePenalty (Qwen3_5CS.compute:1421-1433) in place over rows
 * of device logits [rows][ldl]: for each id with seen[r][id] != 0 (counts,
 * [rows][ld_seen] uint32, device), l = (l > 0 ? l / repetition_penalty :
 * l * repetition_penalty) - presence_penalty.  repetition_penalty must be > 0. */
DU_API int du_apply_penalties(float *logits, int rows, int vocab, int ldl, const uint32_t *seen, int ld_seen,
                              float presence_penalty, float repetition_penalty, void *stream);

/* MarkSampledTokenSeen (Qwen3_5CS.compute:1436-1441) for several rows:
 * seen[r][ids[r]] += 1 (device arrays; ids outside [0, vocab) are skipped).
 * ZeroTokenSeen (:1443-1451) is a memset of seen. */
DU_API int du_mark_seen(uint32_t *seen, int rows, int ld_seen, int vocab, const int32_t *ids, void *stream);

/* RmsNormHidden (G3CS:204-223): y = x * rsqrt(mean(x^2) + eps) * (1 + gamma_m1). */
DU_API int du_rmsnorm(float *y, const float *x, const uint16_t *gamma_m1, int rows, int H, float eps,
                      void *stream);

#ifdef __cplusplus
}
#endif

#endif /* DEEPUNITY_CUDA_H */
