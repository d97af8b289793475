// model.cu -- the decode executor: weights, KV cache, per-step launch
// sequence, CUDA-graph capture and tensor parallelism.
//
// Replaces MiniCPM5Model (InferenceEngine/LLM/MiniCPM5/MiniCPM5Model.cs): the
// 16 dispatches per layer of DispatchLayer (:294-518) become 5 fused kernels
//   1. QKV GEMV  <- RMSNorm(ln1) prologue, split + RoPE + fp16 KV-write epilogue
//   2. flash-decode (split-K, GQA) with the LSE combine
//   3. O GEMV    -> residual add (TP1) / partial sum + NCCL allreduce (TP>1)
//   4. gate|up GEMV <- RMSNorm(ln2) prologue, SiLU(g) * u epilogue
//   5. down GEMV -> residual add / allreduce
// plus embedding gather, the final RMSNorm + lm_head GEMV with per-CTA argmax
// partials, and the greedy pick.  A decode step is captured once per batch
// size as a CUDA graph; positions and KV lengths live in device memory, so
// the same graph replays for every step.
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <chrono>
#include <vector>

#include "attn_impl.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "nccl_shim.h"
#include "step_plan.h"
#include "tp_comm.h"
#include "model_state.h"

namespace du {

static void *dalloc(du_model *m, size_t bytes, int *rc)
{
    void *p = nullptr;
    if (*rc) return nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        *rc = cuda_fail(e, "cudaMalloc");
        return nullptr;
    }
    cudaMemset(p, 0, bytes);
    m->allocs.push_back(p);
    return p;
}

static int64_t qbytes(int quant, int64_t rows, int64_t cols)
{
    return quant == DU_QUANT_INT4 ? rows * cols / 2 : quant == DU_QUANT_INT8 ? rows * cols : rows * cols * 2;
}

static int64_t sbytes(int quant, int group, int64_t rows, int64_t cols)
{
    return quant == DU_QUANT_INT4 ? rows * (cols / group) * 2 : quant == DU_QUANT_INT8 ? rows * 2 : 0;
}

// float32 -> float16 round-to-nearest-even (same rounding as the managed
// converter of MiniCPM5Model.cs:205-234 for all finite inputs)
static uint16_t f32_to_f16(float v)
{
    uint32_t x;
    memcpy(&x, &v, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t m = x & 0x7fffffu;
    if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0u));
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const int t = 14 - e;
        const uint32_t half = 1u << (t - 1);
        uint32_t r = m >> t;
        const uint32_t rem = m & ((1u << t) - 1);
        if (rem > half || (rem == half && (r & 1))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) r++;
    return (uint16_t)(sign | r);
}

static int check_cfg(const du_model_config &c)
{
    DU_CHECK_ARG(c.hidden_size > 0 && c.intermediate_size > 0 && c.num_layers > 0, "config: non-positive dims");
    DU_CHECK_ARG(c.num_heads_q > 0 && c.num_heads_kv > 0 && c.num_heads_q % c.num_heads_kv == 0,
                 "config: num_heads_q must be a multiple of num_heads_kv");
    DU_CHECK_ARG(c.head_dim == 64 || c.head_dim == 128 || c.head_dim == 256, "config: head_dim must be 64, 128 or 256");
    DU_CHECK_ARG(c.kv_quant != DU_KV_INT8 || c.head_dim <= 128, "config: the INT8 KV cache supports head_dim 64/128");
    DU_CHECK_ARG((c.arch_flags & ~(DU_ARCH_QK_NORM | DU_ARCH_SANDWICH | DU_ARCH_GELU | DU_ARCH_ATTN_GATE)) == 0,
                 "config: unknown arch_flags");
    if (c.arch_flags & DU_ARCH_ATTN_GATE)
        DU_CHECK_ARG((c.arch_flags & DU_ARCH_QK_NORM) && (c.tp_size <= 1),
                     "config: DU_ARCH_ATTN_GATE needs DU_ARCH_QK_NORM and a single GPU");
    if (c.rope_rot_dim != 0 && c.rope_rot_dim != c.head_dim) {
        // partial RoPE runs in the qk-norm kernel: rot/2 must be whole lanes of a warp's head
        // (head_dim / 32 values per lane) and a power-of-two number of them
        const int epl = c.head_dim / 32, r2 = c.rope_rot_dim / 2;
        DU_CHECK_ARG(c.rope_rot_dim > 0 && c.rope_rot_dim < c.head_dim && c.rope_rot_dim % 2 == 0 &&
                         (c.arch_flags & DU_ARCH_QK_NORM) && r2 % epl == 0 && ((r2 / epl) & (r2 / epl - 1)) == 0,
                     "config: rope_rot_dim must be head_dim, or an even number below it whose half is a power-of-two "
                     "multiple of head_dim / 32, with DU_ARCH_QK_NORM");
    }
    DU_CHECK_ARG(c.sliding_window >= 0 && c.attn_scale >= 0.0f, "config: negative sliding_window / attn_scale");
    const int G = c.num_heads_q / c.num_heads_kv;
    DU_CHECK_ARG(G == 1 || G == 2 || G == 4 || G == 8, "config: GQA group must be 1, 2, 4 or 8");
    DU_CHECK_ARG(c.vocab_size > 0 && c.kv_capacity > 0 && c.max_batch > 0, "config: vocab/capacity/batch");
    DU_CHECK_ARG(c.quant >= DU_QUANT_FP16 && c.quant <= DU_QUANT_INT4, "config: unknown quant");
    const int tp = c.tp_size <= 0 ? 1 : c.tp_size;
    DU_CHECK_ARG(c.tp_rank >= 0 && c.tp_rank < tp, "config: tp_rank out of range");
    DU_CHECK_ARG(c.num_heads_q % tp == 0 && c.num_heads_kv % tp == 0, "config: heads must divide by tp_size");
    DU_CHECK_ARG(c.intermediate_size % tp == 0 && c.vocab_size % tp == 0, "config: intermediate/vocab % tp");
    const int H = c.hidden_size, I_l = c.intermediate_size / tp, K_o = c.num_heads_q / tp * c.head_dim;
    if (c.quant == DU_QUANT_INT4) {
        DU_CHECK_ARG(c.group_size >= 32 && (c.group_size & (c.group_size - 1)) == 0,
                     "config: int4 group must be a power of two >= 32");
        DU_CHECK_ARG((H / c.group_size) % 2 == 0 && (I_l / c.group_size) % 2 == 0 && (K_o / c.group_size) % 2 == 0,
                     "config: every (sharded) K must hold an even number of int4 groups");
        DU_CHECK_ARG(H % c.group_size == 0 && I_l % c.group_size == 0 && K_o % c.group_size == 0,
                     "config: every (sharded) K must be a multiple of the int4 group");
    }
    DU_CHECK_ARG(H % 32 == 0 && I_l % 32 == 0 && K_o % 32 == 0, "config: K dims must be multiples of 32");
    DU_CHECK_ARG(c.tie_embedding == 0 || tp == 1, "config: tied embedding with tp > 1 is not supported");
    DU_CHECK_ARG(c.kv_quant == 0 || c.kv_quant == DU_KV_FP16 || c.kv_quant == DU_KV_INT8,
                 "config: kv_quant must be DU_KV_FP16 or DU_KV_INT8");
    return DU_OK;
}

// -------------------------------------------------------------- creation

static int qt_of(int quant);

static int model_alloc(du_model *m)
{
    int rc = DU_OK;
    const int H = m->H, hd = m->hd;
    m->layers.resize(m->L);
    const int64_t Ko = (int64_t)m->hq_l * hd;
    for (int l = 0; l < m->L; l++) {
        Layer &ly = m->layers[l];
        ly.w_qkv = (uint8_t *)dalloc(m, qbytes(m->quant, m->qkv_rows, H), &rc);
        ly.s_qkv = (__half *)dalloc(m, sbytes(m->quant, m->group, m->qkv_rows, H), &rc);
        ly.w_o = (uint8_t *)dalloc(m, qbytes(m->quant, H, Ko), &rc);
        ly.s_o = (__half *)dalloc(m, sbytes(m->quant, m->group, H, Ko), &rc);
        ly.w_gu = (uint8_t *)dalloc(m, qbytes(m->quant, 2LL * m->I_l, H), &rc);
        ly.s_gu = (__half *)dalloc(m, sbytes(m->quant, m->group, 2LL * m->I_l, H), &rc);
        ly.w_d = (uint8_t *)dalloc(m, qbytes(m->quant, H, m->I_l), &rc);
        ly.s_d = (__half *)dalloc(m, sbytes(m->quant, m->group, H, m->I_l), &rc);
        ly.ln1 = (__half *)dalloc(m, (size_t)H * 2, &rc);
        ly.ln2 = (__half *)dalloc(m, (size_t)H * 2, &rc);
        if (m->arch & DU_ARCH_QK_NORM) {
            ly.q_norm = (__half *)dalloc(m, (size_t)hd * 2, &rc);
            ly.k_norm = (__half *)dalloc(m, (size_t)hd * 2, &rc);
            m->weight_bytes += 4LL * hd;
        }
        if (m->arch & DU_ARCH_SANDWICH) {
            ly.post_attn = (__half *)dalloc(m, (size_t)H * 2, &rc);
            ly.post_ffn = (__half *)dalloc(m, (size_t)H * 2, &rc);
            m->weight_bytes += 4LL * H;
        }
        m->weight_bytes += qbytes(m->quant, m->qkv_rows, H) + sbytes(m->quant, m->group, m->qkv_rows, H) +
                           qbytes(m->quant, H, Ko) + sbytes(m->quant, m->group, H, Ko) +
                           qbytes(m->quant, 2LL * m->I_l, H) + sbytes(m->quant, m->group, 2LL * m->I_l, H) +
                           qbytes(m->quant, H, m->I_l) + sbytes(m->quant, m->group, H, m->I_l) + 4LL * H;
    }
    m->final_norm = (__half *)dalloc(m, (size_t)H * 2, &rc);
    m->embed = (__half *)dalloc(m, (size_t)m->V * H * 2, &rc);
    m->lm_head = m->cfg.tie_embedding ? m->embed : (__half *)dalloc(m, (size_t)m->V_l * H * 2, &rc);
    m->weight_bytes += 2ull * H + 2ull * m->V_l * H;
    m->rope_cos = (__half *)dalloc(m, (size_t)m->cap * (hd / 2) * 2, &rc);
    m->rope_sin = (__half *)dalloc(m, (size_t)m->cap * (hd / 2) * 2, &rc);
    if (m->window > 0) {
        m->rope_cos_local = (__half *)dalloc(m, (size_t)m->cap * (hd / 2) * 2, &rc);
        m->rope_sin_local = (__half *)dalloc(m, (size_t)m->cap * (hd / 2) * 2, &rc);
    }
    m->kv_layer_elems = (size_t)m->maxb * m->cap * m->hkv_l * hd;
    if (m->kv8) {
        m->k8 = (uint8_t *)dalloc(m, m->kv_layer_elems * m->L, &rc);
        m->v8 = (uint8_t *)dalloc(m, m->kv_layer_elems * m->L, &rc);
        m->ksz = (uint32_t *)dalloc(m, m->kv_layer_elems / hd * m->L * 4, &rc);
        m->vsz = (uint32_t *)dalloc(m, m->kv_layer_elems / hd * m->L * 4, &rc);
    } else {
        m->k_cache = (__half *)dalloc(m, m->kv_layer_elems * m->L * 2, &rc);
        m->v_cache = (__half *)dalloc(m, m->kv_layer_elems * m->L * 2, &rc);
    }
    const int T = m->max_tokens;
    m->d_cache_len = (int *)dalloc(m, sizeof(int) * m->maxb, &rc);
    m->d_ids = (int *)dalloc(m, sizeof(int) * T, &rc);
    m->d_next = (int *)dalloc(m, sizeof(int) * T, &rc);
    m->d_hist = (int *)dalloc(m, sizeof(int) * (size_t)m->maxb * m->cap, &rc);
    m->d_pos = (int *)dalloc(m, sizeof(int) * T, &rc);
    m->d_seq = (int *)dalloc(m, sizeof(int) * T, &rc);
    m->d_kvlen = (int *)dalloc(m, sizeof(int) * T, &rc);
    m->x_res = (float *)dalloc(m, sizeof(float) * T * H, &rc);
    m->part = (float *)dalloc(m, sizeof(float) * T * H, &rc);
    m->q = (float *)dalloc(m, sizeof(float) * T * m->hq_l * hd, &rc);
    m->att = (float *)dalloc(m, sizeof(float) * T * m->hq_l * hd, &rc);
    m->inter = (float *)dalloc(m, sizeof(float) * T * m->I_l, &rc);
    if (m->kv8) m->kv_stage = (float *)dalloc(m, sizeof(float) * T * 2 * m->hkv_l * hd, &rc);
    if (m->arch & DU_ARCH_QK_NORM) m->qkv_buf = (float *)dalloc(m, sizeof(float) * T * m->qkv_rows, &rc);
    if (m->arch & DU_ARCH_ATTN_GATE) m->gate_buf = (float *)dalloc(m, sizeof(float) * T * m->hq_l * hd, &rc);
    // one-row decode steps fold the O projection into flash-decode when the shapes allow
    // (DU_FUSE_ATTN_O=0 in the environment keeps them separate)
    {
        const char *e = getenv("DU_FUSE_ATTN_O");
        const bool want = e == nullptr || atoi(e) != 0;
        m->fuse_o = want && m->tp == 1 && !m->kv8 && !(m->arch & DU_ARCH_SANDWICH) &&
                    flash_decode_fuse_o_supported(1, m->hq_l, m->hkv_l, hd, H, qt_of(m->quant), m->group);
        if (m->fuse_o) {
            m->o_part = (float *)dalloc(m, sizeof(float) * (size_t)m->hkv_l * H, &rc);
            m->o_cnt = (unsigned *)dalloc(m, sizeof(unsigned) * 16, &rc);
        }
    }
    m->logits = (float *)dalloc(m, sizeof(float) * m->maxb * m->V_l, &rc);
    if (m->tp > 1) m->logits_all = (float *)dalloc(m, sizeof(float) * m->tp * m->maxb * m->V_l, &rc);
    m->am_parts = 2 * num_sms();
    // per-row greedy state is sized for the largest forward chunk (all-position logits), and
    // for the tensor-core head (one partial per 128-row vocab tile)
    const int am_cap = m->am_parts > (m->V_l + 127) / 128 ? m->am_parts : (m->V_l + 127) / 128;
    m->am_val = (float *)dalloc(m, sizeof(float) * T * am_cap, &rc);
    m->am_idx = (int *)dalloc(m, sizeof(int) * T * am_cap, &rc);
    m->best_val = (float *)dalloc(m, sizeof(float) * T * 2, &rc);
    m->gbest_val = (float *)dalloc(m, sizeof(float) * T * 2 * m->tp, &rc);
    const int G = m->hq_l / m->hkv_l;
    // flash-decode scratch: decode rows (maxb) use fd_nsplit_decode splits; prefill rows use 1..n
    m->fd_nsplit_decode = fd_choose_splits(m->maxb, m->hkv_l, m->cap);
    m->fd_scratch_fl = 0;
    for (int rows = 1; rows <= T; rows++) {   // every row count a decode graph or prefill chunk can use
        const size_t f = fd_scratch_floats(rows, m->hkv_l, G, hd, fd_choose_splits(rows, m->hkv_l, m->cap));
        if (f > m->fd_scratch_fl) m->fd_scratch_fl = f;
    }
    m->fd_scratch = (float *)dalloc(m, sizeof(float) * m->fd_scratch_fl, &rc);
    m->fd_counters = (unsigned *)dalloc(m, sizeof(unsigned) * (size_t)T * m->hkv_l, &rc);
    m->d_barrier = (unsigned *)dalloc(m, sizeof(unsigned), &rc);
    m->d_err = (int *)dalloc(m, sizeof(int), &rc);
    m->d_seeds = (int32_t *)dalloc(m, sizeof(int32_t) * (m->maxb + SAMPLE_PARAMS), &rc);
    m->d_sparams = reinterpret_cast<float *>(m->d_seeds + m->maxb);
    if (m->tp == 1) m->d_seen = (unsigned *)dalloc(m, sizeof(unsigned) * (size_t)m->maxb * m->V, &rc);
    {   // GEMM activation stage: every K a chunk's GEMM can see (H, I_l, hq_l * hd)
        int64_t kmax = H > m->I_l ? H : m->I_l;
        if ((int64_t)m->hq_l * hd > kmax) kmax = (int64_t)m->hq_l * hd;
        m->gm.rows = (size_t)T;
        m->gm.elems = (size_t)T * kmax;
        m->gm.xh = (__half *)dalloc(m, 2 * m->gm.elems, &rc);
        m->gm.xl = (__half *)dalloc(m, 2 * m->gm.elems, &rc);
        m->gm.xscale = (float *)dalloc(m, sizeof(float) * T, &rc);
        m->gm.err = m->d_err;
        m->gm.partial_floats = GEMM_PARTIAL_FLOATS_PER_SM * (size_t)num_sms();
        m->gm.partials = (float *)dalloc(m, sizeof(float) * m->gm.partial_floats, &rc);
        m->gm.counter_n = 1 << 16;
        m->gm.counters = (unsigned *)dalloc(m, sizeof(unsigned) * m->gm.counter_n, &rc);
    }
    m->d_stamps = (unsigned long long *)dalloc(m, sizeof(unsigned long long) * (5 * (size_t)m->L + 8), &rc);
    if (rc) return rc;
    DU_CUDA_TRY(cudaMallocHost(&m->h_pin_err, sizeof(int)));
    DU_CUDA_TRY(cudaMallocHost(&m->h_pin_ids, sizeof(int) * T));
    DU_CUDA_TRY(cudaMallocHost(&m->h_pin_next, sizeof(int) * m->maxb));
    DU_CUDA_TRY(cudaMallocHost(&m->h_pin_seeds, sizeof(int32_t) * (m->maxb + SAMPLE_PARAMS)));
    m->h_cache_len.assign(m->maxb, 0);

    // RoPE tables on the host with the reference formula (MiniCPM5Model.cs:163-191); the
    // sliding-window layers' tables use the local base (Gemma3Model: ropeCosLocal)
    const int hd2 = hd / 2;
    const int rot = m->cfg.rope_rot_dim > 0 ? m->cfg.rope_rot_dim : hd;
    std::vector<uint16_t> c((size_t)m->cap * hd2), s((size_t)m->cap * hd2);
    for (int table = 0; table < (m->window > 0 ? 2 : 1); table++) {
        const float theta = table == 0 || m->cfg.rope_theta_local <= 0.0f ? m->cfg.rope_theta : m->cfg.rope_theta_local;
        for (int pos = 0; pos < m->cap; pos++)
            for (int i = 0; i < hd2; i++) {
                // over the rotated dims (Qwen3.5 partial RoPE: Qwen3_5Model.cs:228-260); entries
                // i >= rot / 2 are not read then
                const float f = 1.0f / powf(theta, 2.0f * (float)i / (float)rot);
                const float ang = (float)pos * f;
                c[(size_t)pos * hd2 + i] = f32_to_f16(cosf(ang));
                s[(size_t)pos * hd2 + i] = f32_to_f16(sinf(ang));
            }
        DU_CUDA_TRY(cudaMemcpy(table ? m->rope_cos_local : m->rope_cos, c.data(), c.size() * 2, cudaMemcpyHostToDevice));
        DU_CUDA_TRY(cudaMemcpy(table ? m->rope_sin_local : m->rope_sin, s.data(), s.size() * 2, cudaMemcpyHostToDevice));
    }
    DU_CUDA_TRY(cudaDeviceSynchronize());
    return DU_OK;
}

static void model_free(du_model *m)
{
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto *gm : {&m->graphs, &m->sgraphs, &m->pgraphs})
        for (auto &kv : *gm) {
            if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
            if (kv.second.g) cudaGraphDestroy(kv.second.g);
            if (kv.second.d_stages) cudaFree(kv.second.d_stages);
        }
    m->sgraphs.clear();
    m->pgraphs.clear();
    if (m->h_pin_seeds) cudaFreeHost(m->h_pin_seeds);
    m->h_pin_seeds = nullptr;
    if (m->h_pin_err) cudaFreeHost(m->h_pin_err);
    m->h_pin_err = nullptr;
    m->graphs.clear();
    tp_comm_free(&m->tpc);
    if (m->comm) {
        const NcclApi *n = nccl_api();
        if (n) n->CommDestroy(m->comm);
        m->comm = nullptr;
    }
    for (void *p : m->allocs) cudaFree(p);
    m->allocs.clear();
    if (m->h_pin_ids) cudaFreeHost(m->h_pin_ids);
    if (m->h_pin_next) cudaFreeHost(m->h_pin_next);
    m->h_pin_ids = m->h_pin_next = nullptr;
    if (m->stream) cudaStreamDestroy(m->stream);
    m->stream = nullptr;
}

// ------------------------------------------------------------- loading

// Copies rows [r0, r1) x byte-columns [c0, c1) of a row-major source with
// `src_pitch` bytes per row into dst (pitch dst_pitch).
static int copy2d(void *dst, size_t dst_pitch, const void *src, size_t src_pitch, int64_t r0, int64_t r1, int64_t c0,
                  int64_t c1, cudaMemcpyKind kind, cudaStream_t st)
{
    if (r1 <= r0 || c1 <= c0) return DU_OK;
    DU_CUDA_TRY(cudaMemcpy2DAsync(dst, dst_pitch, (const uint8_t *)src + r0 * src_pitch + c0, src_pitch,
                                  (size_t)(c1 - c0), (size_t)(r1 - r0), kind, st));
    return DU_OK;
}

enum TensorKind { T_NONE, T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_LMHEAD };

// Tensor-parallel partition of one global tensor: its shape [rows, cols], the
// window [r0, r1) x [c0, c1) this rank keeps, and where the window lands in the
// rank's concatenated buffer (first row drow, row length dcols).
//   q / k / v, gate / up : whole heads / rows, split by output rows
//   o / down             : split by input columns (every row kept)
//   lm_head              : vocab rows
struct ShardWindow {
    int64_t rows, cols, r0, r1, c0, c1, drow, dcols;
};

static int shard_window(const du_model_config &c, int tk, ShardWindow *w)
{
    const int tp = c.tp_size <= 0 ? 1 : c.tp_size, r = c.tp_rank;
    const int64_t H = c.hidden_size, hd = c.head_dim, I = c.intermediate_size;
    const int64_t hq_l = c.num_heads_q / tp, hkv_l = c.num_heads_kv / tp, I_l = I / tp, V_l = c.vocab_size / tp;
    const int64_t qw = (c.arch_flags & DU_ARCH_ATTN_GATE) ? 2 : 1;     // q rows then gate rows per head
    ShardWindow s = {};
    switch (tk) {
    case T_Q: s = {c.num_heads_q * qw * hd, H, r * hq_l * qw * hd, (r + 1) * hq_l * qw * hd, 0, H, 0, H}; break;
    case T_K: s = {c.num_heads_kv * hd, H, r * hkv_l * hd, (r + 1) * hkv_l * hd, 0, H, hq_l * qw * hd, H}; break;
    case T_V:
        s = {c.num_heads_kv * hd, H, r * hkv_l * hd, (r + 1) * hkv_l * hd, 0, H, (hq_l * qw + hkv_l) * hd, H};
        break;
    case T_O: s = {H, c.num_heads_q * hd, 0, H, r * hq_l * hd, (r + 1) * hq_l * hd, 0, hq_l * hd}; break;
    case T_GATE: s = {I, H, r * I_l, (r + 1) * I_l, 0, H, 0, H}; break;
    case T_UP: s = {I, H, r * I_l, (r + 1) * I_l, 0, H, I_l, H}; break;
    case T_DOWN: s = {H, I, 0, H, r * I_l, (r + 1) * I_l, 0, I_l}; break;
    case T_LMHEAD: s = {c.vocab_size, H, r * V_l, (r + 1) * V_l, 0, H, 0, H}; break;
    default: return fail(DU_ENOTFOUND, "unknown tensor kind");
    }
    *w = s;
    return DU_OK;
}

static int tensor_kind_of(const char *stem)
{
    static const struct { const char *stem; int k; } stems[] = {
        {"self_attn_q_proj", T_Q}, {"self_attn_k_proj", T_K}, {"self_attn_v_proj", T_V},
        {"self_attn_o_proj", T_O}, {"mlp_gate_proj", T_GATE}, {"mlp_up_proj", T_UP}, {"mlp_down_proj", T_DOWN},
        {"lm_head", T_LMHEAD}};
    for (auto &s : stems)
        if (strcmp(stem, s.stem) == 0) return s.k;
    return T_NONE;
}

// Places one IMP tensor (weights, or its scales) into the sharded device layout.
int place_tensor(du_model *m, const char *name, const void *src, size_t bytes, cudaMemcpyKind kind)
{
    cudaStream_t st = m->stream;
    const int H = m->H, hd = m->hd, r = m->rank;
    std::string n(name);
    if (n == "norm.bin") {
        DU_CHECK_ARG(bytes == (size_t)H * 2, "norm.bin: size mismatch");
        DU_CUDA_TRY(cudaMemcpyAsync(m->final_norm, src, bytes, kind, st));
        return DU_OK;
    }
    int part = -1;
    const bool is_embed = sscanf(name, "embed_tokens/part_%d.bin", &part) == 1;
    const bool is_head = !is_embed && sscanf(name, "lm_head/part_%d.bin", &part) == 1;
    if (is_embed || is_head) {
        DU_CHECK_ARG(m->V % 16 == 0, "embedding parts need vocab % 16 == 0 (IMP EMBED_CHUNKS)");
        const int64_t rows = m->V / 16;
        DU_CHECK_ARG(part >= 0 && part < 16 && bytes == (size_t)rows * H * 2, "embedding part: bad index or size");
        const int64_t g0 = (int64_t)part * rows, g1 = g0 + rows;
        if (is_embed) {
            int rc = copy2d((uint8_t *)m->embed + g0 * H * 2, (size_t)H * 2, src, (size_t)H * 2, 0, rows, 0,
                            (int64_t)H * 2, kind, st);
            if (rc) return rc;
            return DU_OK;
        }
        DU_CHECK_ARG(!m->cfg.tie_embedding, "lm_head parts given for a tied-embedding model");
        const int64_t s0 = (int64_t)r * m->V_l, s1 = s0 + m->V_l;      // this rank's vocab shard
        const int64_t a = g0 > s0 ? g0 : s0, b = g1 < s1 ? g1 : s1;
        if (a >= b) return DU_OK;
        return copy2d((uint8_t *)m->lm_head + (a - s0) * H * 2, (size_t)H * 2, src, (size_t)H * 2, a - g0, b - g0, 0,
                      (int64_t)H * 2, kind, st);
    }
    int li = -1;
    char rest[128] = {0};
    if (sscanf(name, "layer_%d/%127s", &li, rest) != 2 || li < 0 || li >= m->L)
        return fail(DU_ENOTFOUND, std::string("unknown tensor: ") + name);
    Layer &ly = m->layers[li];
    std::string t(rest);
    if (t == "input_layernorm.bin" || t == "post_attention_layernorm.bin" || t == "pre_feedforward_layernorm.bin" ||
        t == "post_feedforward_layernorm.bin") {
        DU_CHECK_ARG(bytes == (size_t)H * 2, "layernorm: size mismatch");
        // llama: post_attention_layernorm is the pre-MLP norm; with sandwich norms (Gemma3) it
        // is the norm of the attention output, and pre_feedforward_layernorm the pre-MLP one
        const bool sw = m->arch & DU_ARCH_SANDWICH;
        __half *dst = t == "input_layernorm.bin" ? ly.ln1
                      : t == "post_attention_layernorm.bin" ? (sw ? ly.post_attn : ly.ln2)
                      : t == "pre_feedforward_layernorm.bin" ? (sw ? ly.ln2 : nullptr)
                                                             : ly.post_ffn;
        if (dst == nullptr) return fail(DU_ENOTFOUND, std::string("tensor of a sandwich-norm model: ") + name);
        DU_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, kind, st));
        return DU_OK;
    }
    if (t == "self_attn_q_norm.bin" || t == "self_attn_k_norm.bin") {
        if (!(m->arch & DU_ARCH_QK_NORM)) return fail(DU_ENOTFOUND, std::string("tensor of a qk-norm model: ") + name);
        DU_CHECK_ARG(bytes == (size_t)hd * 2, "qk-norm: size mismatch");
        DU_CUDA_TRY(cudaMemcpyAsync(t[10] == 'q' ? ly.q_norm : ly.k_norm, src, bytes, kind, st));
        return DU_OK;
    }
    static const struct { const char *stem; TensorKind k; } stems[] = {
        {"self_attn_q_proj", T_Q}, {"self_attn_k_proj", T_K}, {"self_attn_v_proj", T_V},
        {"self_attn_o_proj", T_O}, {"mlp_gate_proj", T_GATE}, {"mlp_up_proj", T_UP}, {"mlp_down_proj", T_DOWN}};
    TensorKind tk = T_NONE;
    std::string suffix;
    for (auto &sdef : stems) {
        const size_t len = strlen(sdef.stem);
        if (t.compare(0, len, sdef.stem) == 0) { tk = sdef.k; suffix = t.substr(len); break; }
    }
    if (tk == T_NONE) return fail(DU_ENOTFOUND, std::string("unknown tensor: ") + name);
    const char *wext = m->quant == DU_QUANT_INT4 ? ".int4.bin" : m->quant == DU_QUANT_INT8 ? ".int8.bin" : ".bin";
    const bool is_scale = suffix == ".scales.bin";
    if (!is_scale && suffix != wext) return fail(DU_EINVAL, std::string("tensor format does not match the model quant: ") + name);
    if (is_scale && m->quant == DU_QUANT_FP16) return fail(DU_EINVAL, "fp16 model has no scales");

    // global shape [rows, cols], this rank's row/col window, destination
    ShardWindow sw;
    int rc = shard_window(m->cfg, tk, &sw);
    if (rc) return rc;
    const int64_t rows = sw.rows, cols = sw.cols, r0 = sw.r0, r1 = sw.r1, c0 = sw.c0, c1 = sw.c1;
    const int64_t drow = sw.drow, dcols = sw.dcols;
    uint8_t *dw = nullptr;
    __half *ds = nullptr;
    switch (tk) {
    case T_Q: case T_K: case T_V: dw = ly.w_qkv; ds = ly.s_qkv; break;
    case T_O: dw = ly.w_o; ds = ly.s_o; break;
    case T_GATE: case T_UP: dw = ly.w_gu; ds = ly.s_gu; break;
    default: dw = ly.w_d; ds = ly.s_d; break;
    }
    (void)hd; (void)r;
    if (!is_scale) {
        const int64_t need = qbytes(m->quant, rows, cols);
        DU_CHECK_ARG((int64_t)bytes == need, (std::string("size mismatch for ") + name).c_str());
        const int64_t rb = qbytes(m->quant, 1, cols);          // bytes per source row
        const int64_t db = qbytes(m->quant, 1, dcols);         // bytes per destination row
        const int64_t cb0 = qbytes(m->quant, 1, c0), cb1 = qbytes(m->quant, 1, c1);
        return copy2d(dw + drow * db, (size_t)db, src, (size_t)rb, r0, r1, cb0, cb1, kind, st);
    }
    if (m->quant == DU_QUANT_INT8) {
        DU_CHECK_ARG((int64_t)bytes == rows * 2, (std::string("size mismatch for ") + name).c_str());
        // per-row scales: row-split tensors take their rows; K-split tensors keep every row
        return copy2d((uint8_t *)ds + drow * 2, 2, src, 2, r0, r1, 0, 2, kind, st);
    }
    const int64_t g = m->group;
    DU_CHECK_ARG(cols % g == 0, "int4 scales: cols % group != 0");
    DU_CHECK_ARG((int64_t)bytes == rows * (cols / g) * 2, (std::string("size mismatch for ") + name).c_str());
    return copy2d((uint8_t *)ds + drow * (dcols / g) * 2, (size_t)(dcols / g) * 2, src, (size_t)(cols / g) * 2, r0, r1,
                  (c0 / g) * 2, (c1 / g) * 2, kind, st);
}

// ------------------------------------------------------------ execution

static GemvParams gp_base(du_model *m, const uint8_t *w, const __half *s, int64_t K)
{
    GemvParams p = {};
    p.w = w;
    p.scales = s;
    p.row_bytes = qbytes(m->quant, 1, K);
    p.K = (int)K;
    p.group = m->group;
    return p;
}

static int qt_of(int quant) { return quant == DU_QUANT_INT4 ? Q_I4 : quant == DU_QUANT_INT8 ? Q_I8 : Q_F16; }

static int gemv_max_tokens(int qt, int64_t row_bytes)
{
    int mt = 8;
    while (mt > 1 && gemv_smem_bytes(qt, mt, row_bytes) > 220 * 1024) mt >>= 1;
    return mt;
}

// Launches one GEMV over M tokens in chunks the kernel's smem stage holds.
// Token-indexed pointers of `p` are advanced per chunk.
static int run_gemv(du_model *m, int qt, GemvParams p, int M)
{
    if (M <= 2) {     // tensor-core decode GEMV (INT4)
        GemvParams g = p;
        g.M = M;
        if (tgemv_supported(qt, g)) return launch_tgemv(qt, g, m->gm, m->stream);
    }
    if (M >= gemm_min_tokens()) {     // tensor-core GEMM: every weight streamed once for all M rows
        GemvParams g = p;
        g.M = M;
        if (gemm_supported(qt, g)) return launch_gemm(qt, g, m->gm, m->stream);
    }
    const int mt = gemv_max_tokens(qt, p.row_bytes);
    for (int t0 = 0; t0 < M; t0 += mt) {
        GemvParams c = p;
        c.M = M - t0 < mt ? M - t0 : mt;
        c.x = p.x + (size_t)t0 * p.ldx;
        if (p.y) c.y = p.y + (size_t)t0 * p.ldy;
        if (p.q_out) c.q_out = p.q_out + (size_t)t0 * p.hq * p.hd;
        if (p.kv_stage) c.kv_stage = p.kv_stage + (size_t)t0 * 2 * p.hkv * p.hd;
        if (p.pos) c.pos = p.pos + t0;
        if (p.seq_of) c.seq_of = p.seq_of + t0;
        else c.seq_off = p.seq_off + t0;      // token t0 + m belongs to sequence t0 + m
        if (p.logits) c.logits = p.logits + (size_t)t0 * p.ldl;
        int rc = launch_gemv(qt, c, m->stream);
        if (rc) return rc;
    }
    return DU_OK;
}

static int nccl_check(du_model *m, ncclResult_t r, const char *what)
{
    const NcclApi *n = nccl_api();
    if (r == ncclSuccess) return DU_OK;
    if (r == ncclInProgress) {
        auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            ncclResult_t a = ncclSuccess;
            n->CommGetAsyncError(m->comm, &a);
            if (a == ncclSuccess) return DU_OK;
            if (a != ncclInProgress) return fail(DU_ENCCL, std::string(what) + ": " + n->GetErrorString(a));
            if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
                m->nccl_timeout_ms) {
                n->CommAbort(m->comm);
                m->comm = nullptr;
                m->tp_ready = false;
                return fail(DU_ENCCL, std::string(what) + ": timed out, communicator aborted");
            }
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
    return fail(DU_ENCCL, std::string(what) + ": " + n->GetErrorString(r));
}

static int allreduce_sum(du_model *m, float *buf, size_t n)
{
    const NcclApi *api = nccl_api();
    return nccl_check(m, api->AllReduce(buf, buf, n, ncclFloat32, ncclSum, m->comm, m->stream), "ncclAllReduce");
}

struct StepIO {
    int M;                 // token rows
    const int *ids;        // [M] device
    const int *pos;        // [M] cache slot / rope position
    const int *seq_of;     // [M] or nullptr
    const int *kv_len;     // [M] kv length before kv_len_add
    int kv_len_add;
    int kv_new = -1;       // K/V rows per token row written by this pass's QKV stage (-1: not uniform)
    bool p2p = false;      // TP reductions may take the peer-memory allreduce (decode graphs)
    int fd_nsplit;
    int logits_rows;       // rows whose logits are produced (last token per sequence, or all)
    const int *logit_tok;  // tokens -> which rows of x_res feed the lm_head: nullptr = all M
    int logit_stride;      // if logit_tok == nullptr: take every logit_stride-th token starting at logit_first
    int logit_first;
    int *next_out;         // [logits_rows] greedy ids
    int *feed;             // optional: also write ids here (device loop)
    bool advance;          // cache_len[m] += 1 at the end (decode)
    bool sample = false;   // pick with the stochastic sampler (settings and seeds in device memory)
    bool penalize = false; // sample: repetition / presence penalty over the sequence's seen ids first
};

enum Stage { ST_QKV = 0, ST_ATTN = 1, ST_O = 2, ST_GATEUP = 3, ST_DOWN = 4 };

// Decode reductions of a tensor-parallel model may use the peer-memory path.
static bool tp_peer_ok(const du_model *m, const StepIO &io)
{
    return m->tp > 1 && io.p2p && m->tpc.ready && (size_t)io.M * m->H <= m->tpc.maxn;
}

// The peer-memory reduction runs in the O / down GEMV's epilogue up to 4 ranks, and
// as a separate kernel after the GEMV at more (8B INT4, batch 1: TP2 633 vs 581 tok/s
// fused vs separate, TP8 730 vs 761).  DU_TP_FUSE=1 / 0 in the environment forces
// either.
static bool tp_fuse_enabled(const du_model *m)
{
    static const int force = [] {
        const char *e = getenv("DU_TP_FUSE");
        return e == nullptr ? -1 : (atoi(e) != 0 ? 1 : 0);
    }();
    return force < 0 ? m->tp <= 4 : force == 1;
}

// Layer l's part of the INT8 cache.
static Kv8Cache kv8_layer(const du_model *m, int l)
{
    const size_t rows = m->kv_layer_elems / m->hd;
    return Kv8Cache{m->k8 + (size_t)l * m->kv_layer_elems, m->v8 + (size_t)l * m->kv_layer_elems, m->ksz + (size_t)l * rows,
                    m->vsz + (size_t)l * rows};
}

// One stage of layer l for the token rows of `io`.  With tensor parallelism
// the O and down stages end in an allreduce of the partial sums plus the
// residual add (collective = false leaves both out, for kernel timing).
// GEMV parameters of stage `stage` of layer l for the token rows of `io`
// (shared by the per-kernel path and the persistent decode-step plan).
// Layer l is a sliding-window layer (Gemma3Config.layer_types: every
// sliding_pattern-th layer, 1-based, is full attention).
static bool layer_sliding(const du_model *m, int l)
{
    return m->window > 0 && (m->pattern <= 0 || (l + 1) % m->pattern != 0);
}

static GemvParams stage_gemv_params(du_model *m, const StepIO &io, int l, int stage)
{
    const int H = m->H, hd = m->hd;
    const int64_t Ko = (int64_t)m->hq_l * hd;
    const Layer &ly = m->layers[l];
    const bool sw = layer_sliding(m, l);
    GemvParams p;
    switch (stage) {
    case ST_QKV:   // RMSNorm(ln1) -> QKV GEMV -> RoPE -> q, fp16 K/V into the cache
        p = gp_base(m, ly.w_qkv, ly.s_qkv, H);
        p.x = m->x_res; p.ldx = H; p.gamma = ly.ln1; p.eps = m->cfg.rms_eps;
        p.N = m->qkv_rows;
        if (m->arch & DU_ARCH_QK_NORM) {
            // qk-norm needs whole heads: the rows go out as they are; the qkv-post kernel
            // normalises, rotates and writes the cache
            p.map = MAP_IDENT;
            p.epi = EPI_STORE; p.y = m->qkv_buf; p.ldy = m->qkv_rows;
            break;
        }
        p.map = MAP_ROPE_PAIR; p.map_hd = hd;
        p.epi = EPI_QKV; p.q_out = m->q;
        if (m->kv8) {
            p.kv_stage = m->kv_stage;      // quantized into the INT8 cache by the next kernel
        } else {
            p.k_cache = m->k_cache + (size_t)l * m->kv_layer_elems;
            p.v_cache = m->v_cache + (size_t)l * m->kv_layer_elems;
        }
        p.pos = io.pos; p.seq_of = io.seq_of; p.hq = m->hq_l; p.hkv = m->hkv_l; p.hd = hd; p.cap = m->cap;
        p.rope_cos = sw ? m->rope_cos_local : m->rope_cos;
        p.rope_sin = sw ? m->rope_sin_local : m->rope_sin;
        break;
    case ST_O:
    case ST_DOWN:  // O / down GEMV -> residual add (TP1) or partial sum for the allreduce
        if (stage == ST_O) {
            p = gp_base(m, ly.w_o, ly.s_o, Ko);
            p.x = m->att; p.ldx = (int)Ko;
        } else {
            p = gp_base(m, ly.w_d, ly.s_d, m->I_l);
            p.x = m->inter; p.ldx = m->I_l;
        }
        p.N = H; p.map = MAP_IDENT;
        if (m->arch & DU_ARCH_SANDWICH) { p.epi = EPI_STORE; p.y = m->part; p.ldy = H; }   // norm, then residual
        else if (m->tp == 1) { p.epi = EPI_RESID; p.y = m->x_res; p.ldy = H; }
        else if (tp_peer_ok(m, io) && tp_fuse_enabled(m)) {
            // decode: the allreduce over peer memory runs in the GEMV's epilogue
            p.epi = EPI_TP_RESID; p.y = m->part; p.ldy = H; p.tp = m->tpc.dev; p.resid = m->x_res;
        } else { p.epi = EPI_STORE; p.y = m->part; p.ldy = H; }
        break;
    default:       // ST_GATEUP: RMSNorm(ln2) -> gate|up GEMV -> SiLU(g) * u
        p = gp_base(m, ly.w_gu, ly.s_gu, H);
        p.x = m->x_res; p.ldx = H; p.gamma = ly.ln2; p.eps = m->cfg.rms_eps;
        p.N = 2 * m->I_l; p.map = MAP_GATEUP; p.map_I = m->I_l;
        p.epi = EPI_GATEUP; p.y = m->inter; p.ldy = m->I_l;
        p.act = (m->arch & DU_ARCH_GELU) ? 1 : 0;
        break;
    }
    p.M = io.M;
    return p;
}

// Attention parameters of layer l (scratch split for `nsplit` splits of io.M rows).
static FdParams stage_attn_params(du_model *m, const StepIO &io, int l, int nsplit, int *G)
{
    FdParams a = {};
    const int g = m->hq_l / m->hkv_l;
    a.q = m->q;
    a.k_cache = m->k_cache + (size_t)l * m->kv_layer_elems;
    a.v_cache = m->v_cache + (size_t)l * m->kv_layer_elems;
    a.seq_of = io.seq_of;
    a.kv_len = io.kv_len;
    a.kv_len_add = io.kv_len_add;
    a.hq = m->hq_l; a.hkv = m->hkv_l; a.cap = m->cap;
    a.scale = m->attn_scale;
    a.window = layer_sliding(m, l) ? m->window : 0;
    a.out = m->att;
    a.part_o = m->fd_scratch;
    a.part_ml = m->fd_scratch + (size_t)io.M * m->hkv_l * nsplit * g * m->hd;
    a.counters = m->fd_counters;
    *G = g;
    return a;
}

// One stage of layer l for the token rows of `io`.  With tensor parallelism
// the O and down stages end in an allreduce of the partial sums plus the
// residual add (collective = false leaves both out, for kernel timing).
static int enqueue_stage(du_model *m, const StepIO &io, int l, int stage, bool collective)
{
    const int H = m->H, hd = m->hd, M = io.M, qt = qt_of(m->quant);
    cudaStream_t st = m->stream;
    int rc = DU_OK;
    const bool sw = layer_sliding(m, l);
    const bool fused_o = m->fuse_o && M == 1 && collective && !sw && !(m->arch & DU_ARCH_ATTN_GATE);
    if (stage == ST_O && fused_o) return DU_OK;      // ran inside flash-decode
    if (stage == ST_ATTN && fused_o) {
        const Layer &ly = m->layers[l];
        FuseO o = {};
        o.w = ly.w_o; o.scales = ly.s_o; o.quant = qt; o.group = m->group; o.H = H;
        o.resid = m->x_res; o.part = m->o_part; o.cnt = m->o_cnt; o.err = m->d_err;
        return launch_flash_decode_fuse_o(m->q, m->k_cache + (size_t)l * m->kv_layer_elems,
                                          m->v_cache + (size_t)l * m->kv_layer_elems, io.seq_of, io.kv_len,
                                          io.kv_len_add, m->hq_l, m->hkv_l, hd, m->cap, m->attn_scale, m->att, st,
                                          io.kv_new, o);
    }
    if (stage == ST_ATTN) {
        const int window = sw ? m->window : 0;
        if (m->kv8) {
            const Kv8Cache kv = kv8_layer(m, l);
            rc = launch_flash_decode_cluster(m->q, nullptr, nullptr, io.seq_of, io.kv_len, io.kv_len_add, M, m->hq_l,
                                             m->hkv_l, hd, m->cap, m->attn_scale, m->att, st, io.kv_new, &kv, window);
        } else {
            __half *kc = m->k_cache + (size_t)l * m->kv_layer_elems;
            __half *vc = m->v_cache + (size_t)l * m->kv_layer_elems;
            rc = launch_flash_decode_cluster(m->q, kc, vc, io.seq_of, io.kv_len, io.kv_len_add, M, m->hq_l, m->hkv_l,
                                             hd, m->cap, m->attn_scale, m->att, st, io.kv_new, nullptr, window);
        }
        // Qwen3.5: attention output * sigmoid(gate) before o_proj (ApplyAttnGate)
        if (rc == DU_OK && (m->arch & DU_ARCH_ATTN_GATE))
            rc = launch_attn_gate(m->att, m->gate_buf, (size_t)M * m->hq_l * hd, st);
        return rc;
    }
    if (stage < ST_QKV || stage > ST_DOWN) return fail(DU_EINVAL, "unknown stage");
    GemvParams gp = stage_gemv_params(m, io, l, stage);
    if (gp.epi == EPI_TP_RESID && !collective) gp.epi = EPI_STORE;     // partial sums into m->part only
    if ((rc = run_gemv(m, qt, gp, M))) return rc;
    if (stage == ST_QKV && (m->arch & DU_ARCH_QK_NORM)) {
        // qk-norm (Gemma3): normalise and rotate q / k per head, then the cache write
        const Layer &ly = m->layers[l];
        QkvPost a = {};
        a.qkv = m->qkv_buf; a.M = M; a.hq = m->hq_l; a.hkv = m->hkv_l; a.hd = hd;
        a.q_norm = ly.q_norm; a.k_norm = ly.k_norm; a.eps = m->cfg.rms_eps;
        a.pos = io.pos; a.seq_of = io.seq_of; a.seq_off = 0; a.cap = m->cap;
        a.rope_cos = sw ? m->rope_cos_local : m->rope_cos;
        a.rope_sin = sw ? m->rope_sin_local : m->rope_sin;
        a.q_out = m->q;
        a.gated = (m->arch & DU_ARCH_ATTN_GATE) ? 1 : 0;
        a.gate_out = m->gate_buf;
        a.rot = m->cfg.rope_rot_dim;
        if (m->kv8) a.kv8 = kv8_layer(m, l);
        else {
            a.k_cache = m->k_cache + (size_t)l * m->kv_layer_elems;
            a.v_cache = m->v_cache + (size_t)l * m->kv_layer_elems;
        }
        return launch_qkv_post(a, st);
    }
    if (stage == ST_QKV && m->kv8)     // this pass's K / V rows into the INT8 cache
        return launch_kv_quant_int8(m->kv_stage, M, 2, m->hkv_l, hd, io.pos, 0, io.seq_of, 0, m->cap, kv8_layer(m, l), st);
    if ((stage == ST_O || stage == ST_DOWN) && (m->arch & DU_ARCH_SANDWICH)) {
        // sandwich norms (Gemma3): the block output (summed over the ranks) is normalised,
        // then added to the residual
        if (m->tp > 1 && collective && (rc = allreduce_sum(m, m->part, (size_t)M * H))) return rc;
        const Layer &ly = m->layers[l];
        return launch_norm_add(m->part, stage == ST_O ? ly.post_attn : ly.post_ffn, M, H, m->cfg.rms_eps, m->x_res, st);
    }
    if ((stage == ST_O || stage == ST_DOWN) && m->tp > 1 && collective && gp.epi != EPI_TP_RESID) {
        if (tp_peer_ok(m, io)) return launch_tp_allreduce(&m->tpc, m->part, m->x_res, (size_t)M * H, st);
        if ((rc = allreduce_sum(m, m->part, (size_t)M * H))) return rc;
        if ((rc = launch_add_inplace(m->x_res, m->part, (size_t)M * H, st))) return rc;
    }
    return DU_OK;
}

// final RMSNorm + lm_head GEMV with logits and per-CTA argmax partials.  The
// selected rows (every token, or the last token of each sequence) are read in
// place: row i of the head input is x_res[logit_first + i * logit_stride].
static GemvParams head_gemv_params(du_model *m, const StepIO &io)
{
    const int H = m->H;
    GemvParams p = gp_base(m, (const uint8_t *)m->lm_head, nullptr, H);
    p.row_bytes = 2LL * H;
    p.x = m->x_res + (size_t)io.logit_first * H;
    p.ldx = H * io.logit_stride;
    p.gamma = m->final_norm; p.eps = m->cfg.rms_eps;
    p.N = m->V_l; p.map = MAP_IDENT; p.epi = EPI_LOGITS;
    p.logits = m->logits; p.ldl = m->V_l; p.vocab_off = m->rank * m->V_l;
    p.M = io.logits_rows;
    return p;
}

static int enqueue_head(du_model *m, const StepIO &io);

// The launch sequence for M token rows (decode: one per sequence; prefill: a chunk).
static int enqueue_forward(du_model *m, const StepIO &io)
{
    int rc = launch_embed(io.ids, m->embed, m->cfg.embed_scale, io.M, m->H, m->x_res, m->stream);
    if (rc) return rc;
    for (int l = 0; l < m->L; l++)
        for (int s = ST_QKV; s <= ST_DOWN; s++)
            if ((rc = enqueue_stage(m, io, l, s, true))) return rc;
    return enqueue_head(m, io);
}

// final RMSNorm + lm_head (+ argmax partials) on the selected rows, greedy pick
static int enqueue_head(du_model *m, const StepIO &io)
{
    const int H = m->H, M = io.M;
    cudaStream_t st = m->stream;
    int rc = DU_OK;
    const int R = io.logits_rows;
    GemvParams p = head_gemv_params(m, io);
    int nparts;
    GemvParams g = p;
    g.M = R;
    g.am_val = m->am_val;
    g.am_idx = m->am_idx;
    if (R >= gemm_min_tokens() && gemm_supported(Q_F16, g)) {
        // tensor-core head: one (max, argmax) partial per 128-row vocab tile and row
        nparts = (p.N + 127) / 128;
        if ((rc = launch_gemm(Q_F16, g, m->gm, st))) return rc;
    } else {
        // one CTA count for every token tile (the argmax reads nparts partials per row); a
        // single row uses the token-tile-1 layout's count, so that it runs in one wave
        nparts = gemv_grid_for(p.N, 1, R == 1 ? gemv_ctas_per_sm(Q_F16, 1, p.row_bytes) * num_sms() : m->am_parts);
        p.grid = nparts;
        const int mt = gemv_max_tokens(Q_F16, p.row_bytes);
        for (int t0 = 0; t0 < R; t0 += mt) {
            GemvParams c = p;
            c.M = R - t0 < mt ? R - t0 : mt;
            c.x = p.x + (size_t)t0 * p.ldx;
            c.logits = p.logits + (size_t)t0 * p.ldl;
            c.am_val = m->am_val + (size_t)t0 * nparts;
            c.am_idx = m->am_idx + (size_t)t0 * nparts;
            if ((rc = launch_gemv(Q_F16, c, st))) return rc;
        }
    }
    TokHist hist;
    if (io.advance) {   // decode: record the greedy id at each sequence's input position
        hist.tok = m->d_hist;
        hist.cache_len = m->d_cache_len;
        hist.cap = m->cap;
    }
    if (io.sample) {
        // repetition / presence penalty (settings in device memory), counting this step's
        // input ids as seen; then temperature / top-k / top-p / min-p over the full logits
        // (single GPU)
        if (io.penalize && (rc = launch_penalties(m->logits, R, m->V, m->V_l, m->d_seen, m->V, io.ids,
                                                  m->d_sparams + 4, 0.0f, 1.0f, st)))
            return rc;
        if ((rc = launch_sample(m->logits, R, m->V, m->V_l, 1.0f, 0, 1.0f, 0.0f, m->d_seeds, io.next_out, io.feed, hist,
                                m->d_err, st, m->d_sparams)))
            return rc;
    } else if (m->tp == 1) {
        if ((rc = launch_argmax_final(m->am_val, m->am_idx, R, nparts, io.next_out, io.feed, hist, st))) return rc;
    } else {
        // local best (val, idx) per row, exchange the pairs between ranks, pick the global best
        if ((rc = launch_argmax_final_pairs(m->am_val, m->am_idx, R, nparts, m->best_val, st))) return rc;
        const NcclApi *api = nccl_api();
        if ((rc = nccl_check(m, api->AllGather(m->best_val, m->gbest_val, (size_t)m->max_tokens * 2, ncclFloat32,
                                               m->comm, st), "ncclAllGather")))
            return rc;
        if ((rc = launch_argmax_pick_tp(m->gbest_val, m->tp, m->max_tokens, R, io.next_out, io.feed, hist, st)))
            return rc;
    }
    if (io.advance) {
        if ((rc = launch_step_advance(m->d_cache_len, M, st))) return rc;
    }
    return DU_OK;
}

// One forward per call at a time per handle (LLM Busy guard, LLM.cs:393-406).
int sync_cache_len(du_model *m)
{
    DU_CUDA_TRY(cudaMemcpyAsync(m->d_cache_len, m->h_cache_len.data(), sizeof(int) * m->maxb, cudaMemcpyHostToDevice,
                                m->stream));
    return DU_OK;
}

static StepIO decode_io(du_model *m, int batch)
{
    StepIO io = {};
    io.M = batch;
    io.ids = m->d_ids;
    io.pos = m->d_cache_len;
    io.seq_of = nullptr;
    io.kv_len = m->d_cache_len;
    io.kv_len_add = 1;
    io.kv_new = 1;
    io.p2p = true;
    io.fd_nsplit = fd_choose_splits(batch, m->hkv_l, m->cap);
    io.logits_rows = batch;
    io.logit_stride = 1;
    io.logit_first = 0;
    io.next_out = m->d_next;
    io.feed = m->d_ids;
    io.advance = true;
    return io;
}

// Stage list of the persistent decode-step kernel for the decode rows of `io`.
// Fails (and the caller falls back to per-stage kernels) when the model asks for
// that (no DU_FLAG_PERSISTENT, or DU_FLAG_NO_PERSISTENT), runs tensor-parallel, or the batch does not fit
// one token tile / the shared-memory budget.
static int build_step_plan(du_model *m, const StepIO &io, StepPlan *plan, int *qt_out, int *mt_out, size_t *smem_out,
                           StepStage **d_stages)
{
    *d_stages = nullptr;
    if (!(m->cfg.flags & DU_FLAG_PERSISTENT) || (m->cfg.flags & DU_FLAG_NO_PERSISTENT) || m->tp > 1 || io.M > 8 ||
        m->kv8 || m->arch != 0 || m->window > 0 || m->hd > 128)
        return DU_ESTATE;
    const int qt = qt_of(m->quant);
    const int mt = io.M <= 1 ? 1 : io.M <= 2 ? 2 : io.M <= 4 ? 4 : 8;
    std::vector<StepStage> st;
    StepStage s0 = {};
    s0.type = SG_EMBED;
    st.push_back(s0);
    int nsplit = num_sms() / (io.M * m->hkv_l);
    if (nsplit < 1) nsplit = 1;
    if (nsplit > FD_MAXSPLIT) nsplit = FD_MAXSPLIT;
    size_t xmax = 16;
    for (int l = 0; l < m->L; l++)
        for (int sg = ST_QKV; sg <= ST_DOWN; sg++) {
            StepStage s = {};
            if (sg == ST_ATTN) {
                s.type = SG_ATTN;
                s.a = stage_attn_params(m, io, l, nsplit, &s.G);
                s.nsplit = nsplit;
                s.nq = io.M;
                s.a_new = 1;
            } else {
                s.type = SG_GEMV;
                s.qt = qt;
                s.g = stage_gemv_params(m, io, l, sg);
                const size_t xb = gemv_x_bytes(qt, mt, s.g.row_bytes);
                if (xb > xmax) xmax = xb;
            }
            st.push_back(s);
        }
    StepStage hs = {};
    hs.type = SG_GEMV;
    hs.qt = Q_F16;
    hs.g = head_gemv_params(m, io);
    hs.g.am_val = m->am_val;
    hs.g.am_idx = m->am_idx;
    if (gemv_x_bytes(Q_F16, mt, hs.g.row_bytes) > xmax) xmax = gemv_x_bytes(Q_F16, mt, hs.g.row_bytes);
    st.push_back(hs);
    StepStage as = {};
    as.type = SG_ARGMAX;
    st.push_back(as);

    const size_t ring_l = step_ring_bytes(qt, mt, ds_depth(mt));          // the layers' linears
    const size_t ring_h = step_ring_bytes(Q_F16, mt, ds_head_depth(mt));  // lm_head
    const size_t tiles = (size_t)4 * FD_TILE * (m->hd + 8) * sizeof(__half);    // attention K/V tiles alias the ring
    size_t ring = ring_l > ring_h ? ring_l : ring_h;
    if (tiles > ring) ring = tiles;
    const size_t smem = ring + xmax;
    if (smem > step_smem_limit(qt, mt, m->hd)) return DU_ESTATE;
    if (qt == Q_I4 && ((m->H / m->group) % 2 || (m->I_l / m->group) % 2)) return DU_ESTATE;

    DU_CUDA_TRY(cudaMalloc(d_stages, sizeof(StepStage) * st.size()));
    DU_CUDA_TRY(cudaMemcpy(*d_stages, st.data(), sizeof(StepStage) * st.size(), cudaMemcpyHostToDevice));
    StepPlan p = {};
    p.nstages = (int)st.size();
    p.stages = *d_stages;
    p.ring_bytes = ring;
    p.ids = io.ids;
    p.embed = m->embed;
    p.embed_scale = m->cfg.embed_scale;
    p.M = io.M;
    p.H = m->H;
    p.x_res = m->x_res;
    p.am_val = m->am_val;
    p.am_idx = m->am_idx;
    p.nparts = num_sms();
    p.next_out = io.next_out;
    p.feed = io.feed;
    p.hist = m->d_hist;
    p.cache_len = m->d_cache_len;
    p.cap = m->cap;
    p.advance = io.advance ? 1 : 0;
    p.barrier = m->d_barrier;
    p.err = m->d_err;

    p.stamps = m->d_stamps;
    m->stamp_stages = p.nstages;
    *plan = p;
    *qt_out = qt;
    *mt_out = mt;
    *smem_out = smem;
    return DU_OK;
}

// Reports (and clears) a barrier timeout of the persistent step kernel.
static int check_step_error(du_model *m)
{
    if (*m->h_pin_err == 0) return DU_OK;
    *m->h_pin_err = 0;
    cudaMemset(m->d_err, 0, sizeof(int));
    return fail(DU_ECUDA, "a device wait timed out (grid barrier, tensor-parallel peer or GEMM pipeline); "
                          "the call was aborted");
}

static int get_graph(du_model *m, int batch, cudaGraphExec_t *out, Graph **gout = nullptr, bool sample = false,
                     bool penalize = false)
{
    std::map<int, Graph> &gm = penalize ? m->pgraphs : sample ? m->sgraphs : m->graphs;
    auto it = gm.find(batch);
    if (it != gm.end()) {
        *out = it->second.exec;
        if (gout) *gout = &it->second;
        return DU_OK;
    }
    StepIO io = decode_io(m, batch);
    io.sample = sample || penalize;
    io.penalize = penalize;
    Graph g;
    StepPlan plan;
    int qt = 0, mt = 0;
    size_t smem = 0;
    const bool persistent = !io.sample && build_step_plan(m, io, &plan, &qt, &mt, &smem, &g.d_stages) == DU_OK;
    DU_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc;
    if (persistent) {
        cudaError_t me = cudaMemsetAsync(m->d_barrier, 0, sizeof(unsigned), m->stream);
        rc = me == cudaSuccess ? launch_decode_step(plan, qt, mt, m->hd, smem, m->stream)
                               : cuda_fail(me, "cudaMemsetAsync");
    } else {
        rc = enqueue_forward(m, io);
    }
    cudaError_t e = cudaStreamEndCapture(m->stream, &g.g);
    g.persistent = persistent;
    if (rc) {
        if (g.g) cudaGraphDestroy(g.g);
        if (g.d_stages) cudaFree(g.d_stages);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&g.exec, g.g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g.g);
        return cuda_fail(e, "cudaGraphInstantiate");
    }
    gm[batch] = g;
    *out = g.exec;
    if (gout) *gout = &gm[batch];
    return DU_OK;
}

static int check_ids(du_model *m, const int32_t *ids, size_t n)
{
    for (size_t i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= m->V) return fail(DU_EINVAL, "token id outside [0, vocab_size)");
    return DU_OK;
}

}  // namespace du

using namespace du;

extern "C" {

DU_API int du_model_create(const du_model_config *cfg, du_model **out)
{
    DU_CHECK_ARG(cfg && out, "du_model_create: null argument");
    *out = nullptr;
    int rc = check_cfg(*cfg);
    if (rc) return rc;
    du_model *m = new du_model();
    m->cfg = *cfg;
    cudaGetDevice(&m->device);
    m->tp = cfg->tp_size <= 0 ? 1 : cfg->tp_size;
    m->cfg.tp_size = m->tp;
    m->rank = cfg->tp_rank;
    m->H = cfg->hidden_size; m->I = cfg->intermediate_size; m->L = cfg->num_layers;
    m->hq = cfg->num_heads_q; m->hkv = cfg->num_heads_kv; m->hd = cfg->head_dim; m->V = cfg->vocab_size;
    m->hq_l = m->hq / m->tp; m->hkv_l = m->hkv / m->tp; m->I_l = m->I / m->tp; m->V_l = m->V / m->tp;
    m->qkv_rows = (m->hq_l * ((cfg->arch_flags & DU_ARCH_ATTN_GATE) ? 2 : 1) + 2 * m->hkv_l) * m->hd;
    m->quant = cfg->quant;
    m->group = cfg->quant == DU_QUANT_INT4 ? cfg->group_size : 32;
    m->cap = cfg->kv_capacity;
    m->kv8 = cfg->kv_quant == DU_KV_INT8;
    m->arch = cfg->arch_flags;
    m->window = cfg->sliding_window;
    m->pattern = cfg->sliding_pattern;
    m->attn_scale = cfg->attn_scale > 0.0f ? cfg->attn_scale : powf((float)cfg->head_dim, -0.5f);
    m->maxb = cfg->max_batch;
    m->max_tokens = m->maxb > 256 ? m->maxb : 256;
    if (m->cfg.embed_scale == 0.0f) m->cfg.embed_scale = 1.0f;
    cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete m;
        return cuda_fail(e, "cudaStreamCreate");
    }
    rc = model_alloc(m);
    if (rc) {
        model_free(m);
        delete m;
        return rc;
    }
    *out = m;
    return DU_OK;
}

DU_API int du_model_destroy(du_model *m)
{
    if (!m) return DU_OK;
    if (m->busy.exchange(1) != 0) return fail(DU_EBUSY, "du_model_destroy: model is busy");
    model_free(m);
    delete m;
    return DU_OK;
}

DU_API int du_model_load_tensor(du_model *m, const char *name, const void *host, size_t bytes)
{
    DU_GUARD(m);
    DU_CHECK_ARG(name && host, "du_model_load_tensor: null argument");
    int rc = place_tensor(m, name, host, bytes, cudaMemcpyHostToDevice);
    if (rc) return rc;
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return DU_OK;
}

DU_API int du_model_init_random(du_model *m, uint64_t seed, float std)
{
    DU_GUARD(m);
    cudaStream_t st = m->stream;
    const int H = m->H, hd = m->hd;
    const int64_t big = (int64_t)m->I * H > (int64_t)(m->hq + 2 * m->hkv) * hd * H ? (int64_t)m->I * H
                                                                                   : (int64_t)m->hq * hd * H;
    float *tmp = nullptr;
    uint8_t *qtmp = nullptr;
    __half *stmp = nullptr;
    DU_CUDA_TRY(cudaMalloc(&tmp, sizeof(float) * big));
    int rc = DU_OK;
    if (cudaMalloc(&qtmp, (size_t)big * 2) != cudaSuccess || cudaMalloc(&stmp, (size_t)big / 16 + 1024) != cudaSuccess)
        rc = fail(DU_ENOMEM, "du_model_init_random: temp allocation failed");
    const char *ext = m->quant == DU_QUANT_INT4 ? ".int4.bin" : m->quant == DU_QUANT_INT8 ? ".int8.bin" : ".bin";
    static const char *stems[] = {"self_attn_q_proj", "self_attn_k_proj", "self_attn_v_proj", "self_attn_o_proj",
                                  "mlp_gate_proj", "mlp_up_proj", "mlp_down_proj"};
    uint64_t tid = 0;
    for (int l = 0; l < m->L && !rc; l++) {
        for (int t = 0; t < 7 && !rc; t++) {
            int64_t rows, cols;
            switch (t) {
            case 0: rows = (int64_t)m->hq * hd; cols = H; break;
            case 1: case 2: rows = (int64_t)m->hkv * hd; cols = H; break;
            case 3: rows = H; cols = (int64_t)m->hq * hd; break;
            case 4: case 5: rows = m->I; cols = H; break;
            default: rows = H; cols = m->I; break;
            }
            const uint64_t s = seed * 0x9E3779B97F4A7C15ull + (++tid);
            if ((rc = launch_random_normal(tmp, (size_t)(rows * cols), s, 0, std, st))) break;
            char name[96];
            snprintf(name, sizeof name, "layer_%d/%s%s", l, stems[t], ext);
            if (m->quant == DU_QUANT_FP16) {
                // fp16 linears: convert in place through the half generator for the same values
                if ((rc = launch_random_normal_half((__half *)qtmp, (size_t)(rows * cols), s, 0, std, st))) break;
                rc = place_tensor(m, name, qtmp, (size_t)(rows * cols * 2), cudaMemcpyDeviceToDevice);
                continue;
            }
            if (m->quant == DU_QUANT_INT8) rc = launch_quantize_int8(tmp, rows, cols, (int8_t *)qtmp, stmp, st);
            else rc = launch_quantize_int4(tmp, rows, cols, m->group, qtmp, stmp, st);
            if (rc) break;
            if ((rc = place_tensor(m, name, qtmp, (size_t)qbytes(m->quant, rows, cols), cudaMemcpyDeviceToDevice)))
                break;
            snprintf(name, sizeof name, "layer_%d/%s.scales.bin", l, stems[t]);
            rc = place_tensor(m, name, stmp, (size_t)sbytes(m->quant, m->group, rows, cols), cudaMemcpyDeviceToDevice);
        }
        if (!rc) rc = launch_fill_half(m->layers[l].ln1, H, 0.0f, st);
        if (!rc) rc = launch_fill_half(m->layers[l].ln2, H, 0.0f, st);
    }
    if (!rc) rc = launch_fill_half(m->final_norm, H, 0.0f, st);
    if (!rc) rc = launch_random_normal_half(m->embed, (size_t)m->V * H, seed * 0x9E3779B97F4A7C15ull + 0xE1ull, 0, std, st);
    if (!rc && !m->cfg.tie_embedding)
        rc = launch_random_normal_half(m->lm_head, (size_t)m->V_l * H, seed * 0x9E3779B97F4A7C15ull + 0xE2ull,
                                       (uint64_t)m->rank * m->V_l * H, std, st);
    cudaStreamSynchronize(st);
    cudaFree(tmp);
    if (qtmp) cudaFree(qtmp);
    if (stmp) cudaFree(stmp);
    if (rc) return rc;
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

DU_API int du_tp_init(du_model *m, const void *nccl_unique_id, int timeout_ms)
{
    DU_GUARD(m);
    DU_CHECK_ARG(nccl_unique_id != nullptr, "du_tp_init: null unique id");
    if (m->tp == 1) return DU_OK;
    const NcclApi *n = nccl_api();
    if (!n) return DU_ENCCL;
    ncclUniqueId id;
    memcpy(&id, nccl_unique_id, sizeof id);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    m->nccl_timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
    ncclResult_t r = n->CommInitRankConfig(&m->comm, m->tp, id, m->rank, &config);
    if (r != ncclSuccess && r != ncclInProgress)
        return fail(DU_ENCCL, std::string("ncclCommInitRankConfig: ") + n->GetErrorString(r));
    int rc = nccl_check(m, ncclInProgress, "ncclCommInitRankConfig");
    if (rc) return rc;
    m->tp_ready = true;
    return tp_comm_alloc(&m->tpc, ((size_t)m->maxb * m->H + 3) & ~(size_t)3);
}

DU_API int du_tp_comm_handle(du_model *m, void *handle_out64)
{
    DU_GUARD(m);
    DU_CHECK_ARG(handle_out64 != nullptr, "du_tp_comm_handle: null output");
    if (m->tp == 1 || !m->tp_ready) return fail(DU_ESTATE, "du_tp_comm_handle: call du_tp_init first");
    return tp_comm_handle(&m->tpc, handle_out64);
}

DU_API int du_tp_comm_open(du_model *m, const void *handles, int nranks)
{
    DU_GUARD(m);
    DU_CHECK_ARG(handles != nullptr && nranks == m->tp, "du_tp_comm_open: need one 64-byte handle per rank");
    if (m->tp == 1 || !m->tp_ready) return fail(DU_ESTATE, "du_tp_comm_open: call du_tp_init first");
    if (!m->graphs.empty()) return fail(DU_ESTATE, "du_tp_comm_open: open before the first decode step");
    return tp_comm_open(&m->tpc, handles, nranks, m->rank, m->d_err);
}

DU_API int du_forward(du_model *m, const int32_t *ids, int batch, int seq_len, int use_cache, int last_pos_only,
                      float *logits_out, int32_t *next_ids_out)
{
    DU_GUARD(m);
    DU_CHECK_ARG(ids && batch > 0 && seq_len > 0, "du_forward: bad arguments");
    DU_CHECK_ARG(batch <= m->maxb, "du_forward: batch exceeds max_batch");
    if (m->tp > 1 && !m->tp_ready) return fail(DU_ESTATE, "du_forward: call du_tp_init first");
    int rc = check_ids(m, ids, (size_t)batch * seq_len);
    if (rc) return rc;
    if (!use_cache)
        for (int b = 0; b < batch; b++) m->h_cache_len[b] = 0;   // stateless forward from position 0
    for (int b = 0; b < batch; b++)
        if (m->h_cache_len[b] + seq_len > m->cap) return fail(DU_EINVAL, "du_forward: KV cache capacity exceeded");
    cudaStream_t st = m->stream;
    const int H = m->H;
    // chunk the positions so that batch * chunk <= max_tokens
    int chunk = m->max_tokens / batch;
    if (chunk < 1) chunk = 1;
    std::vector<int> hbuf;
    float *big_logits = nullptr;
    if (!last_pos_only && logits_out) {
        DU_CUDA_TRY(cudaMalloc(&big_logits, sizeof(float) * (size_t)m->max_tokens * m->V_l * (m->tp > 1 ? m->tp + 1 : 1)));
    }
    for (int s0 = 0; s0 < seq_len && !rc; s0 += chunk) {
        const int s1 = s0 + chunk < seq_len ? s0 + chunk : seq_len;
        const int Lc = s1 - s0, M = batch * Lc;
        hbuf.assign((size_t)4 * M, 0);
        for (int b = 0; b < batch; b++)
            for (int l = 0; l < Lc; l++) {
                const int t = b * Lc + l;
                hbuf[t] = ids[(size_t)b * seq_len + s0 + l];
                hbuf[M + t] = m->h_cache_len[b] + s0 + l;           // position / cache slot
                hbuf[2 * M + t] = b;                                // sequence
                hbuf[3 * M + t] = m->h_cache_len[b] + s0 + l + 1;   // causal kv length
            }
        DU_CUDA_TRY(cudaMemcpyAsync(m->d_ids, hbuf.data(), sizeof(int) * M, cudaMemcpyHostToDevice, st));
        DU_CUDA_TRY(cudaMemcpyAsync(m->d_pos, hbuf.data() + M, sizeof(int) * M, cudaMemcpyHostToDevice, st));
        DU_CUDA_TRY(cudaMemcpyAsync(m->d_seq, hbuf.data() + 2 * M, sizeof(int) * M, cudaMemcpyHostToDevice, st));
        DU_CUDA_TRY(cudaMemcpyAsync(m->d_kvlen, hbuf.data() + 3 * M, sizeof(int) * M, cudaMemcpyHostToDevice, st));
        StepIO io = {};
        io.M = M; io.ids = m->d_ids; io.pos = m->d_pos; io.seq_of = m->d_seq; io.kv_len = m->d_kvlen;
        io.kv_len_add = 0;
        int maxkv = 0;
        for (int b = 0; b < batch; b++) maxkv = maxkv > m->h_cache_len[b] + s1 ? maxkv : m->h_cache_len[b] + s1;
        io.fd_nsplit = fd_choose_splits(M, m->hkv_l, maxkv);
        const bool last_chunk = s1 == seq_len;
        if (last_pos_only) {
            io.logits_rows = batch; io.logit_first = Lc - 1; io.logit_stride = Lc;
        } else {
            io.logits_rows = M; io.logit_first = 0; io.logit_stride = 1;
        }
        io.next_out = m->d_next;
        io.feed = nullptr;
        io.advance = false;
        if (!last_pos_only && logits_out) {
            // all-position logits: run the head per chunk into the big buffer
            float *saved = m->logits;
            m->logits = big_logits;
            rc = enqueue_forward(m, io);
            m->logits = saved;
            if (rc) break;
            float *src = big_logits;
            if (m->tp > 1) {
                const NcclApi *api = nccl_api();
                float *dst = big_logits + (size_t)m->max_tokens * m->V_l;
                if ((rc = nccl_check(m, api->AllGather(big_logits, dst, (size_t)m->max_tokens * m->V_l, ncclFloat32,
                                                       m->comm, st), "ncclAllGather")))
                    break;
                src = dst;
            }
            std::vector<float> tmp((size_t)M * m->V_l * m->tp);
            for (int r = 0; r < m->tp; r++)
                DU_CUDA_TRY(cudaMemcpyAsync(tmp.data() + (size_t)r * M * m->V_l, src + (size_t)r * m->max_tokens * m->V_l,
                                            sizeof(float) * M * m->V_l, cudaMemcpyDeviceToHost, st));
            DU_CUDA_TRY(cudaStreamSynchronize(st));
            for (int b = 0; b < batch; b++)
                for (int l = 0; l < Lc; l++)
                    for (int r = 0; r < m->tp; r++)
                        memcpy(logits_out + ((size_t)b * seq_len + s0 + l) * m->V + (size_t)r * m->V_l,
                               tmp.data() + ((size_t)r * M + b * Lc + l) * m->V_l, sizeof(float) * m->V_l);
        } else if (last_chunk || !last_pos_only) {
            rc = enqueue_forward(m, io);
        } else {
            // earlier chunks of a last-position-only prefill: no head needed, but the
            // launch sequence is the same; the logits of the last chunk overwrite these
            rc = enqueue_forward(m, io);
        }
    }
    if (big_logits) {
        cudaStreamSynchronize(st);
        cudaFree(big_logits);
    }
    if (rc) return rc;
    // use_cache == 0 (LLM.Predict): the cache rows served as scratch, nothing stays visible
    for (int b = 0; b < batch; b++) m->h_cache_len[b] = use_cache ? m->h_cache_len[b] + seq_len : 0;
    if ((rc = sync_cache_len(m))) return rc;
    m->last_batch = batch;
    if (next_ids_out) {
        DU_CUDA_TRY(cudaMemcpyAsync(m->h_pin_next, m->d_next, sizeof(int) * batch, cudaMemcpyDeviceToHost, st));
    }
    DU_CUDA_TRY(cudaMemcpyAsync(m->h_pin_err, m->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaStreamSynchronize(st));
    if ((rc = check_step_error(m))) return rc;
    if (next_ids_out) memcpy(next_ids_out, m->h_pin_next, sizeof(int) * batch);
    if (last_pos_only && logits_out) {
        m->busy.store(0);
        _guard.ok = false;
        return du_read_logits(m, logits_out, batch);
    }
    (void)H;
    return DU_OK;
}

DU_API int du_read_logits(du_model *m, float *host_out, int batch)
{
    DU_GUARD(m);
    DU_CHECK_ARG(host_out && batch > 0 && batch <= m->maxb, "du_read_logits: bad arguments");
    cudaStream_t st = m->stream;
    if (m->tp == 1) {
        DU_CUDA_TRY(cudaMemcpyAsync(host_out, m->logits, sizeof(float) * batch * m->V_l, cudaMemcpyDeviceToHost, st));
        DU_CUDA_TRY(cudaStreamSynchronize(st));
        return DU_OK;
    }
    const NcclApi *api = nccl_api();
    int rc = nccl_check(m, api->AllGather(m->logits, m->logits_all, (size_t)m->maxb * m->V_l, ncclFloat32, m->comm, st),
                        "ncclAllGather");
    if (rc) return rc;
    std::vector<float> tmp((size_t)m->tp * m->maxb * m->V_l);
    DU_CUDA_TRY(cudaMemcpyAsync(tmp.data(), m->logits_all, sizeof(float) * tmp.size(), cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaStreamSynchronize(st));
    for (int b = 0; b < batch; b++)
        for (int r = 0; r < m->tp; r++)
            memcpy(host_out + (size_t)b * m->V + (size_t)r * m->V_l, tmp.data() + ((size_t)r * m->maxb + b) * m->V_l,
                   sizeof(float) * m->V_l);
    return DU_OK;
}

DU_API int du_decode_step(du_model *m, const int32_t *ids, int batch, int32_t *next_ids)
{
    DU_GUARD(m);
    DU_CHECK_ARG(ids && next_ids && batch > 0 && batch <= m->maxb, "du_decode_step: bad arguments");
    if (m->tp > 1 && !m->tp_ready) return fail(DU_ESTATE, "du_decode_step: call du_tp_init first");
    int rc = check_ids(m, ids, batch);
    if (rc) return rc;
    for (int b = 0; b < batch; b++)
        if (m->h_cache_len[b] + 1 > m->cap) return fail(DU_EINVAL, "du_decode_step: KV cache capacity exceeded");
    cudaGraphExec_t exec;
    if ((rc = get_graph(m, batch, &exec))) return rc;
    cudaStream_t st = m->stream;
    memcpy(m->h_pin_ids, ids, sizeof(int) * batch);
    DU_CUDA_TRY(cudaMemcpyAsync(m->d_ids, m->h_pin_ids, sizeof(int) * batch, cudaMemcpyHostToDevice, st));
    DU_CUDA_TRY(cudaGraphLaunch(exec, st));
    DU_CUDA_TRY(cudaMemcpyAsync(m->h_pin_next, m->d_next, sizeof(int) * batch, cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaMemcpyAsync(m->h_pin_err, m->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaStreamSynchronize(st));
    if ((rc = check_step_error(m))) {
        sync_cache_len(m);   // the aborted step may or may not have advanced the device copy
        cudaStreamSynchronize(st);
        return rc;
    }
    memcpy(next_ids, m->h_pin_next, sizeof(int) * batch);
    for (int b = 0; b < batch; b++) m->h_cache_len[b] += 1;
    m->last_batch = batch;
    return DU_OK;
}

}  // extern "C"

namespace du {

// One sampled decode step (du_decode_step_sample / _ex): settings and seeds go to
// device memory, then the captured graph of this batch size runs.
static int decode_step_sample_impl(du_model *m, const int32_t *ids, int batch, float temperature, int top_k,
                                   float top_p, float min_p, bool penalize, float presence, float repetition,
                                   const int32_t *seeds, int32_t *next_ids, const char *name)
{
    DU_CHECK_ARG(ids && seeds && next_ids && batch > 0 && batch <= m->maxb, std::string(name) + ": bad arguments");
    if (m->tp > 1) return fail(DU_ESTATE, std::string(name) + ": stochastic sampling runs on a single GPU");
    if (!sample_supported(temperature, top_k, top_p, m->V))
        return fail(DU_EINVAL, std::string(name) + ": top_p < 1 needs top_k in 1..64 (the reference's parallel sampler)");
    if (penalize && !(repetition > 0.0f)) return fail(DU_EINVAL, std::string(name) + ": repetition_penalty must be > 0");
    int rc = check_ids(m, ids, batch);
    if (rc) return rc;
    for (int b = 0; b < batch; b++)
        if (m->h_cache_len[b] + 1 > m->cap) return fail(DU_EINVAL, std::string(name) + ": KV cache capacity exceeded");
    cudaGraphExec_t exec;
    if ((rc = get_graph(m, batch, &exec, nullptr, true, penalize))) return rc;
    cudaStream_t st = m->stream;
    memcpy(m->h_pin_ids, ids, sizeof(int) * batch);
    memcpy(m->h_pin_seeds, seeds, sizeof(int32_t) * batch);
    float *hp = reinterpret_cast<float *>(m->h_pin_seeds + m->maxb);
    hp[0] = temperature;
    hp[1] = (float)top_k;
    hp[2] = top_p;
    hp[3] = min_p;
    hp[4] = penalize ? presence : 0.0f;
    hp[5] = penalize ? repetition : 1.0f;
    DU_CUDA_TRY(cudaMemcpyAsync(m->d_ids, m->h_pin_ids, sizeof(int) * batch, cudaMemcpyHostToDevice, st));
    DU_CUDA_TRY(cudaMemcpyAsync(m->d_seeds, m->h_pin_seeds, sizeof(int32_t) * (m->maxb + SAMPLE_PARAMS),
                                cudaMemcpyHostToDevice, st));
    DU_CUDA_TRY(cudaGraphLaunch(exec, st));
    DU_CUDA_TRY(cudaMemcpyAsync(m->h_pin_next, m->d_next, sizeof(int) * batch, cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaMemcpyAsync(m->h_pin_err, m->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaStreamSynchronize(st));
    if ((rc = check_step_error(m))) {
        sync_cache_len(m);
        cudaStreamSynchronize(st);
        return rc;
    }
    memcpy(next_ids, m->h_pin_next, sizeof(int) * batch);
    for (int b = 0; b < batch; b++) m->h_cache_len[b] += 1;
    m->last_batch = batch;
    return DU_OK;
}

}  // namespace du

extern "C" {

DU_API int du_decode_step_sample(du_model *m, const int32_t *ids, int batch, float temperature, int top_k,
                                 float top_p, float min_p, const int32_t *seeds, int32_t *next_ids)
{
    DU_GUARD(m);
    return decode_step_sample_impl(m, ids, batch, temperature, top_k, top_p, min_p, false, 0.0f, 1.0f, seeds, next_ids,
                                   "du_decode_step_sample");
}

DU_API int du_decode_step_sample_ex(du_model *m, const int32_t *ids, int batch, float temperature, int top_k,
                                    float top_p, float min_p, float presence_penalty, float repetition_penalty,
                                    const int32_t *seeds, int32_t *next_ids)
{
    DU_GUARD(m);
    return decode_step_sample_impl(m, ids, batch, temperature, top_k, top_p, min_p, true, presence_penalty,
                                   repetition_penalty, seeds, next_ids, "du_decode_step_sample_ex");
}

DU_API int du_decode_loop(du_model *m, const int32_t *ids, int batch, int n_steps, int32_t *tokens_out)
{
    DU_GUARD(m);
    DU_CHECK_ARG(ids && tokens_out && batch > 0 && batch <= m->maxb && n_steps >= 0, "du_decode_loop: bad arguments");
    if (m->tp > 1 && !m->tp_ready) return fail(DU_ESTATE, "du_decode_loop: call du_tp_init first");
    int rc = check_ids(m, ids, batch);
    if (rc) return rc;
    for (int b = 0; b < batch; b++)
        if (m->h_cache_len[b] + n_steps > m->cap) return fail(DU_EINVAL, "du_decode_loop: KV cache capacity exceeded");
    if (n_steps == 0) return DU_OK;
    cudaGraphExec_t exec;
    if ((rc = get_graph(m, batch, &exec))) return rc;
    cudaStream_t st = m->stream;
    memcpy(m->h_pin_ids, ids, sizeof(int) * batch);
    DU_CUDA_TRY(cudaMemcpyAsync(m->d_ids, m->h_pin_ids, sizeof(int) * batch, cudaMemcpyHostToDevice, st));
    // back-to-back graph replays; each step's argmax feeds the next step's input on
    // the device and is recorded at its input position of the token history
    for (int s = 0; s < n_steps; s++) DU_CUDA_TRY(cudaGraphLaunch(exec, st));
    std::vector<int> h((size_t)batch * n_steps);
    for (int b = 0; b < batch; b++)
        DU_CUDA_TRY(cudaMemcpyAsync(h.data() + (size_t)b * n_steps, m->d_hist + (size_t)b * m->cap + m->h_cache_len[b],
                                    sizeof(int) * n_steps, cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaMemcpyAsync(m->h_pin_err, m->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    DU_CUDA_TRY(cudaStreamSynchronize(st));
    if ((rc = check_step_error(m))) {
        sync_cache_len(m);
        cudaStreamSynchronize(st);
        return rc;
    }
    for (int s = 0; s < n_steps; s++)
        for (int b = 0; b < batch; b++) tokens_out[(size_t)s * batch + b] = h[(size_t)b * n_steps + s];
    for (int b = 0; b < batch; b++) m->h_cache_len[b] += n_steps;
    m->last_batch = batch;
    return DU_OK;
}

DU_API int du_reset_cache(du_model *m)
{
    DU_GUARD(m);
    for (int b = 0; b < m->maxb; b++) m->h_cache_len[b] = 0;
    int rc = sync_cache_len(m);
    if (rc) return rc;
    // ZeroTokenSeen (Qwen3_5CS.compute:1443-1451, on ResetCache): penalties start fresh
    if (m->d_seen)
        DU_CUDA_TRY(cudaMemsetAsync(m->d_seen, 0, sizeof(unsigned) * (size_t)m->maxb * m->V, m->stream));
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return DU_OK;
}

DU_API int du_cache_len(du_model *m, int seq, int *out)
{
    DU_GUARD(m);
    DU_CHECK_ARG(out && seq >= 0 && seq < m->maxb, "du_cache_len: bad arguments");
    *out = m->h_cache_len[seq];
    return DU_OK;
}

DU_API int du_model_stream(du_model *m, void **stream_out)
{
    DU_CHECK_ARG(m && stream_out, "du_model_stream: null argument");
    *stream_out = m->stream;
    return DU_OK;
}

DU_API int du_model_weight_bytes(du_model *m, uint64_t *out)
{
    DU_CHECK_ARG(m && out, "du_model_weight_bytes: null argument");
    *out = m->weight_bytes;
    return DU_OK;
}

DU_API int du_tp_shard_window(const du_model_config *cfg, const char *tensor, int64_t *out6)
{
    DU_CHECK_ARG(cfg && tensor && out6, "du_tp_shard_window: null argument");
    int rc = check_cfg(*cfg);
    if (rc) return rc;
    const int tk = tensor_kind_of(tensor);
    if (tk == T_NONE) return fail(DU_ENOTFOUND, std::string("du_tp_shard_window: unknown tensor ") + tensor);
    ShardWindow w;
    if ((rc = shard_window(*cfg, tk, &w))) return rc;
    out6[0] = w.rows; out6[1] = w.cols; out6[2] = w.r0; out6[3] = w.r1; out6[4] = w.c0; out6[5] = w.c1;
    return DU_OK;
}

DU_API int du_model_graph_info(du_model *m, int batch, int *kernel_nodes, int *total_nodes)
{
    DU_GUARD(m);
    DU_CHECK_ARG(kernel_nodes && total_nodes && batch > 0 && batch <= m->maxb, "du_model_graph_info: bad arguments");
    if (m->tp > 1 && !m->tp_ready) return fail(DU_ESTATE, "du_model_graph_info: call du_tp_init first");
    cudaGraphExec_t exec;
    Graph *g = nullptr;
    int rc = get_graph(m, batch, &exec, &g);
    if (rc) return rc;
    size_t n = 0;
    DU_CUDA_TRY(cudaGraphGetNodes(g->g, nullptr, &n));
    std::vector<cudaGraphNode_t> nodes(n);
    DU_CUDA_TRY(cudaGraphGetNodes(g->g, nodes.data(), &n));
    int k = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        DU_CUDA_TRY(cudaGraphNodeGetType(nd, &t));
        if (t == cudaGraphNodeTypeKernel) k++;
    }
    *kernel_nodes = k;
    *total_nodes = (int)n;
    return DU_OK;
}

DU_API int du_model_stage_times(du_model *m, float *us_out, int max_stages, int *n_out)
{
    DU_GUARD(m);
    DU_CHECK_ARG(us_out && n_out && max_stages >= 0, "du_model_stage_times: bad arguments");
    *n_out = 0;
    if (m->stamp_stages <= 0) return DU_OK;
    std::vector<unsigned long long> ts((size_t)m->stamp_stages + 1);
    DU_CUDA_TRY(cudaMemcpy(ts.data(), m->d_stamps, sizeof(unsigned long long) * ts.size(), cudaMemcpyDeviceToHost));
    const int n = m->stamp_stages < max_stages ? m->stamp_stages : max_stages;
    for (int s = 0; s < n; s++) us_out[s] = (float)((double)(ts[s + 1] - ts[s]) * 1e-3);
    *n_out = n;
    return DU_OK;
}

DU_API int du_model_kernel_times(du_model *m, int batch, int reps, float *ms_out)
{
    DU_GUARD(m);
    DU_CHECK_ARG(ms_out && batch > 0 && batch <= m->maxb && reps > 0, "du_model_kernel_times: bad arguments");
    for (int b = 0; b < batch; b++)
        if (m->h_cache_len[b] + 1 > m->cap) return fail(DU_EINVAL, "du_model_kernel_times: KV cache is full");
    StepIO io = decode_io(m, batch);
    io.feed = nullptr;
    io.advance = false;
    cudaStream_t st = m->stream;
    cudaEvent_t e0, e1;
    DU_CUDA_TRY(cudaEventCreate(&e0));
    DU_CUDA_TRY(cudaEventCreate(&e1));
    int rc = DU_OK;
    for (int s = 0; s <= 5 && !rc; s++) {
        for (int pass = 0; pass < 2 && !rc; pass++) {          // pass 0 warms up
            cudaEventRecord(e0, st);
            for (int r = 0; r < reps && !rc; r++)
                for (int l = 0; l < m->L && !rc; l++)
                    rc = s < 5 ? enqueue_stage(m, io, l, s, false) : (l == 0 ? enqueue_head(m, io) : DU_OK);
            cudaEventRecord(e1, st);
        }
        if (rc) break;
        cudaEventSynchronize(e1);
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e0, e1);
        ms_out[s] = ms / (float)(reps * (s < 5 ? m->L : 1));
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc) return rc;
    DU_CUDA_TRY(cudaStreamSynchronize(st));
    return DU_OK;
}

}  // extern "C"
