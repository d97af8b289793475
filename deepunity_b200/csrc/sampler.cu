// sampler.cu -- stochastic token sampling after the lm_head: temperature, top-k,
// top-p, min-p (SampleToken / SampleTokenSerial, Gemma3CS.compute:932-1132) and
// the greedy pick (ArgMax, G3CS:911-928) when temperature <= 0.
//
// One CTA per sequence (row of logits).
//  * top_k in 1..64 (the reference's parallel path): scaled logits s = l / T,
//    probabilities exp(s - max s) / sum over the WHOLE vocabulary; the top_k
//    largest s are the candidates, in descending order with ties in the ArgMax
//    tree order (am_rank).  The reference finds them with top_k argmax passes
//    over the vocabulary; here an exact radix select on the order-preserving key
//    of s finds the top_k-th largest value in four 8-bit passes, the elements at
//    or above it are gathered and sorted (bitonic, in shared memory).  Then thread
//    0 applies the min-p cut (p < p_max * min_p), the top-p cut (stop once the
//    kept mass reaches top_p; the crossing token is kept) and draws r = runif() *
//    kept mass against the candidates' running sum.
//  * top_k <= 0 (or >= vocab) with top_p >= 1 (the reference's serial path for a
//    pure temperature / min-p sampler): probabilities exp((l - max l) / T) / sum,
//    the min-p filter, renormalisation, and r = runif() against the cumulative
//    distribution in index order (block prefix sums over contiguous slices).
//  * Other combinations (a nucleus without a top-k bound) are rejected by the
//    host with DU_EINVAL.
// runif is the reference's hash of a signed 32-bit seed (G3CS:177-186).
#include <cstdint>

#include "internal.h"

namespace du {

constexpr int SM_THREADS = 512;
constexpr int SM_MAXK = 64;
constexpr int SM_CAP = 4096;          // candidates gathered at or above the top_k-th value

__device__ __forceinline__ float sm_runif(int32_t seed)
{
    uint32_t s = (uint32_t)seed;
    s ^= 2747636419u;
    s *= 2654435769u;
    s ^= (uint32_t)((int32_t)s >> 16);
    s *= 2654435769u;
    s ^= (uint32_t)((int32_t)s >> 16);
    s *= 2654435769u;
    return __int2float_rn((int32_t)s) * (1.0f / 4294967296.0f) + 0.5f;
}

// order-preserving map of an fp32 value to uint32 (larger value -> larger key)
__device__ __forceinline__ uint32_t sm_key(float v)
{
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct SmShared {
    float red[SM_THREADS / 32];
    float fscal[4];
    unsigned hist[256];
    unsigned uscal[4];
    unsigned long long ck[SM_CAP];   // (key << 32) | (~am_rank): descending = value desc, then tree order
    float cand_p[SM_MAXK];
    int cand_i[SM_MAXK];
    float csum[SM_THREADS];
};

__device__ __forceinline__ float sm_block_max(float v, SmShared &sh)
{
    v = warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = sh.red[0];
    for (int w = 1; w < SM_THREADS / 32; w++) r = fmaxf(r, sh.red[w]);
    return r;
}

__device__ __forceinline__ float sm_block_sum(float v, SmShared &sh)
{
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.0f;
    for (int w = 0; w < SM_THREADS / 32; w++) r += sh.red[w];
    return r;
}

struct SampleParams {
    const float *logits;   // [rows][ldl]
    int ldl, V;
    float temperature, top_p, min_p;
    int top_k;
    const int32_t *seeds;  // [rows] (device)
    int32_t *out;          // [rows]
    int *feed;             // optional: also write the id here (device-resident loop)
    TokHist hist;          // optional: token history
    int *err;              // set when more than SM_CAP logits tie at the top_k-th value
    const float *dparams;  // optional device copy of (temperature, top_k, top_p, min_p): overrides the above
};

__global__ void __launch_bounds__(SM_THREADS) sample_kernel(SampleParams sp)
{
    if (sp.dparams != nullptr) {          // settings live in device memory (one captured graph serves all)
        sp.temperature = sp.dparams[0];
        sp.top_k = (int)sp.dparams[1];
        sp.top_p = sp.dparams[2];
        sp.min_p = sp.dparams[3];
    }
    extern __shared__ __align__(16) unsigned char sm_raw[];
    SmShared &sh = *reinterpret_cast<SmShared *>(sm_raw);
    const int row = blockIdx.x, tid = threadIdx.x;
    const float *lg = sp.logits + (size_t)row * sp.ldl;
    const int V = sp.V;
    int chosen = 0;

    if (!(sp.temperature > 0.0f)) {
        // greedy: ArgMax with the tree tie-break
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = tid; i < V; i += SM_THREADS)
            if (am_better(lg[i], i, bv, bi)) { bv = lg[i]; bi = i; }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if ((tid & 31) == 0) { sh.red[tid >> 5] = bv; sh.ck[tid >> 5] = (unsigned)bi; }
        __syncthreads();
        if (tid == 0) {
            bv = sh.red[0];
            bi = (int)sh.ck[0];
            for (int w = 1; w < SM_THREADS / 32; w++)
                if (am_better(sh.red[w], (int)sh.ck[w], bv, bi)) { bv = sh.red[w]; bi = (int)sh.ck[w]; }
            chosen = bi;
        }
    } else if (sp.top_k >= 1 && sp.top_k <= SM_MAXK) {
        const float inv_t = 1.0f / sp.temperature;
        // 1. max and full-vocabulary sum of exp of the scaled logits
        float mx = -3.0e38f;
        for (int i = tid; i < V; i += SM_THREADS) mx = fmaxf(mx, lg[i] * inv_t);
        const float gmax = sm_block_max(mx, sh);
        float se = 0.0f;
        for (int i = tid; i < V; i += SM_THREADS) se += expf(lg[i] * inv_t - gmax);
        const float sum_exp = fmaxf(sm_block_sum(se, sh), 1e-12f);
        const int K = sp.top_k < V ? sp.top_k : V;
        // 2. radix select: key T of the K-th largest scaled logit, and how many ties to take
        uint32_t prefix = 0;
        int need = K;
        for (int d = 3; d >= 0; d--) {
            for (int b = tid; b < 256; b += SM_THREADS) sh.hist[b] = 0u;
            __syncthreads();
            const int sh_hi = 8 * (d + 1);
            for (int i = tid; i < V; i += SM_THREADS) {
                const uint32_t k = sm_key(lg[i] * inv_t);
                if (d == 3 || (k >> sh_hi) == prefix) atomicAdd(&sh.hist[(k >> (8 * d)) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                unsigned cum = 0;
                int b = 255;
                for (; b > 0; b--) {
                    if (cum + sh.hist[b] >= (unsigned)need) break;
                    cum += sh.hist[b];
                }
                sh.uscal[0] = (prefix << 8) | (uint32_t)b;
                sh.uscal[1] = (unsigned)need - cum;
            }
            __syncthreads();
            prefix = sh.uscal[0];
            need = (int)sh.uscal[1];
            __syncthreads();
        }
        const uint32_t tkey = prefix;
        // 3. gather every element with key >= T (K - need above it, the rest ties)
        if (tid == 0) sh.uscal[2] = 0u;
        __syncthreads();
        for (int i = tid; i < V; i += SM_THREADS) {
            const uint32_t k = sm_key(lg[i] * inv_t);
            if (k >= tkey) {
                const unsigned pos = atomicAdd(&sh.uscal[2], 1u);
                if (pos < (unsigned)SM_CAP)
                    sh.ck[pos] = ((unsigned long long)k << 32) | (unsigned long long)(~am_rank(i));
            }
        }
        __syncthreads();
        unsigned n = sh.uscal[2];
        if (n > (unsigned)SM_CAP) {
            if (tid == 0 && sp.err) atomicExch(sp.err, 3);
            n = SM_CAP;
        }
        unsigned np = 1;
        while (np < n) np <<= 1;
        for (unsigned i = n + tid; i < np; i += SM_THREADS) sh.ck[i] = 0ull;
        __syncthreads();
        // 4. bitonic sort, descending
        for (unsigned size = 2; size <= np; size <<= 1)
            for (unsigned stride = size >> 1; stride > 0; stride >>= 1) {
                for (unsigned i = tid; i < np; i += SM_THREADS) {
                    const unsigned jx = i ^ stride;
                    if (jx > i) {
                        const bool desc = (i & size) == 0;
                        const unsigned long long a = sh.ck[i], b = sh.ck[jx];
                        if (desc ? a < b : a > b) { sh.ck[i] = b; sh.ck[jx] = a; }
                    }
                }
                __syncthreads();
            }
        // 5. candidates: the first K entries; index back from am_rank (a bijection on 0..2^31)
        if (tid < K) {
            const unsigned long long e = sh.ck[tid];
            const uint32_t rank = ~(uint32_t)e;
            // am_rank(i) = (brev8(i & 255) << 24) | (i >> 8)
            const uint32_t lo8 = __brev(rank & 0xFF000000u) & 255u;
            const int idx = (int)(((rank & 0x00FFFFFFu) << 8) | lo8);
            sh.cand_i[tid] = idx;
            sh.cand_p[tid] = expf(lg[idx] * inv_t - gmax) / sum_exp;
        }
        __syncthreads();
        if (tid == 0) {
            const float min_thresh = sp.min_p > 0.0f ? sh.cand_p[0] * sp.min_p : 0.0f;
            float cum = 0.0f;
            int count = 0;
            for (int c = 0; c < K; c++) {
                const float pc = sh.cand_p[c];
                if (sp.min_p > 0.0f && pc < min_thresh) break;
                if (sp.top_p < 1.0f && cum >= sp.top_p) break;
                cum += pc;
                count++;
            }
            if (count == 0) count = 1;
            const float r = sm_runif(sp.seeds[row]) * cum;
            float cdf = 0.0f;
            chosen = sh.cand_i[count - 1];
            for (int c = 0; c < count; c++) {
                cdf += sh.cand_p[c];
                if (cdf >= r) { chosen = sh.cand_i[c]; break; }
            }
        }
    } else {
        // full-vocabulary sampler (pure temperature, optional min-p), index-order draw
        const float inv_t = 1.0f / sp.temperature;
        float mx = -3.0e38f;
        for (int i = tid; i < V; i += SM_THREADS) mx = fmaxf(mx, lg[i]);
        const float max_l = sm_block_max(mx, sh);
        float se = 0.0f;
        for (int i = tid; i < V; i += SM_THREADS) se += expf((lg[i] - max_l) * inv_t);
        const float inv_sum = 1.0f / fmaxf(sm_block_sum(se, sh), 1e-12f);
        // max probability is exp(0) * inv_sum; min-p keeps p >= p_max * min_p
        const float th = sp.min_p > 0.0f ? inv_sum * sp.min_p : 0.0f;
        // contiguous slices: kept mass per slice, block prefix, then the crossing slice walks
        const int per = (V + SM_THREADS - 1) / SM_THREADS;
        const int i0 = tid * per, i1 = min(V, i0 + per);
        float part = 0.0f;
        for (int i = i0; i < i1; i++) {
            const float pr = expf((lg[i] - max_l) * inv_t) * inv_sum;
            if (pr >= th) part += pr;
        }
        sh.csum[tid] = part;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.0f;
            for (int t = 0; t < SM_THREADS; t++) {
                const float v = sh.csum[t];
                sh.csum[t] = tot;           // exclusive prefix
                tot += v;
            }
            sh.fscal[0] = tot;
        }
        __syncthreads();
        const float new_sum = sh.fscal[0];
        if (new_sum <= 0.0f) {
            if (tid == 0) chosen = 0;
        } else {
            const float r = sm_runif(sp.seeds[row]) * new_sum;   // == drawing on the renormalised cdf
            const float base = sh.csum[tid];
            const float next = tid + 1 < SM_THREADS ? sh.csum[tid + 1] : new_sum;
            if (tid == 0) sh.uscal[3] = (unsigned)(V - 1);
            __syncthreads();
            if (i0 < i1 && base < r && next >= r) {
                float cdf = base;
                int pick = i1 - 1;
                for (int i = i0; i < i1; i++) {
                    const float pr = expf((lg[i] - max_l) * inv_t) * inv_sum;
                    if (pr >= th) cdf += pr;
                    if (cdf >= r) { pick = i; break; }
                }
                atomicMin(&sh.uscal[3], (unsigned)pick);
            } else if (tid == 0 && r <= 0.0f) {
                atomicMin(&sh.uscal[3], 0u);
            }
            __syncthreads();
            if (tid == 0) chosen = (int)sh.uscal[3];
        }
    }
    if (tid == 0) {
        sp.out[row] = chosen;
        if (sp.feed) sp.feed[row] = chosen;
        if (sp.hist.tok) sp.hist.tok[(size_t)row * sp.hist.cap + sp.hist.cache_len[row]] = chosen;
    }
}

bool sample_supported(float temperature, int top_k, float top_p, int V)
{
    if (!(temperature > 0.0f)) return true;
    if (top_k >= 1 && top_k <= SM_MAXK) return true;
    return (top_k <= 0 || top_k >= V) && top_p >= 1.0f;
}

int launch_sample(const float *logits, int rows, int V, int ldl, float temperature, int top_k, float top_p,
                  float min_p, const int32_t *seeds, int32_t *out, int *feed, TokHist hist, int *err, cudaStream_t st,
                  const float *dparams)
{
    if (rows <= 0) return DU_OK;
    if (dparams == nullptr && !sample_supported(temperature, top_k, top_p, V))
        return fail(DU_EINVAL, "sample: top_p < 1 needs top_k in 1..64 (the reference's parallel sampler)");
    SampleParams sp;
    sp.logits = logits;
    sp.ldl = ldl;
    sp.V = V;
    sp.temperature = temperature;
    sp.top_p = top_p;
    sp.min_p = min_p;
    sp.top_k = top_k;
    sp.seeds = seeds;
    sp.out = out;
    sp.feed = feed;
    sp.hist = hist;
    sp.err = err;
    sp.dparams = dparams;
    const size_t smem = sizeof(SmShared);
    int rc = ensure_func_attrs((const void *)sample_kernel, (int)smem);
    if (rc) return rc;
    sample_kernel<<<rows, SM_THREADS, smem, st>>>(sp);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// Repetition + presence penalty (ApplyRepetitionPresencePenalty, Qwen3_5CS.compute:1421-1433),
// in place on rows of logits, for the ids already seen in the row's sequence:
// l = l > 0 ? l / repetition : l * repetition, then l -= presence (once per id,
// whatever its count).  seen [rows][ld_seen] occurrence counts.  in_ids (optional,
// decode steps): the step's input id per row, which was the previous pick; it counts
// as seen here and one thread adds it to seen (MarkSampledTokenSeen,
// Qwen3_5CS.compute:1436-1441, moved from after the pick to the next step's start).
// The penalty depends only on whether a count is non-zero, so the increment racing
// with the reads of the same word cannot change a result.  dp (optional): device
// (presence, repetition) overriding the scalars (one captured graph for all settings).
constexpr int PEN_THREADS = 256;
constexpr int PEN_PER_THREAD = 4;

__global__ void __launch_bounds__(PEN_THREADS) penalty_kernel(float *logits, int V, int ldl, unsigned *seen, int ld_seen,
                                                              const int *in_ids, const float *dp, float presence,
                                                              float repetition)
{
    if (dp != nullptr) {
        presence = dp[0];
        repetition = dp[1];
    }
    const int row = blockIdx.y;
    float *lg = logits + (size_t)row * ldl;
    const unsigned *sn = seen + (size_t)row * ld_seen;
    const int in = in_ids != nullptr ? in_ids[row] : -1;
    const int base = blockIdx.x * PEN_THREADS * PEN_PER_THREAD + threadIdx.x;
#pragma unroll
    for (int k = 0; k < PEN_PER_THREAD; k++) {
        const int i = base + k * PEN_THREADS;
        if (i < V && (sn[i] != 0u || i == in)) {
            float l = lg[i];
            l = l > 0.0f ? l / repetition : l * repetition;
            lg[i] = l - presence;
        }
    }
    if (in_ids != nullptr && blockIdx.x == 0 && threadIdx.x == 0 && in >= 0 && in < V)
        seen[(size_t)row * ld_seen + in] += 1u;
}

int launch_penalties(float *logits, int rows, int V, int ldl, unsigned *seen, int ld_seen, const int *in_ids,
                     const float *dp, float presence, float repetition, cudaStream_t st)
{
    if (rows <= 0) return DU_OK;
    const dim3 grid((V + PEN_THREADS * PEN_PER_THREAD - 1) / (PEN_THREADS * PEN_PER_THREAD), rows);
    penalty_kernel<<<grid, PEN_THREADS, 0, st>>>(logits, V, ldl, seen, ld_seen, in_ids, dp, presence, repetition);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

// MarkSampledTokenSeen (Qwen3_5CS.compute:1436-1441) for several rows: seen[r][ids[r]] += 1.
__global__ void mark_seen_kernel(unsigned *seen, int rows, int ld_seen, int V, const int32_t *ids)
{
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        const int id = ids[r];
        if (id >= 0 && id < V) atomicAdd(&seen[(size_t)r * ld_seen + id], 1u);
    }
}

}  // namespace du

using namespace du;

extern "C" DU_API int du_apply_penalties(float *logits, int rows, int vocab, int ldl, const uint32_t *seen, int ld_seen,
                                         float presence_penalty, float repetition_penalty, void *stream)
{
    DU_CHECK_ARG(logits && seen && rows >= 0 && vocab > 0 && ldl >= vocab && ld_seen >= vocab,
                 "du_apply_penalties: bad arguments");
    DU_CHECK_ARG(repetition_penalty > 0.0f, "du_apply_penalties: repetition_penalty must be > 0");
    return launch_penalties(logits, rows, vocab, ldl, const_cast<unsigned *>(seen), ld_seen, nullptr, nullptr,
                            presence_penalty, repetition_penalty, static_cast<cudaStream_t>(stream));
}

extern "C" DU_API int du_mark_seen(uint32_t *seen, int rows, int ld_seen, int vocab, const int32_t *ids, void *stream)
{
    DU_CHECK_ARG(seen && ids && rows >= 0 && vocab > 0 && ld_seen >= vocab, "du_mark_seen: bad arguments");
    if (rows == 0) return DU_OK;
    mark_seen_kernel<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(seen, rows, ld_seen, vocab, ids);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

extern "C" DU_API int du_sample(int32_t *out, const float *logits, int rows, int vocab, int ldl, float temperature,
                                int top_k, float top_p, float min_p, const int32_t *seeds, void *stream)
{
    DU_CHECK_ARG(out && logits && seeds && rows >= 0 && vocab > 0 && ldl >= vocab, "du_sample: bad arguments");
    if (!sample_supported(temperature, top_k, top_p, vocab))
        return fail(DU_EINVAL, "du_sample: top_p < 1 needs top_k in 1..64 (the reference's parallel sampler)");
    return launch_sample(logits, rows, vocab, ldl, temperature, top_k, top_p, min_p, seeds, out, nullptr, TokHist{},
                         nullptr, static_cast<cudaStream_t>(stream), nullptr);
}
