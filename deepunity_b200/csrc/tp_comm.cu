// tp_comm.cu -- one-shot allreduce over NVLink peer memory for decode-sized
// tensor-parallel reductions.
//
// The two collectives of a tensor-parallel layer (after o_proj and down_proj)
// carry tokens x hidden fp32 values: 16 KB at batch 1.  At that size
// ncclAllReduce costs a fixed ~10 us per call.  With 64 calls per step that is
// more than the GEMV time TP saves.  Each rank maps every peer's communication
// buffer (CUDA IPC) and one kernel does, per element i of its slice:
//   1. push: one 64-bit store of (sequence number << 32 | value) into slot
//      [parity][my rank][i] of every rank's receive buffer (NVLink stores; the
//      own slot is a local store).  A naturally aligned 64-bit scalar access is
//      single-copy atomic, so the sequence number in the same word flags the
//      value: no fence and no separate flag are needed;
//   2. wait + reduce: poll slot [parity][r][i] of the own buffer for every
//      rank r until it carries this sequence number (bounded; sets the error
//      word on timeout), and add the values in rank order, so every rank
//      computes bit-identical residuals: dst[i] += sum.
//   3. the last CTA to finish advances the rank's sequence counter.
// Receive slots alternate by the sequence parity: a rank can run at most one
// allreduce ahead of a peer (it cannot finish allreduce k + 1 before the peer
// has contributed to it, which the peer does only after it finished k), so the
// slot a fast rank writes is never the one a slow rank is still reading.
// Sequence numbers only grow, so slots never need resetting.  Every rank runs
// the same sequence of allreduces (the same graphs and prefill chunks).
#include <cstring>

#include "internal.h"
#include "tp_comm.h"

namespace du {

constexpr unsigned TP_SPIN_LIMIT = 1u << 24;

struct TpArgs {
    uint2 *peer_recv[TP_MAX_RANKS];      // rank r's receive region ([2][TP_MAX_RANKS][maxn] (value, seq) words)
    const uint2 *my_recv;
    unsigned *seq;                       // this rank's last completed sequence number
    unsigned *done;                      // CTAs finished in this launch (last one resets it)
    int *err;
    const float *src;                    // this rank's partial sums [n]
    float *dst;                          // residual [n] (+= the sum)
    int n, rank, nranks;
    size_t maxn;
};

__global__ void __launch_bounds__(256) tp_allreduce_kernel(const TpArgs a)
{
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nthr = gridDim.x * blockDim.x;
    const unsigned s = *(volatile unsigned *)a.seq + 1u;
    const size_t par = s & 1u;
    // 1. push (value, seq) words
    for (int i = tid; i < a.n; i += nthr) {
        const unsigned v = __float_as_uint(a.src[i]);
        for (int r = 0; r < a.nranks; r++) {
            uint2 *d = a.peer_recv[r] + (par * TP_MAX_RANKS + a.rank) * a.maxn + i;
            const unsigned long long word = ((unsigned long long)s << 32) | v;      // one 64-bit access: seen whole
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(d), "l"(word) : "memory");
        }
    }
    // 2. wait for every rank's word and reduce in rank order
    bool ok = true;
    for (int i = tid; i < a.n; i += nthr) {
        float sum = 0.0f;
        for (int r = 0; r < a.nranks; r++) {
            const uint2 *w = a.my_recv + (par * TP_MAX_RANKS + r) * a.maxn + i;
            unsigned v = 0, n = 0;
            for (;;) {
                unsigned long long word;
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(w) : "memory");
                v = (unsigned)word;
                if ((unsigned)(word >> 32) == s) break;
                if (++n > TP_SPIN_LIMIT || (n & 1023) == 0 && *(volatile int *)a.err) {
                    atomicExch(a.err, 1);
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
            sum += __uint_as_float(v);
        }
        if (!ok) break;
        a.dst[i] += sum;
    }
    // 3. the last CTA advances the sequence
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.done, 1u) == gridDim.x - 1u) {
            *a.done = 0u;
            *(volatile unsigned *)a.seq = s;
        }
    }
}

size_t tp_comm_bytes(size_t maxn)
{
    return sizeof(uint2) * 2 * TP_MAX_RANKS * maxn;
}

int tp_comm_alloc(TpComm *c, size_t maxn)
{
    c->maxn = maxn;
    const size_t bytes = tp_comm_bytes(maxn);
    DU_CUDA_TRY(cudaMalloc(&c->buf, bytes));
    DU_CUDA_TRY(cudaMemset(c->buf, 0, bytes));
    DU_CUDA_TRY(cudaMalloc(&c->ctl, sizeof(unsigned) * 2));
    DU_CUDA_TRY(cudaMemset(c->ctl, 0, sizeof(unsigned) * 2));
    return DU_OK;
}

int tp_comm_handle(TpComm *c, void *out64)
{
    if (!c->buf) return fail(DU_ESTATE, "tp comm: buffer not allocated");
    cudaIpcMemHandle_t h;
    DU_CUDA_TRY(cudaIpcGetMemHandle(&h, c->buf));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    memcpy(out64, &h, 64);
    return DU_OK;
}

int tp_comm_open(TpComm *c, const void *handles, int nranks, int rank)
{
    if (nranks < 2 || nranks > TP_MAX_RANKS || rank < 0 || rank >= nranks)
        return fail(DU_EINVAL, "tp comm: 2..8 ranks");
    for (int r = 0; r < nranks; r++) {
        if (r == rank) {
            c->peer[r] = c->buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char *>(handles) + 64 * r, 64);
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            tp_comm_close(c);
            return cuda_fail(e, "cudaIpcOpenMemHandle");
        }
        c->peer[r] = p;
        c->opened[r] = true;
    }
    c->nranks = nranks;
    c->rank = rank;
    c->ready = true;
    return DU_OK;
}

void tp_comm_close(TpComm *c)
{
    for (int r = 0; r < TP_MAX_RANKS; r++) {
        if (c->opened[r] && c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]);
        c->opened[r] = false;
        c->peer[r] = nullptr;
    }
    c->ready = false;
}

void tp_comm_free(TpComm *c)
{
    tp_comm_close(c);
    if (c->buf) cudaFree(c->buf);
    if (c->ctl) cudaFree(c->ctl);
    c->buf = nullptr;
    c->ctl = nullptr;
}

int launch_tp_allreduce(TpComm *c, const float *src, float *dst, size_t n, int *err, cudaStream_t st)
{
    if (!c->ready || n > c->maxn) return fail(DU_ESTATE, "tp allreduce: peer buffers not open or too small");
    TpArgs a = {};
    for (int r = 0; r < c->nranks; r++) a.peer_recv[r] = static_cast<uint2 *>(c->peer[r]);
    a.my_recv = a.peer_recv[c->rank];
    a.seq = c->ctl;
    a.done = c->ctl + 1;
    a.err = err;
    a.src = src;
    a.dst = dst;
    a.n = (int)n;
    a.rank = c->rank;
    a.nranks = c->nranks;
    a.maxn = c->maxn;
    int ncta = (int)((n + 255) / 256);
    if (ncta > 64) ncta = 64;
    if (ncta < 1) ncta = 1;
    tp_allreduce_kernel<<<ncta, 256, 0, st>>>(a);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

}  // namespace du
