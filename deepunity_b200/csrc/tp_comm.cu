// tp_comm.cu -- one-shot allreduce over NVLink peer memory for decode-sized
// tensor-parallel reductions.
//
// The two collectives of a tensor-parallel layer (after o_proj and down_proj)
// carry tokens x hidden fp32 values: 16 KB at batch 1.  At that size
// ncclAllReduce costs a fixed ~10 us per call.  With 64 calls per step that is
// more than the GEMV time TP saves.  Each rank maps every peer's communication
// buffer (CUDA IPC).  The decode graph fuses the reduction into the O / down
// GEMV epilogue (gemv_impl.cuh); this file holds the buffers, the handle
// exchange and a standalone kernel for the same protocol (tp_fuse.cuh), which
// does, per element i of its slice:
//   1. push this rank's value to every rank's receive buffer;
//   2. wait for every rank's value and add them in rank order: dst[i] += sum;
//   3. the last CTA to finish advances the rank's sequence counter.
// Every rank runs the same sequence of reductions (the same graphs and prefill
// chunks).
#include <cstdlib>
#include <cstring>

#include "internal.h"
#include "tp_comm.h"
#include "tp_fuse.cuh"

namespace du {

__global__ void __launch_bounds__(256) tp_allreduce_kernel(const TpFuse t, const float *src, float *dst, int n)
{
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nthr = gridDim.x * blockDim.x;
    const unsigned s = tp_next_seq(t);
    for (int i = tid; i < n; i += nthr) tp_push(t, s, i, src[i]);
    for (int i = tid; i < n; i += nthr) {
        float sum;
        if (!tp_wait_sum(t, s, i, sum)) break;
        dst[i] += sum;
    }
    tp_launch_done(t, s);
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
    DU_CUDA_TRY(cudaMalloc(&c->dev, sizeof(TpFuse)));
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

unsigned tp_spin_limit()
{
    const char *e = getenv("DU_TP_SPIN_LIMIT");
    const long long v = e ? atoll(e) : 0;
    return v > 0 && v < (1ll << 31) ? (unsigned)v : TP_SPIN_LIMIT;
}

int tp_comm_open(TpComm *c, const void *handles, int nranks, int rank, int *err)
{
    if (nranks < 2 || nranks > TP_MAX_RANKS || rank < 0 || rank >= nranks)
        return fail(DU_EINVAL, "tp comm: 2..8 ranks");
    if (!c->buf || !c->dev || !err) return fail(DU_ESTATE, "tp comm: buffer not allocated");
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
    TpFuse h = {};
    for (int r = 0; r < nranks; r++) h.peer_recv[r] = static_cast<uint2 *>(c->peer[r]);
    h.seq = c->ctl;
    h.done = c->ctl + 1;
    h.err = err;
    h.maxn = c->maxn;
    h.rank = rank;
    h.nranks = nranks;
    h.spin_limit = tp_spin_limit();
    cudaError_t e = cudaMemcpy(c->dev, &h, sizeof(h), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        tp_comm_close(c);
        return cuda_fail(e, "tp comm: handle upload");
    }
    c->host = h;
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
    if (c->dev) cudaFree(c->dev);
    c->buf = nullptr;
    c->ctl = nullptr;
    c->dev = nullptr;
}

int launch_tp_allreduce(TpComm *c, const float *src, float *dst, size_t n, cudaStream_t st)
{
    if (!c->ready || n > c->maxn) return fail(DU_ESTATE, "tp allreduce: peer buffers not open or too small");
    int ncta = (int)((n + 255) / 256);
    if (ncta > 64) ncta = 64;
    if (ncta < 1) ncta = 1;
    tp_allreduce_kernel<<<ncta, 256, 0, st>>>(c->host, src, dst, (int)n);
    DU_CUDA_TRY(cudaGetLastError());
    return DU_OK;
}

}  // namespace du

using namespace du;

// One-process check of the bounded peer wait (no reference counterpart).  A
// two-rank communicator is built from two local buffers; this process plays
// rank 0 and nothing ever plays rank 1, so every wait for rank 1's value must
// give up after spin_limit polls, set the error word and let the kernel return.
// *timed_out = the error word the host reads back (1 when the wait ran out).
extern "C" DU_API int du_tp_wait_selftest(unsigned spin_limit, int *timed_out)
{
    DU_CHECK_ARG(timed_out != nullptr && spin_limit > 0, "du_tp_wait_selftest: bad arguments");
    *timed_out = 0;
    const size_t maxn = 256;
    void *bufs[2] = {nullptr, nullptr};
    unsigned *ctl = nullptr;
    int *err = nullptr;
    float *src = nullptr, *dst = nullptr;
    int rc = DU_OK;
    auto alloc = [&](void **p, size_t bytes) {
        if (rc) return;
        cudaError_t e = cudaMalloc(p, bytes);
        if (e == cudaSuccess) e = cudaMemset(*p, 0, bytes);
        if (e != cudaSuccess) rc = cuda_fail(e, "du_tp_wait_selftest: allocation");
    };
    alloc(&bufs[0], tp_comm_bytes(maxn));
    alloc(&bufs[1], tp_comm_bytes(maxn));
    alloc((void **)&ctl, 2 * sizeof(unsigned));
    alloc((void **)&err, sizeof(int));
    alloc((void **)&src, maxn * sizeof(float));
    alloc((void **)&dst, maxn * sizeof(float));
    if (!rc) {
        TpFuse h = {};
        h.peer_recv[0] = static_cast<uint2 *>(bufs[0]);
        h.peer_recv[1] = static_cast<uint2 *>(bufs[1]);
        h.seq = ctl;
        h.done = ctl + 1;
        h.err = err;
        h.maxn = maxn;
        h.rank = 0;
        h.nranks = 2;
        h.spin_limit = spin_limit;
        tp_allreduce_kernel<<<1, 256>>>(h, src, dst, (int)maxn);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(timed_out, err, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = cuda_fail(e, "du_tp_wait_selftest");
    }
    for (void *p : {bufs[0], bufs[1], (void *)ctl, (void *)err, (void *)src, (void *)dst})
        if (p) cudaFree(p);
    return rc;
}
