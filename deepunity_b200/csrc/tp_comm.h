// tp_comm.h -- peer-memory allreduce for decode-sized tensor-parallel reductions (tp_comm.cu).
#pragma once

#include <cstddef>

#include "common.cuh"

namespace du {

struct TpComm {
    void *buf = nullptr;             // [2 parities][TP_MAX_RANKS][maxn] (value, sequence) 8-byte words
    unsigned *ctl = nullptr;         // [0] last completed sequence, [1] CTA completion count
    void *peer[TP_MAX_RANKS] = {};   // every rank's buf (own = buf), mapped through CUDA IPC
    bool opened[TP_MAX_RANKS] = {};
    TpFuse host = {};                // handles of the open peers
    TpFuse *dev = nullptr;           // device copy of `host` (read by the fused GEMV epilogue)
    size_t maxn = 0;                 // floats per slot
    int nranks = 0, rank = 0;
    bool ready = false;
};

size_t tp_comm_bytes(size_t maxn);
// polls of one peer word before a wait gives up (DU_TP_SPIN_LIMIT, else TP_SPIN_LIMIT)
unsigned tp_spin_limit();
int tp_comm_alloc(TpComm *c, size_t maxn);
int tp_comm_handle(TpComm *c, void *out64);
// maps the peers' buffers; waits that time out set *err
int tp_comm_open(TpComm *c, const void *handles, int nranks, int rank, int *err);
void tp_comm_close(TpComm *c);
void tp_comm_free(TpComm *c);
// dst[0..n) += sum over ranks of src (every rank's src), in rank order
int launch_tp_allreduce(TpComm *c, const float *src, float *dst, size_t n, cudaStream_t st);

}  // namespace du
