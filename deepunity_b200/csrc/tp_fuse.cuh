// tp_fuse.cuh -- device side of the peer-memory tensor-parallel reduction
// (host side and the standalone kernel: tp_comm.cu; fused into the O / down
// GEMV epilogue: gemv_impl.cuh).
//
// Element i of reduction number s travels as one 64-bit word (s << 32 | value
// bits), which rank `from` stores into slot [s & 1][from][i] of every rank's
// receive buffer.  A naturally aligned 64-bit access is single-copy atomic, so
// a reader that sees sequence s in the word also sees the value: no fence and no
// separate flag.  Readers add the ranks' values in rank order, so every rank
// computes a bit-identical sum.  Slots alternate by parity: a rank cannot finish
// reduction s + 1 before every peer has contributed to it, which a peer does
// only after it has finished reduction s, so a slot that is being rewritten is
// never one that a slower rank still reads.
#pragma once

#include "common.cuh"

namespace du {

// Default number of polls of one peer word before a wait gives up (several
// seconds); DU_TP_SPIN_LIMIT in the environment overrides it when the peers are
// opened.
constexpr unsigned TP_SPIN_LIMIT = 1u << 24;

__device__ __forceinline__ size_t tp_slot(const TpFuse &t, unsigned s, int from, size_t i)
{
    return ((size_t)(s & 1u) * TP_MAX_RANKS + from) * t.maxn + i;
}

// sends this rank's value of element i of reduction s to every rank
__device__ __forceinline__ void tp_push(const TpFuse &t, unsigned s, size_t i, float v)
{
    const unsigned long long word = ((unsigned long long)s << 32) | __float_as_uint(v);
    const size_t off = tp_slot(t, s, t.rank, i);
    for (int r = 0; r < t.nranks; r++)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(t.peer_recv[r] + off), "l"(word) : "memory");
}

// sum over the ranks, in rank order, of element i of reduction s.  Each wait is
// bounded: on timeout (or when another thread already failed) it sets *t.err
// and returns false.
__device__ __forceinline__ bool tp_wait_sum(const TpFuse &t, unsigned s, size_t i, float &sum)
{
    float acc = 0.0f;
    for (int r = 0; r < t.nranks; r++) {
        const uint2 *w = t.peer_recv[t.rank] + tp_slot(t, s, r, i);
        for (unsigned n = 0;;) {
            unsigned long long word;
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(w) : "memory");
            if ((unsigned)(word >> 32) == s) {
                acc += __uint_as_float((unsigned)word);
                break;
            }
            if (++n > t.spin_limit || ((n & 1023) == 0 && *(volatile int *)t.err)) {
                atomicExch(t.err, 1);
                return false;
            }
        }
    }
    sum = acc;
    return true;
}

// sequence number of the reduction a launch performs; read after the launch's
// dependency on the previous reduction's launch has resolved
__device__ __forceinline__ unsigned tp_next_seq(const TpFuse &t) { return *(volatile const unsigned *)t.seq + 1u; }

// the last CTA of a reducing launch advances the sequence; every thread of
// every CTA calls it after its waits
__device__ __forceinline__ void tp_launch_done(const TpFuse &t, unsigned s)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(t.done, 1u) == gridDim.x - 1u) {
            *t.done = 0u;
            *(volatile unsigned *)t.seq = s;
        }
    }
}

}  // namespace du
