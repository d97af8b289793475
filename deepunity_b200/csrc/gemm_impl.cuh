// gemm_impl.cuh -- device helpers of the tensor-core dequant GEMM (gemm.cu):
// mbarriers, TMA tile loads, tcgen05 (TMEM allocation, MMA, commit, loads) and
// the exact weight unpack into fp16 operand pairs.
//
// Exact operands.  An INT4 weight is w = (n - 8) * d with d an fp16 group scale
// (readQ4 / readW, Gemma3CS.compute:84-101).  (n - 8) has at most 3 significant
// bits and d 11, so w needs up to 14 bits: more than one fp16 holds.  The unpack
// writes w = hi + lo with hi = fp16(w) and lo = fp16(w - hi); the difference has
// at most 3 significant bits, so the pair is exact (for weights in the fp16
// normal range).  INT8 weights q (|q| <= 127) are exact in one fp16 and keep
// their row scale for the epilogue (wScale, G3CS:92-101); fp16 weights are used
// as they are.  Activations are split the same way (x = hi + lo, ~22 bits), so
// the MMAs A_hi.B_hi + A_hi.B_lo (+ A_lo.B_hi for INT4) reproduce the fp32 dot
// product to ~2^-22 relative.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace du {

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase of parity `parity` of barrier `bar`.  Gives up after
// `limit_ns` nanoseconds of polling, or as soon as another role of the CTA has
// given up (*abort set): then it records the failure in *err (device memory, when
// given) and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_f, int *err,
                                          uint64_t limit_ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (unsigned n = 1;; n++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 63) == 0) {
            if (*abort_f) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                *abort_f = 1;
                if (err) atomicExch(err, 2);
                return false;
            }
        }
    }
}

// 16-byte shared-memory load that the compiler keeps in program order with the
// other volatile asm (the raw stage it reads is handed back to the TMA producer
// right after)
__device__ __forceinline__ uint4 lds128_volatile(const void *p)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p))
                 : "memory");
    return v;
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// --------------------------------------------------------------------- TMA

// 2-D tiled load of the box at (x, y) into shared memory, completing on `bar`
// (x: innermost coordinate, always a multiple of 16 bytes here).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, uint32_t bar, int x, int y,
                                            uint64_t pol)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// ----------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// arrives on `bar` once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void tc_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// D[tmem] (+)= A[smem desc] . B[smem desc]^T, fp16 inputs, fp32 accumulators
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
                 : "memory");
}
// this thread's TMEM lane, 32 consecutive 32-bit columns
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
                 "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzled layout: rows of 128 bytes (64 fp16 of K), 8-row groups 1024 bytes
// apart.  Start address, leading-byte offset (unused for this layout), stride-
// byte offset, descriptor version 1, swizzle mode 2 (128 B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr)
{
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor of kind::f16: fp32 accumulators, fp16 A and B, both
// K-major, M = 128 rows, N = n columns.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n)
{
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// ---------------------------------------------------------- exact unpack

// Byte address of 16-byte chunk c (8 fp16 of K) of row r in a 128-byte
// swizzled tile: rows 128 bytes apart, chunk index XOR (r mod 8).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// 8 INT4 weights (one 32-bit word: low nibble = even column, as readQ4) times the
// fp16 scale d2 = (d, d) -> exact fp16 pairs hi + lo, columns in order.
// 0x6400 | n is the fp16 1024 + n; subtracting 1032 leaves n - 8 exactly.
__device__ __forceinline__ void dq_int4_word(uint32_t w, __half2 d2, uint4 &hi, uint4 &lo)
{
    const uint32_t m = 0x000F000Fu, mg = 0x64006400u;
    const uint32_t t0 = (w & m) | mg, t1 = ((w >> 4) & m) | mg;     // columns (0, 4), (1, 5)
    const uint32_t t2 = ((w >> 8) & m) | mg, t3 = ((w >> 12) & m) | mg;   // (2, 6), (3, 7)
    const uint32_t q[4] = {__byte_perm(t0, t1, 0x5410), __byte_perm(t2, t3, 0x5410), __byte_perm(t0, t1, 0x7632),
                           __byte_perm(t2, t3, 0x7632)};
    const __half2 off = u2h(0x64086408u);   // (1032, 1032)
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half2 qi = __hsub2(u2h(q[i]), off);
        const __half2 a = __hmul2(qi, d2);
        const __half2 b = __hfma2(qi, d2, u2h(h2u(a) ^ 0x80008000u));   // qi * d - hi, one rounding
        h[i] = h2u(a);
        l[i] = h2u(b);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// 8 INT8 weights (two 32-bit words, byte order = column order, as readQ8) -> fp16 q exactly.
// (b ^ 0x80) is b + 128 in 0..255; 0x6400 | that is 1024 + b + 128; minus 1152 leaves b.
__device__ __forceinline__ uint4 dq_int8_2words(uint32_t w0, uint32_t w1)
{
    const uint32_t x0 = w0 ^ 0x80808080u, x1 = w1 ^ 0x80808080u;
    const __half2 off = u2h(0x64806480u);   // (1152, 1152)
    const uint32_t q[4] = {__byte_perm(x0, 0x64646464u, 0x4140), __byte_perm(x0, 0x64646464u, 0x4342),
                           __byte_perm(x1, 0x64646464u, 0x4140), __byte_perm(x1, 0x64646464u, 0x4342)};
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = h2u(__hsub2(u2h(q[i]), off));
    return make_uint4(h[0], h[1], h[2], h[3]);
}

}  // namespace du
