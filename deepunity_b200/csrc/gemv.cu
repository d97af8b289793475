// gemv.cu -- standalone decode GEMV kernel (device code in gemv_impl.cuh) and its launcher.
#include <cstdlib>

#ifdef DU_GEMV_STAMPS
#include "gemv_stamps.cuh"     // timing build: per-CTA phase stamps (libdeepunity_cuda_stamps.so)
#endif
#include "gemv_impl.cuh"
#include "internal.h"

namespace du {

// NW warps per CTA: GV_WARPS (two CTAs per SM) or GV_WARPS_WIDE (one CTA per SM,
// one activation stage per SM and a deeper ring).  TPR: EPI_TP_RESID, the
// tensor-parallel reduction in the epilogue (a separate instantiation, so that
// the other epilogues compile as without it).
template <int QT, int MT, int RW, int D, int NW, bool TPR>
__global__ void __launch_bounds__(NW * 32) qgemv_kernel(const GemvParams p)
{
    extern __shared__ __align__(16) unsigned char gv_smem[];
    __shared__ GemvShared<MT, NW> sh;
    GemvStream<QT, MT, RW, D, NW, TPR> gs;
    GV_STAMP(0);
    gs.prefetch(p, gv_smem, blockIdx.x, gridDim.x);
    GV_STAMP(1);
    // activations of the previous kernel are complete from here on
    pdl_wait();
    GV_STAMP(2);
    gs.run(p, gv_smem + gemv_ring_bytes<QT, RW, D, NW>(), sh, blockIdx.x, gridDim.x, [] { pdl_trigger(); });
    GV_STAMP(5);
}

// ------------------------------------------------------------------ launch

static constexpr int rw_of(int mt) { return mt == 1 ? 4 : 2; }
static constexpr size_t SMEM_PER_SM = 227 * 1024;
static constexpr size_t GV_SMEM_MAX = 220 * 1024;     // dynamic shared memory per CTA (static scratch + margin below)

static size_t ring_bytes(int qt, int mt, int d, int nw = GV_WARPS)
{
    const size_t slots = (size_t)nw * d * rw_of(mt) * 32;
    return slots * 16 + (qt == Q_I4 ? slots * 4 : 0);
}

static size_t x_bytes(int qt, int mt, int64_t row_bytes)
{
    const int nchunk = (int)(row_bytes >> 4);
    const int xu4 = qt == Q_I4 ? 7 : qt == Q_I8 ? 3 : 2;
    return (size_t)mt * nchunk * xu4 * 16;
}

// 8-warp CTAs with depth 4 when two per SM fit in shared memory.  Else (large K,
// where two CTAs per SM would hold two copies of a large activation stage): one
// decode token (MT = 1) uses the wide layout, one 16-warp CTA per SM with depth
// 6..4 as shared memory allows (measured on the 8B down projection, K = 14336:
// 14.4 vs 14.7 us; at K = 4096 the two-CTA layout is faster, 7.1 vs 7.9 us for
// o_proj); other token tiles use two CTAs at depth 3 if that fits, else one at 4.
// DU_GEMV_WIDE=0 in the environment turns the wide layout off.
struct GvCfg {
    int nw, d, cps;
};

static bool wide_enabled()
{
    static const bool on = [] {     // read once (thread-safe static initialisation)
        const char *e = getenv("DU_GEMV_WIDE");
        return e ? atoi(e) != 0 : true;
    }();
    return on;
}

static GvCfg choose_cfg(int qt, int mt, int64_t row_bytes)
{
    const size_t x = x_bytes(qt, mt, row_bytes);
    if (2 * (ring_bytes(qt, mt, 4) + x + 1024) <= SMEM_PER_SM) return {GV_WARPS, 4, 2};
    if (mt == 1 && wide_enabled())
        for (int d = 6; d >= 4; d--)
            if (ring_bytes(qt, mt, d, GV_WARPS_WIDE) + x <= GV_SMEM_MAX) return {GV_WARPS_WIDE, d, 1};
    if (2 * (ring_bytes(qt, mt, 3) + x + 1024) <= SMEM_PER_SM) return {GV_WARPS, 3, 2};
    return {GV_WARPS, 4, 1};
}

size_t gemv_x_bytes(int qt, int mt, int64_t row_bytes) { return x_bytes(qt, mt, row_bytes); }

int gemv_ctas_per_sm(int qt, int mt, int64_t row_bytes) { return choose_cfg(qt, mt, row_bytes).cps; }

size_t gemv_smem_bytes(int qt, int mt, int64_t row_bytes)
{
    const GvCfg c = choose_cfg(qt, mt, row_bytes);
    return ring_bytes(qt, mt, c.d, c.nw) + x_bytes(qt, mt, row_bytes);
}

static bool g_pdl = true;
void gemv_set_pdl(bool on) { g_pdl = on; }
bool pdl_enabled() { return g_pdl; }

int gemv_rows_per_group(int M) { return rw_of(M <= 1 ? 1 : 2); }

template <int QT, int MT, int D, int NW, bool TPR>
static int launch_kernel(const GemvParams &p, int grid, size_t smem, cudaStream_t st)
{
    auto kern = qgemv_kernel<QT, MT, rw_of(MT), D, NW, TPR>;
    int rc = ensure_func_attrs((const void *)kern, (int)GV_SMEM_MAX);
    if (rc) return rc;
    if (TPR) {
        // each CTA waits for the other ranks' values of its rows: all CTAs must be
        // resident at once, so the grid is capped at one wave
        int per_sm = 0;
        DU_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NW * 32, smem));
        if (per_sm < 1) return fail(DU_EINVAL, "gemv: tensor-parallel epilogue kernel does not fit on an SM");
        if (grid > per_sm * num_sms()) grid = per_sm * num_sms();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl ? 1 : 0;
    DU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
    return DU_OK;
}

template <int QT, int MT, bool TPR>
static int launch_cfg(const GemvParams &p, int grid, const GvCfg &c, size_t smem, cudaStream_t st)
{
    if constexpr (MT == 1) {
        if (c.nw == GV_WARPS_WIDE) {
            if (c.d == 6) return launch_kernel<QT, MT, 6, GV_WARPS_WIDE, TPR>(p, grid, smem, st);
            if (c.d == 5) return launch_kernel<QT, MT, 5, GV_WARPS_WIDE, TPR>(p, grid, smem, st);
            return launch_kernel<QT, MT, 4, GV_WARPS_WIDE, TPR>(p, grid, smem, st);
        }
    }
    return c.d == 3 ? launch_kernel<QT, MT, 3, GV_WARPS, TPR>(p, grid, smem, st)
                    : launch_kernel<QT, MT, 4, GV_WARPS, TPR>(p, grid, smem, st);
}

template <int QT, int MT>
static int launch_mt(const GemvParams &p, int grid, const GvCfg &c, size_t smem, cudaStream_t st)
{
    return p.epi == EPI_TP_RESID ? launch_cfg<QT, MT, true>(p, grid, c, smem, st)
                                 : launch_cfg<QT, MT, false>(p, grid, c, smem, st);
}

// CTAs for N rows at token tile M: `want` (0 = 2 per SM), never more than one per row group
int gemv_grid_for(int N, int M, int want)
{
    const int RW = gemv_rows_per_group(M);
    const int ng = (N + RW - 1) / RW;
    const int grid = want > 0 ? want : 2 * num_sms();
    return grid > ng ? ng : grid;
}

int launch_gemv(int qt, GemvParams p, cudaStream_t st)
{
    if (p.M <= 0 || p.N <= 0) return DU_OK;
    if (p.M > 8) return fail(DU_EINVAL, "gemv: M > 8 must be split by the caller");
    if (qt == Q_I4 && (p.group < 32 || (p.group & (p.group - 1)) || ((p.K / p.group) & 1)))
        return fail(DU_EINVAL, "gemv: int4 group must be a power of two >= 32 with an even number of groups per row");
    const int mt = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
    const GvCfg c = choose_cfg(qt, mt, p.row_bytes);
    const size_t smem = ring_bytes(qt, mt, c.d, c.nw) + x_bytes(qt, mt, p.row_bytes);
    if (smem > GV_SMEM_MAX) return fail(DU_EINVAL, "gemv: M*K too large for the shared-memory stage");
    const int grid = gemv_grid_for(p.N, mt, p.grid > 0 ? p.grid : c.cps * num_sms());
#define DU_GV_CASE(Q, M_)                                        \
    if (qt == Q && mt == M_) return launch_mt<Q, M_>(p, grid, c, smem, st);
    DU_GV_CASE(Q_I4, 1) DU_GV_CASE(Q_I4, 2) DU_GV_CASE(Q_I4, 4) DU_GV_CASE(Q_I4, 8)
    DU_GV_CASE(Q_I8, 1) DU_GV_CASE(Q_I8, 2) DU_GV_CASE(Q_I8, 4) DU_GV_CASE(Q_I8, 8)
    DU_GV_CASE(Q_F16, 1) DU_GV_CASE(Q_F16, 2) DU_GV_CASE(Q_F16, 4) DU_GV_CASE(Q_F16, 8)
#undef DU_GV_CASE
    return fail(DU_EINVAL, "gemv: unsupported quant kind");
}

}  // namespace du
