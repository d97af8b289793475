// gemv.cu -- standalone decode GEMV kernel (device code in gemv_impl.cuh) and its launcher.
#include "gemv_impl.cuh"
#include "internal.h"

namespace du {

template <int QT, int MT, int RW, int D>
__global__ void __launch_bounds__(GV_THREADS) qgemv_kernel(const GemvParams p)
{
    extern __shared__ __align__(16) unsigned char gv_smem[];
    __shared__ GemvShared<MT> sh;
    GemvStream<QT, MT, RW, D> gs;
    gs.prefetch(p, gv_smem, blockIdx.x, gridDim.x);
    // activations of the previous kernel are complete from here on
    pdl_wait();
    gs.run(p, gv_smem + gemv_ring_bytes<QT, RW, D>(), sh, blockIdx.x, gridDim.x, [] { pdl_trigger(); });
}

// ------------------------------------------------------------------ launch

// Ring depth D: 4 when two CTAs per SM fit in shared memory, else 3 if that
// makes two fit (large K), else 4 with one CTA per SM.
static constexpr int rw_of(int mt) { return mt == 1 ? 4 : 2; }
static constexpr size_t SMEM_PER_SM = 227 * 1024;

static size_t ring_bytes(int qt, int mt, int d)
{
    const size_t slots = (size_t)GV_WARPS * d * rw_of(mt) * 32;
    return slots * 16 + (qt == Q_I4 ? slots * 4 : 0);
}

static size_t x_bytes(int qt, int mt, int64_t row_bytes)
{
    const int nchunk = (int)(row_bytes >> 4);
    const int xu4 = qt == Q_I4 ? 7 : qt == Q_I8 ? 3 : 2;
    return (size_t)mt * nchunk * xu4 * 16;
}

static int choose_depth(int qt, int mt, int64_t row_bytes, int *cps)
{
    const size_t x = x_bytes(qt, mt, row_bytes);
    for (int d = 4; d >= 3; d--)
        if (2 * (ring_bytes(qt, mt, d) + x + 1024) <= SMEM_PER_SM) { *cps = 2; return d; }
    *cps = 1;
    return 4;
}

size_t gemv_x_bytes(int qt, int mt, int64_t row_bytes) { return x_bytes(qt, mt, row_bytes); }

size_t gemv_smem_bytes(int qt, int mt, int64_t row_bytes)
{
    int cps = 1;
    const int d = choose_depth(qt, mt, row_bytes, &cps);
    return ring_bytes(qt, mt, d) + x_bytes(qt, mt, row_bytes);
}

static bool g_pdl = true;
void gemv_set_pdl(bool on) { g_pdl = on; }
bool pdl_enabled() { return g_pdl; }

int gemv_rows_per_group(int M) { return rw_of(M <= 1 ? 1 : 2); }

template <int QT, int MT, int D>
static int launch_kernel(const GemvParams &p, int grid, size_t smem, cudaStream_t st)
{
    auto kern = qgemv_kernel<QT, MT, rw_of(MT), D>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        DU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        attr_set[dev & 63] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GV_THREADS);
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

template <int QT, int MT>
static int launch_mt(const GemvParams &p, int grid, int depth, size_t smem, cudaStream_t st)
{
    return depth == 3 ? launch_kernel<QT, MT, 3>(p, grid, smem, st) : launch_kernel<QT, MT, 4>(p, grid, smem, st);
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
    int cps = 1;
    const int depth = choose_depth(qt, mt, p.row_bytes, &cps);
    const size_t smem = ring_bytes(qt, mt, depth) + x_bytes(qt, mt, p.row_bytes);
    if (smem > 220 * 1024) return fail(DU_EINVAL, "gemv: M*K too large for the shared-memory stage");
    const int grid = gemv_grid_for(p.N, mt, p.grid > 0 ? p.grid : cps * num_sms());
#define DU_GV_CASE(Q, M_)                                        \
    if (qt == Q && mt == M_) return launch_mt<Q, M_>(p, grid, depth, smem, st);
    DU_GV_CASE(Q_I4, 1) DU_GV_CASE(Q_I4, 2) DU_GV_CASE(Q_I4, 4) DU_GV_CASE(Q_I4, 8)
    DU_GV_CASE(Q_I8, 1) DU_GV_CASE(Q_I8, 2) DU_GV_CASE(Q_I8, 4) DU_GV_CASE(Q_I8, 8)
    DU_GV_CASE(Q_F16, 1) DU_GV_CASE(Q_F16, 2) DU_GV_CASE(Q_F16, 4) DU_GV_CASE(Q_F16, 8)
#undef DU_GV_CASE
    return fail(DU_EINVAL, "gemv: unsupported quant kind");
}

}  // namespace du
