// capi.cu -- error plumbing, device queries, NCCL loader and the kernel-level
// C entry points of libdeepunity_cuda.
#include <dlfcn.h>

#include <atomic>

#include <map>
#include <mutex>
#include <utility>
#include <string>
#include <vector>

#include "gemv.cuh"
#include "internal.h"
#include "nccl_shim.h"

namespace du {

static thread_local std::string t_last_error;

void set_error(const std::string &msg) { t_last_error = msg; }

int fail(int code, const std::string &msg)
{
    t_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *what)
{
    t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? DU_ENOMEM : DU_ECUDA;
}

int num_sms()
{
    static std::atomic<int> cache[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int n = cache[dev & 63].load(std::memory_order_relaxed);
    if (n == 0) {
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
        cache[dev & 63].store(n, std::memory_order_relaxed);   // every thread computes the same value
    }
    return n;
}

// Raises a kernel's dynamic shared-memory limit (and optionally allows
// non-portable cluster sizes) once per (kernel, device).  Launchers may run on
// several host threads at once, so the record is guarded.
int ensure_func_attrs(const void *kern, int smem_bytes, bool nonportable_cluster)
{
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, int> done;
    int dev = 0;
    DU_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_pair(kern, dev);
    const auto it = done.find(key);
    if (it != done.end() && it->second >= smem_bytes) return DU_OK;
    DU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
    if (nonportable_cluster) DU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    done[key] = smem_bytes;
    return DU_OK;
}

// Grow-only per-device scratch for the kernel-level entry points.  Slot 0/1
// are independent regions; freshly grown memory is zeroed (the flash-decode
// counters rely on that and reset themselves after each launch).
void *device_scratch(size_t bytes, int slot)
{
    static std::mutex mu;
    static void *ptr[64][8] = {};
    static size_t cap[64][8] = {};
    std::lock_guard<std::mutex> lk(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    dev &= 63;
    if (cap[dev][slot] < bytes) {
        if (ptr[dev][slot]) {
            cudaDeviceSynchronize();
            cudaFree(ptr[dev][slot]);
        }
        ptr[dev][slot] = nullptr;
        cap[dev][slot] = 0;
        if (cudaMalloc(&ptr[dev][slot], bytes) != cudaSuccess) return nullptr;
        cudaMemset(ptr[dev][slot], 0, bytes);
        cudaDeviceSynchronize();
        cap[dev][slot] = bytes;
    }
    return ptr[dev][slot];
}

const NcclApi *nccl_api()
{
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
#define DU_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
        DU_SYM(GetUniqueId, "ncclGetUniqueId");
        DU_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
        DU_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
        DU_SYM(AllReduce, "ncclAllReduce");
        DU_SYM(AllGather, "ncclAllGather");
        DU_SYM(CommAbort, "ncclCommAbort");
        DU_SYM(CommDestroy, "ncclCommDestroy");
        DU_SYM(CommFinalize, "ncclCommFinalize");
        DU_SYM(GetErrorString, "ncclGetErrorString");
#undef DU_SYM
        api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.AllReduce &&
                 api.AllGather && api.CommAbort && api.CommDestroy && api.GetErrorString;
    });
    if (!api.ok) {
        set_error("NCCL (libnccl.so.2) could not be loaded");
        return nullptr;
    }
    return &api;
}

static int x_to_f32(const void *x, int x_dtype, size_t n, const float **out, cudaStream_t st)
{
    if (x_dtype == DU_DTYPE_F32) {
        *out = static_cast<const float *>(x);
        return DU_OK;
    }
    if (x_dtype != DU_DTYPE_F16 && x_dtype != DU_DTYPE_BF16) return fail(DU_EINVAL, "unsupported x_dtype");
    float *buf = static_cast<float *>(device_scratch(n * sizeof(float), 1));
    if (!buf) return fail(DU_ENOMEM, "scratch allocation failed");
    int rc = launch_convert_to_f32(x, x_dtype, n, buf, st);
    if (rc) return rc;
    *out = buf;
    return DU_OK;
}

static int gemv_entry(int qt, float *y, const void *x, int x_dtype, const void *w, const void *scales,
                      int scale_f32, int group, int M, int N, int K, void *stream)
{
    DU_CHECK_ARG(y && x && w && M >= 0 && N >= 0 && K > 0, "gemv: null pointer or negative size");
    const int cols_per_chunk = qt == Q_I4 ? 32 : qt == Q_I8 ? 16 : 8;
    DU_CHECK_ARG(K % cols_per_chunk == 0, "gemv: K must be a multiple of 32 (int4) / 16 (int8) / 8 (fp16)");
    if (qt == Q_I4) DU_CHECK_ARG(group > 0 && group % 32 == 0 && K % group == 0, "gemv: group must be a multiple of 32 dividing K");
    if (qt != Q_F16) DU_CHECK_ARG(scales != nullptr, "gemv: scales required");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const float *xf = nullptr;
    int rc = x_to_f32(x, x_dtype, (size_t)M * K, &xf, st);
    if (rc) return rc;
    const int64_t row_bytes = qt == Q_I4 ? K / 2 : qt == Q_I8 ? K : 2 * (int64_t)K;
    if (M <= 2 && qt == Q_I4) {
        // tensor-core decode GEMV
        GemvParams p = {};
        p.x = xf; p.ldx = K;
        p.w = static_cast<const uint8_t *>(w);
        p.scales = scales;
        p.row_bytes = row_bytes;
        p.K = K; p.N = N; p.M = M; p.group = group;
        p.map = MAP_IDENT;
        p.epi = EPI_STORE;
        p.y = y;
        p.ldy = N;
        if (tgemv_supported(qt, p)) {
            GemmScratch g;
            g.partial_floats = GEMM_PARTIAL_FLOATS_PER_SM * (size_t)num_sms();
            g.counter_n = 1 << 16;
            char *ps = static_cast<char *>(device_scratch(4 * g.partial_floats + 4 * g.counter_n, 4));
            if (!ps) return fail(DU_ENOMEM, "gemv: scratch allocation failed");
            g.partials = reinterpret_cast<float *>(ps);
            g.counters = reinterpret_cast<unsigned *>(ps + 4 * g.partial_floats);
            return launch_tgemv(qt, p, g, st);
        }
    }
    if (M >= gemm_min_tokens()) {
        // tensor-core GEMM: weights streamed once for all M rows
        GemvParams p = {};
        p.x = xf; p.ldx = K;
        p.w = static_cast<const uint8_t *>(w);
        p.scales = scales;
        p.scale_f32 = scale_f32;
        p.row_bytes = row_bytes;
        p.K = K; p.N = N; p.M = M; p.group = group;
        p.map = MAP_IDENT;
        p.epi = EPI_STORE;
        p.y = y;
        p.ldy = N;
        if (gemm_supported(qt, p)) {
            GemmScratch g;
            g.elems = (size_t)M * K;
            g.rows = (size_t)M;
            char *buf = static_cast<char *>(device_scratch(4 * g.elems + 4 * g.rows + 16, 3));
            if (!buf) return fail(DU_ENOMEM, "gemm: scratch allocation failed");
            g.xh = reinterpret_cast<__half *>(buf);
            g.xl = g.xh + g.elems;
            g.xscale = reinterpret_cast<float *>(buf + 4 * g.elems);
            g.partial_floats = GEMM_PARTIAL_FLOATS_PER_SM * (size_t)num_sms();
            g.counter_n = 1 << 16;
            char *ps = static_cast<char *>(device_scratch(4 * g.partial_floats + 4 * g.counter_n, 4));
            if (!ps) return fail(DU_ENOMEM, "gemm: scratch allocation failed");
            g.partials = reinterpret_cast<float *>(ps);
            g.counters = reinterpret_cast<unsigned *>(ps + 4 * g.partial_floats);
            return launch_gemm(qt, p, g, st);
        }
    }
    int mt = 8;
    while (mt > 1 && gemv_smem_bytes(qt, mt, row_bytes) > 220 * 1024) mt >>= 1;
    if (gemv_smem_bytes(qt, mt, row_bytes) > 220 * 1024) return fail(DU_EINVAL, "gemv: K too large");
    for (int m0 = 0; m0 < M; m0 += mt) {
        GemvParams p = {};
        p.x = xf + (size_t)m0 * K;
        p.ldx = K;
        p.w = static_cast<const uint8_t *>(w);
        p.scales = scales;
        p.scale_f32 = scale_f32;
        p.row_bytes = row_bytes;
        p.K = K; p.N = N; p.M = M - m0 < mt ? M - m0 : mt; p.group = group;
        p.map = MAP_IDENT;
        p.epi = EPI_STORE;
        p.y = y + (size_t)m0 * N;
        p.ldy = N;
        rc = launch_gemv(qt, p, st);
        if (rc) return rc;
    }
    return DU_OK;
}

}  // namespace du

using namespace du;

extern "C" {

DU_API const char *du_last_error(void) { return t_last_error.c_str(); }

DU_API const char *du_version(void) { return "deepunity_b200 0.1 (sm_100a)"; }

DU_API int du_init(int device_ordinal)
{
    int n = 0;
    DU_CUDA_TRY(cudaGetDeviceCount(&n));
    DU_CHECK_ARG(device_ordinal >= 0 && device_ordinal < n, "du_init: device ordinal out of range");
    DU_CUDA_TRY(cudaSetDevice(device_ordinal));
    cudaDeviceProp prop;
    DU_CUDA_TRY(cudaGetDeviceProperties(&prop, device_ordinal));
    if (prop.major != 10) return fail(DU_ESTATE, std::string("du_init: built for sm_100a, device is ") + prop.name);
    DU_CUDA_TRY(cudaFree(nullptr));
    return DU_OK;
}

DU_API int du_gemv_q8(float *y, const void *x, int x_dtype, const int8_t *w, const void *scales, int scale_dtype,
                      int M, int N, int K, void *stream)
{
    DU_CHECK_ARG(scale_dtype == DU_DTYPE_F16 || scale_dtype == DU_DTYPE_F32, "du_gemv_q8: scale_dtype F16 or F32");
    return gemv_entry(Q_I8, y, x, x_dtype, w, scales, scale_dtype == DU_DTYPE_F32, 0, M, N, K, stream);
}

DU_API int du_gemv_q4(float *y, const void *x, int x_dtype, const uint8_t *w, const uint16_t *scales_f16, int group,
                      int M, int N, int K, void *stream)
{
    return gemv_entry(Q_I4, y, x, x_dtype, w, scales_f16, 0, group, M, N, K, stream);
}

DU_API int du_gemv_f16(float *y, const void *x, int x_dtype, const uint16_t *w, int M, int N, int K, void *stream)
{
    return gemv_entry(Q_F16, y, x, x_dtype, w, nullptr, 0, 0, M, N, K, stream);
}

DU_API int du_flash_decode(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                           const int32_t *kv_len, int batch, int hq, int hkv, int hd, int capacity, float scale,
                           void *stream)
{
    DU_CHECK_ARG(out && q && k_cache && v_cache && kv_len, "du_flash_decode: null pointer");
    DU_CHECK_ARG(batch >= 0 && hq > 0 && hkv > 0 && capacity > 0, "du_flash_decode: bad sizes");
    DU_CHECK_ARG(hq % hkv == 0, "du_flash_decode: hq must be a multiple of hkv");
    // the model's kernel: the splits of a (sequence, kv head) combine inside a
    // thread-block cluster, so no global scratch is needed
    return launch_flash_decode_cluster(q, reinterpret_cast<const __half *>(k_cache),
                                       reinterpret_cast<const __half *>(v_cache), nullptr, kv_len, 0, batch, hq, hkv,
                                       hd, capacity, scale, out, static_cast<cudaStream_t>(stream));
}

DU_API int du_flash_decode_window(float *out, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                  const int32_t *kv_len, int batch, int hq, int hkv, int hd, int capacity, float scale,
                                  int window, void *stream)
{
    DU_CHECK_ARG(out && q && k_cache && v_cache && kv_len, "du_flash_decode_window: null pointer");
    DU_CHECK_ARG(batch >= 0 && hq > 0 && hkv > 0 && capacity > 0, "du_flash_decode_window: bad sizes");
    DU_CHECK_ARG(hq % hkv == 0, "du_flash_decode_window: hq must be a multiple of hkv");
    return launch_flash_decode_cluster(q, reinterpret_cast<const __half *>(k_cache),
                                       reinterpret_cast<const __half *>(v_cache), nullptr, kv_len, 0, batch, hq, hkv,
                                       hd, capacity, scale, out, static_cast<cudaStream_t>(stream), -1, nullptr,
                                       window > 0 ? window : 0);
}

DU_API int du_kv_write_int8(const float *kv_new, int seq_len, int hkv, int hd, int cache_len, uint8_t *cache,
                            uint32_t *sz, void *stream)
{
    DU_CHECK_ARG(kv_new && cache && sz, "du_kv_write_int8: null pointer");
    DU_CHECK_ARG(seq_len >= 0 && hkv > 0 && hd > 0 && cache_len >= 0, "du_kv_write_int8: bad sizes");
    Kv8Cache kv = {cache, nullptr, sz, nullptr};
    // one sequence, K rows only: rows land at positions cache_len + m
    return launch_kv_quant_int8(kv_new, seq_len, 1, hkv, hd, nullptr, cache_len, nullptr, 0, 0, kv,
                                static_cast<cudaStream_t>(stream));
}

DU_API int du_flash_decode_kv8(float *out, const float *q, const uint8_t *k8, const uint32_t *ksz, const uint8_t *v8,
                               const uint32_t *vsz, const int32_t *kv_len, int batch, int hq, int hkv, int hd,
                               int capacity, float scale, void *stream)
{
    DU_CHECK_ARG(out && q && k8 && ksz && v8 && vsz && kv_len, "du_flash_decode_kv8: null pointer");
    DU_CHECK_ARG(batch >= 0 && hq > 0 && hkv > 0 && capacity > 0, "du_flash_decode_kv8: bad sizes");
    DU_CHECK_ARG(hq % hkv == 0, "du_flash_decode_kv8: hq must be a multiple of hkv");
    Kv8Cache kv = {const_cast<uint8_t *>(k8), const_cast<uint8_t *>(v8), const_cast<uint32_t *>(ksz),
                   const_cast<uint32_t *>(vsz)};
    return launch_flash_decode_cluster(q, nullptr, nullptr, nullptr, kv_len, 0, batch, hq, hkv, hd, capacity, scale, out,
                                       static_cast<cudaStream_t>(stream), -1, &kv);
}

DU_API int du_dequant(float *out, const void *w, const void *scales, int quant, int scale_dtype, int group,
                      int64_t row0, int nrows, int K, void *stream)
{
    DU_CHECK_ARG(out && w && nrows >= 0 && row0 >= 0 && K > 0 && K % 8 == 0, "du_dequant: bad arguments");
    DU_CHECK_ARG(quant == DU_QUANT_FP16 || quant == DU_QUANT_INT8 || quant == DU_QUANT_INT4, "du_dequant: quant");
    if (quant != DU_QUANT_FP16) DU_CHECK_ARG(scales != nullptr, "du_dequant: scales required");
    if (quant == DU_QUANT_INT4)
        DU_CHECK_ARG(group >= 8 && group % 8 == 0 && K % group == 0, "du_dequant: group must be a multiple of 8 dividing K");
    if (quant == DU_QUANT_INT8)
        DU_CHECK_ARG(scale_dtype == DU_DTYPE_F16 || scale_dtype == DU_DTYPE_F32, "du_dequant: scale_dtype F16 or F32");
    const int qt = quant == DU_QUANT_INT4 ? Q_I4 : quant == DU_QUANT_INT8 ? Q_I8 : Q_F16;
    return launch_dequant_rows(qt, w, scales, scale_dtype == DU_DTYPE_F32, group, row0, nrows, K, out,
                               static_cast<cudaStream_t>(stream));
}

DU_API int du_quantize_int8(const float *w, int64_t rows, int64_t cols, int8_t *q, uint16_t *scales_f16,
                            void *stream)
{
    DU_CHECK_ARG(w && q && scales_f16 && rows >= 0 && cols > 0, "du_quantize_int8: bad arguments");
    return launch_quantize_int8(w, rows, cols, q, reinterpret_cast<__half *>(scales_f16),
                                static_cast<cudaStream_t>(stream));
}

DU_API int du_quantize_int4(const float *w, int64_t rows, int64_t cols, int group, uint8_t *packed,
                            uint16_t *scales_f16, void *stream)
{
    DU_CHECK_ARG(w && packed && scales_f16 && rows >= 0 && cols > 0, "du_quantize_int4: bad arguments");
    return launch_quantize_int4(w, rows, cols, group, packed, reinterpret_cast<__half *>(scales_f16),
                                static_cast<cudaStream_t>(stream));
}

DU_API int du_rmsnorm(float *y, const float *x, const uint16_t *gamma_m1, int rows, int H, float eps, void *stream)
{
    DU_CHECK_ARG(y && x && gamma_m1 && rows >= 0 && H > 0, "du_rmsnorm: bad arguments");
    return launch_rmsnorm(x, reinterpret_cast<const __half *>(gamma_m1), rows, H, eps, y,
                          static_cast<cudaStream_t>(stream));
}

DU_API int du_nccl_unique_id(void *out128)
{
    DU_CHECK_ARG(out128 != nullptr, "du_nccl_unique_id: null output");
    const NcclApi *n = nccl_api();
    if (!n) return DU_ENCCL;
    ncclUniqueId id;
    ncclResult_t r = n->GetUniqueId(&id);
    if (r != ncclSuccess) return fail(DU_ENCCL, std::string("ncclGetUniqueId: ") + n->GetErrorString(r));
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out128, &id, 128);
    return DU_OK;
}

}  // extern "C"
