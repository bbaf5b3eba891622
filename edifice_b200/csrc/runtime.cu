// runtime.cu -- library-wide host utilities of libedifice_b200.so: version and
// status strings, the per-device error word, tensor-map encoding through the
// runtime's driver entry point, and the per-device SM-count cache.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "edb_common.cuh"

__device__ unsigned int g_edb_device_errors = 0;

namespace edb {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* gaddr,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                      const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return CUDA_ERROR_NOT_SUPPORTED;
    // The driver call needs a current context on this thread.  A thread that
    // has only ever asked the runtime for the device number (e.g. an autograd
    // worker) has none yet; cudaSetDevice makes the primary context current.
    thread_local int ctx_dev = -1;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CUDA_ERROR_INVALID_CONTEXT;
    if (dev != ctx_dev) {
        if (cudaSetDevice(dev) != cudaSuccess) return CUDA_ERROR_INVALID_CONTEXT;
        ctx_dev = dev;
    }
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return g_encode(map, dtype, rank, gaddr, dims, strides_bytes, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

namespace {

using PFN_ctx_current = CUresult (*)(CUcontext*);
using PFN_ctx_id = CUresult (*)(CUcontext, unsigned long long*);
PFN_ctx_current g_ctx_current = nullptr;
PFN_ctx_id g_ctx_id = nullptr;
std::once_flag g_ctx_once;

// Unique id of the calling thread's current context, 0 if none or unknown.
unsigned long long current_context_id() {
    std::call_once(g_ctx_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            g_ctx_current = reinterpret_cast<PFN_ctx_current>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_id = reinterpret_cast<PFN_ctx_id>(fn);
    });
    if (!g_ctx_current || !g_ctx_id) return 0;
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
    if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

SymbolCache g_error_word_cache;

}  // namespace

int symbol_address(const void* symbol, SymbolCache& cache, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    const bool cacheable = dev >= 0 && dev < 64;
    unsigned long long id = current_context_id();
    if (cacheable && id != 0) {
        std::lock_guard<std::mutex> lk(cache.m);
        if (cache.ctx_id[dev] == id && cache.addr[dev] != nullptr) {
            *out = cache.addr[dev];
            return EDB_OK;
        }
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, symbol);
    if (e != cudaSuccess) return (int)e;
    if (p == nullptr) return EDB_ERR_UNSUPPORTED;
    id = current_context_id();  // the lookup makes the primary context current
    if (cacheable && id != 0) {
        std::lock_guard<std::mutex> lk(cache.m);
        cache.ctx_id[dev] = id;
        cache.addr[dev] = p;
    }
    *out = p;
    return EDB_OK;
}

unsigned int* device_error_word() {
    void* p = nullptr;
    if (symbol_address(&g_edb_device_errors, g_error_word_cache, &p) != EDB_OK) return nullptr;
    return static_cast<unsigned int*>(p);
}

namespace {
std::atomic<long long> g_wait_limit{-1};  // < 0: EDB_WAIT_NS
}  // namespace

unsigned long long wait_limit_ns() {
    const long long v = g_wait_limit.load(std::memory_order_relaxed);
    return v < 0 ? EDB_WAIT_NS : (unsigned long long)v;
}

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace edb

extern "C" const char* edb_version(void) { return "edifice_b200 0.1 sm_100a"; }

extern "C" const char* edb_status_string(int status) {
    switch (status) {
        case EDB_OK: return "ok";
        case EDB_ERR_NULL_POINTER: return "null pointer argument";
        case EDB_ERR_BAD_SHAPE: return "invalid shape";
        case EDB_ERR_BAD_DTYPE: return "invalid dtype";
        case EDB_ERR_MISALIGNED: return "pointer not aligned as required";
        case EDB_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
        case EDB_ERR_UNSUPPORTED: return "configuration not supported";
        case EDB_ERR_DEVICE_TIMEOUT: return "a bounded device wait gave up";
        default:
            if (status > 0 && status < 1000) return cudaGetErrorString((cudaError_t)status);
            return "unknown status";
    }
}

extern "C" int edb_set_wait_limit_ns(long long limit_ns) {
    edb::g_wait_limit.store(limit_ns < 0 ? -1 : limit_ns, std::memory_order_relaxed);
    return EDB_OK;
}

extern "C" int edb_get_device_errors(unsigned int* flags_out, int clear) {
    if (!flags_out) return EDB_ERR_NULL_POINTER;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return (int)e;
    e = cudaMemcpyFromSymbol(flags_out, g_edb_device_errors, sizeof(unsigned int));
    if (e != cudaSuccess) return (int)e;
    if (clear) {
        unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_edb_device_errors, &zero, sizeof(unsigned int));
    }
    return (int)e;
}

// ------------------------------------------------------------ storage conversion
namespace {
template <typename S, typename D>
__global__ void edb_convert_kernel(const S* __restrict__ src, D* __restrict__ dst, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) st_scalar<D>(dst + i, ld_scalar<S>(src + i));
}
}  // namespace

extern "C" int edb_convert(int src_dtype, const void* src, int dst_dtype, void* dst, size_t n,
                           void* stream) {
    if ((src_dtype != EDB_F32 && src_dtype != EDB_BF16) ||
        (dst_dtype != EDB_F32 && dst_dtype != EDB_BF16))
        return EDB_ERR_BAD_DTYPE;
    if (n == 0) return EDB_OK;
    if (!src || !dst) return EDB_ERR_NULL_POINTER;
    cudaStream_t st = (cudaStream_t)stream;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    using bf = __nv_bfloat16;
    if (src_dtype == EDB_F32 && dst_dtype == EDB_F32)
        edb_convert_kernel<float, float><<<blocks, 256, 0, st>>>((const float*)src, (float*)dst, n);
    else if (src_dtype == EDB_F32)
        edb_convert_kernel<float, bf><<<blocks, 256, 0, st>>>((const float*)src, (bf*)dst, n);
    else if (dst_dtype == EDB_F32)
        edb_convert_kernel<bf, float><<<blocks, 256, 0, st>>>((const bf*)src, (float*)dst, n);
    else
        edb_convert_kernel<bf, bf><<<blocks, 256, 0, st>>>((const bf*)src, (bf*)dst, n);
    return edb::status_from_cuda(cudaGetLastError());
}
