// edb_common.cuh -- shared device/host helpers for the edifice_b200 kernels.
//
// sm_100a only.  Inline PTX for mbarriers and TMA (cp.async.bulk.tensor), the
// 128-bit vector I/O used by the bandwidth-bound scans, the bounded-wait error
// flag, and host-side tensor-map encoding through the driver entry point.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "edifice_b200.h"

// ---------------------------------------------------------------- errors
// Device-side error word, one per device (defined in runtime.cu; kernels get
// its address as an argument from edb::device_error_word()).  Bounded waits
// that give up OR a bit in here instead of spinning forever; the host reads and
// clears it with edb_get_device_errors().  Bits are EDB_DEVERR_*.
static __device__ __forceinline__ void edb_flag_error(unsigned* err, unsigned bit) {
    if (err) atomicOr(err, bit);
}

// ---------------------------------------------------------------- smem / PTX
static __device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

static __device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

static __device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

static __device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

static __device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

static __device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

static __device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe of an mbarrier phase (never suspends the thread).
static __device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

static __device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wall-clock limit of every device-side wait (2 s).
#define EDB_WAIT_NS 2000000000ull

// Bounded wait on an mbarrier phase.  Returns false (and flags the device
// error word) when the wait has lasted EDB_WAIT_NS on the global timer; the
// caller must then leave its loop at the next CTA-uniform point instead of
// waiting again.
static __device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity,
                                                         unsigned* err, unsigned errbit) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > EDB_WAIT_NS) break;
    }
    edb_flag_error(err, errbit);
    return false;
}

// As mbar_wait_bounded with a caller-chosen limit (edb_set_wait_limit_ns):
// limit_ns = 0 gives up as soon as one probe finds the phase incomplete, which
// is how a test makes a wait run out on purpose.
static __device__ __forceinline__ bool mbar_wait_limited(uint64_t* bar, unsigned parity,
                                                         unsigned* err, unsigned errbit,
                                                         uint64_t limit_ns) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (limit_ns != 0 && global_ns() - t0 <= limit_ns)
        if (mbar_try_wait(bar, parity)) return true;
    edb_flag_error(err, errbit);
    return false;
}

// 2D tiled TMA load global -> shared, completion counted on `bar` (bytes).
static __device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map,
                                                   uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

static __device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map,
                                                   uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// 16-byte asynchronous copy global -> shared (cp.async.cg); src_bytes < 16
// zero-fills the rest (0: nothing is read, the whole 16 bytes become zero).
static __device__ __forceinline__ void cp_async16(void* dst, const void* src, unsigned src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
static __device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most `PENDING` of this thread's committed groups are in flight.
template <int PENDING>
static __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(PENDING) : "memory");
}

static __device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- packed f32 pairs
// sm_100 executes fma/mul/add on a pair of f32 values as one instruction, with
// the rounding of the scalar forms.  The compiler builtins (not inline PTX) let
// the register allocator keep pairs in place: wrapping the PTX .f32x2 forms in
// asm with mov.b64 packing hid the pairs from it and cost register moves.
// a * b + c, element-wise
static __device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    return __ffma2_rn(a, b, c);
}
static __device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
static __device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
static __device__ __forceinline__ float2 dup2(float x) { return make_float2(x, x); }

// ---------------------------------------------------------------- vector I/O
// A 16-byte vector of storage elements widened to f32.
template <typename T>
struct Vec16;

template <>
struct Vec16<float> {
    static constexpr int N = 4;
    static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
        f[0] = __uint_as_float(v.x);
        f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z);
        f[3] = __uint_as_float(v.w);
    }
    static __device__ __forceinline__ uint4 pack(const float* f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                          __float_as_uint(f[3]));
    }
};

template <>
struct Vec16<__nv_bfloat16> {
    static constexpr int N = 8;
    static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ uint4 pack(const float* f) {
        return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]),
                          pack2(f[6], f[7]));
    }
};

template <typename T>
static __device__ __forceinline__ float ld_scalar(const T* p);
template <>
__device__ __forceinline__ float ld_scalar<float>(const float* p) {
    return *p;
}
template <>
__device__ __forceinline__ float ld_scalar<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
}

template <typename T>
static __device__ __forceinline__ void st_scalar(T* p, float v);
template <>
__device__ __forceinline__ void st_scalar<float>(float* p, float v) {
    *p = v;
}
template <>
__device__ __forceinline__ void st_scalar<__nv_bfloat16>(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16(v);
}

static __device__ __forceinline__ uint4 ld_global_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

static __device__ __forceinline__ void st_global_v4(void* p, const uint4& v) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// ---------------------------------------------------------------- host side
namespace edb {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank,
                      void* gaddr, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                      const cuuint32_t* box, CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int dtype) { return dtype == EDB_BF16 ? 2 : 4; }

// SM count of the current device (cached per device).
int sm_count();

// Per-device cache of one __device__ symbol's address, keyed on the unique id
// of the context it was looked up in.
struct SymbolCache {
    std::mutex m;
    unsigned long long ctx_id[64] = {};
    void* addr[64] = {};
};

// Device address of a __device__ symbol of this library in the current
// device's current context (0 or a cudaError_t).  The address is cached per
// device together with the context's unique id (cuCtxGetId, through the
// runtime's driver entry point), so a cudaDeviceReset or any other re-creation
// of the context is noticed and the symbol looked up again; when the id cannot
// be read the symbol is looked up on every call.  The first lookup in a
// context may load this library's module: it should not happen inside a
// stream capture.
int symbol_address(const void* symbol, SymbolCache& cache, void** out);

// Device address of the current device's error word (see symbol_address).
unsigned int* device_error_word();

// Wall-clock limit of the waits that take one (edb_set_wait_limit_ns): the
// default EDB_WAIT_NS unless the host set another.
unsigned long long wait_limit_ns();

// Map a cudaError_t to the ABI's int status.
inline int status_from_cuda(cudaError_t e) { return e == cudaSuccess ? EDB_OK : (int)e; }

}  // namespace edb
