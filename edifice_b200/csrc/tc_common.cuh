// tc_common.cuh -- 5th-generation tensor core (tcgen05) helpers for sm_100a.
//
// Inline PTX for TMEM allocation, tcgen05.mma (kind::f16, bf16 x bf16 -> f32,
// both operands from shared memory), commits to mbarriers, TMEM <-> register
// moves, and the shared-memory matrix descriptors for the 128-byte swizzled
// layouts that TMA writes (SWIZZLE_128B).
//
// Descriptor conventions (sm_100 "version 1" shared-memory descriptor):
//   bits  0-13  start address >> 4      bits 16-29  leading byte offset >> 4
//   bits 32-45  stride byte offset >> 4  bits 46-47  version = 1
//   bits 49-51  base offset = 0          bit  52     LBO mode = 0
//   bits 61-63  layout: 2 = SWIZZLE_128B
// K-major SW128 tile (rows x 64 bf16, 128 B per row, 8-row swizzle atoms of
// 1 KB): SBO = 1024 B, LBO unused; advancing K by 16 elements adds 32 B to the
// start address.  MN-major SW128 (the MN dimension contiguous, 64 elements per
// 128-B row of the atom, K rows): LBO = byte distance between 64-element MN
// blocks, SBO = distance between 8-row K groups (1024 B when rows are packed).
#pragma once

#include "edb_common.cuh"

namespace tc {

// ---------------------------------------------------------------- TMEM alloc
static __device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
static __device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
static __device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

static __device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
static __device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- MMA
// D[tmem] (+)= A[smem desc] * B[smem desc]; accumulate != 0 keeps D.
static __device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc,
                                                   uint64_t b_desc, uint32_t idesc,
                                                   uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32 (f32 operands read with
// 10 explicit mantissa bits); the layouts (K- or MN-major) are in `idesc`.
static __device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc,
                                                   uint64_t b_desc, uint32_t idesc,
                                                   uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// All MMAs issued so far by this thread arrive on `bar` when complete.
static __device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// Instruction descriptor, kind::f16: bf16 A/B, f32 D, dense.
//   a_mn / b_mn: 1 if that operand is MN-major (else K-major).
static __host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
    return (1u << 4)                       // D format f32
           | (1u << 7)                     // A bf16
           | (1u << 10)                    // B bf16
           | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16)
           | ((uint32_t)(N >> 3) << 17)    // N / 8
           | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// Shared-memory descriptor for a SWIZZLE_128B operand tile.
static __device__ __forceinline__ uint64_t sdesc_sw128(const void* smem_ptr, uint32_t lbo_bytes,
                                                       uint32_t sbo_bytes) {
    const uint32_t a = smem_u32(smem_ptr);
    uint64_t d = 0;
    d |= (uint64_t)((a >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // version
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}

// ---------------------------------------------------------------- TMEM <-> regs
// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane
// (base lane + t), columns [col, col + 32).
static __device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

static __device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 32 lanes x 16 consecutive columns.
static __device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// 32 lanes x 8 consecutive columns (loops over column groups stay small).
static __device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

// 32 lanes x 8 consecutive columns (a store needing few live registers).
static __device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                     taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                 "r"(r[7])
                 : "memory");
}

static __device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
static __device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- TMA store
static __device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src,
                                                    int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// global[tile at {x,y,z}] += smem tile (f32 add), bulk-group completion
static __device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src,
                                                         int x, int y, int z) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group"
        " [%0, {%2, %3, %4}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// wait until every committed bulk group has finished READING its smem source
static __device__ __forceinline__ void tma_store_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
static __device__ __forceinline__ void tma_store_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
static __device__ __forceinline__ void tma_store_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------- misc
static __device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
static __device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

static __device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a
// SWIZZLE_128B tile whose rows are 128 bytes (base 1024-byte aligned).
static __device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// Named barrier among `count` threads (warp multiples), id 1..15.
static __device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 3D bf16 tensor map [nbh][L][d] (d contiguous) with SWIZZLE_128B boxes of
// 64 columns x box_rows rows; rows past L read as zero and are not written.
inline int make_attn_map(CUtensorMap* m, const void* p, int d, int L, int nbh, int box_rows) {
    const cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)L, (cuuint64_t)nbh};
    const cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)L * d * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    CUresult r = edb::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p),
                                   dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    return r == CUDA_SUCCESS ? EDB_OK : EDB_ERR_UNSUPPORTED;
}

// 3D f32 tensor map [nbh][L][d] with SWIZZLE_128B boxes of 32 columns x box_rows.
inline int make_attn_map_f32(CUtensorMap* m, const void* p, int d, int L, int nbh, int box_rows) {
    const cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)L, (cuuint64_t)nbh};
    const cuuint64_t strides[2] = {(cuuint64_t)d * 4, (cuuint64_t)L * d * 4};
    const cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
    CUresult r = edb::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(p),
                                   dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    return r == CUDA_SUCCESS ? EDB_OK : EDB_ERR_UNSUPPORTED;
}

}  // namespace tc
