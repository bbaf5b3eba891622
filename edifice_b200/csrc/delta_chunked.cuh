// delta_chunked.cuh -- pieces shared by the chunked DeltaNet kernels
// (delta_chunked.cu: forward, delta_chunked_bwd.cu: backward).
//
// Tiles are f32 in HBM and reach shared memory as SWIZZLE_128B boxes of 32
// columns (128 B) x R rows, so a [R][n] operand is n/32 boxes of R*128 bytes.
// Every tcgen05 operand is K-major (kind::tf32: 8 elements = 32 B per K step).
#pragma once

#include "tc_common.cuh"

namespace dchunk {

constexpr int C = 64;    // chunk length
constexpr int D = 128;   // head dim (d_k = d_v)
constexpr int BOX_C = C * 128;   // 8 KB: [C rows][32 f32]
constexpr int BOX_D = D * 128;   // 16 KB: [D rows][32 f32]

inline size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

// Residual buffer (s_ckpt) of the chunked path, per (b, h) unit u of n units:
//   S^T at the start of chunk c (and the final one), [n][NC + 1][D][D]
//   then the chunk errors U~ = U0 - W S_0^T, [n][NC][C][D]
static __host__ __device__ __forceinline__ size_t ckpt_state_floats(long long units, int NC) {
    return (size_t)units * (NC + 1) * D * D;
}
inline size_t ckpt_bytes(long long units, int NC) {
    return (ckpt_state_floats(units, NC) + (size_t)units * NC * C * D) * sizeof(float);
}

static __host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4)                      // D format f32
           | (2u << 7) | (2u << 10)       // A, B tf32 (both K-major)
           | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::tf32, A K-major in TMEM.
static __device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem,
                                                   uint64_t b_desc, uint32_t idesc,
                                                   uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32.
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

// Descriptor of K step kk (8 f32) of a K-major SW128 operand made of boxes.
static __device__ __forceinline__ uint64_t kdesc(const uint8_t* base, int box_bytes, int kk) {
    return tc::sdesc_sw128(base + (kk >> 2) * box_bytes + (kk & 3) * 32, 16, 1024);
}

// Byte offset of the 4 f32 (row, k..k+3), k % 4 == 0, in such an operand of
// `rows` rows.
static __device__ __forceinline__ uint32_t kmaj_off4(int row, int k, int rows) {
    return (uint32_t)(k >> 5) * (uint32_t)(rows * 128) + tc::sw128_off(row, (k & 31) >> 2);
}

// 2D f32 map over a [rows][cols] array, boxes of 32 columns x box_rows rows.
inline int make_box_map(CUtensorMap* m, const float* p, long long rows, int cols,
                        int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    CUresult r = edb::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p),
                                   dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    return r == CUDA_SUCCESS ? EDB_OK : EDB_ERR_UNSUPPORTED;
}

// Thread i holds row i of a [D][ncol] TMEM accumulator (columns col..);
// stores it transposed: dst[c * D + i] for c < ncol (coalesced over i).
template <int NCOL>
static __device__ __forceinline__ void store_rows_transposed(float* dst, uint32_t taddr,
                                                             float scale = 1.0f) {
#pragma unroll
    for (int cc = 0; cc < NCOL / 32; ++cc) {
        uint32_t x[32];
        tc::tmem_ld32(taddr + cc * 32, x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) dst[(cc * 32 + e) * D] = scale * __uint_as_float(x[e]);
    }
}

// ---------------------------------------------------------------- chunk prep (SIMT)
// Shared by the forward and backward prep kernels (256 threads, one chunk).
// Shared-memory operands are f32 with padded rows: [C][PP] for C x D tiles,
// [C][PC] for C x C (odd strides: column walks are bank-conflict free).
constexpr int kPrepThreads = 256;
constexpr int PP = D + 1;
constexpr int PC = C + 1;

// Load rows t0.. of a bf16 [.., heads, D] tensor (token stride H*D) into
// dst[C][PP] as f32; rows past L are zero.  If gcopy != nullptr, also stores
// the f32 rows to gcopy[C][D].
static __device__ __forceinline__ void load_chunk_rows(float* dst, const __nv_bfloat16* src,
                                                       long long row0, long long tok_stride,
                                                       int nvalid, float* gcopy) {
    for (int idx = threadIdx.x; idx < C * (D / 8); idx += kPrepThreads) {
        const int t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
        float f[8];
        if (t < nvalid) {
            Vec16<__nv_bfloat16>::unpack(
                *reinterpret_cast<const uint4*>(src + row0 + t * tok_stride + j8), f);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[t * PP + j8 + e] = f[e];
        if (gcopy != nullptr) {
            *reinterpret_cast<float4*>(gcopy + t * D + j8) = make_float4(f[0], f[1], f[2], f[3]);
            *reinterpret_cast<float4*>(gcopy + t * D + j8 + 4) =
                make_float4(f[4], f[5], f[6], f[7]);
        }
    }
}

// Gs = K K^T (all entries), Ms = tril(Q K^T) with the diagonal.
static __device__ __forceinline__ void prep_products(const float* Ks, const float* Qs, float* Gs,
                                                     float* Ms) {
    const int t = threadIdx.x >> 2, sl = threadIdx.x & 3;
    float g[16], m[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) g[e] = m[e] = 0.0f;
    for (int j = 0; j < D; ++j) {
        const float kt = Ks[t * PP + j], qt = Qs[t * PP + j];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const float ks = Ks[(sl + 4 * e) * PP + j];
            g[e] = fmaf(kt, ks, g[e]);
            m[e] = fmaf(qt, ks, m[e]);
        }
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        const int s = sl + 4 * e;
        Gs[t * PC + s] = g[e];
        Ms[t * PC + s] = s <= t ? m[e] : 0.0f;
    }
}

// Tm = (I + A)^-1 with A = tril(diag(beta) Gs, -1): forward substitution, one
// column per thread (threads 0..C-1).  Caller syncs before and after.
static __device__ __forceinline__ void prep_solve(const float* Gs, const float* bs, float* Tm) {
    if (threadIdx.x < C) {
        const int j = threadIdx.x;
        for (int t = 0; t < C; ++t) {
            float acc = (t == j) ? 1.0f : 0.0f;
            const float bt = bs[t];
            for (int s = j; s < t; ++s) acc = fmaf(-bt * Gs[t * PC + s], Tm[s * PC + j], acc);
            Tm[t * PC + j] = t >= j ? acc : 0.0f;
        }
    }
}

// out[e] = (T diag(beta) X)[t][jl + 4 e] for thread (t = tid / 4, jl = tid % 4).
static __device__ __forceinline__ void prep_apply_tb(const float* Tm, const float* bs,
                                                     const float* Xs, float (&out)[32]) {
    const int t = threadIdx.x >> 2, jl = threadIdx.x & 3;
#pragma unroll
    for (int e = 0; e < 32; ++e) out[e] = 0.0f;
    for (int s = 0; s <= t; ++s) {
        const float tb = Tm[t * PC + s] * bs[s];
#pragma unroll
        for (int e = 0; e < 32; ++e) out[e] = fmaf(tb, Xs[s * PP + jl + 4 * e], out[e]);
    }
}

}  // namespace dchunk
