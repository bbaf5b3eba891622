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

// ---------------------------------------------------------------- chunk-local SIMT
// Shared by the prep kernels and the backward's C x C kernel (256 threads,
// one chunk).  Shared-memory tiles are f32: C x D tiles with rows of PP = 132
// floats (16-byte aligned; float4 index 33 t + j/4 puts 8 consecutive rows
// on 8 different bank groups), C x C tiles with rows of PC = 65 floats (odd:
// scalar column walks are bank-conflict free).  Thread (ty, tx) = (tid / 16,
// tid % 16) owns output rows ty + 16 r and, for C x D outputs, columns
// 4 tx + 64 c + e (two float4s per row), for C x C outputs columns tx + 16 c.
constexpr int kPrepThreads = 256;
constexpr int PP = D + 4;
constexpr int PC = C + 1;

static __device__ __forceinline__ float4 ld4(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}
static __device__ __forceinline__ void st4(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
}
static __device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
}

// Load rows of a bf16 [.., heads, D] tensor (token stride tok_stride, first
// row at row0) into dst[C][PP] as f32; rows >= nvalid are zero.  If gcopy is
// not null, also stores the f32 rows to gcopy[C][D].
// All of a thread's global loads are issued before the first use, so the
// latencies overlap (one loop iteration per load would serialise them).
static __device__ __forceinline__ void load_chunk_rows(float* dst, const __nv_bfloat16* src,
                                                       long long row0, long long tok_stride,
                                                       int nvalid, float* gcopy) {
    constexpr int N = C * (D / 8) / kPrepThreads;
    uint4 raw[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const int idx = threadIdx.x + n * kPrepThreads;
        const int t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
        raw[n] = t < nvalid ? *reinterpret_cast<const uint4*>(src + row0 + t * tok_stride + j8)
                            : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const int idx = threadIdx.x + n * kPrepThreads;
        const int t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
        float f[8];
        Vec16<__nv_bfloat16>::unpack(raw[n], f);
        const float4 lo = make_float4(f[0], f[1], f[2], f[3]), hi = make_float4(f[4], f[5], f[6], f[7]);
        st4(dst + t * PP + j8, lo);
        st4(dst + t * PP + j8 + 4, hi);
        if (gcopy != nullptr) {
            st4(gcopy + t * D + j8, lo);
            st4(gcopy + t * D + j8 + 4, hi);
        }
    }
}

// out[j][t] = scale * src[t][j] for a [C][PP] tile (out is [D][C]); each
// store instruction is coalesced over t.
static __device__ __forceinline__ void store_transposed(float* out, const float* src,
                                                        float scale) {
    for (int idx = threadIdx.x; idx < C * (D / 4); idx += blockDim.x) {
        const int t = idx % C, j4 = (idx / C) * 4;
        const float4 f = ld4(src + t * PP + j4);
        out[(j4 + 0) * C + t] = scale * f.x;
        out[(j4 + 1) * C + t] = scale * f.y;
        out[(j4 + 2) * C + t] = scale * f.z;
        out[(j4 + 3) * C + t] = scale * f.w;
    }
}

// Gs = K K^T (every entry), Ms = tril(Q K^T) with the diagonal.
static __device__ __forceinline__ void prep_products(const float* Ks, const float* Qs, float* Gs,
                                                     float* Ms) {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    float g[4][4], m[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) g[r][c] = m[r][c] = 0.0f;
    for (int j = 0; j < D; j += 4) {
        float4 kt[4], qt[4], ks[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            kt[r] = ld4(Ks + (ty + 16 * r) * PP + j);
            qt[r] = ld4(Qs + (ty + 16 * r) * PP + j);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) ks[c] = ld4(Ks + (tx + 16 * c) * PP + j);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                g[r][c] = dot4(kt[r], ks[c], g[r][c]);
                m[r][c] = dot4(qt[r], ks[c], m[r][c]);
            }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int t = ty + 16 * r, s = tx + 16 * c;
            Gs[t * PC + s] = g[r][c];
            Ms[t * PC + s] = s <= t ? m[r][c] : 0.0f;
        }
}

// One block diagonal d = i - j of the blocked solve below: every block (i, i - d)
//   Y_ij = sum_{k=j}^{i-1} N_ik T_kj,   T_ij = T_ii Y_ij,   N = -diag(beta) G
// with each thread's NE entries accumulated side by side (independent chains
// over unrolled 16-step block products).
template <int LEV, int NTH>
static __device__ __forceinline__ void prep_solve_level(const float* Gs, const float* bs,
                                                        float* Ys, float* Tm) {
    constexpr int NE = (4 - LEV) * 256 / NTH;
    static_assert(NE * NTH == (4 - LEV) * 256, "thread count divides the level");
    const int tid = threadIdx.x;
    float acc[NE];
    int g0[NE], t0[NE];
#pragma unroll
    for (int m = 0; m < NE; ++m) {
        const int e = tid + NTH * m, i = LEV + (e >> 8), j = i - LEV, r = (e >> 4) & 15, c = e & 15;
        g0[m] = (16 * i + r) * PC + 16 * j;
        t0[m] = 16 * j * PC + 16 * j + c;
        acc[m] = 0.0f;
    }
#pragma unroll
    for (int kk = 0; kk < LEV; ++kk)
#pragma unroll
        for (int s = 0; s < 16; ++s)
#pragma unroll
            for (int m = 0; m < NE; ++m)
                acc[m] = fmaf(Gs[g0[m] + 16 * kk + s], Tm[t0[m] + (16 * kk + s) * PC], acc[m]);
#pragma unroll
    for (int m = 0; m < NE; ++m) {
        const int e = tid + NTH * m, i = LEV + (e >> 8), r = (e >> 4) & 15;
        Ys[e] = -bs[16 * i + r] * acc[m];
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < NE; ++m) {
        const int e = tid + NTH * m, i = LEV + (e >> 8), r = (e >> 4) & 15, c = e & 15;
        g0[m] = (16 * i + r) * PC + 16 * i;  // row r of T_ii (zero above its diagonal)
        t0[m] = (e & ~255) + c;              // column c of Y_ij
        acc[m] = 0.0f;
    }
#pragma unroll
    for (int s = 0; s < 16; ++s)
#pragma unroll
        for (int m = 0; m < NE; ++m) acc[m] = fmaf(Tm[g0[m] + s], Ys[t0[m] + 16 * s], acc[m]);
#pragma unroll
    for (int m = 0; m < NE; ++m) {
        const int e = tid + NTH * m, i = LEV + (e >> 8), j = i - LEV, r = (e >> 4) & 15, c = e & 15;
        Tm[(16 * i + r) * PC + 16 * j + c] = acc[m];
    }
    __syncthreads();
}

// Tm = (I + A)^-1 with A = tril(diag(beta) Gs, -1), in 16 x 16 blocks: the
// four diagonal blocks by substitution (one thread per column, 16 steps), then
// the blocks below the diagonal one block diagonal at a time (block row i of
// (I + A) T = I gives T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj).  NTH threads
// (128 or 256); Ys is scratch of 768 floats.  Caller syncs before; syncs
// inside.  Tm is written in full (zero above the diagonal).
template <int NTH>
static __device__ __forceinline__ void prep_solve(const float* Gs, const float* bs, float* Ys,
                                                  float* Tm) {
    const int tid = threadIdx.x;
    if (tid < C) {
        const int o = 16 * (tid >> 4), j = tid & 15;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) x[r] = r == j ? 1.0f : 0.0f;
#pragma unroll
        for (int s = 0; s < 15; ++s)
#pragma unroll
            for (int r = s + 1; r < 16; ++r)
                x[r] = fmaf(-bs[o + r] * Gs[(o + r) * PC + o + s], x[s], x[r]);
#pragma unroll
        for (int r = 0; r < 16; ++r) Tm[(o + r) * PC + o + j] = x[r];
    } else {
        // the six blocks above the diagonal are zero
        for (int idx = tid - C; idx < 6 * 256; idx += NTH - C) {
            const int blk = idx >> 8, r = (idx >> 4) & 15, c = idx & 15;
            const int bi = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
            const int bj = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
            Tm[(16 * bi + r) * PC + 16 * bj + c] = 0.0f;
        }
    }
    __syncthreads();
    prep_solve_level<1, NTH>(Gs, bs, Ys, Tm);
    prep_solve_level<2, NTH>(Gs, bs, Ys, Tm);
    prep_solve_level<3, NTH>(Gs, bs, Ys, Tm);
}

// out = (T diag(beta) X) for this thread's rows ty + 16 r and columns
// 4 tx + 64 c + e: out[r][4 c + e].  T is lower triangular, so row t only
// needs s <= t.
static __device__ __forceinline__ void prep_apply_tb(const float* Tm, const float* bs,
                                                     const float* Xs, float (&out)[4][8]) {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int e = 0; e < 8; ++e) out[r][e] = 0.0f;
    for (int s = 0; s <= ty + 48; ++s) {
        float tb[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) tb[r] = Tm[(ty + 16 * r) * PC + s] * bs[s];
        const float4 x0 = ld4(Xs + s * PP + 4 * tx), x1 = ld4(Xs + s * PP + 64 + 4 * tx);
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int e = 0; e < 8; ++e) out[r][e] = fmaf(tb[r], xv[e], out[r][e]);
    }
}

// Writes a thread's [4][8] C x D tile (rows ty + 16 r, columns 4 tx + 64 c + e)
// into a [C][PP] shared tile, times scale.
static __device__ __forceinline__ void put_tile(float* dst, const float (&v)[4][8], float scale) {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c)
            st4(dst + (ty + 16 * r) * PP + 64 * c + 4 * tx,
                make_float4(scale * v[r][4 * c], scale * v[r][4 * c + 1],
                            scale * v[r][4 * c + 2], scale * v[r][4 * c + 3]));
}

}  // namespace dchunk
