// delta_chunked_post.cu -- last stage of the chunked DeltaNet backward: the
// per-chunk C x C chain and the final dQ, dK, dV, dbeta.
//
// Inputs per chunk (f32 scratch from the earlier stages of
// delta_chunked_bwd.cu): dQa = dO S_0, dW = -dU~ S_0 (and its transpose),
// dK1 = U~ dS_C, dM = tril(dO U~^T), dU~ (and its transpose), T, K K^T, K (row and
// transposed f32 copies), Q^T; plus v, beta (bf16).
//   dT_b = dW K^T + dU~ V^T                        tcgen05, M=64,  K=2x128
//   dbeta_s = sum_t dT_b[t][s] T[t][s],  dT = dT_b diag(beta)
//   dA = -(T^T dT) T^T (strictly lower),  dbeta_t += sum_{s<t} dA[t][s] (K K^T)[t][s]
//   E = dG + dG^T,  dG = diag(beta) dA             SIMT (64 x 64 x 64)
//   dQ^T = K^T dM^T                 (+ dQa)        tcgen05, M=128, K=64
//   dV^T = dU~^T T_b                               tcgen05, M=128, K=64
//   dK^T = Q^T dM + dW^T T_b + K^T E  (+ dK1)       tcgen05, M=128, K=3x64
// Every tcgen05 operand is a K-major f32 SWIZZLE_128B tile: the earlier stages
// write the orientations needed here, so tiles arrive by TMA without
// transposes; the B tiles of the last products (dM, dM^T, T_b^T, E) are written
// by the threads.  One CTA (256 threads) per chunk; the K^T / Q^T tiles of the
// last products load while the SIMT chain runs.
#include <math.h>

#include "delta_chunked.cuh"

using namespace dchunk;

namespace {

constexpr int THREADS = 256;
constexpr int A_TILE = 4 * BOX_C;            // 32 KB: a [C][D] or [D][C] f32 tile
constexpr int B_TILE = 2 * BOX_C;            // 16 KB: a [C][C] f32 tile
// A tiles.  Phase 1: 0 dW | 1 dU~ | 2 K | 3 V.  Then 2 K^T | 3 Q^T (loading during
// the chain, whose scratch occupies tiles 0-1), and 0 dU~^T | 1 dW^T.
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + 4 * A_TILE;    // 4 B tiles: dM | dM^T | T_b^T | E
constexpr int OFF_BS = OFF_B + 4 * B_TILE;   // beta [C]
constexpr int OFF_BAR = OFF_BS + C * 4;
constexpr int SMEM = OFF_BAR + 64;
constexpr int TM_DTB = 0, TM_Q = 64, TM_V = 128, TM_K = 192, TM_COLS = 256;
// SIMT scratch of the C x C chain (floats, inside A tiles 0-1)
constexpr int SC_T = 0, SC_DT = C * PC, SC_X = 2 * C * PC;
static_assert((3 * C * PC) * 4 <= 2 * A_TILE, "chain scratch fits A tiles 0-1");

struct PostMaps {
    CUtensorMap dW, dU, Kf;          // phase 1: [C][D] row tiles (box rows C)
    CUtensorMap KT, dUT, QT, dWT;    // phase 2: [D][C] tiles (box rows D)
};

static __device__ __forceinline__ float4 f4(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}

// A thread's share of a 64 x 64 tile: rows ty + 16 r, columns tx + 16 c (r, c < 4).
__global__ void __launch_bounds__(THREADS, 1)
    delta_post2_kernel(const __grid_constant__ PostMaps maps, const __nv_bfloat16* __restrict__ v,
                       const __nv_bfloat16* __restrict__ beta, const float* __restrict__ dQa,
                       const float* __restrict__ dK1, const float* __restrict__ dMg,
                       const float* __restrict__ Tg, const float* __restrict__ Gg,
                       __nv_bfloat16* __restrict__ gq, __nv_bfloat16* __restrict__ gk,
                       __nv_bfloat16* __restrict__ gv, __nv_bfloat16* __restrict__ gbeta, int L,
                       int H, int NC, unsigned* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* sc = reinterpret_cast<float*>(smem + OFF_A);  // chain scratch (A tiles 0-1)
    float* bs = reinterpret_cast<float*>(smem + OFF_BS);
    uint64_t* bar_ld = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // [3] TMA groups
    uint64_t* bar_mma = bar_ld + 3;
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bar_mma + 1);  // [0] tmem, [1] abort
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ty = tid >> 4, tx = tid & 15;
    const long long ch = ((long long)b * H + h) * NC + c;
    const int t0 = c * C, nvalid = min(C, L - t0);
    const long long ts = (long long)H * D;
    const long long row0 = (((long long)b * L + t0) * H + h) * D;
    uint8_t* At = smem + OFF_A;

    if ((smem_u32(smem) & 1023u) != 0) {
        if (tid == 0) edb_flag_error(err, EDB_DEVERR_DELTA_PIPE);
        return;
    }
    if (warp == 0) {
        tc::tmem_alloc(s_misc, TM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        s_misc[1] = 0;
        for (int i = 0; i < 3; ++i) mbar_init(&bar_ld[i], 1);
        mbar_init(bar_mma, 1);
        fence_mbar_init();
        // phase 1 tiles: dW, dU~, K rows of this chunk
        mbar_arrive_expect_tx(&bar_ld[0], 3 * A_TILE);
        const int rc = (int)(ch * C);
        for (int bx = 0; bx < 4; ++bx) {
            tma_load_2d(At + 0 * A_TILE + bx * BOX_C, &maps.dW, &bar_ld[0], bx * 32, rc);
            tma_load_2d(At + 1 * A_TILE + bx * BOX_C, &maps.dU, &bar_ld[0], bx * 32, rc);
            tma_load_2d(At + 2 * A_TILE + bx * BOX_C, &maps.Kf, &bar_ld[0], bx * 32, rc);
        }
    }
    // V rows (bf16 -> f32) into A tile 3; beta
    {
        constexpr int N = C * (D / 8) / THREADS;
        uint4 rv[N];
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
            rv[n] = t < nvalid ? *reinterpret_cast<const uint4*>(v + row0 + t * ts + j8)
                               : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
            float f[8];
            Vec16<__nv_bfloat16>::unpack(rv[n], f);
            uint8_t* vt = At + 3 * A_TILE;
            st4(reinterpret_cast<float*>(vt + kmaj_off4(t, j8, C)), make_float4(f[0], f[1], f[2], f[3]));
            st4(reinterpret_cast<float*>(vt + kmaj_off4(t, j8 + 4, C)), make_float4(f[4], f[5], f[6], f[7]));
        }
    }
    if (tid < C)
        bs[tid] = tid < nvalid ? __bfloat162float(beta[((long long)b * L + t0 + tid) * H + h])
                               : 0.0f;
    // this thread's share of dM, and of T for the chain (loads issued early)
    float dm[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) dm[r][cc] = dMg[(ch * C + ty + 16 * r) * C + tx + 16 * cc];
    float4 tv[C * C / 4 / THREADS];
#pragma unroll
    for (int n = 0; n < C * C / 4 / THREADS; ++n) tv[n] = f4(Tg + ch * C * C + 4 * (tid + n * THREADS));
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_misc[0];
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;

    // ---- phase 1: dT_b = dW K^T + dU~ V^T  (M = 64); then K^T, Q^T start loading
    if (tid == 0) {
        bool ok = mbar_wait_bounded(&bar_ld[0], 0, err, EDB_DEVERR_DELTA_PIPE);
        if (ok) {
            tc::fence_after_sync();
            constexpr uint32_t id64 = idesc_tf32(64, C);
#pragma unroll
            for (int kk = 0; kk < D / 8; ++kk) {
                mma_tf32_ss(tmem + TM_DTB, kdesc(At + 0 * A_TILE, BOX_C, kk),
                            kdesc(At + 2 * A_TILE, BOX_C, kk), id64, kk > 0);
                mma_tf32_ss(tmem + TM_DTB, kdesc(At + 1 * A_TILE, BOX_C, kk),
                            kdesc(At + 3 * A_TILE, BOX_C, kk), id64, 1);
            }
            tc::commit(bar_mma);
            if (!mbar_wait_bounded(bar_mma, 0, err, EDB_DEVERR_DELTA_PIPE)) {
                mbar_wait_bounded(bar_mma, 0, err, EDB_DEVERR_DELTA_PIPE);
                ok = false;
            }
        } else {
            mbar_wait_bounded(&bar_ld[0], 0, err, EDB_DEVERR_DELTA_PIPE);
        }
        if (ok) {
            mbar_arrive_expect_tx(&bar_ld[1], 2 * A_TILE);
            const int rd = (int)(ch * D);
            for (int bx = 0; bx < 2; ++bx) {
                tma_load_2d(At + 2 * A_TILE + bx * BOX_D, &maps.KT, &bar_ld[1], bx * 32, rd);
                tma_load_2d(At + 3 * A_TILE + bx * BOX_D, &maps.QT, &bar_ld[1], bx * 32, rd);
            }
        } else {
            s_misc[1] = 1;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const bool aborted = s_misc[1] != 0;
    float* Ts = sc + SC_T;
    float* Ds = sc + SC_DT;
    float* Xs = sc + SC_X;
    if (!aborted) {
        // dT_b out of TMEM (M = 64: lanes 32w + r, r < 16, hold row 16w + r); T in
        if (warp < 4) {
            uint32_t x0[32], x1[32];
            tc::tmem_ld32(tmem + TM_DTB + lane_base, x0);
            tc::tmem_ld32(tmem + TM_DTB + lane_base + 32, x1);
            tc::tmem_wait_ld();
            if (lane < 16) {
                const int t = 16 * warp + lane;
#pragma unroll
                for (int s = 0; s < 32; ++s) {
                    Ds[t * PC + s] = __uint_as_float(x0[s]);
                    Ds[t * PC + 32 + s] = __uint_as_float(x1[s]);
                }
            }
        }
#pragma unroll
        for (int n = 0; n < C * C / 4 / THREADS; ++n) {
            const int e0 = 4 * (tid + n * THREADS);
            float* d = Ts + (e0 / C) * PC + e0 % C;
            d[0] = tv[n].x;
            d[1] = tv[n].y;
            d[2] = tv[n].z;
            d[3] = tv[n].w;
        }
        __syncthreads();
        // dbeta through T_b: column s = tid / 4, four threads per column
        float dbeta_part;
        {
            const int s = tid >> 2, qd = tid & 3;
            float acc = 0.0f;
            for (int t = qd; t < C; t += 4) acc = fmaf(Ds[t * PC + s], Ts[t * PC + s], acc);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            dbeta_part = acc + __shfl_xor_sync(0xffffffffu, acc, 2);
        }
        __syncthreads();
        for (int idx = tid; idx < C * C; idx += THREADS) Ds[(idx / C) * PC + idx % C] *= bs[idx % C];
        __syncthreads();
        {  // X = T^T dT
            float a[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) a[r][cc] = 0.0f;
            for (int t = 0; t < C; ++t) {
                float at[4], bd[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) at[r] = Ts[t * PC + ty + 16 * r];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) bd[cc] = Ds[t * PC + tx + 16 * cc];
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) a[r][cc] = fmaf(at[r], bd[cc], a[r][cc]);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) Xs[(ty + 16 * r) * PC + tx + 16 * cc] = a[r][cc];
        }
        __syncthreads();
        {  // dA = -X T^T, strictly lower (into Ds: dT is no longer needed)
            float a[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) a[r][cc] = 0.0f;
            for (int s = 0; s < C; ++s) {
                float ax[4], bt[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) ax[r] = Xs[(ty + 16 * r) * PC + s];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) bt[cc] = Ts[(tx + 16 * cc) * PC + s];
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) a[r][cc] = fmaf(ax[r], bt[cc], a[r][cc]);
            }
            __syncthreads();  // every read of Ds (dT) and Xs (X) is done
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const int row = ty + 16 * r, col = tx + 16 * cc;
                    Ds[row * PC + col] = col < row ? -a[r][cc] : 0.0f;
                }
        }
        __syncthreads();
        // dbeta through A: row t = tid / 4 (same threads as the column sums above)
        {
            const int t = tid >> 2, qd = tid & 3;
            const float* g = Gg + (ch * C + t) * C + 16 * qd;
            float acc = 0.0f;
#pragma unroll
            for (int s4 = 0; s4 < 16; s4 += 4) {
                const float4 gv4 = f4(g + s4);
                const float* da = Ds + t * PC + 16 * qd + s4;
                acc = fmaf(da[0], gv4.x, fmaf(da[1], gv4.y, fmaf(da[2], gv4.z, fmaf(da[3], gv4.w, acc))));
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (qd == 0 && t < nvalid)
                gbeta[((long long)b * L + t0 + t) * H + h] = __float2bfloat16(acc + dbeta_part);
        }
        for (int idx = tid; idx < C * C; idx += THREADS) {
            const int t = idx / C, s = idx % C;
            Xs[t * PC + s] = bs[t] * Ds[t * PC + s] + bs[s] * Ds[s * PC + t];
        }
        __syncthreads();
        // ---- B tiles of phase 2 (K-major [n][k]): dM [t][s], dM^T [s][t],
        // T_b^T [s][t] = T[t][s] beta_s, E [s][t] (symmetric)
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int row = ty + 16 * r, col = tx + 16 * cc;
                *reinterpret_cast<float*>(smem + OFF_B + 0 * B_TILE + kmaj_off4(row, col & ~3, C) + (col & 3) * 4) = dm[r][cc];
                *reinterpret_cast<float*>(smem + OFF_B + 1 * B_TILE + kmaj_off4(col, row & ~3, C) + (row & 3) * 4) = dm[r][cc];
            }
        for (int idx = tid; idx < C * C / 4; idx += THREADS) {
            const int s = idx / (C / 4), t4 = (idx % (C / 4)) * 4;
            const float bsv = bs[s];
            st4(reinterpret_cast<float*>(smem + OFF_B + 2 * B_TILE + kmaj_off4(s, t4, C)),
                make_float4(Ts[t4 * PC + s] * bsv, Ts[(t4 + 1) * PC + s] * bsv,
                            Ts[(t4 + 2) * PC + s] * bsv, Ts[(t4 + 3) * PC + s] * bsv));
            st4(reinterpret_cast<float*>(smem + OFF_B + 3 * B_TILE + kmaj_off4(s, t4, C)),
                make_float4(Xs[s * PC + t4], Xs[s * PC + t4 + 1], Xs[s * PC + t4 + 2],
                            Xs[s * PC + t4 + 3]));
        }
    }
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // ---- phase 2: dU~^T, dW^T into A tiles 0-1 (the chain scratch is dead), then
    // dQ^T, dV^T, dK^T  (M = 128)
    if (tid == 0 && !aborted) {
        mbar_arrive_expect_tx(&bar_ld[2], 2 * A_TILE);
        const int rd = (int)(ch * D);
        for (int bx = 0; bx < 2; ++bx) {
            tma_load_2d(At + 0 * A_TILE + bx * BOX_D, &maps.dUT, &bar_ld[2], bx * 32, rd);
            tma_load_2d(At + 1 * A_TILE + bx * BOX_D, &maps.dWT, &bar_ld[2], bx * 32, rd);
        }
        bool ok = mbar_wait_bounded(&bar_ld[1], 0, err, EDB_DEVERR_DELTA_PIPE);
        const bool ok2 = mbar_wait_bounded(&bar_ld[2], 0, err, EDB_DEVERR_DELTA_PIPE);
        ok = ok && ok2;
        if (ok) {
            tc::fence_after_sync();
            constexpr uint32_t id128 = idesc_tf32(128, C);
            const uint8_t* ut = At + 0 * A_TILE;
            const uint8_t* wt = At + 1 * A_TILE;
            const uint8_t* kt = At + 2 * A_TILE;
            const uint8_t* qt = At + 3 * A_TILE;
#pragma unroll
            for (int kk = 0; kk < C / 8; ++kk) {
                const uint64_t dM = kdesc(smem + OFF_B + 0 * B_TILE, BOX_C, kk);
                const uint64_t dMT = kdesc(smem + OFF_B + 1 * B_TILE, BOX_C, kk);
                const uint64_t TbT = kdesc(smem + OFF_B + 2 * B_TILE, BOX_C, kk);
                const uint64_t E = kdesc(smem + OFF_B + 3 * B_TILE, BOX_C, kk);
                const uint64_t kA = kdesc(kt, BOX_D, kk);
                mma_tf32_ss(tmem + TM_Q, kA, dM, id128, kk > 0);
                mma_tf32_ss(tmem + TM_V, kdesc(ut, BOX_D, kk), TbT, id128, kk > 0);
                mma_tf32_ss(tmem + TM_K, kdesc(qt, BOX_D, kk), dMT, id128, kk > 0);
                mma_tf32_ss(tmem + TM_K, kdesc(wt, BOX_D, kk), TbT, id128, 1);
                mma_tf32_ss(tmem + TM_K, kA, E, id128, 1);
            }
            tc::commit(bar_mma);
            if (!mbar_wait_bounded(bar_mma, 1, err, EDB_DEVERR_DELTA_PIPE)) {
                mbar_wait_bounded(bar_mma, 1, err, EDB_DEVERR_DELTA_PIPE);
                ok = false;
            }
        }
        if (!ok) s_misc[1] = 1;
    }
    // the epilogue's addends, loaded while the last products run: thread (lane
    // quarter, half) -> column j = TMEM lane, tokens [32 half, 32 half + 32)
    const int j = (warp & 3) * 32 + lane, hf = warp >> 2;
    float aq[32], ak[32];
    if (!aborted) {
        const float* qa = dQa + ch * C * D + (long long)hf * 32 * D + j;
        const float* k1 = dK1 + ch * C * D + (long long)hf * 32 * D + j;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            aq[e] = qa[e * D];
            ak[e] = k1[e * D];
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (!s_misc[1]) {
        uint32_t xq[32], xv[32], xk[32];
        tc::tmem_ld32(tmem + TM_Q + lane_base + hf * 32, xq);
        tc::tmem_ld32(tmem + TM_V + lane_base + hf * 32, xv);
        tc::tmem_ld32(tmem + TM_K + lane_base + hf * 32, xk);
        tc::tmem_wait_ld();
        __nv_bfloat16* oq = gq + row0 + j;
        __nv_bfloat16* ok_ = gk + row0 + j;
        __nv_bfloat16* ov = gv + row0 + j;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const int t = hf * 32 + e;
            if (t < nvalid) {
                oq[t * ts] = __float2bfloat16(aq[e] + __uint_as_float(xq[e]));
                ov[t * ts] = __float2bfloat16(__uint_as_float(xv[e]));
                ok_[t * ts] = __float2bfloat16(ak[e] + __uint_as_float(xk[e]));
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, TM_COLS);
    }
}

}  // namespace

// Library-internal launcher (called by edb_delta_chunked_bwd).
int edb_delta_chunked_post2(const void* v, const void* beta, const float* dQa, const float* dW,
                            const float* dWT, const float* dK1, const float* dM, const float* T,
                            const float* G, const float* dU, const float* dUT, const float* Kf,
                            const float* KT, const float* QT, void* gq, void* gk, void* gv,
                            void* gbeta, int B, int L, int H, cudaStream_t st) {
    const int NC = (L + C - 1) / C;
    const long long nch = (long long)B * H * NC;
    PostMaps m;
    int s;
    if ((s = make_box_map(&m.dW, dW, nch * C, D, C))) return s;
    if ((s = make_box_map(&m.dU, dU, nch * C, D, C))) return s;
    if ((s = make_box_map(&m.Kf, Kf, nch * C, D, C))) return s;
    if ((s = make_box_map(&m.KT, KT, nch * D, C, D))) return s;
    if ((s = make_box_map(&m.dUT, dUT, nch * D, C, D))) return s;
    if ((s = make_box_map(&m.QT, QT, nch * D, C, D))) return s;
    if ((s = make_box_map(&m.dWT, dWT, nch * D, C, D))) return s;
    cudaError_t e = cudaFuncSetAttribute(delta_post2_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return (int)e;
    delta_post2_kernel<<<dim3(NC, H, B), THREADS, SMEM, st>>>(
        m, (const __nv_bfloat16*)v, (const __nv_bfloat16*)beta, dQa, dK1, dM, T, G,
        (__nv_bfloat16*)gq, (__nv_bfloat16*)gk, (__nv_bfloat16*)gv, (__nv_bfloat16*)gbeta, L, H,
        NC, edb::device_error_word());
    return edb::status_from_cuda(cudaGetLastError());
}
