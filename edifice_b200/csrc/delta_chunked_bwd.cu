// delta_chunked_bwd.cu -- DeltaNet delta rule in chunked WY form on tcgen05 (backward).
//
// Gradient of the forward in delta_chunked.cu (same notation: per chunk
// A, T, T_b, W, U0, M, U~, S_0 -> S_C), given dO and the forward's residuals
// (S^T at every chunk start, U~ per chunk).  Reverse-mode through
//   O = Q S_0^T + M U~,  S_C = S_0 + U~^T K,  U~ = U0 - W S_0^T,
//   W = T_b K,  U0 = T_b V,  T_b = T diag(beta),  T = (I + A)^-1,
//   A = tril(diag(beta) K K^T, -1),  M = tril(Q K^T):
//   dU~  = M^T dO + K dS_C^T
//   dS_0 = dS_C + dO^T Q - dU~^T W                       (carried backwards)
//   dW   = -dU~ S_0,     dM = tril(dO U~^T),     dV = T_b^T dU~
//   dT_b = dW K^T + dU~ V^T,   dT = dT_b diag(beta),   dA = -T^T dT T^T (strictly lower)
//   dQ   = dO S_0 + dM K
//   dK   = U~ dS_C + dM^T Q + T_b^T dW + (dG + dG^T) K,   dG = diag(beta) dA
//   dbeta_s = sum_t dT_b[t][s] T[t][s] + sum_{r<s} dA[s][r] (K K^T)[s][r]
// The key gradient is the exact one, as in delta_rule.cu.
//
// Kernels (one stream, in order):
//   delta_prep_kernel<false> (delta_prep.cuh) per chunk, tcgen05 kind::f16:
//                           K K^T, M, T, W; writes the K-major f32 operands of
//                           the state kernel and T, K K^T.
//   delta_state_bwd_kernel  per (b, h), chunks in reverse, tcgen05 kind::tf32,
//                           dS in TMEM (lanes = value dim):
//                             D_U = dS K^T + dO^T M        (= dU~^T)   N=64
//                             dS += dO^T Q + D_U (-W)                  N=128
//                           stores dS_C^T, dU~ and dU~^T per chunk.
//   delta_post_kernel       (delta_chunked_post.cu) per chunk: the products
//                           with S_0 / dS_C, dT_b, dQ, dK, dV on tcgen05, the
//                           C x C chain (dA, dbeta) SIMT.
//
// GatedDeltaNet (GATED; fused_scan.ex:1347-1431 is the reference's backward):
// with the forward's gamma_t, Gamma, K' = diag(gamma) K, K~ = diag(gamma_C/gamma) K,
// Q~ = diag(gamma) Q, M = tril(Q K^T) o Gamma, W = T diag(beta) K':
//   dU~  = M^T dO + K~ dS_C^T
//   dS_0 = gamma_C dS_C + dO^T Q~ - dU~^T W
//   dT_b = dW K'^T + dU~ V^T,  dM~ = dM o Gamma,  dG = (diag(beta) dA) o Gamma
//   dQ   = diag(gamma) dO S_0 + dM~ K
//   dK   = diag(gamma_C/gamma) U~ dS_C + dM~^T Q + diag(gamma) T_b^T dW + (dG + dG^T) K
//   dg_t = <dQ~_t, q~_t> + <dK'_t, k'_t> - <dK~_t, k~_t> + rowsum - colsum of dM o M
//          and of dA o A (A = tril(diag(beta)(K K^T o Gamma), -1)), and at t = C - 1
//          also sum_s <dK~_s, k~_s> + gamma_C <dS_C, S_0>
//   dalpha_s = (sum_{t >= s} dg_t) / alpha_s        (g_t = sum_{s<=t} log alpha_s)
// The prep writes K' (Kf), K~ (Kd), Q~^T (QdT) and g; the state kernel reads K~,
// Q~^T and -W^T, and scales dS by gamma_C between P1 (which needs dS_C) and P2.
#include <math.h>

#include "delta_chunked.cuh"
#include "delta_prep.cuh"

using namespace dchunk;

namespace {

// ------------------------------------------------------------------ scratch
struct BwdScratch {
    // prep outputs
    float* Kf;    // [nch][C][D]  K (f32)
    float* KT;    // [nch][D][C]  K^T
    float* dOT;   // [nch][D][C]  dO^T
    float* QT;    // [nch][D][C]  Q^T
    float* WnT;   // [nch][D][C]  -W^T
    float* MT;    // [nch][C][C]  M^T
    float* T;     // [nch][C][C]  T (unscaled)
    float* G;     // [nch][C][C]  K K^T
    // state kernel outputs
    float* dSCT;  // [nch][D][D]  dS_C^T
    float* dU;    // [nch][C][D]  dU~
    float* dUT;   // [nch][D][C]  dU~^T
    // gated only
    float* Kd;    // [nch][C][D]  K~ = diag(gamma_C / gamma) K
    float* QdT;   // [nch][D][C]  Q~^T
    float* gl;    // [nch][C]     g
};

size_t bwd_scratch_bytes(long long nch, bool gated) {
    return 7 * a256((size_t)nch * C * D * 4) + 3 * a256((size_t)nch * C * C * 4) +
           a256((size_t)nch * D * D * 4) +
           (gated ? 2 * a256((size_t)nch * C * D * 4) + a256((size_t)nch * C * 4) : 0);
}

BwdScratch carve_bwd(void* ws, long long nch, bool gated) {
    char* p = static_cast<char*>(ws);
    const size_t cd = a256((size_t)nch * C * D * 4), cc = a256((size_t)nch * C * C * 4);
    auto take = [&](size_t bytes) {
        float* r = reinterpret_cast<float*>(p);
        p += bytes;
        return r;
    };
    BwdScratch s;
    s.Kf = take(cd);
    s.KT = take(cd);
    s.dOT = take(cd);
    s.QT = take(cd);
    s.WnT = take(cd);
    s.dU = take(cd);
    s.dUT = take(cd);
    s.MT = take(cc);
    s.T = take(cc);
    s.G = take(cc);
    s.dSCT = take(a256((size_t)nch * D * D * 4));
    s.Kd = gated ? take(cd) : nullptr;
    s.QdT = gated ? take(cd) : nullptr;
    s.gl = gated ? take(a256((size_t)nch * C * 4)) : nullptr;
    return s;
}

// ------------------------------------------------------------------ state bwd
struct StateBwdMaps {
    CUtensorMap Kf, dOT, MT, QT, WnT;
};

// grid (H, B), one CTA per (b, h), chunks in reverse.  Warp roles as in the
// forward state kernel:
//   warps 0-3  read dS (= dS_C of the chunk) out of TMEM at every step and
//              store dS_C^T;
//   warps 4-7  read the finished D_U = dU~^T of each step out (dU~ and
//              dU~^T) while P2 of that step runs;
//   warp 8     lane 0 issues the TMA loads and the MMAs.
// D_U is double-buffered by step parity:
//   P1(n): D_U[b] = dS K^T + dO^T M            (dS read as A from TMEM)
//   P2(n): dS += dO^T Q + D_U[b] (-W)          (after dS_C^T is read out)
// mbarriers: fullX[2], fullY (TMA), p1[b], p2[b] (tcgen05.commit), s_read
// (dS read out, 4 warp arrivals), u_free[b] (D_U[b] read out, 4 arrivals).
namespace sb {
constexpr int THREADS = 288;
// X stage (double-buffered): K [C][D] | dO^T [D][C] | M^T [C][C]
constexpr int XO_K = 0, XO_O = 4 * BOX_C, XO_M = XO_O + 2 * BOX_D;
constexpr int X_BYTES = XO_M + 2 * BOX_C;  // 80 KB
// Y stage (single): Q^T [D][C] | -W^T [D][C]
constexpr int YO_Q = 0, YO_W = 2 * BOX_D;
constexpr int Y_BYTES = YO_W + 2 * BOX_D;  // 64 KB
constexpr int OFF_Y = 2 * X_BYTES;
constexpr int OFF_BARS = OFF_Y + Y_BYTES;
constexpr int SMEM = OFF_BARS + 128;
constexpr int TM_S = 0, TM_U = 128, TM_COLS = 256;  // D_U: 2 x 64 columns
}  // namespace sb

template <bool GATED>
__global__ void __launch_bounds__(sb::THREADS, 1)
    delta_state_bwd_kernel(const __grid_constant__ StateBwdMaps maps, const float* __restrict__ gl,
                           float* __restrict__ dSCT, float* __restrict__ dU,
                           float* __restrict__ dUT, int H, int NC, unsigned* err) {
    using namespace sb;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BARS);
    uint64_t* fullX = bars;       // [2]
    uint64_t* fullY = bars + 2;
    uint64_t* p1 = bars + 3;      // [2]
    uint64_t* p2 = bars + 5;      // [2]
    uint64_t* s_read = bars + 7;
    uint64_t* u_free = bars + 8;  // [2]
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 10);
    volatile uint32_t* s_abort = s_tmem + 1;
    const int h = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long ch0 = ((long long)b * H + h) * NC;

    if ((smem_u32(smem) & 1023u) != 0) {
        if (tid == 0) edb_flag_error(err, EDB_DEVERR_DELTA_PIPE);
        return;
    }
    if (warp == 0) {
        tc::tmem_alloc(s_tmem, TM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        *s_abort = 0;
        for (int e = 0; e < 10; ++e) mbar_init(&bars[e], e >= 7 ? 4 : 1);
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *s_tmem;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int i = (warp & 3) * 32 + lane;  // TMEM lane = value-dim row of dS
    if (warp < 4) {  // dS = 0: no gradient reaches the final state
        uint32_t z[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) z[e] = 0u;
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) tc::tmem_st32(tmem + TM_S + lane_base + cc * 32, z);
        tc::tmem_wait_st();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    auto wait = [&](uint64_t* bar, uint32_t parity) {
        if (mbar_wait_bounded(bar, parity, err, EDB_DEVERR_DELTA_PIPE)) return true;
        *s_abort = 1;
        return false;
    };
    // The same decisions taken by a whole warp: the .sync.aligned TMEM loads and
    // stores that follow them need every lane, so no lane may leave alone.
    auto wait_w = [&](uint64_t* bar, uint32_t parity) {
        const bool ok = mbar_wait_bounded(bar, parity, err, EDB_DEVERR_DELTA_PIPE);
        if (__all_sync(0xffffffffu, ok)) return true;
        *s_abort = 1;
        return false;
    };
    auto abort_w = [&]() { return __any_sync(0xffffffffu, *s_abort != 0u); };

    if (warp == 8) {
        // ---------------------------------------------------------- TMA + MMA
        if (lane == 0) {
            // copies issued / waited per barrier
            int x_issued[2] = {0, 0}, x_landed[2] = {0, 0}, y_issued = 0, y_landed = 0;
            int committed = 0, done = 0;
            auto issue_x = [&](int c, int n) {
                uint8_t* st = smem + (n & 1) * X_BYTES;
                uint64_t* bar = &fullX[n & 1];
                const int rc = (int)((ch0 + c) * C), rd = (int)((ch0 + c) * D);
                mbar_arrive_expect_tx(bar, X_BYTES);
                for (int bx = 0; bx < 4; ++bx)
                    tma_load_2d(st + XO_K + bx * BOX_C, &maps.Kf, bar, bx * 32, rc);
                for (int bx = 0; bx < 2; ++bx) {
                    tma_load_2d(st + XO_O + bx * BOX_D, &maps.dOT, bar, bx * 32, rd);
                    tma_load_2d(st + XO_M + bx * BOX_C, &maps.MT, bar, bx * 32, rc);
                }
                ++x_issued[n & 1];
            };
            auto issue_y = [&](int c) {
                uint8_t* st = smem + OFF_Y;
                const int rd = (int)((ch0 + c) * D);
                mbar_arrive_expect_tx(fullY, Y_BYTES);
                for (int bx = 0; bx < 2; ++bx) {
                    tma_load_2d(st + YO_Q + bx * BOX_D, &maps.QT, fullY, bx * 32, rd);
                    tma_load_2d(st + YO_W + bx * BOX_D, &maps.WnT, fullY, bx * 32, rd);
                }
                ++y_issued;
            };
            prefetch_tmap(&maps.Kf);
            prefetch_tmap(&maps.dOT);
            prefetch_tmap(&maps.MT);
            prefetch_tmap(&maps.QT);
            prefetch_tmap(&maps.WnT);
            issue_x(NC - 1, 0);
            issue_y(NC - 1);
            if (NC > 1) issue_x(NC - 2, 1);
            constexpr uint32_t idN64 = idesc_tf32(128, C);
            constexpr uint32_t idN128 = idesc_tf32(128, D);
            for (int n = 0; n < NC; ++n) {
                const int c = NC - 1 - n, bf = n & 1;
                const uint32_t par = (n >> 1) & 1;
                const uint8_t* xs = smem + bf * X_BYTES;
                const uint8_t* ys = smem + OFF_Y;
                const uint32_t tU = tmem + TM_U + bf * 64;
                if (!wait(&fullX[bf], x_landed[bf] & 1)) break;
                ++x_landed[bf];
                // D_U[bf] was read out at step n - 2
                if (n >= 2 && !wait(&u_free[bf], ((n - 2) >> 1) & 1)) break;
                tc::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk)
                    mma_tf32_ts(tU, tmem + TM_S + kk * 8, kdesc(xs + XO_K, BOX_C, kk), idN64,
                                kk > 0);
#pragma unroll
                for (int kk = 0; kk < C / 8; ++kk)
                    mma_tf32_ss(tU, kdesc(xs + XO_O, BOX_D, kk), kdesc(xs + XO_M, BOX_C, kk),
                                idN64, 1);
                tc::commit(&p1[bf]);
                committed = 2 * n + 1;
                if (!wait(&p1[bf], par)) break;
                done = 2 * n + 1;
                if (!wait(fullY, y_landed & 1)) break;
                ++y_landed;
                if (!wait(s_read, n & 1)) break;
                tc::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < C / 8; ++kk) {
                    mma_tf32_ss(tmem + TM_S, kdesc(xs + XO_O, BOX_D, kk),
                                kdesc(ys + YO_Q, BOX_D, kk), idN128, 1);
                    mma_tf32_ts(tmem + TM_S, tU + kk * 8, kdesc(ys + YO_W, BOX_D, kk), idN128, 1);
                }
                tc::commit(&p2[bf]);
                committed = 2 * n + 2;
                if (!wait(&p2[bf], par)) break;
                done = 2 * n + 2;
                if (c >= 1) issue_y(c - 1);
                if (c >= 2) issue_x(c - 2, n + 2);
            }
            if (*s_abort) {
                // bounded waits for the copies and MMAs still in flight
                for (int bb = 0; bb < 2; ++bb)
                    for (; x_landed[bb] < x_issued[bb]; ++x_landed[bb])
                        mbar_wait_bounded(&fullX[bb], x_landed[bb] & 1, err,
                                          EDB_DEVERR_DELTA_PIPE);
                for (; y_landed < y_issued; ++y_landed)
                    mbar_wait_bounded(fullY, y_landed & 1, err, EDB_DEVERR_DELTA_PIPE);
                if (committed > done) {
                    const int nn = (committed - 1) >> 1;
                    uint64_t* bar = (committed & 1) ? &p1[nn & 1] : &p2[nn & 1];
                    mbar_wait_bounded(bar, (nn >> 1) & 1, err, EDB_DEVERR_DELTA_PIPE);
                }
            }
        }
    } else if (warp < 4) {
        // ---------------------------------------------------------- dS_C^T
        for (int n = 0; n < NC; ++n) {
            if (n > 0 && !wait_w(&p2[(n - 1) & 1], ((n - 1) >> 1) & 1)) break;
            if (abort_w()) break;
            tc::fence_after_sync();
            // dS is read into registers and released (s_read) before its 64 KB of
            // stores are issued, so P2 never waits on the global store queue
            uint32_t x[D / 32][32];
#pragma unroll
            for (int cc = 0; cc < D / 32; ++cc)
                tc::tmem_ld32(tmem + TM_S + lane_base + cc * 32, x[cc]);
            tc::tmem_wait_ld();
            if (GATED) {
                // dS <- gamma_C dS once P1(n) has read dS_C
                const float gC = __expf(gl[(ch0 + NC - 1 - n) * C + C - 1]);
                if (!wait_w(&p1[n & 1], (n >> 1) & 1)) break;
                tc::fence_after_sync();
#pragma unroll
                for (int cc = 0; cc < D / 32; ++cc)
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8) {
                        uint32_t y[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            y[e] = __float_as_uint(gC * __uint_as_float(x[cc][8 * g8 + e]));
                        tc::tmem_st8(tmem + TM_S + lane_base + cc * 32 + 8 * g8, y);
                    }
                tc::tmem_wait_st();
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_read);
            float* dst = dSCT + (ch0 + NC - 1 - n) * D * D + i;
#pragma unroll
            for (int cc = 0; cc < D / 32; ++cc)
#pragma unroll
                for (int e = 0; e < 32; ++e) dst[(cc * 32 + e) * D] = __uint_as_float(x[cc][e]);
        }
    } else {
        // ---------------------------------------------------------- dU~, dU~^T
        for (int n = 0; n < NC; ++n) {
            // D_U[n & 1] is final once P1(n) is done (P2(n) only reads it)
            if (!wait_w(&p1[n & 1], (n >> 1) & 1)) break;
            if (abort_w()) break;
            tc::fence_after_sync();
            // D_U row i -> dU~[c][t][i] (coalesced over i) and dU~^T[c][i][t]
            const int c = NC - 1 - n;
            float* ut = dUT + ((ch0 + c) * D + i) * C;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t x[32];
                tc::tmem_ld32(tmem + TM_U + (n & 1) * 64 + lane_base + half * 32, x);
                tc::tmem_wait_ld();
                float* du = dU + (ch0 + c) * C * D + (long long)half * 32 * D + i;
#pragma unroll
                for (int e = 0; e < 32; ++e) du[e * D] = __uint_as_float(x[e]);
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                    st4(ut + half * 32 + e,
                        make_float4(__uint_as_float(x[e]), __uint_as_float(x[e + 1]),
                                    __uint_as_float(x[e + 2]), __uint_as_float(x[e + 3])));
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&u_free[n & 1]);
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

// ---------------------------------------------------------------- library-internal
int edb_delta_chunked_post(const float* resid, const void* dO, const void* v, const void* beta,
                           const void* alpha, const float* dSCT, const float* dU, const float* dUT,
                           const float* Kf, const float* KT, const float* QT, const float* T,
                           const float* G, const float* MT, const float* gl, void* gq, void* gk,
                           void* gv, void* gbeta, void* galpha, int B, int L, int H,
                           cudaStream_t st);

size_t edb_delta_chunked_bwd_ws(int B, int L, int H, int gated) {
    return bwd_scratch_bytes((long long)B * H * ((L + C - 1) / C), gated != 0);
}

int edb_delta_chunked_bwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* alpha, const void* dO, const float* resid, void* gq,
                          void* gk, void* gv, void* gbeta, void* galpha, int B, int L, int H,
                          void* ws, cudaStream_t st) {
    const int NC = (L + C - 1) / C;
    const long long units = (long long)B * H, nch = units * NC;
    if ((units * (NC + 1)) * D > 0x7fffffffLL) return EDB_ERR_UNSUPPORTED;
    const bool gated = alpha != nullptr;
    BwdScratch w = carve_bwd(ws, nch, gated);
    unsigned* err = edb::device_error_word();
    cudaError_t e;
    PrepOut po{};
    po.KT = w.KT;
    po.Kf = w.Kf;
    po.XT = w.dOT;
    po.QT = w.QT;
    po.MT = w.MT;
    po.WnT = w.WnT;
    po.T = w.T;
    po.G = w.G;
    po.Kd = w.Kd;
    po.QdT = w.QdT;
    po.gl = w.gl;
    int s = launch_delta_prep<false>(q, k, dO, beta, alpha, po, B, L, H, st);
    if (s != EDB_OK) return s;

    // gated: the state kernel takes K~ and Q~^T, the post kernel K' (in Kf), K^T, Q^T
    StateBwdMaps sm;
    if ((s = make_box_map(&sm.Kf, gated ? w.Kd : w.Kf, nch * C, D, C))) return s;
    if ((s = make_box_map(&sm.dOT, w.dOT, nch * D, C, D))) return s;
    if ((s = make_box_map(&sm.MT, w.MT, nch * C, C, C))) return s;
    if ((s = make_box_map(&sm.QT, gated ? w.QdT : w.QT, nch * D, C, D))) return s;
    if ((s = make_box_map(&sm.WnT, w.WnT, nch * D, C, D))) return s;
    auto kern = gated ? delta_state_bwd_kernel<true> : delta_state_bwd_kernel<false>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  sb::SMEM)) != cudaSuccess)
        return (int)e;
    kern<<<dim3(H, B), sb::THREADS, sb::SMEM, st>>>(sm, w.gl, w.dSCT, w.dU, w.dUT, H, NC, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return (int)e;

    return edb_delta_chunked_post(resid, dO, v, beta, alpha, w.dSCT, w.dU, w.dUT, w.Kf, w.KT,
                                  w.QT, w.T, w.G, w.MT, w.gl, gq, gk, gv, gbeta, galpha, B, L, H,
                                  st);
}
