// delta_chunked.cu -- DeltaNet delta rule in chunked WY form on tcgen05 (forward).
//
// Same semantics as delta_rule.cu (lib/edifice/cuda/fused_scan.ex:2212-2236,
// lib/edifice/recurrent/delta_net.ex:231-273; the reference's CUDA kernel,
// native/cuda/fused_delta_rule_scan.cu, walks tokens one by one).  This path
// serves bf16 io, one beta per (token, head), head_dim 128.
//
// Per chunk of C = 64 tokens (K, Q, V: C x d rows; S_0 the state before the
// chunk, [d_v][d_k]):
//   A   = tril(diag(beta) K K^T, -1),   T = (I + A)^-1,   T_b = T diag(beta)
//   W   = T_b K,   U0 = T_b V,   M = tril(Q K^T) (diagonal included)
//   U~  = U0 - W S_0^T            (the chunk's beta-scaled errors)
//   O   = Q S_0^T + M U~
//   S_C = S_0 + U~^T K
// which is the token recurrence S_t = S_{t-1} + beta_t (v_t - S_{t-1} k_t) k_t^T,
// o_t = S_t q_t, regrouped (T solves the within-chunk dependence of the errors).
//
// Kernels:
//   delta_prep_fwd_kernel   one CTA per chunk (all chunks at once), tcgen05
//                           kind::tf32 for K K^T, Q K^T, W and U0, SIMT for the
//                           unit-triangular solve for T; writes -W, Q, K^T, U0^T
//                           and M (f32) to scratch.
//   delta_state_fwd_kernel  one CTA per (b, h), chunks in order, tcgen05
//                           kind::tf32 with every operand K-major.  S lives in
//                           TMEM (lanes = value dim, columns = key dim) as the f32
//                           accumulator and is fed back as the A operand:
//                             D_U  = U0^T + S (-W)^T        M=128, N=64,  K=128
//                             D_O  = S Q^T + D_U M^T        M=128, N=64,  K=128/64
//                             S   += D_U (K^T)^T            M=128, N=128, K=64
//                           -W, Q, K^T, M arrive by TMA (SWIZZLE_128B f32 boxes)
//                           in a 2-stage ring; U0^T rows are stored into TMEM
//                           by the threads.  With a residual buffer it also
//                           stores S^T at every chunk start (and the final S^T)
//                           and each chunk's U~ for the backward.  TF32
//                           operands (10-bit mantissa), f32 accumulation.
#include <math.h>

#include "delta_chunked.cuh"

using namespace dchunk;

namespace {

// ------------------------------------------------------------------ scratch
struct FwdScratch {
    float* Wn;   // [nch][C][D]  -W
    float* Q;    // [nch][C][D]
    float* KT;   // [nch][D][C]
    float* U0T;  // [nch][D][C]
    float* M;    // [nch][C][C]  tril(Q K^T), diagonal included
};

size_t fwd_scratch_bytes(long long nch) {
    return 4 * a256((size_t)nch * C * D * 4) + a256((size_t)nch * C * C * 4);
}

FwdScratch carve_fwd(void* ws, long long nch) {
    char* p = static_cast<char*>(ws);
    const size_t cd = a256((size_t)nch * C * D * 4);
    FwdScratch s;
    s.Wn = reinterpret_cast<float*>(p);
    s.Q = reinterpret_cast<float*>(p + cd);
    s.KT = reinterpret_cast<float*>(p + 2 * cd);
    s.U0T = reinterpret_cast<float*>(p + 3 * cd);
    s.M = reinterpret_cast<float*>(p + 4 * cd);
    return s;
}

// ------------------------------------------------------------------ prep (tcgen05)
// grid (NC, H, B), 128 threads, one chunk per CTA, all chunks at once.  The
// threads stage f32 K-major SWIZZLE_128B operand tiles in shared memory (bf16 ->
// f32 is exact, and so is the tf32 view of a bf16 value), the products run on
// tcgen05 kind::tf32 with the accumulators in TMEM:
//   G = K K^T, Mq = Q K^T                M=64,  N=64, K=128   TMEM cols [0,64), [64,128)
//   W^T = K^T T_b^T, U0^T = V^T T_b^T    M=128, N=64, K=64    TMEM cols [128,192), [192,256)
// and the unit-triangular solve for T between them is SIMT on G read out of TMEM.
// Rows past L load as zero with beta 0, which makes their W / U0 rows zero, so
// the padded tail leaves S untouched.
namespace prep {
constexpr int THREADS = 128;
constexpr int OFF_K = 0;                    // [C][D]  K-major (K = d)
constexpr int OFF_Q = OFF_K + 4 * BOX_C;    // [C][D]
constexpr int OFF_KT = OFF_Q + 4 * BOX_C;   // [D][C]  K-major (K = token)
constexpr int OFF_VT = OFF_KT + 2 * BOX_D;  // [D][C]
constexpr int OFF_TB = OFF_VT + 2 * BOX_D;  // [C][C]  T diag(beta)
constexpr int OFF_F = OFF_TB + 2 * BOX_C;   // f32: V [C][D] K-major while staging, then G | T | Ys
constexpr int F_FLOATS = 2 * C * PC + C * C;
static_assert(F_FLOATS >= C * D, "V rows fit the solve scratch");
constexpr int OFF_BS = OFF_F + F_FLOATS * 4;
constexpr int OFF_BAR = OFF_BS + C * 4;
constexpr int SMEM = OFF_BAR + 64;
constexpr int TM_G = 0, TM_M = 64, TM_W = 128, TM_U = 192, TM_COLS = 256;
}  // namespace prep

__global__ void __launch_bounds__(prep::THREADS, 1)
    delta_prep_fwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                          const __nv_bfloat16* __restrict__ v,
                          const __nv_bfloat16* __restrict__ beta, FwdScratch ws, int L, int H,
                          int NC, unsigned* err) {
    using namespace prep;
    extern __shared__ __align__(1024) uint8_t smem[];
    float* F = reinterpret_cast<float*>(smem + OFF_F);
    float* Gs = F;                   // [C][PC]
    float* Tm = F + C * PC;          // [C][PC]
    float* Ys = F + 2 * C * PC;      // solve scratch
    float* bs = reinterpret_cast<float*>(smem + OFF_BS);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(mbar + 1);  // [0] tmem base, [1] abort
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long ch = ((long long)b * H + h) * NC + c;
    const int t0 = c * C, nvalid = min(C, L - t0);
    const long long row0 = (((long long)b * L + t0) * H + h) * D, ts = (long long)H * D;

    if ((smem_u32(smem) & 1023u) != 0) {  // SW128 tiles need 1 KB alignment
        if (tid == 0) edb_flag_error(err, EDB_DEVERR_DELTA_PIPE);
        return;
    }
    if (warp == 0) {
        tc::tmem_alloc(s_misc, TM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        s_misc[1] = 0;
        mbar_init(mbar, 1);
        fence_mbar_init();
    }
    // ---- K, Q -> swizzled row tiles, V -> plain rows; the f32 Q rows also to HBM
    {
        constexpr int N = C * (D / 8) / THREADS;
        uint4 rk[N], rq[N], rv[N];
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
            const bool ok = t < nvalid;
            const long long off = row0 + t * ts + j8;
            rk[n] = ok ? *reinterpret_cast<const uint4*>(k + off) : make_uint4(0u, 0u, 0u, 0u);
            rq[n] = ok ? *reinterpret_cast<const uint4*>(q + off) : make_uint4(0u, 0u, 0u, 0u);
            rv[n] = ok ? *reinterpret_cast<const uint4*>(v + off) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
            float f[8];
            Vec16<__nv_bfloat16>::unpack(rk[n], f);
            st4(reinterpret_cast<float*>(smem + OFF_K + kmaj_off4(t, j8, C)), make_float4(f[0], f[1], f[2], f[3]));
            st4(reinterpret_cast<float*>(smem + OFF_K + kmaj_off4(t, j8 + 4, C)), make_float4(f[4], f[5], f[6], f[7]));
            Vec16<__nv_bfloat16>::unpack(rq[n], f);
            const float4 q0 = make_float4(f[0], f[1], f[2], f[3]), q1 = make_float4(f[4], f[5], f[6], f[7]);
            st4(reinterpret_cast<float*>(smem + OFF_Q + kmaj_off4(t, j8, C)), q0);
            st4(reinterpret_cast<float*>(smem + OFF_Q + kmaj_off4(t, j8 + 4, C)), q1);
            st4(ws.Q + (ch * C + t) * D + j8, q0);
            st4(ws.Q + (ch * C + t) * D + j8 + 4, q1);
            Vec16<__nv_bfloat16>::unpack(rv[n], f);
            st4(reinterpret_cast<float*>(smem + OFF_F + kmaj_off4(t, j8, C)), make_float4(f[0], f[1], f[2], f[3]));
            st4(reinterpret_cast<float*>(smem + OFF_F + kmaj_off4(t, j8 + 4, C)), make_float4(f[4], f[5], f[6], f[7]));
        }
    }
    if (tid < C)
        bs[tid] = tid < nvalid ? __bfloat162float(beta[((long long)b * L + t0 + tid) * H + h])
                               : 0.0f;
    __syncthreads();
    // ---- K^T, V^T tiles.  A warp takes 32 consecutive tokens t and 4 columns
    // j: one float4 read per row tile (8 rows cover the 8 swizzled 16-byte
    // slots), 4 scalar writes into one 128-byte row of each transposed tile
    // (conflict free), and K^T[j][t] to HBM coalesced over t.
    for (int idx = tid; idx < C * (D / 4); idx += THREADS) {
        const int t = idx % C, j4 = (idx / C) * 4;
        const float4 k4 = ld4(reinterpret_cast<const float*>(smem + OFF_K + kmaj_off4(t, j4, C)));
        const float4 v4 = ld4(reinterpret_cast<const float*>(smem + OFF_F + kmaj_off4(t, j4, C)));
        const float kv[4] = {k4.x, k4.y, k4.z, k4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
        const uint32_t o = (t & 3) * 4;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            *reinterpret_cast<float*>(smem + OFF_KT + kmaj_off4(j4 + e, t & ~3, D) + o) = kv[e];
            *reinterpret_cast<float*>(smem + OFF_VT + kmaj_off4(j4 + e, t & ~3, D) + o) = vv[e];
            ws.KT[(ch * D + j4 + e) * C + t] = kv[e];
        }
    }
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_misc[0];
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    if (tid == 0) {
        constexpr uint32_t id64 = idesc_tf32(64, C);
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
            const uint64_t kd = kdesc(smem + OFF_K, BOX_C, kk);
            mma_tf32_ss(tmem + TM_G, kd, kd, id64, kk > 0);
            mma_tf32_ss(tmem + TM_M, kdesc(smem + OFF_Q, BOX_C, kk), kd, id64, kk > 0);
        }
        tc::commit(mbar);
        if (!mbar_wait_bounded(mbar, 0, err, EDB_DEVERR_DELTA_PIPE)) {
            mbar_wait_bounded(mbar, 0, err, EDB_DEVERR_DELTA_PIPE);
            s_misc[1] = 1;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (!s_misc[1]) {
        // ---- G -> shared (solve input), Mq -> HBM (masked); M=64 accumulators:
        // lanes 32w + r (r < 16) hold row 16w + r
        uint32_t g0[32], g1[32];
        tc::tmem_ld32(tmem + TM_G + lane_base, g0);
        tc::tmem_ld32(tmem + TM_G + lane_base + 32, g1);
        tc::tmem_wait_ld();
        if (lane < 16) {
            const int t = 16 * warp + lane;
#pragma unroll
            for (int s = 0; s < 32; ++s) {
                Gs[t * PC + s] = __uint_as_float(g0[s]);
                Gs[t * PC + 32 + s] = __uint_as_float(g1[s]);
            }
        }
        tc::tmem_ld32(tmem + TM_M + lane_base, g0);
        tc::tmem_ld32(tmem + TM_M + lane_base + 32, g1);
        tc::tmem_wait_ld();
        if (lane < 16) {
            const int t = 16 * warp + lane;
            float* mg = ws.M + (ch * C + t) * C;
#pragma unroll
            for (int s = 0; s < 32; s += 4) {
                st4(mg + s, make_float4(s <= t ? __uint_as_float(g0[s]) : 0.f,
                                        s + 1 <= t ? __uint_as_float(g0[s + 1]) : 0.f,
                                        s + 2 <= t ? __uint_as_float(g0[s + 2]) : 0.f,
                                        s + 3 <= t ? __uint_as_float(g0[s + 3]) : 0.f));
                st4(mg + 32 + s, make_float4(s + 32 <= t ? __uint_as_float(g1[s]) : 0.f,
                                             s + 33 <= t ? __uint_as_float(g1[s + 1]) : 0.f,
                                             s + 34 <= t ? __uint_as_float(g1[s + 2]) : 0.f,
                                             s + 35 <= t ? __uint_as_float(g1[s + 3]) : 0.f));
            }
        }
    }
    __syncthreads();
    if (!s_misc[1]) {
        prep_solve<THREADS>(Gs, bs, Ys, Tm);
        // ---- T diag(beta) -> K-major tile [t][s]
        for (int idx = tid; idx < C * (C / 4); idx += THREADS) {
            const int t = idx / (C / 4), s4 = (idx % (C / 4)) * 4;
            st4(reinterpret_cast<float*>(smem + OFF_TB + kmaj_off4(t, s4, C)),
                make_float4(Tm[t * PC + s4] * bs[s4], Tm[t * PC + s4 + 1] * bs[s4 + 1],
                            Tm[t * PC + s4 + 2] * bs[s4 + 2], Tm[t * PC + s4 + 3] * bs[s4 + 3]));
        }
        fence_proxy_async();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (tid == 0) {
            constexpr uint32_t id128 = idesc_tf32(128, C);
#pragma unroll
            for (int kk = 0; kk < C / 8; ++kk) {
                const uint64_t tb = kdesc(smem + OFF_TB, BOX_C, kk);
                mma_tf32_ss(tmem + TM_W, kdesc(smem + OFF_KT, BOX_D, kk), tb, id128, kk > 0);
                mma_tf32_ss(tmem + TM_U, kdesc(smem + OFF_VT, BOX_D, kk), tb, id128, kk > 0);
            }
            tc::commit(mbar);
            if (!mbar_wait_bounded(mbar, 1, err, EDB_DEVERR_DELTA_PIPE)) {
                mbar_wait_bounded(mbar, 1, err, EDB_DEVERR_DELTA_PIPE);
                s_misc[1] = 1;
            }
        }
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (!s_misc[1]) {
            // W^T row j -> -W[t][j] (coalesced over j); U0^T row i -> U0^T[i][t]
            const int j = tid;
            store_rows_transposed<C>(ws.Wn + ch * C * D + j, tmem + TM_W + lane_base, -1.0f);
            float* ug = ws.U0T + (ch * D + j) * C;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t x[32];
                tc::tmem_ld32(tmem + TM_U + lane_base + half * 32, x);
                tc::tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                    st4(ug + half * 32 + e,
                        make_float4(__uint_as_float(x[e]), __uint_as_float(x[e + 1]),
                                    __uint_as_float(x[e + 2]), __uint_as_float(x[e + 3])));
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

// ------------------------------------------------------------------ state fwd
struct StateMaps {
    CUtensorMap Wn, Q, KT, M;
};

// grid (H, B), one CTA per (b, h), chunks in order.  Warp roles:
//   warps 0-3  read S out of TMEM at every chunk start and store S^T (residual);
//   warps 4-7  store U0^T rows into TMEM ahead of each chunk, and read the
//              finished O and U~ of the previous chunk out (o, residual U~);
//   warp 8     lane 0 issues the TMA loads (2-stage ring) and the MMAs.
// The TMEM accumulators U and O are double-buffered by chunk parity, so the
// read-out of chunk c - 1 and the S^T store of chunk c run while the tensor
// core works on chunk c:
//   P1(c): D_U[b] = U0^T + S (-W)^T,  D_O[b] = S Q^T      (S read as A from TMEM)
//   P2(c): D_O[b] += D_U[b] M^T,  S += D_U[b] (K^T)^T      (after S^T is read out)
// mbarriers (per buffer where two chunks could otherwise alias one phase):
//   full[s]       TMA stage s landed          u0_ready[b]  U0^T rows in D_U[b]
//   p1[b], p2[b]  tcgen05.commit of P1 / P2   s_read       S^T of this chunk read
namespace sf {
constexpr int THREADS = 288;
constexpr int OFF_W = 0;
constexpr int OFF_Q = OFF_W + 4 * BOX_C;
constexpr int OFF_KT = OFF_Q + 4 * BOX_C;
constexpr int OFF_M = OFF_KT + 2 * BOX_D;
constexpr int STAGE_BYTES = OFF_M + 2 * BOX_C;  // 112 KB
constexpr int OFF_BARS = 2 * STAGE_BYTES;
constexpr int SMEM = OFF_BARS + 128;
constexpr int TM_S = 0, TM_U = 128, TM_O = 256, TM_COLS = 512;  // U, O: 2 x 64 columns
}  // namespace sf

__global__ void __launch_bounds__(sf::THREADS, 1)
    delta_state_fwd_kernel(const __grid_constant__ StateMaps maps, const float* __restrict__ U0T,
                           float* __restrict__ resid, __nv_bfloat16* __restrict__ o, int L, int H,
                           int NC, unsigned* err) {
    using namespace sf;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BARS);
    uint64_t* full = bars;          // [2]
    uint64_t* u0_ready = bars + 2;  // [2]
    uint64_t* p1 = bars + 4;        // [2]
    uint64_t* p2 = bars + 6;        // [2]
    uint64_t* s_read = bars + 8;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 9);
    volatile uint32_t* s_abort = s_tmem + 1;
    const int h = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long bh = (long long)b * H + h;
    const long long ch0 = bh * NC;
    // residuals: S^T per chunk start [units][NC+1][D][D], then U~ [units][NC][C][D]
    float* st_T = resid != nullptr ? resid + bh * (NC + 1) * D * D : nullptr;
    float* ures = resid != nullptr
                      ? resid + ckpt_state_floats(gridDim.x * (long long)gridDim.y, NC) +
                            ch0 * C * D
                      : nullptr;

    if ((smem_u32(smem) & 1023u) != 0) {  // SW128 boxes need 1 KB alignment
        if (tid == 0) edb_flag_error(err, EDB_DEVERR_DELTA_PIPE);
        return;
    }
    if (warp == 0) {
        tc::tmem_alloc(s_tmem, TM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        *s_abort = 0;
        for (int e = 0; e < 9; ++e) mbar_init(&bars[e], (e >= 2 && e < 4) || e == 8 ? 4 : 1);
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *s_tmem;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int i = (warp & 3) * 32 + lane;  // TMEM lane = value-dim row of S
    if (warp < 4) {  // S = 0
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

    if (warp == 8) {
        // ---------------------------------------------------------- TMA + MMA
        if (lane == 0) {
            auto issue = [&](int c) {
                uint8_t* st = smem + (c & 1) * STAGE_BYTES;
                uint64_t* bar = &full[c & 1];
                const int rc = (int)((ch0 + c) * C), rd = (int)((ch0 + c) * D);
                mbar_arrive_expect_tx(bar, STAGE_BYTES);
                for (int bx = 0; bx < 4; ++bx) {
                    tma_load_2d(st + OFF_W + bx * BOX_C, &maps.Wn, bar, bx * 32, rc);
                    tma_load_2d(st + OFF_Q + bx * BOX_C, &maps.Q, bar, bx * 32, rc);
                }
                for (int bx = 0; bx < 2; ++bx) {
                    tma_load_2d(st + OFF_KT + bx * BOX_D, &maps.KT, bar, bx * 32, rd);
                    tma_load_2d(st + OFF_M + bx * BOX_C, &maps.M, bar, bx * 32, rc);
                }
            };
            prefetch_tmap(&maps.Wn);
            prefetch_tmap(&maps.Q);
            prefetch_tmap(&maps.KT);
            prefetch_tmap(&maps.M);
            int issued = 0, landed = 0, committed = 0, done = 0;
            issue(0);
            issued = 1;
            if (NC > 1) {
                issue(1);
                issued = 2;
            }
            constexpr uint32_t idN64 = idesc_tf32(128, C);
            constexpr uint32_t idN128 = idesc_tf32(128, D);
            for (int c = 0; c < NC; ++c) {
                const int bf = c & 1;
                const uint32_t par = (c >> 1) & 1;
                const uint8_t* st = smem + bf * STAGE_BYTES;
                const uint32_t tU = tmem + TM_U + bf * 64, tO = tmem + TM_O + bf * 64;
                if (!wait(&full[bf], par)) break;
                landed = c + 1;
                if (!wait(&u0_ready[bf], par)) break;
                tc::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk) {
                    mma_tf32_ts(tU, tmem + TM_S + kk * 8, kdesc(st + OFF_W, BOX_C, kk), idN64, 1);
                    mma_tf32_ts(tO, tmem + TM_S + kk * 8, kdesc(st + OFF_Q, BOX_C, kk), idN64,
                                kk > 0);
                }
                tc::commit(&p1[bf]);
                committed = 2 * c + 1;
                if (!wait(&p1[bf], par)) break;
                done = 2 * c + 1;
                if (!wait(s_read, c & 1)) break;
                tc::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < C / 8; ++kk) {
                    mma_tf32_ts(tO, tU + kk * 8, kdesc(st + OFF_M, BOX_C, kk), idN64, 1);
                    mma_tf32_ts(tmem + TM_S, tU + kk * 8, kdesc(st + OFF_KT, BOX_D, kk), idN128,
                                1);
                }
                tc::commit(&p2[bf]);
                committed = 2 * c + 2;
                if (!wait(&p2[bf], par)) break;
                done = 2 * c + 2;
                if (c + 2 < NC) {
                    issue(c + 2);
                    issued = c + 3;
                }
            }
            if (*s_abort) {
                // wait (bounded) for the copies and MMAs still in flight before the
                // shared memory and TMEM they target are released
                for (int cc = landed; cc < issued; ++cc)
                    mbar_wait_bounded(&full[cc & 1], (cc >> 1) & 1, err, EDB_DEVERR_DELTA_PIPE);
                if (committed > done) {
                    const int cc = (committed - 1) >> 1;
                    uint64_t* bar = (committed & 1) ? &p1[cc & 1] : &p2[cc & 1];
                    mbar_wait_bounded(bar, (cc >> 1) & 1, err, EDB_DEVERR_DELTA_PIPE);
                }
            }
        }
    } else if (warp < 4) {
        // ---------------------------------------------------------- S^T residual
        for (int c = 0; c <= NC; ++c) {
            if (c > 0 && !wait(&p2[(c - 1) & 1], ((c - 1) >> 1) & 1)) break;
            if (*s_abort) break;
            tc::fence_after_sync();
            if (st_T != nullptr)
                store_rows_transposed<D>(st_T + (long long)c * D * D + i, tmem + TM_S + lane_base);
            if (c == NC) break;
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_read);
        }
    } else {
        // ---------------------------------------------------------- U0^T in, O / U~ out
        float4 u[16];
        auto load_u0 = [&](int c) {
            const float4* src = reinterpret_cast<const float4*>(U0T + ((ch0 + c) * D + i) * C);
#pragma unroll
            for (int e = 0; e < 16; ++e) u[e] = src[e];
        };
        auto readout = [&](int c) {  // O^T row i -> o[b, cC + t, h, i]; U~^T row i -> U~[c][t][i]
            const int bf = c & 1;
            const int nt = min(C, L - c * C);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t x[32];
                tc::tmem_ld32(tmem + TM_O + bf * 64 + lane_base + half * 32, x);
                tc::tmem_wait_ld();
                __nv_bfloat16* op =
                    o + (((long long)b * L + c * C + half * 32) * H + h) * D + i;
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    if (half * 32 + t < nt) *op = __float2bfloat16(__uint_as_float(x[t]));
                    op += H * D;
                }
            }
            if (ures != nullptr)
                store_rows_transposed<C>(ures + (long long)c * C * D + i,
                                         tmem + TM_U + bf * 64 + lane_base);
        };
        load_u0(0);
        for (int c = 0; c < NC; ++c) {
            const int bf = c & 1;
            // P1(c - 1) was issued, so u0_ready[bf ^ 1] is consumed and the
            // buffer pair bf (last used by chunk c - 2, read out already) is free
            if (c > 0 && !wait(&p1[bf ^ 1], ((c - 1) >> 1) & 1)) break;
            if (*s_abort) break;
            {
                uint32_t r[32];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        r[4 * e] = __float_as_uint(u[8 * half + e].x);
                        r[4 * e + 1] = __float_as_uint(u[8 * half + e].y);
                        r[4 * e + 2] = __float_as_uint(u[8 * half + e].z);
                        r[4 * e + 3] = __float_as_uint(u[8 * half + e].w);
                    }
                    tc::tmem_st32(tmem + TM_U + bf * 64 + lane_base + half * 32, r);
                }
                tc::tmem_wait_st();
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&u0_ready[bf]);
            if (c > 0) {
                if (!wait(&p2[bf ^ 1], ((c - 1) >> 1) & 1)) break;
                tc::fence_after_sync();
                readout(c - 1);
            }
            // the next rows land while P1(c) runs
            if (c + 1 < NC) load_u0(c + 1);
        }
        if (!*s_abort && wait(&p2[(NC - 1) & 1], ((NC - 1) >> 1) & 1)) {
            tc::fence_after_sync();
            readout(NC - 1);
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
// Whether the chunked path serves a call.
bool edb_delta_chunked_ok(int dtype, int beta_per_element, int head_dim) {
    return dtype == EDB_BF16 && !beta_per_element && head_dim == D;
}

size_t edb_delta_chunked_ckpt_bytes(int B, int L, int H) {
    return ckpt_bytes((long long)B * H, (L + C - 1) / C);
}

size_t edb_delta_chunked_fwd_ws(int B, int L, int H) {
    return fwd_scratch_bytes((long long)B * H * ((L + C - 1) / C));
}

int edb_delta_chunked_fwd(const void* q, const void* k, const void* v, const void* beta, void* o,
                          float* resid, int B, int L, int H, void* ws, cudaStream_t st) {
    const int NC = (L + C - 1) / C;
    const long long nch = (long long)B * H * NC;
    if (nch * D > 0x7fffffffLL) return EDB_ERR_UNSUPPORTED;  // TMA row coordinate is int32
    FwdScratch w = carve_fwd(ws, nch);
    cudaError_t e = cudaFuncSetAttribute(delta_prep_fwd_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, prep::SMEM);
    if (e != cudaSuccess) return (int)e;
    delta_prep_fwd_kernel<<<dim3(NC, H, B), prep::THREADS, prep::SMEM, st>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
        (const __nv_bfloat16*)beta, w, L, H, NC, edb::device_error_word());
    if ((e = cudaGetLastError()) != cudaSuccess) return (int)e;
    StateMaps maps;
    int s;
    if ((s = make_box_map(&maps.Wn, w.Wn, nch * C, D, C))) return s;
    if ((s = make_box_map(&maps.Q, w.Q, nch * C, D, C))) return s;
    if ((s = make_box_map(&maps.KT, w.KT, nch * D, C, D))) return s;
    if ((s = make_box_map(&maps.M, w.M, nch * C, C, C))) return s;
    e = cudaFuncSetAttribute(delta_state_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             sf::SMEM);
    if (e != cudaSuccess) return (int)e;
    delta_state_fwd_kernel<<<dim3(H, B), sf::THREADS, sf::SMEM, st>>>(
        maps, w.U0T, resid, (__nv_bfloat16*)o, L, H, NC, edb::device_error_word());
    return edb::status_from_cuda(cudaGetLastError());
}
