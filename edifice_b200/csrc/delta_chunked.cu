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
//   delta_prep_kernel<true> (delta_prep.cuh) one CTA per chunk (all chunks at
//                           once), tcgen05 kind::f16 for K K^T, Q K^T, W and U0
//                           (T_b as a bf16 hi/lo pair), SIMT for the blocked
//                           unit-triangular solve for T; writes -W, Q, K^T, U0^T
//                           and M (f32) to scratch.
//   delta_state_fwd_kernel  one CTA per (b, h), chunks in order, tcgen05
//                           kind::tf32 with every operand K-major.  S lives in
//                           TMEM (lanes = value dim, columns = key dim) as the f32
//                           accumulator and is fed back as the A operand:
//                             [D_U | D_O] = [U0^T | 0] + S [-W; Q]^T   M=128, N=128, K=128
//                             D_O += D_U M^T                M=128, N=64,  K=64
//                             S   += D_U (K^T)^T            M=128, N=128, K=64
//                           -W, Q, K^T, M arrive by TMA (SWIZZLE_128B f32 boxes)
//                           in a 2-stage ring; U0^T rows are stored into TMEM
//                           by the threads.  With a residual buffer it also
//                           stores S^T at every chunk start (and the final S^T)
//                           and each chunk's U~ for the backward.  TF32
//                           operands (10-bit mantissa), f32 accumulation.
//
// GatedDeltaNet (one decay alpha per token and head; fused_scan.ex:2256-2284,
// gated_delta_net.ex:382-394), same kernels with GATED: inside a chunk
// gamma_t = prod_{s<=t} alpha_s, Gamma_ts = gamma_t / gamma_s (s <= t), and
//   A = tril(diag(beta)(K K^T o Gamma), -1),  W = T diag(beta gamma) K,  U0 = T diag(beta) V
//   U~ = U0 - W S_0^T,  O = diag(gamma) Q S_0^T + (tril(Q K^T) o Gamma) U~
//   S_C = gamma_C S_0 + U~^T diag(gamma_C / gamma) K
// (the recurrence S_t = alpha_t S_{t-1} + beta_t (v_t - alpha_t S_{t-1} k_t) k_t^T
// unrolled over the chunk).  The prep folds every gamma into its operands; the
// state kernel scales S by gamma_C between P1 (which needs S_0) and P2.
#include <math.h>

#include "delta_chunked.cuh"
#include "delta_prep.cuh"

using namespace dchunk;

namespace {

// ------------------------------------------------------------------ scratch
struct FwdScratch {
    float* Wn;   // [nch][C][D]  -W
    float* Q;    // [nch][C][D]
    float* KT;   // [nch][D][C]
    float* U0T;  // [nch][D][C]
    float* M;    // [nch][C][C]  tril(Q K^T), diagonal included
    float* gl;   // [nch][C]     gated: in-chunk log-decay cumsum
};

size_t fwd_scratch_bytes(long long nch) {
    return 4 * a256((size_t)nch * C * D * 4) + a256((size_t)nch * C * C * 4) +
           a256((size_t)nch * C * 4);
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
    s.gl = reinterpret_cast<float*>(p + 4 * cd + a256((size_t)nch * C * C * 4));
    return s;
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
//   P1(c): [D_U | D_O][b] = [U0^T | 0] + S [-W; Q]^T      (S read as A from TMEM)
//   P2(c): D_O[b] += D_U[b] M^T,  S += D_U[b] (K^T)^T      (after S^T is read out)
// mbarriers (per buffer where two chunks could otherwise alias one phase):
//   full[s]       TMA stage s landed          u0_ready[b]  U0^T rows in D_U[b]
//   p1[b], p2[b]  tcgen05.commit of P1 / P2   s_read       S^T of this chunk read
namespace sf {
constexpr int THREADS = 288;
// -W and Q share their K slices: box bx of -W (rows 0-63) is followed by box bx of
// Q (rows 64-127), so each 128-byte K slice of the pair is one N = 128 operand
// and P1 is a single product S [-W; Q]^T = [D_U | D_O]
constexpr int OFF_WQ = 0;
constexpr int OFF_KT = OFF_WQ + 8 * BOX_C;
constexpr int OFF_M = OFF_KT + 2 * BOX_D;
constexpr int STAGE_BYTES = OFF_M + 2 * BOX_C;  // 112 KB
constexpr int OFF_BARS = 2 * STAGE_BYTES;
constexpr int SMEM = OFF_BARS + 128;
// TMEM: S, then two buffers of [D_U (64 columns) | D_O (64 columns)]
constexpr int TM_S = 0, TM_U = 128, TM_COLS = 512;
constexpr int TM_BUF = 128, TM_OFF_O = 64;
}  // namespace sf

template <bool GATED>
__global__ void __launch_bounds__(sf::THREADS, 1)
    delta_state_fwd_kernel(const __grid_constant__ StateMaps maps, const float* __restrict__ U0T,
                           const float* __restrict__ gl, float* __restrict__ resid,
                           __nv_bfloat16* __restrict__ o, int L, int H, int NC, unsigned* err) {
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
            auto issue = [&](int c) {
                uint8_t* st = smem + (c & 1) * STAGE_BYTES;
                uint64_t* bar = &full[c & 1];
                const int rc = (int)((ch0 + c) * C), rd = (int)((ch0 + c) * D);
                mbar_arrive_expect_tx(bar, STAGE_BYTES);
                for (int bx = 0; bx < 4; ++bx) {
                    tma_load_2d(st + OFF_WQ + (2 * bx) * BOX_C, &maps.Wn, bar, bx * 32, rc);
                    tma_load_2d(st + OFF_WQ + (2 * bx + 1) * BOX_C, &maps.Q, bar, bx * 32, rc);
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
                const uint32_t tU = tmem + TM_U + bf * TM_BUF, tO = tU + TM_OFF_O;
                if (!wait(&full[bf], par)) break;
                landed = c + 1;
                if (!wait(&u0_ready[bf], par)) break;
                tc::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk) {
                    // [D_U | D_O] += S [-W; Q]^T: D_U holds U0^T, D_O zeros (the
                    // U0 warps store both halves), so every step accumulates
                    mma_tf32_ts(tU, tmem + TM_S + kk * 8, kdesc(st + OFF_WQ, 2 * BOX_C, kk),
                                idN128, 1);
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
            if (c > 0 && !wait_w(&p2[(c - 1) & 1], ((c - 1) >> 1) & 1)) break;
            if (abort_w()) break;
            tc::fence_after_sync();
            // S is read into registers and released (s_read) before its 64 KB of
            // stores are issued, so P2 never waits on the global store queue
            uint32_t x[D / 32][32];
            if (GATED || st_T != nullptr) {
#pragma unroll
                for (int cc = 0; cc < D / 32; ++cc)
                    tc::tmem_ld32(tmem + TM_S + lane_base + cc * 32, x[cc]);
                tc::tmem_wait_ld();
            }
            if (GATED && c < NC) {
                // S <- gamma_C S once P1(c) has read S_0
                const float gC = __expf(gl[(ch0 + c) * C + C - 1]);
                if (!wait_w(&p1[c & 1], (c >> 1) & 1)) break;
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
            if (c < NC) {
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_read);
            }
            if (st_T != nullptr) {
                float* dst = st_T + (long long)c * D * D + i;
#pragma unroll
                for (int cc = 0; cc < D / 32; ++cc)
#pragma unroll
                    for (int e = 0; e < 32; ++e) dst[(cc * 32 + e) * D] = __uint_as_float(x[cc][e]);
            }
            if (c == NC) break;
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
                tc::tmem_ld32(tmem + TM_U + bf * TM_BUF + TM_OFF_O + lane_base + half * 32, x);
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
                                         tmem + TM_U + bf * TM_BUF + lane_base);
        };
        load_u0(0);
        for (int c = 0; c < NC; ++c) {
            const int bf = c & 1;
            // P1(c - 1) was issued, so u0_ready[bf ^ 1] is consumed and the
            // buffer pair bf (last used by chunk c - 2, read out already) is free
            if (c > 0 && !wait_w(&p1[bf ^ 1], ((c - 1) >> 1) & 1)) break;
            if (abort_w()) break;
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
                    tc::tmem_st32(tmem + TM_U + bf * TM_BUF + lane_base + half * 32, r);
                }
                uint32_t z[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) z[e] = 0u;
#pragma unroll
                for (int half = 0; half < 2; ++half)
                    tc::tmem_st32(tmem + TM_U + bf * TM_BUF + TM_OFF_O + lane_base + half * 32, z);
                tc::tmem_wait_st();
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&u0_ready[bf]);
            // the next rows are in flight while P1(c) runs and chunk c - 1 is read out
            if (c + 1 < NC) load_u0(c + 1);
            if (c > 0) {
                if (!wait_w(&p2[bf ^ 1], ((c - 1) >> 1) & 1)) break;
                tc::fence_after_sync();
                readout(c - 1);
            }
        }
        if (!abort_w() && wait_w(&p2[(NC - 1) & 1], ((NC - 1) >> 1) & 1)) {
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

int edb_delta_chunked_fwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* alpha, void* o, float* resid, int B, int L, int H, void* ws,
                          cudaStream_t st) {
    const int NC = (L + C - 1) / C;
    const long long nch = (long long)B * H * NC;
    if (nch * D > 0x7fffffffLL) return EDB_ERR_UNSUPPORTED;  // TMA row coordinate is int32
    FwdScratch w = carve_fwd(ws, nch);
    PrepOut po{};
    po.KT = w.KT;
    po.Q = w.Q;
    po.M = w.M;
    po.Wn = w.Wn;
    po.U0T = w.U0T;
    po.gl = w.gl;
    int s = launch_delta_prep<true>(q, k, v, beta, alpha, po, B, L, H, st);
    if (s != EDB_OK) return s;
    StateMaps maps;
    if ((s = make_box_map(&maps.Wn, w.Wn, nch * C, D, C))) return s;
    if ((s = make_box_map(&maps.Q, w.Q, nch * C, D, C))) return s;
    if ((s = make_box_map(&maps.KT, w.KT, nch * D, C, D))) return s;
    if ((s = make_box_map(&maps.M, w.M, nch * C, C, C))) return s;
    auto kern = alpha != nullptr ? delta_state_fwd_kernel<true> : delta_state_fwd_kernel<false>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sf::SMEM);
    if (e != cudaSuccess) return (int)e;
    kern<<<dim3(H, B), sf::THREADS, sf::SMEM, st>>>(maps, w.U0T, w.gl, resid, (__nv_bfloat16*)o,
                                                     L, H, NC, edb::device_error_word());
    return edb::status_from_cuda(cudaGetLastError());
}
