// delta_prep.cuh -- the per-chunk preparation kernel of the chunked DeltaNet
// path, forward (delta_chunked.cu) and backward (delta_chunked_bwd.cu).
//
// One CTA (128 threads, two per SM) per chunk of C = 64 tokens, all chunks at
// once.  The bf16 rows of K, Q and X (X = V forward, dO backward) are staged
// as bf16 K-major SWIZZLE_128B tiles [C][D]; the products run on tcgen05
// kind::f16 with f32 accumulators in TMEM:
//   G  = K K^T,  Mq = Q K^T                       M=64,  N=64, K=128 (exact: bf16 inputs)
//   W^T = K^T T_b^T  (and U0^T = V^T T_b^T)        M=128, N=64, K=64
// For the last two, K / V are read MN-major from the same tiles (no
// transpose) and T_b = T diag(beta) enters as a pair of bf16 tiles, hi =
// bf16(T_b) and lo = bf16(T_b - hi), so the product carries about 16
// significant bits of T_b.  T = (I + A)^-1, A = tril(diag(beta) G, -1), is
// the blocked SIMT solve between the two groups of products.
// Outputs (f32 scratch, chunk ch of nch):
//   forward   Q [C][D], K^T [D][C], M [C][C] (tril(Q K^T), diagonal kept),
//             -W [C][D], U0^T [D][C]
//   backward  K [C][D], K^T, Q^T, dO^T [D][C], M^T [C][C], T [C][C],
//             G [C][C], -W^T [D][C]
// Rows past L load as zero with beta 0, so their W / U0 rows are zero.
//
// GATED (GatedDeltaNet, one decay alpha per token and head): with the chunk's
// log-decay cumsum g_t = sum_{s<=t} log alpha_s, gamma_t = exp(g_t) and
// Gamma_ts = exp(g_t - g_s) (<= 1 for s <= t, so nothing overflows):
//   A = tril(diag(beta)(K K^T o Gamma), -1),  M = tril(Q K^T) o Gamma,
//   W = T diag(beta gamma) K,  U0 = T diag(beta) V,
// the forward's Q rows are diag(gamma) Q and its K^T copy (diag(gamma_C / gamma) K)^T;
// the backward writes K' = diag(gamma) K rows (Kf), K~ = diag(gamma_C / gamma) K rows
// (Kd), Q^T and (diag(gamma) Q)^T (QdT), (M o Gamma)^T, K K^T o Gamma below the
// diagonal (G) and -W^T with the gamma above.  g goes to gl[nch][C] (both).
// Rows past L take alpha = 1 (log 0), so g_{C-1} = g of the last real token.
#pragma once

#include "delta_chunked.cuh"

namespace dchunk {

namespace prep {
constexpr int THREADS = 128;
constexpr int BOXB = C * 128;  // 8 KB: [C rows][64 bf16]
constexpr int OFF_K = 0;                 // bf16 [C][D]: 2 boxes
constexpr int OFF_Q = OFF_K + 2 * BOXB;
constexpr int OFF_X = OFF_Q + 2 * BOXB;
constexpr int OFF_TH = OFF_X + 2 * BOXB;  // bf16 [C][C]: T_b hi
constexpr int OFF_TL = OFF_TH + BOXB;     //                T_b lo
constexpr int OFF_F = OFF_TL + BOXB;      // f32: Gs [C][PC] | Tm [C][PC] | Ys [768]
constexpr int F_FLOATS = 2 * C * PC + 768;
constexpr int OFF_BS = OFF_F + F_FLOATS * 4;
constexpr int OFF_GL = OFF_BS + C * 4;    // f32 [C]: warp-wise inclusive scans of log alpha
constexpr int OFF_GAM = OFF_GL + C * 4;   // f32 [C]: gamma_t
constexpr int OFF_KAP = OFF_GAM + C * 4;  // f32 [C]: gamma_C / gamma_t
constexpr int OFF_BAR = OFF_KAP + C * 4;
constexpr int SMEM = OFF_BAR + 64;
static_assert(2 * (SMEM + 1024) <= 228 * 1024, "two CTAs per SM");
constexpr int TM_G = 0, TM_M = 64, TM_W = 128, TM_U = 192, TM_COLS = 256;
}  // namespace prep

struct PrepOut {
    float* KT;   // [nch][D][C]  both
    float* Q;    // [nch][C][D]  forward
    float* M;    // [nch][C][C]  forward
    float* Wn;   // [nch][C][D]  forward: -W
    float* U0T;  // [nch][D][C]  forward
    float* Kf;   // [nch][C][D]  backward
    float* XT;   // [nch][D][C]  backward: dO^T
    float* QT;   // [nch][D][C]  backward
    float* MT;   // [nch][C][C]  backward
    float* WnT;  // [nch][D][C]  backward: -W^T
    float* T;    // [nch][C][C]  backward
    float* G;    // [nch][C][C]  backward
    // gated only
    float* Kd;   // [nch][C][D]  backward: diag(gamma_C / gamma) K
    float* QdT;  // [nch][D][C]  backward: (diag(gamma) Q)^T
    float* gl;   // [nch][C]     both: g_t
};

// Byte offset of bf16 columns d8..d8+7 (d8 % 8 == 0) of row t in a [C][D]
// bf16 K-major SW128 tile (boxes of 64 columns).
static __device__ __forceinline__ uint32_t bf_off8(int t, int d8) {
    return (uint32_t)(d8 >> 6) * prep::BOXB + tc::sw128_off(t, (d8 & 63) >> 3);
}

// out[(d8 + e) * C + t] = f32 of tile element (t, d8 + e), times tsc[t] when
// tsc is given: a warp takes 32 consecutive t (8 rows cover the 8 swizzled
// 16-byte slots of one column octet), each store instruction is coalesced over t.
static __device__ __forceinline__ void store_tile_transposed(float* out, const uint8_t* tile,
                                                             const float* tsc = nullptr) {
    for (int idx = threadIdx.x; idx < C * (D / 8); idx += prep::THREADS) {
        const int t = idx % C, d8 = (idx / C) * 8;
        float f[8];
        Vec16<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(tile + bf_off8(t, d8)), f);
        const float sc = tsc != nullptr ? tsc[t] : 1.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) out[(d8 + e) * C + t] = sc * f[e];
    }
}

// g_t of the chunk from the warp-wise scans in gls (warps 0 and 1 each scanned
// 32 tokens).
static __device__ __forceinline__ float gcum(const float* gls, int t) {
    return gls[t] + (t >= 32 ? gls[31] : 0.0f);
}

template <bool FWD, bool GATED>
__global__ void __launch_bounds__(prep::THREADS, 2)
    delta_prep_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                      const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ beta,
                      const __nv_bfloat16* __restrict__ alpha, PrepOut out, int L, int H, int NC,
                      unsigned* err) {
    using namespace prep;
    extern __shared__ __align__(1024) uint8_t smem[];
    float* Gs = reinterpret_cast<float*>(smem + OFF_F);  // [C][PC]
    float* Tm = Gs + C * PC;                            // [C][PC]
    float* Ys = Tm + C * PC;                            // solve scratch
    float* bs = reinterpret_cast<float*>(smem + OFF_BS);
    float* gls = reinterpret_cast<float*>(smem + OFF_GL);
    float* gam = reinterpret_cast<float*>(smem + OFF_GAM);
    float* kap = reinterpret_cast<float*>(smem + OFF_KAP);
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
    if (GATED) {
        // log-decay scan: warps 0 and 1 each scan 32 tokens; gamma and gamma_C / gamma
        if (warp < 2) {
            float lg = tid < nvalid
                           ? logf(__bfloat162float(alpha[((long long)b * L + t0 + tid) * H + h]))
                           : 0.0f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, lg, o);
                if (lane >= o) lg += y;
            }
            gls[tid] = lg;
        }
        __syncthreads();
        if (tid < C) {
            const float gt = gcum(gls, tid), gC = gcum(gls, C - 1);
            gam[tid] = __expf(gt);
            kap[tid] = __expf(gC - gt);
            out.gl[ch * C + tid] = gt;
        }
        __syncthreads();
    }
    // ---- K, Q, X rows -> bf16 tiles; f32 Q (forward) or K (backward) rows to HBM
    {
        constexpr int N = C * (D / 8) / THREADS;
        uint4 rk[N], rq[N], rx[N];
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), d8 = (idx % (D / 8)) * 8;
            const bool ok = t < nvalid;
            const long long off = row0 + t * ts + d8;
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            rk[n] = ok ? *reinterpret_cast<const uint4*>(k + off) : z;
            rq[n] = ok ? *reinterpret_cast<const uint4*>(q + off) : z;
            rx[n] = ok ? *reinterpret_cast<const uint4*>(x + off) : z;
        }
        if (tid < C)
            bs[tid] = tid < nvalid ? __bfloat162float(beta[((long long)b * L + t0 + tid) * H + h])
                                   : 0.0f;
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), d8 = (idx % (D / 8)) * 8;
            const uint32_t o = bf_off8(t, d8);
            *reinterpret_cast<uint4*>(smem + OFF_K + o) = rk[n];
            *reinterpret_cast<uint4*>(smem + OFF_Q + o) = rq[n];
            *reinterpret_cast<uint4*>(smem + OFF_X + o) = rx[n];
            float f[8];
            Vec16<__nv_bfloat16>::unpack(FWD ? rq[n] : rk[n], f);
            float* g = (FWD ? out.Q : out.Kf) + (ch * C + t) * D + d8;
            const float sg = GATED ? gam[t] : 1.0f;  // diag(gamma) Q  or  K' = diag(gamma) K
            st4(g, make_float4(sg * f[0], sg * f[1], sg * f[2], sg * f[3]));
            st4(g + 4, make_float4(sg * f[4], sg * f[5], sg * f[6], sg * f[7]));
            if (GATED && !FWD) {
                const float sk = kap[t];
                float* gd = out.Kd + (ch * C + t) * D + d8;
                st4(gd, make_float4(sk * f[0], sk * f[1], sk * f[2], sk * f[3]));
                st4(gd + 4, make_float4(sk * f[4], sk * f[5], sk * f[6], sk * f[7]));
            }
        }
    }
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_misc[0];
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    if (tid == 0) {
        constexpr uint32_t id64 = tc::idesc_bf16(64, C, 0, 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t ko = (kk >> 2) * BOXB + (kk & 3) * 32;
            const uint64_t kd = tc::sdesc_sw128(smem + OFF_K + ko, 16, 1024);
            tc::mma_bf16_ss(tmem + TM_G, kd, kd, id64, kk > 0);
            tc::mma_bf16_ss(tmem + TM_M, tc::sdesc_sw128(smem + OFF_Q + ko, 16, 1024), kd, id64,
                            kk > 0);
        }
        tc::commit(mbar);
    }
    // ---- transposed f32 copies, while the products run
    store_tile_transposed(out.KT + ch * D * C, smem + OFF_K, GATED && FWD ? kap : nullptr);
    if (!FWD) {
        store_tile_transposed(out.QT + ch * D * C, smem + OFF_Q);
        store_tile_transposed(out.XT + ch * D * C, smem + OFF_X);
        if (GATED) store_tile_transposed(out.QdT + ch * D * C, smem + OFF_Q, gam);
    }
    if (tid == 0 && !mbar_wait_bounded(mbar, 0, err, EDB_DEVERR_DELTA_PIPE)) {
        mbar_wait_bounded(mbar, 0, err, EDB_DEVERR_DELTA_PIPE);
        s_misc[1] = 1;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (!s_misc[1]) {
        // ---- G -> shared (solve input); M -> HBM, masked (forward [t][s],
        // backward transposed [s][t]).  M=64 accumulators: lanes 32w + r
        // (r < 16) hold row 16w + r.
        uint32_t g0[32], g1[32];
        tc::tmem_ld32(tmem + TM_G + lane_base, g0);
        tc::tmem_ld32(tmem + TM_G + lane_base + 32, g1);
        tc::tmem_wait_ld();
        const int t = 16 * warp + lane;
        const float gt = GATED ? gcum(gls, t) : 0.0f;
        // Gamma_ts for s <= t (1 elsewhere, where the masks leave nothing anyway)
        auto gmul = [&](int s) { return GATED && s < t ? __expf(gt - gcum(gls, s)) : 1.0f; };
        if (lane < 16) {
#pragma unroll
            for (int s = 0; s < 32; ++s) {
                Gs[t * PC + s] = __uint_as_float(g0[s]) * gmul(s);
                Gs[t * PC + 32 + s] = __uint_as_float(g1[s]) * gmul(s + 32);
            }
        }
        tc::tmem_ld32(tmem + TM_M + lane_base, g0);
        tc::tmem_ld32(tmem + TM_M + lane_base + 32, g1);
        tc::tmem_wait_ld();
        if (GATED && lane < 16) {
#pragma unroll
            for (int s = 0; s < 32; ++s) {
                g0[s] = __float_as_uint(__uint_as_float(g0[s]) * gmul(s));
                g1[s] = __float_as_uint(__uint_as_float(g1[s]) * gmul(s + 32));
            }
        }
        if (lane < 16) {
            if (FWD) {
                float* mg = out.M + (ch * C + t) * C;
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
            } else {
                float* mt = out.MT + ch * C * C + t;
#pragma unroll
                for (int s = 0; s < 32; ++s) {
                    mt[s * C] = s <= t ? __uint_as_float(g0[s]) : 0.f;
                    mt[(s + 32) * C] = s + 32 <= t ? __uint_as_float(g1[s]) : 0.f;
                }
            }
        }
    }
    __syncthreads();
    if (!s_misc[1]) {
        if (!FWD)
            for (int idx = tid; idx < C * C; idx += THREADS)
                out.G[ch * C * C + idx] = Gs[(idx / C) * PC + idx % C];
        prep_solve<THREADS>(Gs, bs, Ys, Tm);
        // ---- T_b = T diag(beta) as bf16 hi / lo K-major tiles [t][s]; T to HBM.
        // Gated: W takes T diag(beta gamma), in the Q tiles' space (free once M is
        // done) when U0 needs the plain T_b too (forward), else in T_b's place.
        constexpr int OFF_WH = GATED && FWD ? OFF_Q : OFF_TH;
        constexpr int OFF_WL = GATED && FWD ? OFF_Q + BOXB : OFF_TL;
        for (int idx = tid; idx < C * (C / 8); idx += THREADS) {
            const int t = idx / (C / 8), s8 = (idx % (C / 8)) * 8;
            float hi[8], lo[8];
            const uint32_t o = tc::sw128_off(t, s8 >> 3);
            if (GATED) {
                float wh[8], wl[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float v = Tm[t * PC + s8 + e] * bs[s8 + e] * gam[s8 + e];
                    wh[e] = __bfloat162float(__float2bfloat16(v));
                    wl[e] = v - wh[e];
                }
                *reinterpret_cast<uint4*>(smem + OFF_WH + o) = Vec16<__nv_bfloat16>::pack(wh);
                *reinterpret_cast<uint4*>(smem + OFF_WL + o) = Vec16<__nv_bfloat16>::pack(wl);
            }
            if (!GATED || FWD) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float v = Tm[t * PC + s8 + e] * bs[s8 + e];
                    hi[e] = __bfloat162float(__float2bfloat16(v));
                    lo[e] = v - hi[e];
                }
                *reinterpret_cast<uint4*>(smem + OFF_TH + o) = Vec16<__nv_bfloat16>::pack(hi);
                *reinterpret_cast<uint4*>(smem + OFF_TL + o) = Vec16<__nv_bfloat16>::pack(lo);
            }
            if (!FWD) {
                float* tg = out.T + (ch * C + t) * C + s8;
                st4(tg, make_float4(Tm[t * PC + s8], Tm[t * PC + s8 + 1], Tm[t * PC + s8 + 2],
                                    Tm[t * PC + s8 + 3]));
                st4(tg + 4, make_float4(Tm[t * PC + s8 + 4], Tm[t * PC + s8 + 5],
                                        Tm[t * PC + s8 + 6], Tm[t * PC + s8 + 7]));
            }
        }
        fence_proxy_async();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (tid == 0) {
            // W^T = K^T T_b^T (and U0^T = V^T T_b^T): A MN-major from the row tile
            constexpr uint32_t id128 = tc::idesc_bf16(128, C, 1, 0);
#pragma unroll
            for (int kk = 0; kk < C / 16; ++kk) {
                const uint64_t th = tc::sdesc_sw128(smem + OFF_TH + kk * 32, 16, 1024);
                const uint64_t tl = tc::sdesc_sw128(smem + OFF_TL + kk * 32, 16, 1024);
                const uint64_t wh = tc::sdesc_sw128(smem + OFF_WH + kk * 32, 16, 1024);
                const uint64_t wl = tc::sdesc_sw128(smem + OFF_WL + kk * 32, 16, 1024);
                const uint64_t ka = tc::sdesc_sw128(smem + OFF_K + kk * 2048, BOXB, 1024);
                tc::mma_bf16_ss(tmem + TM_W, ka, wh, id128, kk > 0);
                tc::mma_bf16_ss(tmem + TM_W, ka, wl, id128, 1);
                if (FWD) {
                    const uint64_t va = tc::sdesc_sw128(smem + OFF_X + kk * 2048, BOXB, 1024);
                    tc::mma_bf16_ss(tmem + TM_U, va, th, id128, kk > 0);
                    tc::mma_bf16_ss(tmem + TM_U, va, tl, id128, 1);
                }
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
            // TMEM lane j = column j of W: -W[t][j] (forward, coalesced over j)
            // or -W^T[j][t] (backward, rows); U0^T[j][t]
            const int j = tid;
            if (FWD) {
                store_rows_transposed<C>(out.Wn + ch * C * D + j, tmem + TM_W + lane_base, -1.0f);
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t xw[32];
                tc::tmem_ld32(tmem + (FWD ? TM_U : TM_W) + lane_base + half * 32, xw);
                tc::tmem_wait_ld();
                const float sc = FWD ? 1.0f : -1.0f;
                float* dst = (FWD ? out.U0T : out.WnT) + (ch * D + j) * C + half * 32;
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                    st4(dst + e, make_float4(sc * __uint_as_float(xw[e]), sc * __uint_as_float(xw[e + 1]),
                                             sc * __uint_as_float(xw[e + 2]),
                                             sc * __uint_as_float(xw[e + 3])));
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

// Launches the kernel over every chunk (gated when alpha is not null).  Returns
// an edb status.
template <bool FWD, bool GATED>
inline int launch_delta_prep_t(const void* q, const void* k, const void* x, const void* beta,
                               const void* alpha, const PrepOut& out, int B, int L, int H,
                               cudaStream_t st) {
    const int NC = (L + C - 1) / C;
    cudaError_t e = cudaFuncSetAttribute(delta_prep_kernel<FWD, GATED>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, prep::SMEM);
    if (e != cudaSuccess) return (int)e;
    delta_prep_kernel<FWD, GATED><<<dim3(NC, H, B), prep::THREADS, prep::SMEM, st>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)x,
        (const __nv_bfloat16*)beta, (const __nv_bfloat16*)alpha, out, L, H, NC,
        edb::device_error_word());
    return edb::status_from_cuda(cudaGetLastError());
}

template <bool FWD>
inline int launch_delta_prep(const void* q, const void* k, const void* x, const void* beta,
                             const void* alpha, const PrepOut& out, int B, int L, int H,
                             cudaStream_t st) {
    return alpha != nullptr
               ? launch_delta_prep_t<FWD, true>(q, k, x, beta, alpha, out, B, L, H, st)
               : launch_delta_prep_t<FWD, false>(q, k, x, beta, nullptr, out, B, L, H, st);
}

}  // namespace dchunk
