// delta_chunked_post.cu -- last stage of the chunked DeltaNet backward: every
// per-chunk product and the final dQ, dK, dV, dbeta, in one kernel.
//
// Inputs per chunk: the forward's residuals S_0^T and U~, the state pass's
// dS_C^T and dU~ (and dU~^T), the prep's K (row and transposed f32 copies),
// Q^T, T and K K^T, plus dO, v, beta (bf16).  Products, all on tcgen05
// kind::tf32 with f32 accumulators in TMEM (one CTA of 256 threads per chunk):
//   dQa^T = (dO S_0)^T, dW^T = -(dU~ S_0)^T, dK1^T = (U~ dS_C)^T   M=128, N=64, K=128
//   dM    = tril(dO U~^T)                                         M=64,  N=64, K=128
//   dT_b  = dW K^T + dU~ V^T                                      M=64,  N=64, K=2x128
//   X' = T^T dT_b,  dbeta_s = X'[s][s] (= sum_t dT_b[t][s] T[t][s])
//   dA = -X' T_b^T (strictly lower; = -(T^T dT) T^T with dT = dT_b diag(beta)),
//   dbeta_t += sum_{s<t} dA[t][s] (K K^T)[t][s]
//   E = dG + dG^T,  dG = diag(beta) dA                             SIMT (64 x 64 x 64)
//   dQ^T = dQa^T + K^T dM^T                                       M=128, N=64, K=64
//   dV^T = dU~^T T_b                                              M=128, N=64, K=64
//   dK^T = dK1^T + Q^T dM + dW^T T_b + K^T E                      M=128, N=64, K=3x64
// dQa, dK1 accumulate in place into the dQ / dK accumulators, dW^T is read
// back from TMEM as the A operand of its product, and dM goes from TMEM
// straight into the B tiles, so none of them reaches HBM.  Every shared-memory
// operand is a K-major f32 SWIZZLE_128B tile; the tiles of the later products
// load (TMA) into the space of the first products' operands while the
// threads work.
//
// GATED (GatedDeltaNet): the prep hands over K' = diag(gamma) K rows (Kf),
// K K^T o Gamma (G), (M o Gamma)^T and g; the same products then give
// dQa~ = dO S_0 and dK~ = U~ dS_C unscaled, and three more accumulators keep
// the parts of dQ and dK whose row scale differs:
//   dQ = gamma (.) dQa~ + dM~ K                         (dM~ = dM o Gamma)
//   dK = dM~^T Q + E K + (gamma_C/gamma) (.) dK~ + gamma (.) T_b^T dW
// with E = dG~ + dG~^T, dG~ = (diag(beta) dA) o Gamma.  The log-decay gradient dg
// gathers in shared memory (row and column sums of dM o M and dA o A, the row
// dots with q and k at the read-out, gamma_C <dS_C, S_0> from the phase-A tiles)
// and dalpha_s = (sum_{t>=s} dg_t) / alpha_s.
#include <math.h>

#include "delta_chunked.cuh"

using namespace dchunk;

namespace {

constexpr int THREADS = 256;
constexpr int R_BYTES = 4 * BOX_D;  // 64 KB
// Shared memory, in the order the regions are used:
//   R0  S_0^T [D][D]                  -> K^T [D][C] | Q^T [D][C]
//   R1  dS_C^T [D][D]                 -> dW [C][D] | dU~^T [D][C]; B tiles T_b^T | E in the dW half
//   R2  U~ [C][D]                     -> K [C][D]  -> chain scratch (with R3)
//   R3  dU~ [C][D]
//   R4  dO [C][D] (threads, from bf16) -> V [C][D] (threads) -> B tiles dM | dM^T
constexpr int OFF_R0 = 0, OFF_R1 = OFF_R0 + R_BYTES, OFF_R2 = OFF_R1 + R_BYTES;
constexpr int OFF_R3 = OFF_R2 + 4 * BOX_C, OFF_R4 = OFF_R3 + 4 * BOX_C;
constexpr int OFF_KT = OFF_R0, OFF_QT = OFF_R0 + 2 * BOX_D;
constexpr int OFF_DW = OFF_R1, OFF_DUT = OFF_R1 + 2 * BOX_D;
constexpr int OFF_TBT = OFF_R1, OFF_E = OFF_R1 + 2 * BOX_C;
constexpr int OFF_DM = OFF_R4, OFF_DMT = OFF_R4 + 2 * BOX_C;
constexpr int OFF_BS = OFF_R4 + 4 * BOX_C;  // beta [C]
constexpr int OFF_GS = OFF_BS + C * 4;      // gated: g [C] in log2 units
constexpr int OFF_GAM = OFF_GS + C * 4;     // gated: gamma [C]
// gated: dg partials per warp [THREADS / 32][C], summed in a fixed order at the end
// (no atomics: the gradient is the same bits every run)
constexpr int OFF_DG = OFF_GAM + C * 4;
constexpr int OFF_BAR = OFF_DG + (THREADS / 32) * C * 4;
constexpr int SMEM = OFF_BAR + 64;
static_assert(SMEM <= 227 * 1024, "fits the per-CTA shared-memory limit");
constexpr int PHASE_A_TX = 8 * BOX_D + 8 * BOX_C;  // S_0^T, dS_C^T, U~, dU~
constexpr int TM_Q = 0, TM_W = 64, TM_K = 128, TM_M = 192, TM_DTB = 256, TM_V = 320,
              TM_COLS = 512;
// gated: dM~ K (dQ), dM~^T Q + E K (dK) and T_b^T dW (dK, in dM's columns once read)
constexpr int TM_Q2 = 384, TM_KB = 448, TM_KW = TM_M;
// gated read-out: per-(token, column) dg partials [C][DGP] in the chain scratch
constexpr int DGP = D + 4;
static_assert(C * DGP * 4 <= 8 * BOX_C, "dg partials fit R2-R3");
// SIMT scratch of the C x C chain (floats, in R2..R3): three [C][PS] arrays
// and one [C]
constexpr int PS = C + 4;
static_assert((3 * C * PS + C) * 4 <= 8 * BOX_C, "chain scratch fits R2-R3");

struct PostMaps {
    CUtensorMap S0T, dSCT, Ut, dU;  // phase A
    CUtensorMap Kf;                 // dT_b
    CUtensorMap KT, QT, dUT;        // last products
};

static __device__ __forceinline__ float4 f4(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}
static __device__ __forceinline__ void st_f32(uint8_t* base, uint32_t off, float v) {
    *reinterpret_cast<float*>(base + off) = v;
}

template <bool GATED>
__global__ void __launch_bounds__(THREADS, 1)
    delta_post_kernel(const __grid_constant__ PostMaps maps, const __nv_bfloat16* __restrict__ dO,
                      const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ beta,
                      const __nv_bfloat16* __restrict__ alpha, const float* __restrict__ Tg,
                      const float* __restrict__ Gg, const float* __restrict__ MTg,
                      const float* __restrict__ glg, __nv_bfloat16* __restrict__ gq,
                      __nv_bfloat16* __restrict__ gk, __nv_bfloat16* __restrict__ gv,
                      __nv_bfloat16* __restrict__ gbeta, __nv_bfloat16* __restrict__ galpha, int L,
                      int H, int NC, unsigned* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    float* sc = reinterpret_cast<float*>(smem + OFF_R2);
    float* bs = reinterpret_cast<float*>(smem + OFF_BS);
    float* gs = reinterpret_cast<float*>(smem + OFF_GS);
    float* gam_s = reinterpret_cast<float*>(smem + OFF_GAM);
    float* dgw = reinterpret_cast<float*>(smem + OFF_DG);
    uint64_t* bar_ld = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // [3] TMA groups
    uint64_t* bar_mma = bar_ld + 3;
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bar_mma + 1);  // [0] tmem, [1] abort
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long bh = (long long)b * H + h;
    const long long ch = bh * NC + c;
    const int t0 = c * C, nvalid = min(C, L - t0);
    const long long ts = (long long)H * D;
    const long long row0 = (((long long)b * L + t0) * H + h) * D;
    int ld_issued = 0, ld_landed = 0;  // bit g: TMA group g (thread 0)

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
        mbar_arrive_expect_tx(&bar_ld[0], PHASE_A_TX);
        const int rs = (int)((bh * (NC + 1) + c) * D), rd = (int)(ch * D), rc = (int)(ch * C);
        for (int bx = 0; bx < 4; ++bx) {
            tma_load_2d(smem + OFF_R0 + bx * BOX_D, &maps.S0T, &bar_ld[0], bx * 32, rs);
            tma_load_2d(smem + OFF_R1 + bx * BOX_D, &maps.dSCT, &bar_ld[0], bx * 32, rd);
            tma_load_2d(smem + OFF_R2 + bx * BOX_C, &maps.Ut, &bar_ld[0], bx * 32, rc);
            tma_load_2d(smem + OFF_R3 + bx * BOX_C, &maps.dU, &bar_ld[0], bx * 32, rc);
        }
        ld_issued = 1;
    }
    // dO rows (bf16) -> f32 K-major tile in R4; V rows and T held in registers
    constexpr int NR = C * (D / 8) / THREADS;
    uint4 rv[NR];
    {
        uint4 ro[NR];
#pragma unroll
        for (int n = 0; n < NR; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
            const bool ok = t < nvalid;
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            ro[n] = ok ? *reinterpret_cast<const uint4*>(dO + row0 + t * ts + j8) : z;
            rv[n] = ok ? *reinterpret_cast<const uint4*>(v + row0 + t * ts + j8) : z;
        }
#pragma unroll
        for (int n = 0; n < NR; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
            float f[8];
            Vec16<__nv_bfloat16>::unpack(ro[n], f);
            st4(reinterpret_cast<float*>(smem + OFF_R4 + kmaj_off4(t, j8, C)), make_float4(f[0], f[1], f[2], f[3]));
            st4(reinterpret_cast<float*>(smem + OFF_R4 + kmaj_off4(t, j8 + 4, C)), make_float4(f[4], f[5], f[6], f[7]));
        }
    }
    if (tid < C)
        bs[tid] = tid < nvalid ? __bfloat162float(beta[((long long)b * L + t0 + tid) * H + h])
                               : 0.0f;
    if (GATED) {
        if (tid < C) {
            // log2 units: every decay ratio below is one ex2
            const float g2 = glg[ch * C + tid] * 1.4426950408889634f;
            gs[tid] = g2;
            gam_s[tid] = tc::ex2(g2);
        }
        for (int i = tid; i < (THREADS / 32) * C; i += THREADS) dgw[i] = 0.0f;
    }
    constexpr int NT = C * C / 4 / THREADS;
    float4 tv[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) tv[n] = f4(Tg + ch * C * C + 4 * (tid + n * THREADS));
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_misc[0];
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int hf = warp >> 2;  // column half of an M=128 accumulator this warp reads

    // ---- phase A: the products with S_0 and dS_C; then K, K^T, Q^T, dU~^T load
    // into the freed space
    if (tid == 0) {
        bool ok = mbar_wait_bounded(&bar_ld[0], 0, err, EDB_DEVERR_DELTA_PIPE);
        if (ok) {
            ld_landed = 1;
            tc::fence_after_sync();
            constexpr uint32_t id128 = idesc_tf32(128, C), id64 = idesc_tf32(64, C);
#pragma unroll
            for (int kk = 0; kk < D / 8; ++kk) {
                const uint64_t s0 = kdesc(smem + OFF_R0, BOX_D, kk);
                const uint64_t dof = kdesc(smem + OFF_R4, BOX_C, kk);
                const uint64_t u = kdesc(smem + OFF_R2, BOX_C, kk);
                mma_tf32_ss(tmem + TM_Q, s0, dof, id128, kk > 0);
                mma_tf32_ss(tmem + TM_W, s0, kdesc(smem + OFF_R3, BOX_C, kk), id128, kk > 0);
                mma_tf32_ss(tmem + TM_K, kdesc(smem + OFF_R1, BOX_D, kk), u, id128, kk > 0);
                mma_tf32_ss(tmem + TM_M, dof, u, id64, kk > 0);
            }
            tc::commit(bar_mma);
            if (!mbar_wait_bounded(bar_mma, 0, err, EDB_DEVERR_DELTA_PIPE)) {
                mbar_wait_bounded(bar_mma, 0, err, EDB_DEVERR_DELTA_PIPE);
                ok = false;
            }
        }
        if (!ok) s_misc[1] = 1;
    }
    if (GATED) {
        // dg_{C-1} += gamma_C <dS_C, S_0>: the two phase-A tiles share one
        // (swizzled) layout, so the dot runs over their bytes in order.  Warps
        // 1-7, while warp 0's lane 0 waits on the products.
        float acc = 0.0f;
        if (warp > 0) {
            if (mbar_wait_bounded(&bar_ld[0], 0, err, EDB_DEVERR_DELTA_PIPE)) {
                const float4* a4 = reinterpret_cast<const float4*>(smem + OFF_R0);
                const float4* b4 = reinterpret_cast<const float4*>(smem + OFF_R1);
#pragma unroll 4
                for (int i = tid - 32; i < R_BYTES / 16; i += THREADS - 32) acc = dot4(a4[i], b4[i], acc);
            } else {
                s_misc[1] = 1;
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0 && warp > 0) dgw[warp * C + C - 1] += gam_s[C - 1] * acc;
        __syncthreads();  // the phase-A tiles are read: their space takes the next loads
    }
    if (tid == 0) {
        if (!s_misc[1]) {
            const int rd = (int)(ch * D), rc = (int)(ch * C);
            mbar_arrive_expect_tx(&bar_ld[1], 4 * BOX_C);
            for (int bx = 0; bx < 4; ++bx)
                tma_load_2d(smem + OFF_R2 + bx * BOX_C, &maps.Kf, &bar_ld[1], bx * 32, rc);
            mbar_arrive_expect_tx(&bar_ld[2], 6 * BOX_D);
            for (int bx = 0; bx < 2; ++bx) {
                tma_load_2d(smem + OFF_KT + bx * BOX_D, &maps.KT, &bar_ld[2], bx * 32, rd);
                tma_load_2d(smem + OFF_QT + bx * BOX_D, &maps.QT, &bar_ld[2], bx * 32, rd);
                tma_load_2d(smem + OFF_DUT + bx * BOX_D, &maps.dUT, &bar_ld[2], bx * 32, rd);
            }
            ld_issued = 7;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const bool aborted = s_misc[1] != 0;
    if (!aborted) {
        // dW = -(dU~ S_0): TMEM lane j holds column j for tokens [32 hf, 32 hf + 32).
        // Negated in TMEM (the dW^T operand of dK) and stored as the dW row tile.
        const int j = (warp & 3) * 32 + lane;
        uint32_t x[32];
        tc::tmem_ld32(tmem + TM_W + lane_base + hf * 32, x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            x[e] ^= 0x80000000u;
            st_f32(smem + OFF_DW, kmaj_off4(hf * 32 + e, j & ~3, C) + (j & 3) * 4,
                   __uint_as_float(x[e]));
        }
        tc::tmem_st32(tmem + TM_W + lane_base + hf * 32, x);
        tc::tmem_wait_st();
        // V rows -> f32 K-major tile in R4 (dO is no longer needed)
#pragma unroll
        for (int n = 0; n < NR; ++n) {
            const int idx = tid + n * THREADS, t = idx / (D / 8), j8 = (idx % (D / 8)) * 8;
            float f[8];
            Vec16<__nv_bfloat16>::unpack(rv[n], f);
            st4(reinterpret_cast<float*>(smem + OFF_R4 + kmaj_off4(t, j8, C)), make_float4(f[0], f[1], f[2], f[3]));
            st4(reinterpret_cast<float*>(smem + OFF_R4 + kmaj_off4(t, j8 + 4, C)), make_float4(f[4], f[5], f[6], f[7]));
        }
    }
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // ---- dT_b = dW K^T + dU~ V^T  (M = 64)
    if (tid == 0 && !aborted) {
        bool ok = mbar_wait_bounded(&bar_ld[1], 0, err, EDB_DEVERR_DELTA_PIPE);
        if (ok) {
            ld_landed |= 2;
            tc::fence_after_sync();
            constexpr uint32_t id64 = idesc_tf32(64, C);
#pragma unroll
            for (int kk = 0; kk < D / 8; ++kk) {
                mma_tf32_ss(tmem + TM_DTB, kdesc(smem + OFF_DW, BOX_C, kk),
                            kdesc(smem + OFF_R2, BOX_C, kk), id64, kk > 0);
                mma_tf32_ss(tmem + TM_DTB, kdesc(smem + OFF_R3, BOX_C, kk),
                            kdesc(smem + OFF_R4, BOX_C, kk), id64, 1);
            }
            tc::commit(bar_mma);
            if (!mbar_wait_bounded(bar_mma, 1, err, EDB_DEVERR_DELTA_PIPE)) {
                mbar_wait_bounded(bar_mma, 1, err, EDB_DEVERR_DELTA_PIPE);
                ok = false;
            }
        }
        if (!ok) s_misc[1] = 1;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const bool aborted2 = s_misc[1] != 0;
    if (!aborted2) {
        // ---- the C x C chain.  Thread (a, b) = (tid / 16, tid % 16) owns rows
        // 4a..4a+3 and columns 4b..4b+3 of each 64 x 64 product; row-major f32
        // scratch with rows of PS floats (float4 aligned), products by float4
        // loads and packed f32x2 FMAs over the triangular ranges only.
        float* Ts = sc;               // T [t][s]; then X'^T [t'][s]
        float* Ds = sc + C * PS;      // dT_b [t][t']; then dA [t][s]
        float* Tb = sc + 2 * C * PS;  // T_b^T [s][t] = T[t][s] beta_s
        float* dbT = sc + 3 * C * PS; // [C]: sum_t dT_b[t][s] T[t][s]
        const int a = tid >> 4, bq = tid & 15;
        if (warp < 4) {
            // dT_b and dM out of TMEM (M = 64: lanes 32w + r, r < 16, hold row 16w + r);
            // dM into the B tiles dM [t][s] and dM^T [s][t]
            uint32_t x0[32], x1[32];
            tc::tmem_ld32(tmem + TM_DTB + lane_base, x0);
            tc::tmem_ld32(tmem + TM_DTB + lane_base + 32, x1);
            tc::tmem_wait_ld();
            const int t = 16 * warp + lane;
            if (lane < 16) {
#pragma unroll
                for (int s4 = 0; s4 < 32; s4 += 4) {
                    st4(Ds + t * PS + s4, make_float4(__uint_as_float(x0[s4]), __uint_as_float(x0[s4 + 1]),
                                                      __uint_as_float(x0[s4 + 2]), __uint_as_float(x0[s4 + 3])));
                    st4(Ds + t * PS + 32 + s4,
                        make_float4(__uint_as_float(x1[s4]), __uint_as_float(x1[s4 + 1]),
                                    __uint_as_float(x1[s4 + 2]), __uint_as_float(x1[s4 + 3])));
                }
            }
            tc::tmem_ld32(tmem + TM_M + lane_base, x0);
            tc::tmem_ld32(tmem + TM_M + lane_base + 32, x1);
            tc::tmem_wait_ld();
            if (lane < 16) {
#pragma unroll
                for (int s4 = 0; s4 < C; s4 += 4) {
                    float m[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int s = s4 + e;
                        m[e] = s <= t ? __uint_as_float(s < 32 ? x0[s] : x1[s - 32]) : 0.0f;
                        if (!GATED)
                            st_f32(smem + OFF_DMT, kmaj_off4(s, t & ~3, C) + (t & 3) * 4, m[e]);
                    }
                    st4(reinterpret_cast<float*>(smem + OFF_DM + kmaj_off4(t, s4, C)),
                        make_float4(m[0], m[1], m[2], m[3]));
                }
            }
        }
        // T rows; T_b^T (scratch and the K-major B tile [s][t])
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int e0 = 4 * (tid + n * THREADS), t = e0 / C, s0 = e0 % C;
            st4(Ts + t * PS + s0, tv[n]);
            const float tvv[4] = {tv[n].x, tv[n].y, tv[n].z, tv[n].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float tb = tvv[e] * bs[s0 + e];
                Tb[(s0 + e) * PS + t] = tb;
                st_f32(smem + OFF_TBT, kmaj_off4(s0 + e, t & ~3, C) + (t & 3) * 4, tb);
            }
        }
        // gated: M[4a + r][4bq + cc] = (M o Gamma)^T[4bq + cc][4a + r], in flight
        // across the barrier
        float4 mt4[GATED ? 4 : 1];
        if constexpr (GATED) {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) mt4[cc] = f4(MTg + (ch * C + 4 * bq + cc) * C + 4 * a);
        }
        __syncthreads();
        if constexpr (GATED) {
            // this thread's 4 x 4 block of dM (raw, masked): dM~ = dM o Gamma into both
            // B tiles; dg_t += rowsum(dM o M), dg_s -= colsum(dM o M)
            float dmv[4][4], rs[4], cs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float4 x = ld4(reinterpret_cast<const float*>(smem + OFF_DM + kmaj_off4(4 * a + r, 4 * bq, C)));
                dmv[r][0] = x.x, dmv[r][1] = x.y, dmv[r][2] = x.z, dmv[r][3] = x.w;
                const float mr[4] = {r == 0 ? mt4[0].x : r == 1 ? mt4[0].y : r == 2 ? mt4[0].z : mt4[0].w,
                                     r == 0 ? mt4[1].x : r == 1 ? mt4[1].y : r == 2 ? mt4[1].z : mt4[1].w,
                                     r == 0 ? mt4[2].x : r == 1 ? mt4[2].y : r == 2 ? mt4[2].z : mt4[2].w,
                                     r == 0 ? mt4[3].x : r == 1 ? mt4[3].y : r == 2 ? mt4[3].z : mt4[3].w};
                const int t = 4 * a + r;
                rs[r] = 0.0f;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const float pr = dmv[r][cc] * mr[cc];
                    rs[r] += pr;
                    cs[cc] += pr;
                    const int s2 = 4 * bq + cc;
                    dmv[r][cc] = s2 <= t ? dmv[r][cc] * tc::ex2(gs[t] - gs[s2]) : 0.0f;
                }
                st4(reinterpret_cast<float*>(smem + OFF_DM + kmaj_off4(t, 4 * bq, C)),
                    make_float4(dmv[r][0], dmv[r][1], dmv[r][2], dmv[r][3]));
            }
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
                st4(reinterpret_cast<float*>(smem + OFF_DMT + kmaj_off4(4 * bq + cc, 4 * a, C)),
                    make_float4(dmv[0][cc], dmv[1][cc], dmv[2][cc], dmv[3][cc]));
#pragma unroll
            for (int r = 0; r < 4; ++r) {
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], o);
            }
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) cs[cc] += __shfl_xor_sync(0xffffffffu, cs[cc], 16);
            // this warp's row of partials: column sums, then (other lanes, maybe the
            // same entries) row sums
            if (lane < 16) {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) dgw[warp * C + 4 * bq + cc] -= cs[cc];
            }
            __syncwarp();
            if (bq == 0) {
#pragma unroll
                for (int r = 0; r < 4; ++r) dgw[warp * C + 4 * a + r] += rs[r];
            }
        }
        float2 acc[4][2];
        {
            // X' = T^T dT_b (T[t][s] = 0 for t < s): the rows of block a need t in
            // [4a, 64), so warp w takes row blocks w and 15 - w (64 - 4w + 4 + 4w = 68
            // steps in all, the same for every warp) and its half-warps each walk half
            // of both ranges; one xor-16 round adds the halves.  Half 0 then owns
            // block w, half 1 block 15 - w.  The diagonal of X' is dbeta's T_b term.
            const int hh = lane >> 4;
            const int aA = warp, aB = 15 - warp;
            const int mA = 2 * aA + C / 2, mB = 2 * aB + C / 2;  // midpoints of [4a, 64)
            float2 xa[4][2], xb[4][2];
#pragma unroll
            for (int r = 0; r < 4; ++r)
                xa[r][0] = xa[r][1] = xb[r][0] = xb[r][1] = make_float2(0.0f, 0.0f);
            auto walk = [&](int blk, int t0, int t1, float2 (&x)[4][2]) {
                for (int t = t0; t < t1; ++t) {
                    const float4 tt = ld4(Ts + t * PS + 4 * blk), dd = ld4(Ds + t * PS + 4 * bq);
                    const float2 d01 = make_float2(dd.x, dd.y), d23 = make_float2(dd.z, dd.w);
                    const float tr[4] = {tt.x, tt.y, tt.z, tt.w};
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        x[r][0] = fma2(dup2(tr[r]), d01, x[r][0]);
                        x[r][1] = fma2(dup2(tr[r]), d23, x[r][1]);
                    }
                }
            };
            walk(aA, hh ? mA : 4 * aA, hh ? C : mA, xa);
            walk(aB, hh ? mB : 4 * aB, hh ? C : mB, xb);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    xa[r][k].x += __shfl_xor_sync(0xffffffffu, xa[r][k].x, 16);
                    xa[r][k].y += __shfl_xor_sync(0xffffffffu, xa[r][k].y, 16);
                    xb[r][k].x += __shfl_xor_sync(0xffffffffu, xb[r][k].x, 16);
                    xb[r][k].y += __shfl_xor_sync(0xffffffffu, xb[r][k].y, 16);
                    acc[r][k] = hh ? xb[r][k] : xa[r][k];
                }
        }
        const int ax = lane >> 4 ? 15 - warp : warp;  // row block of this thread's X'
        if (ax == bq) {
            dbT[4 * ax] = acc[0][0].x;
            dbT[4 * ax + 1] = acc[1][0].y;
            dbT[4 * ax + 2] = acc[2][1].x;
            dbT[4 * ax + 3] = acc[3][1].y;
        }
        __syncthreads();  // T is no longer read: X'^T goes in its place
        st4(Ts + (4 * bq) * PS + 4 * ax, make_float4(acc[0][0].x, acc[1][0].x, acc[2][0].x, acc[3][0].x));
        st4(Ts + (4 * bq + 1) * PS + 4 * ax, make_float4(acc[0][0].y, acc[1][0].y, acc[2][0].y, acc[3][0].y));
        st4(Ts + (4 * bq + 2) * PS + 4 * ax, make_float4(acc[0][1].x, acc[1][1].x, acc[2][1].x, acc[3][1].x));
        st4(Ts + (4 * bq + 3) * PS + 4 * ax, make_float4(acc[0][1].y, acc[1][1].y, acc[2][1].y, acc[3][1].y));
        __syncthreads();
        // this thread's 4 x 4 block of K K^T (o Gamma, gated), in flight across dA
        float4 g4[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) g4[r] = f4(Gg + (ch * C + 4 * a + r) * C + 4 * bq);
        {
            // dA = -X' T_b^T, strictly lower (T_b[col][s] = 0 for s > col): block
            // (a, bq) is nonzero for bq <= a only and sums s in [0, 4 bq + 4).  Balanced
            // as X' above (warp w: row blocks w and 15 - w, half-warps split each range),
            // then masked, negated and written over dT_b (no longer read), from where
            // every thread takes back its own (a, bq) block.
            const int hh = lane >> 4;
            const int aA = warp, aB = 15 - warp;
            const int n = 4 * bq + 4, mid = 2 * bq + 2;
            float2 ya[4][2], yb[4][2];
#pragma unroll
            for (int r = 0; r < 4; ++r)
                ya[r][0] = ya[r][1] = yb[r][0] = yb[r][1] = make_float2(0.0f, 0.0f);
            auto walk = [&](int blk, float2 (&y)[4][2]) {
                if (bq > blk) return;
                for (int s2 = hh ? mid : 0; s2 < (hh ? n : mid); ++s2) {
                    const float4 xv = ld4(Ts + s2 * PS + 4 * blk), tb = ld4(Tb + s2 * PS + 4 * bq);
                    const float2 t01 = make_float2(tb.x, tb.y), t23 = make_float2(tb.z, tb.w);
                    const float xr[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        y[r][0] = fma2(dup2(xr[r]), t01, y[r][0]);
                        y[r][1] = fma2(dup2(xr[r]), t23, y[r][1]);
                    }
                }
            };
            walk(aA, ya);
            walk(aB, yb);
            const int ax = hh ? aB : aA;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                float v4[4];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    ya[r][k].x += __shfl_xor_sync(0xffffffffu, ya[r][k].x, 16);
                    ya[r][k].y += __shfl_xor_sync(0xffffffffu, ya[r][k].y, 16);
                    yb[r][k].x += __shfl_xor_sync(0xffffffffu, yb[r][k].x, 16);
                    yb[r][k].y += __shfl_xor_sync(0xffffffffu, yb[r][k].y, 16);
                    const float2 y2 = hh ? yb[r][k] : ya[r][k];
                    v4[2 * k] = y2.x;
                    v4[2 * k + 1] = y2.y;
                }
                float m[4];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) m[cc] = 4 * bq + cc < 4 * ax + r ? -v4[cc] : 0.0f;
                st4(Ds + (4 * ax + r) * PS + 4 * bq, make_float4(m[0], m[1], m[2], m[3]));
            }
        }
        __syncthreads();  // dA complete in Ds
        float dA[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float4 v = ld4(Ds + (4 * a + r) * PS + 4 * bq);
            dA[r][0] = v.x, dA[r][1] = v.y, dA[r][2] = v.z, dA[r][3] = v.w;
        }
        // dbeta_t = sum_s dT_b[t][s]-term (diagonal of X') + sum_{s<t} dA[t][s] (K K^T)[t][s]
        {
            // gated: G holds K K^T o Gamma below the diagonal, A = diag(beta) G there;
            // dg_t += rowsum(dA o A), dg_s -= colsum(dA o A)
            float p[4], cs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float4 g = g4[r];
                p[r] = dA[r][0] * g.x + dA[r][1] * g.y + dA[r][2] * g.z + dA[r][3] * g.w;
                if (GATED) {
                    const float bt = bs[4 * a + r];
                    cs[0] = fmaf(bt * dA[r][0], g.x, cs[0]);
                    cs[1] = fmaf(bt * dA[r][1], g.y, cs[1]);
                    cs[2] = fmaf(bt * dA[r][2], g.z, cs[2]);
                    cs[3] = fmaf(bt * dA[r][3], g.w, cs[3]);
                }
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) p[r] += __shfl_xor_sync(0xffffffffu, p[r], o);
            }
            if (GATED) {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) cs[cc] += __shfl_xor_sync(0xffffffffu, cs[cc], 16);
                if (lane < 16) {
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) dgw[warp * C + 4 * bq + cc] -= cs[cc];
                }
                __syncwarp();
                if (bq == 0) {
#pragma unroll
                    for (int r = 0; r < 4; ++r) dgw[warp * C + 4 * a + r] += bs[4 * a + r] * p[r];
                }
            }
            __syncthreads();  // dA and dbT complete
            if (bq == 0) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int t = 4 * a + r;
                    if (t < nvalid)
                        gbeta[((long long)b * L + t0 + t) * H + h] = __float2bfloat16(p[r] + dbT[t]);
                }
            }
        }
        // E = dG + dG^T, dG = diag(beta) dA, into its B tile (symmetric)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            const float4 tr = ld4(Ds + (4 * bq + cc) * PS + 4 * a);  // dA[4b+cc][4a..4a+3]
            const float trv[4] = {tr.x, tr.y, tr.z, tr.w};
            const float bc = bs[4 * bq + cc];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                dA[r][cc] = bs[4 * a + r] * dA[r][cc] + bc * trv[r];
                if (GATED) {
                    // one of the two terms is nonzero: Gamma of the pair, later index first
                    const int t = 4 * a + r, s2 = 4 * bq + cc;
                    dA[r][cc] *= tc::ex2(t >= s2 ? gs[t] - gs[s2] : gs[s2] - gs[t]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
            st4(reinterpret_cast<float*>(smem + OFF_E + kmaj_off4(4 * a + r, 4 * bq, C)),
                make_float4(dA[r][0], dA[r][1], dA[r][2], dA[r][3]));
    }
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // ---- dQ^T += K^T dM^T, dV^T = dU~^T T_b, dK^T += Q^T dM + dW^T T_b + K^T E
    if (tid == 0 && !aborted2) {
        bool ok = mbar_wait_bounded(&bar_ld[2], 0, err, EDB_DEVERR_DELTA_PIPE);
        if (ok) {
            ld_landed |= 4;
            tc::fence_after_sync();
            constexpr uint32_t id128 = idesc_tf32(128, C);
#pragma unroll
            for (int kk = 0; kk < C / 8; ++kk) {
                const uint64_t dM = kdesc(smem + OFF_DM, BOX_C, kk);
                const uint64_t dMT = kdesc(smem + OFF_DMT, BOX_C, kk);
                const uint64_t TbT = kdesc(smem + OFF_TBT, BOX_C, kk);
                const uint64_t E = kdesc(smem + OFF_E, BOX_C, kk);
                const uint64_t kA = kdesc(smem + OFF_KT, BOX_D, kk);
                if (!GATED) {
                    mma_tf32_ss(tmem + TM_Q, kA, dM, id128, 1);
                    mma_tf32_ss(tmem + TM_V, kdesc(smem + OFF_DUT, BOX_D, kk), TbT, id128, kk > 0);
                    mma_tf32_ss(tmem + TM_K, kdesc(smem + OFF_QT, BOX_D, kk), dMT, id128, 1);
                    mma_tf32_ts(tmem + TM_K, tmem + TM_W + kk * 8, TbT, id128, 1);
                    mma_tf32_ss(tmem + TM_K, kA, E, id128, 1);
                } else {
                    mma_tf32_ss(tmem + TM_Q2, kA, dM, id128, kk > 0);
                    mma_tf32_ss(tmem + TM_V, kdesc(smem + OFF_DUT, BOX_D, kk), TbT, id128, kk > 0);
                    mma_tf32_ss(tmem + TM_KB, kdesc(smem + OFF_QT, BOX_D, kk), dMT, id128, kk > 0);
                    mma_tf32_ss(tmem + TM_KB, kA, E, id128, 1);
                    mma_tf32_ts(tmem + TM_KW, tmem + TM_W + kk * 8, TbT, id128, kk > 0);
                }
            }
            tc::commit(bar_mma);
            if (!mbar_wait_bounded(bar_mma, 0, err, EDB_DEVERR_DELTA_PIPE)) {
                mbar_wait_bounded(bar_mma, 0, err, EDB_DEVERR_DELTA_PIPE);
                ok = false;
            }
        }
        if (!ok) s_misc[1] = 1;
    }
    if (tid == 0 && s_misc[1]) {
        // abort: wait (bounded) for the copies still in flight
        for (int g = 0; g < 3; ++g)
            if ((ld_issued >> g & 1) && !(ld_landed >> g & 1))
                mbar_wait_bounded(&bar_ld[g], 0, err, EDB_DEVERR_DELTA_PIPE);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (!GATED && !s_misc[1]) {
        // thread (lane quarter, half) -> column j = TMEM lane, tokens [32 hf, 32 hf + 32)
        const int j = (warp & 3) * 32 + lane;
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
                oq[t * ts] = __float2bfloat16(__uint_as_float(xq[e]));
                ov[t * ts] = __float2bfloat16(__uint_as_float(xv[e]));
                ok_[t * ts] = __float2bfloat16(__uint_as_float(xk[e]));
            }
        }
    }
    if (GATED && !s_misc[1]) {
        // thread (lane quarter, half) -> column j = TMEM lane, tokens t = 32 hf + 16 g + e
        // (sixteen columns of each accumulator at a time); q_t[j], k_t[j] from the Q^T,
        // K^T tiles; the dg partial of (t, j) into scratch (the chain's, dead now)
        const int j = (warp & 3) * 32 + lane;
        const float gC = gs[C - 1];
        float k1tot = 0.0f;
        __nv_bfloat16* oq = gq + row0 + j;
        __nv_bfloat16* ov = gv + row0 + j;
        __nv_bfloat16* ok_ = gk + row0 + j;
#pragma unroll 1
        for (int g16 = 0; g16 < 2; ++g16) {
            const uint32_t col = lane_base + hf * 32 + 16 * g16;
            uint32_t xq[16], xq2[16], xv[16], xk1[16], xkb[16], xkw[16];
            tc::tmem_ld16(tmem + TM_Q + col, xq);
            tc::tmem_ld16(tmem + TM_Q2 + col, xq2);
            tc::tmem_ld16(tmem + TM_V + col, xv);
            tc::tmem_ld16(tmem + TM_K + col, xk1);
            tc::tmem_ld16(tmem + TM_KB + col, xkb);
            tc::tmem_ld16(tmem + TM_KW + col, xkw);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int t = hf * 32 + 16 * g16 + e;
                const float gam = gam_s[t], kap = tc::ex2(gC - gs[t]);
                const uint32_t to = (t & 3) * 4;
                const float qv = *reinterpret_cast<const float*>(smem + OFF_QT + kmaj_off4(j, t & ~3, D) + to);
                const float kv = *reinterpret_cast<const float*>(smem + OFF_KT + kmaj_off4(j, t & ~3, D) + to);
                const float dqa = gam * __uint_as_float(xq[e]);        // gamma dQa~
                const float k1 = kap * __uint_as_float(xk1[e]);        // (gamma_C/gamma) dK~
                const float kw = gam * __uint_as_float(xkw[e]);        // gamma T_b^T dW
                sc[t * DGP + j] = fmaf(dqa, qv, kv * (kw - k1));
                k1tot = fmaf(kv, k1, k1tot);
                if (t < nvalid) {
                    oq[t * ts] = __float2bfloat16(dqa + __uint_as_float(xq2[e]));
                    ov[t * ts] = __float2bfloat16(__uint_as_float(xv[e]));
                    ok_[t * ts] = __float2bfloat16(__uint_as_float(xkb[e]) + k1 + kw);
                }
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) k1tot += __shfl_xor_sync(0xffffffffu, k1tot, o);
        if (lane == 0) dgw[warp * C + C - 1] += k1tot;
    }
    tc::fence_before_sync();
    __syncthreads();
    if (GATED) {
        if (!s_misc[1]) {
            // dg_t += sum_j of the partials: four threads per token, j = 4 jj + quarter
            // (bank-conflict free), then a two-step shuffle
            const int t = tid >> 2, qq = tid & 3;
            float acc = 0.0f;
#pragma unroll 8
            for (int jj = 0; jj < D / 4; ++jj) acc += sc[t * DGP + 4 * jj + qq];
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (qq == 0) dgw[warp * C + t] += acc;
        }
        __syncthreads();
    }
    if (GATED && !s_misc[1] && warp < 2) {
        // dlog alpha_s = sum_{t >= s} dg_t (a reverse scan), dalpha_s = that / alpha_s
        // dg_s: the warps' partials in a fixed order
        const int s = tid;
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < THREADS / 32; ++w) acc += dgw[w * C + s];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_down_sync(0xffffffffu, acc, o);
            if (lane + o < 32) acc += y;
        }
        if (warp == 0) {
            float tail = 0.0f;
#pragma unroll
            for (int w = 0; w < THREADS / 32; ++w) tail += dgw[w * C + 32 + lane];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) tail += __shfl_xor_sync(0xffffffffu, tail, o);
            acc += tail;
        }
        if (s < nvalid) {
            const long long ai = ((long long)b * L + t0 + s) * H + h;
            galpha[ai] = __float2bfloat16(acc / __bfloat162float(alpha[ai]));
        }
    }
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, TM_COLS);
    }
}

}  // namespace

// Library-internal launcher (called by edb_delta_chunked_bwd).
int edb_delta_chunked_post(const float* resid, const void* dO, const void* v, const void* beta,
                           const void* alpha, const float* dSCT, const float* dU, const float* dUT,
                           const float* Kf, const float* KT, const float* QT, const float* T,
                           const float* G, const float* MT, const float* gl, void* gq, void* gk,
                           void* gv, void* gbeta, void* galpha, int B, int L, int H,
                           cudaStream_t st) {
    const int NC = (L + C - 1) / C;
    const long long units = (long long)B * H, nch = units * NC;
    PostMaps m;
    int s;
    if ((s = make_box_map(&m.S0T, resid, units * (NC + 1) * D, D, D))) return s;
    if ((s = make_box_map(&m.dSCT, dSCT, nch * D, D, D))) return s;
    if ((s = make_box_map(&m.Ut, resid + ckpt_state_floats(units, NC), nch * C, D, C))) return s;
    if ((s = make_box_map(&m.dU, dU, nch * C, D, C))) return s;
    if ((s = make_box_map(&m.Kf, Kf, nch * C, D, C))) return s;
    if ((s = make_box_map(&m.KT, KT, nch * D, C, D))) return s;
    if ((s = make_box_map(&m.QT, QT, nch * D, C, D))) return s;
    if ((s = make_box_map(&m.dUT, dUT, nch * D, C, D))) return s;
    auto kern = alpha != nullptr ? delta_post_kernel<true> : delta_post_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return (int)e;
    kern<<<dim3(NC, H, B), THREADS, SMEM, st>>>(
        m, (const __nv_bfloat16*)dO, (const __nv_bfloat16*)v, (const __nv_bfloat16*)beta,
        (const __nv_bfloat16*)alpha, T, G, MT, gl, (__nv_bfloat16*)gq, (__nv_bfloat16*)gk,
        (__nv_bfloat16*)gv, (__nv_bfloat16*)gbeta, (__nv_bfloat16*)galpha, L, H, NC,
        edb::device_error_word());
    return edb::status_from_cuda(cudaGetLastError());
}
