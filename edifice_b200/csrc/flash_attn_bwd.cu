// flash_attn_bwd.cu -- backward of causal/full GQA attention.
//
// Reference semantics (edifice project paths):
//   lib/edifice/cuda/fused_scan.ex:3527-3574 (flash_attention_backward_fallback):
//     P = softmax(QK^T*scale); dV = P^T dO; dP = dO V^T;
//     dS = P (.) (dP - rowsum(dP (.) P)) * scale; dQ = dS K; dK = dS^T Q
//   native/cuda/fused_flash_attention_backward.cu:49-408 (equal heads).
// rowsum(dP (.) P) equals D = rowsum(dO (.) O), which a prep kernel computes.
// GQA: dK, dV of kv head hk sum over its Hq/Hkv query heads.
//
// B200 path (bf16, head_dim 64/128) -- one CTA per (kv tile of 128 rows,
// kv head, batch), longest causal work first; per (query head of the group,
// query tile of 64 rows) five tcgen05 MMAs with TMEM accumulators:
//   S^T  = K Q^T    (128x64, K-major x K-major)        TMEM cols [2D, 2D+64)
//   dP^T = V dO^T   (128x64)                            TMEM cols [2D+64, 2D+128)
//   dV  += P^T dO   (128xD, P^T from smem, dO MN-major) TMEM cols [0, D)
//   dK  += dS^T Q   (128xD)                             TMEM cols [D, 2D)
//   dQ_i = dS K     (64xD, dS^T read as an MN-major A)  TMEM cols [2D+128, 3D+128)
// Warps 0-3 turn S^T, dP^T (TMEM lane = kv row) into P^T and dS^T (bf16,
// 128-byte swizzled smem); warps 4-7 stage each dQ_i in swizzled smem and add
// it into an f32 accumulator with one TMA bulk reduce-add per 32 columns, and at
// the end write dK, dV; warp 8 streams Q_i / dO_i / lse / D through a 3-stage
// TMA ring; warp 9 issues the MMAs.  S^T/dP^T of
// the next tile is issued as soon as the compute warps have read the current
// one, so it overlaps their exponentials.  A last kernel converts dQ to the io
// dtype.  Other shapes run SIMT kernels with the same math.
#include <math.h>

#include "tc_common.cuh"

namespace {

constexpr int BKV = 128;
constexpr int BQ = 64;
// A Q/dO stage is released only after its second use (the dV/dK MMAs), so
// three stages are needed to keep the next tiles' TMA loads off the critical path.
constexpr int QD_STAGES = 3;
// warps 0-7 P^T/dS^T (two per TMEM lane quarter, 32 query columns each),
// 8-11 dQ staging/reduce + dK/dV epilogue, 12 TMA producer, 13 MMA issuer
constexpr int kBwdThreads = 448;
constexpr int kComputeWarps = 8;
constexpr int kDqWarp0 = 8, kProducerWarp = 12, kMmaWarp = 13;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdMaps {
    CUtensorMap q, k, v, dO, dq;  // dq: the f32 accumulator, 32-column SW128 boxes
};

template <int HD>
struct BwdSmem {
    static constexpr int NB = HD / 64;
    static constexpr int KV_BYTES = BKV * HD * 2;
    static constexpr int QD_BYTES = BQ * HD * 2;
    static constexpr int T_BYTES = BKV * BQ * 2;  // P^T or dS^T tile
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = OFF_K + KV_BYTES;
    static constexpr int OFF_Q = OFF_V + KV_BYTES;
    static constexpr int OFF_DO = OFF_Q + QD_STAGES * QD_BYTES;
    static constexpr int OFF_PT = OFF_DO + QD_STAGES * QD_BYTES;
    static constexpr int OFF_DS = OFF_PT + T_BYTES;
    static constexpr int OFF_DQ = OFF_DS + T_BYTES;           // f32 dQ staging [HD/32][BQ][32]
    static constexpr int DQ_BYTES = BQ * HD * 4;
    static constexpr int OFF_LSE = OFF_DQ + DQ_BYTES;
    static constexpr int OFF_D = OFF_LSE + QD_STAGES * BQ * 4;
    static constexpr int OFF_BAR = OFF_D + QD_STAGES * BQ * 4;
    // kv_full, qd_full[2], qd_empty[2], sdp_full, sdp_free, pds_full, mm2_done,
    // dq_full, dq_free, all_done
    static constexpr int NBAR = 1 + 2 * QD_STAGES + 7;
    static constexpr int TOTAL = OFF_BAR + NBAR * 8 + 16;
    static constexpr int TM_DV = 0, TM_DK = HD, TM_S = 2 * HD, TM_DP = 2 * HD + 64,
                         TM_DQ = 2 * HD + 128;
    static constexpr int TMEM_COLS = 512;
};

// FOX: FoX attention (fused_scan.ex:3870-3984): P of key row j takes the bias
// -cs[b, h, j] of its query head h (one plain load per head and thread), and
// each compute thread adds up the dS of its key row over its 32 query columns of
// every tile of a head, storing that partial (half hf of the query columns) to
// cs_part[hf][b, h, j]; fox_dcs_kernel then forms grad_cs = -(sum) / scale.  No
// wait or barrier is added.
template <int HD, bool CAUSAL, bool FOX = false>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ BwdMaps maps, const float* __restrict__ lse,
                       const float* __restrict__ Dv, float* __restrict__ dq_acc,
                       __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int L,
                       int Hq, int Hkv, float scale, unsigned* err,
                       const float* __restrict__ cs = nullptr, float* __restrict__ cs_part = nullptr) {
    using S = BwdSmem<HD>;
    constexpr int NB = S::NB;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sK = smem + S::OFF_K;
    uint8_t* sV = smem + S::OFF_V;
    uint8_t* sQ = smem + S::OFF_Q;
    uint8_t* sdO = smem + S::OFF_DO;
    uint8_t* sPt = smem + S::OFF_PT;
    uint8_t* sDs = smem + S::OFF_DS;
    uint8_t* sDq = smem + S::OFF_DQ;
    float* sLse = reinterpret_cast<float*>(smem + S::OFF_LSE);
    float* sD = reinterpret_cast<float*>(smem + S::OFF_D);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* kv_full = bars;
    uint64_t* qd_full = bars + 1;
    uint64_t* qd_empty = bars + 1 + QD_STAGES;
    uint64_t* sdp_full = bars + 1 + 2 * QD_STAGES;
    uint64_t* sdp_free = sdp_full + 1;
    uint64_t* pds_full = sdp_full + 2;
    uint64_t* mm2_done = sdp_full + 3;
    uint64_t* dq_full = sdp_full + 4;
    uint64_t* dq_free = sdp_full + 5;
    uint64_t* all_done = sdp_full + 6;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + S::NBAR);
    int* s_abort = reinterpret_cast<int*>(s_tmem + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Blocks launch in linear-index order (x fastest).  The kv tile is taken as the
    // slowest index: with a causal mask kv tile 0 has the most query tiles, so the
    // longest CTAs of every (kv head, batch) go first and the short ones fill the
    // tail (FoX backward 7.78 -> 7.47 ms at the configs[3] shapes; causal attention
    // 7.83-7.97 -> 7.78-7.83 ms)
    const int nrow = gridDim.y * gridDim.z;
    const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    const int kt = lin / nrow, rem = lin - kt * nrow;
    const int hk = rem % Hkv, b = rem / Hkv;
    const int G = Hq / Hkv;
    const int bhk = b * Hkv + hk;
    const int nq = (L + BQ - 1) / BQ;
    const int i0 = CAUSAL ? (kt * BKV) / BQ : 0;
    const int nqi = nq - i0;
    const int N = G * nqi;
    const float scale_log2 = scale * kLog2e;

    if ((smem_u32(smem) & 1023u) != 0) {
        if (tid == 0) edb_flag_error(err, EDB_DEVERR_ATTN_PIPE);
        return;
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(s_tmem, S::TMEM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 256) {
        mbar_init(kv_full, 1);
        for (int s = 0; s < QD_STAGES; ++s) {
            mbar_init(&qd_full[s], 1);
            mbar_init(&qd_empty[s], 1);
        }
        mbar_init(sdp_full, 1);
        mbar_init(sdp_free, kComputeWarps);
        mbar_init(pds_full, kComputeWarps);
        mbar_init(mm2_done, 1);
        mbar_init(dq_full, 1);
        mbar_init(dq_free, 4);
        mbar_init(all_done, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *s_tmem;
    volatile int* abort_flag = s_abort;

    if (warp == kProducerWarp) {
        // ------------------------------------------------ producer (whole warp)
        if (lane == 0) {
            prefetch_tmap(&maps.q);
            prefetch_tmap(&maps.k);
            prefetch_tmap(&maps.v);
            prefetch_tmap(&maps.dO);
            mbar_arrive_expect_tx(kv_full, 2 * S::KV_BYTES);
            for (int bx = 0; bx < NB; ++bx) {
                tma_load_3d(sK + bx * (BKV * 128), &maps.k, kv_full, bx * 64, kt * BKV, bhk);
                tma_load_3d(sV + bx * (BKV * 128), &maps.v, kv_full, bx * 64, kt * BKV, bhk);
            }
        }
        int issued = 0;
        // this lane's rows of -lse log2(e) and -D scale for a tile, loaded one tile
        // ahead so their latency hides behind the wait for a free stage
        float pl[BQ / 32], pd[BQ / 32];
        auto fetch = [&](int n) {
            const int g = n / nqi, i = i0 + n % nqi;
            const long long row0 = (long long)(b * Hq + hk * G + g) * L;
#pragma unroll
            for (int r = 0; r < BQ / 32; ++r) {
                const int qr = i * BQ + lane + 32 * r;
                const bool ok = qr < L;
                // stored as -lse log2(e) and -D scale: P = ex2(S scale log2(e) + .),
                // dS = P (dP scale + .); rows past L give P = 0
                pl[r] = ok ? -lse[row0 + qr] * kLog2e : -INFINITY;
                pd[r] = ok ? -Dv[row0 + qr] * scale : 0.0f;
            }
        };
        if (N > 0) fetch(0);
        for (int n = 0; n < N; ++n) {
            const int s = n % QD_STAGES;
            int go = 1;
            if (lane == 0 && n >= QD_STAGES) {
                if (*abort_flag ||
                    !mbar_wait_bounded(&qd_empty[s], ((n / QD_STAGES) - 1) & 1, err,
                                       EDB_DEVERR_ATTN_PIPE)) {
                    *abort_flag = 1;
                    go = 0;
                }
            }
            go = __shfl_sync(0xffffffffu, go, 0);
            if (!go) break;
            const int g = n / nqi, i = i0 + n % nqi;
            const int bh = b * Hq + hk * G + g;
#pragma unroll
            for (int r = 0; r < BQ / 32; ++r) {
                sLse[s * BQ + lane + 32 * r] = pl[r];
                sD[s * BQ + lane + 32 * r] = pd[r];
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&qd_full[s], 2 * S::QD_BYTES);
                for (int bx = 0; bx < NB; ++bx) {
                    tma_load_3d(sQ + s * S::QD_BYTES + bx * (BQ * 128), &maps.q, &qd_full[s],
                                bx * 64, i * BQ, bh);
                    tma_load_3d(sdO + s * S::QD_BYTES + bx * (BQ * 128), &maps.dO, &qd_full[s],
                                bx * 64, i * BQ, bh);
                }
            }
            issued = n + 1;
            if (n + 1 < N) fetch(n + 1);
        }
        if (lane == 0) {
            for (int n = max(0, issued - QD_STAGES); n < issued; ++n)
                mbar_wait_bounded(&qd_full[n % QD_STAGES], (n / QD_STAGES) & 1, err,
                                  EDB_DEVERR_ATTN_PIPE);
            mbar_wait_bounded(kv_full, 0, err, EDB_DEVERR_ATTN_PIPE);
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idSP = tc::idesc_bf16(BKV, BQ, 0, 0);   // S^T, dP^T
            constexpr uint32_t idKV = tc::idesc_bf16(BKV, HD, 0, 1);   // dV, dK
            constexpr uint32_t idQ = tc::idesc_bf16(BQ, HD, 1, 1);     // dQ (head_dim 64)
            constexpr uint32_t idQt = tc::idesc_bf16(HD, BQ, 1, 1);    // dQ^T (head_dim 128)
            auto issue_sdp = [&](int n) {
                const int s = n % QD_STAGES;
                const uint8_t* q = sQ + s * S::QD_BYTES;
                const uint8_t* o = sdO + s * S::QD_BYTES;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const int off_kv = (kk >> 2) * (BKV * 128) + (kk & 3) * 32;
                    const int off_q = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
                    tc::mma_bf16_ss(tmem + S::TM_S, tc::sdesc_sw128(sK + off_kv, 16, 1024),
                                    tc::sdesc_sw128(q + off_q, 16, 1024), idSP, kk > 0);
                    tc::mma_bf16_ss(tmem + S::TM_DP, tc::sdesc_sw128(sV + off_kv, 16, 1024),
                                    tc::sdesc_sw128(o + off_q, 16, 1024), idSP, kk > 0);
                }
                tc::commit(sdp_full);
            };
            bool ok = mbar_wait_bounded(kv_full, 0, err, EDB_DEVERR_ATTN_PIPE) &&
                      (N == 0 || mbar_wait_bounded(&qd_full[0], 0, err, EDB_DEVERR_ATTN_PIPE));
            if (ok && N > 0) {
                tc::fence_after_sync();
                issue_sdp(0);
            }
            for (int n = 0; ok && n < N; ++n) {
                if (n + 1 < N) {
                    ok = !*abort_flag &&
                         mbar_wait_bounded(&qd_full[(n + 1) % QD_STAGES],
                                           ((n + 1) / QD_STAGES) & 1, err, EDB_DEVERR_ATTN_PIPE) &&
                         mbar_wait_bounded(sdp_free, n & 1, err, EDB_DEVERR_ATTN_PIPE);
                    if (!ok) break;
                    tc::fence_after_sync();
                    issue_sdp(n + 1);
                }
                ok = mbar_wait_bounded(pds_full, n & 1, err, EDB_DEVERR_ATTN_PIPE) &&
                     (n == 0 || mbar_wait_bounded(dq_free, (n - 1) & 1, err, EDB_DEVERR_ATTN_PIPE));
                if (!ok) break;
                tc::fence_after_sync();
                const int s = n % QD_STAGES;
                const uint8_t* q = sQ + s * S::QD_BYTES;
                const uint8_t* o = sdO + s * S::QD_BYTES;
                // dQ first, its barrier committed at once: the dQ warps drain it while
                // dV and dK run.  head_dim 128 computes dQ^T = K^T dS^T, M = 128 (the
                // head dim): the tensor core's full-rate shape, where dS K would be
                // M = 64 (half rate); both operands are MN-major in the same tiles.
                if constexpr (HD == 128) {
#pragma unroll
                    for (int kk = 0; kk < BKV / 16; ++kk)
                        tc::mma_bf16_ss(tmem + S::TM_DQ, tc::sdesc_sw128(sK + kk * 2048, BKV * 128, 1024),
                                        tc::sdesc_sw128(sDs + kk * 2048, BQ * 128, 1024), idQt,
                                        kk > 0);
                } else {
#pragma unroll
                    for (int kk = 0; kk < BKV / 16; ++kk)
                        tc::mma_bf16_ss(tmem + S::TM_DQ, tc::sdesc_sw128(sDs + kk * 2048, BQ * 128, 1024),
                                        tc::sdesc_sw128(sK + kk * 2048, BKV * 128, 1024), idQ, kk > 0);
                }
                tc::commit(dq_full);
#pragma unroll
                for (int kk = 0; kk < BQ / 16; ++kk) {
                    tc::mma_bf16_ss(tmem + S::TM_DV, tc::sdesc_sw128(sPt + kk * 32, 16, 1024),
                                    tc::sdesc_sw128(o + kk * 2048, BQ * 128, 1024), idKV,
                                    (n > 0 || kk > 0));
                    tc::mma_bf16_ss(tmem + S::TM_DK, tc::sdesc_sw128(sDs + kk * 32, 16, 1024),
                                    tc::sdesc_sw128(q + kk * 2048, BQ * 128, 1024), idKV,
                                    (n > 0 || kk > 0));
                }
                tc::commit(mm2_done);
                tc::commit(&qd_empty[s]);
            }
            if (!ok) *abort_flag = 1;
            tc::commit(all_done);
            mbar_wait_bounded(all_done, 0, err, EDB_DEVERR_ATTN_PIPE);
        }
    } else if (warp < kComputeWarps) {
        // ------------------------------------------------ P^T / dS^T compute
        // warp (quarter q = warp % 4, half hf = warp / 4): kv row r = 32 q + lane
        // (TMEM lane), query columns [32 hf, 32 hf + 32) of the tile
        const int qw = warp & 3, hf = warp >> 2;
        const int r = qw * 32 + lane;
        const int kv_idx = kt * BKV + r;
        const uint32_t lb = (uint32_t)(qw * 32) << 16;
        const int c0 = hf * 32;
        const float2 sl2 = dup2(scale_log2), sc2 = dup2(scale);
        float2 nb2 = dup2(0.0f);  // FoX: -cs[b, h, kv] log2(e) of the current query head
        float dsum = 0.0f;        // FoX: this thread's dS sum over the head's query columns
        const long long rows_all = (long long)gridDim.z * Hq * L;
        for (int n = 0; n < N; ++n) {
            const int s = n % QD_STAGES;
            const int i = i0 + n % nqi;
            const int gq = n / nqi;
            if (FOX && n % nqi == 0)
                nb2 = dup2(kv_idx < L ? -__ldg(cs + ((long long)b * Hq + hk * G + gq) * L + kv_idx) *
                                            kLog2e
                                      : 0.0f);
            // go / give-up decisions are the whole warp's (__all_sync): a lane that
            // left the loop alone would leave the others in tcgen05.ld
            const bool got =
                !*abort_flag &&
                mbar_wait_bounded(&qd_full[s], (n / QD_STAGES) & 1, err, EDB_DEVERR_ATTN_PIPE) &&
                mbar_wait_bounded(sdp_full, n & 1, err, EDB_DEVERR_ATTN_PIPE);
            if (!__all_sync(0xffffffffu, got)) {
                *abort_flag = 1;
                break;
            }
            tc::fence_after_sync();
            uint32_t sr[32], dr[32];
            tc::tmem_ld32(tmem + S::TM_S + lb + c0, sr);
            tc::tmem_ld32(tmem + S::TM_DP + lb + c0, dr);
            tc::tmem_wait_ld();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(sdp_free);
            const float* nl2 = sLse + s * BQ + c0;   // -lse log2(e)
            const float* ndd = sD + s * BQ + c0;     // -D scale
            // masks only on the diagonal and for a ragged last kv tile; query rows
            // past L carry -lse = -inf and give P = 0 by themselves
            const bool need_mask = (kt * BKV + BKV > L) || (CAUSAL && i * BQ < kt * BKV + BKV);
            // P and dS in registers first: this math overlaps the previous tile's
            // dV / dK / dQ products, which still read P^T and dS^T in shared memory;
            // only the stores below wait for them (mm2_done)
            uint4 pt4[4], ds4[4];
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const float4 la = *reinterpret_cast<const float4*>(nl2 + ch * 8);
                const float4 lb4 = *reinterpret_cast<const float4*>(nl2 + ch * 8 + 4);
                const float4 da = *reinterpret_cast<const float4*>(ndd + ch * 8);
                const float4 db = *reinterpret_cast<const float4*>(ndd + ch * 8 + 4);
                const float2 lv[4] = {make_float2(la.x, la.y), make_float2(la.z, la.w),
                                      make_float2(lb4.x, lb4.y), make_float2(lb4.z, lb4.w)};
                const float2 dv2[4] = {make_float2(da.x, da.y), make_float2(da.z, da.w),
                                       make_float2(db.x, db.y), make_float2(db.z, db.w)};
                uint32_t pk[4], dk2[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int cc = ch * 8 + 2 * e;  // column within this warp's 32
                    const float2 sv = make_float2(__uint_as_float(sr[cc]), __uint_as_float(sr[cc + 1]));
                    const float2 dp = make_float2(__uint_as_float(dr[cc]), __uint_as_float(dr[cc + 1]));
                    const float2 arg = fma2(sv, sl2, FOX ? add2(lv[e], nb2) : lv[e]);
                    float2 p = make_float2(tc::ex2(arg.x), tc::ex2(arg.y));
                    if (need_mask) {
                        const int q_idx = i * BQ + c0 + cc;
                        const bool ok = kv_idx < L;
                        if (!ok || (CAUSAL && q_idx < kv_idx)) p.x = 0.0f;
                        if (!ok || (CAUSAL && q_idx + 1 < kv_idx)) p.y = 0.0f;
                    }
                    const float2 ds = mul2(p, fma2(dp, sc2, dv2[e]));
                    if (FOX) dsum += ds.x + ds.y;
                    pk[e] = tc::pack_bf16x2(p.x, p.y);
                    dk2[e] = tc::pack_bf16x2(ds.x, ds.y);
                }
                pt4[ch] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                ds4[ch] = make_uint4(dk2[0], dk2[1], dk2[2], dk2[3]);
            }
            if (n > 0 && !__all_sync(0xffffffffu, mbar_wait_bounded(mm2_done, (n - 1) & 1, err,
                                                                    EDB_DEVERR_ATTN_PIPE))) {
                *abort_flag = 1;
                break;
            }
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const int chunk = hf * 4 + ch;  // 16-byte chunk of the 128-byte row
                *reinterpret_cast<uint4*>(sPt + tc::sw128_off(r, chunk)) = pt4[ch];
                *reinterpret_cast<uint4*>(sDs + tc::sw128_off(r, chunk)) = ds4[ch];
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(pds_full);
            if (FOX && n % nqi == nqi - 1) {  // the head's last query tile
                if (kv_idx < L)
                    cs_part[hf * rows_all + ((long long)b * Hq + hk * G + gq) * L + kv_idx] = dsum;
                dsum = 0.0f;
            }
        }
    } else {
        // ------------------------------------------------ dQ reduction + dK/dV epilogue (warps 4-7)
        const int w = warp - kDqWarp0;
        const uint32_t lb = (uint32_t)(w * 32) << 16;
        // A warp whose wait gives up keeps taking the two named barriers of every
        // remaining tile (doing nothing else), so no other dQ warp is left waiting.
        bool ok = true;
        for (int n = 0; n < N; ++n) {
            const int g = n / nqi, i = i0 + n % nqi;
            const int bh = b * Hq + hk * G + g;
            if (ok && !__all_sync(0xffffffffu, !*abort_flag && mbar_wait_bounded(dq_full, n & 1, err,
                                                                                 EDB_DEVERR_ATTN_PIPE))) {
                *abort_flag = 1;
                ok = false;
            }
            if (ok) {
                tc::fence_after_sync();
                // the previous tile's bulk reduce must be done reading the staging tile
                if (w == 0 && lane == 0) tc::tma_store_wait_read_all();
            }
            tc::named_bar(2, 128);
            if (ok) {
                if constexpr (HD == 128) {
                    // dQ^T: TMEM lane 32 w + lane is head-dim column d, its 64 columns the
                    // tile's query rows; the thread writes column d of every row into
                    // staging box w (float `lane` of each 128-byte row, conflict free)
                    uint32_t qv[2][32];
                    tc::tmem_ld32(tmem + S::TM_DQ + lb, qv[0]);
                    tc::tmem_ld32(tmem + S::TM_DQ + lb + 32, qv[1]);
                    tc::tmem_wait_ld();
                    uint8_t* box = sDq + w * (BQ * 128) + (lane & 3) * 4;
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            *reinterpret_cast<uint32_t*>(box + tc::sw128_off(h2 * 32 + e, lane >> 2)) =
                                qv[h2][e];
                } else
                // dQ_i in two halves of HD/2 columns (register budget); M = 64
                // accumulator: lanes 32w + t (t < 16) hold query row 16w + t of the tile
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t qv[HD / 64][32];
#pragma unroll
                    for (int cc = 0; cc < HD / 64; ++cc)
                        tc::tmem_ld32(tmem + S::TM_DQ + lb + (hh * (HD / 64) + cc) * 32, qv[cc]);
                    tc::tmem_wait_ld();
                    if (lane < 16) {
                        const int r = 16 * w + lane;
#pragma unroll
                        for (int cc = 0; cc < HD / 64; ++cc)
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                *reinterpret_cast<uint4*>(sDq + (hh * (HD / 64) + cc) * (BQ * 128) +
                                                          tc::sw128_off(r, j)) =
                                    make_uint4(qv[cc][4 * j], qv[cc][4 * j + 1], qv[cc][4 * j + 2],
                                               qv[cc][4 * j + 3]);
                    }
                }
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(dq_free);
                fence_proxy_async();
            }
            tc::named_bar(2, 128);
            // dq_acc[bh, i*BQ .., :] += staging tile (rows past L are clipped)
            if (ok && w == 0 && lane == 0 && *abort_flag == 0) {
#pragma unroll
                for (int cc = 0; cc < HD / 32; ++cc)
                    tc::tma_reduce_add_3d(&maps.dq, sDq + cc * (BQ * 128), cc * 32, i * BQ, bh);
                tc::tma_store_commit();
            }
        }
        if (w == 0 && lane == 0) tc::tma_store_wait_all();
        if (ok && __all_sync(0xffffffffu, mbar_wait_bounded(all_done, 0, err, EDB_DEVERR_ATTN_PIPE))) {
            tc::fence_after_sync();
            const int r = w * 32 + lane;
            const int kv_idx = kt * BKV + r;
#pragma unroll
            for (int which = 0; which < 2; ++which) {
                __nv_bfloat16* dst = (which == 0 ? dv : dk) + ((long long)bhk * L + kv_idx) * HD;
                const uint32_t col = which == 0 ? S::TM_DV : S::TM_DK;
#pragma unroll
                for (int cc = 0; cc < HD / 32; ++cc) {
                    uint32_t x[32];
                    tc::tmem_ld32(tmem + col + lb + cc * 32, x);
                    tc::tmem_wait_ld();
                    if (kv_idx < L) {
#pragma unroll
                        for (int e = 0; e < 32; e += 8)
                            st_global_v4(dst + cc * 32 + e,
                                         make_uint4(tc::pack_bf16x2(__uint_as_float(x[e]), __uint_as_float(x[e + 1])),
                                                    tc::pack_bf16x2(__uint_as_float(x[e + 2]), __uint_as_float(x[e + 3])),
                                                    tc::pack_bf16x2(__uint_as_float(x[e + 4]), __uint_as_float(x[e + 5])),
                                                    tc::pack_bf16x2(__uint_as_float(x[e + 6]), __uint_as_float(x[e + 7]))));
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

// D = rowsum(dO (.) O), one warp per 4 rows (8 lanes x 16 bytes per 128-wide row)
template <typename T>
__global__ void attn_bwd_rowdot_kernel(const T* __restrict__ o, const T* __restrict__ dO,
                                       float* __restrict__ D, long long rows, int d) {
    const long long row = (long long)blockIdx.x * blockDim.y + threadIdx.y;
    if (row >= rows) return;
    float acc = 0.0f;
    for (int e = threadIdx.x; e < d; e += blockDim.x)
        acc = fmaf(ld_scalar<T>(o + row * d + e), ld_scalar<T>(dO + row * d + e), acc);
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (threadIdx.x == 0) D[row] = acc;
}

template <typename T>
__global__ void dq_convert_kernel(const float* __restrict__ acc, T* __restrict__ dq, long long n) {
    const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        const float4 v = *reinterpret_cast<const float4*>(acc + i);
        st_scalar<T>(dq + i, v.x);
        st_scalar<T>(dq + i + 1, v.y);
        st_scalar<T>(dq + i + 2, v.z);
        st_scalar<T>(dq + i + 3, v.w);
    } else {
        for (long long j = i; j < n; ++j) st_scalar<T>(dq + j, acc[j]);
    }
}

// ------------------------------------------------------------ SIMT backward
// lse of every query row (natural log), one thread per row
template <typename T, int HDMAX>
__global__ void attn_lse_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                     float* __restrict__ lse, int L, int Hq, int Hkv, int d,
                                     int causal, float scale) {
    const int hq = blockIdx.y, b = blockIdx.z;
    const int hk = hq / (Hq / Hkv);
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= L) return;
    const T* qi = q + (((long long)b * Hq + hq) * L + i) * d;
    const T* kb = k + ((long long)b * Hkv + hk) * L * d;
    float qv[HDMAX];
    for (int e = 0; e < HDMAX; ++e) qv[e] = e < d ? ld_scalar<T>(qi + e) * scale * kLog2e : 0.0f;
    float m = -INFINITY, l = 0.0f;
    const int jend = causal ? i + 1 : L;
    for (int j = 0; j < jend; ++j) {
        float s = 0.0f;
        for (int e = 0; e < d; ++e) s = fmaf(qv[e], ld_scalar<T>(kb + (long long)j * d + e), s);
        const float mn = fmaxf(m, s);
        l = l * exp2f(m - mn) + exp2f(s - mn);
        m = mn;
    }
    lse[((long long)b * Hq + hq) * L + i] = (m + log2f(l)) / kLog2e;
}

template <typename T, int HDMAX>
__global__ void attn_bwd_dq_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                        const T* __restrict__ v, const T* __restrict__ dO,
                                        const float* __restrict__ lse, const float* __restrict__ Dv,
                                        T* __restrict__ dq, int L, int Hq, int Hkv, int d,
                                        int causal, float scale,
                                        const float* __restrict__ cs = nullptr) {
    const int hq = blockIdx.y, b = blockIdx.z;
    const int hk = hq / (Hq / Hkv);
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= L) return;
    const long long row = ((long long)b * Hq + hq) * L + i;
    const T* kb = k + ((long long)b * Hkv + hk) * L * d;
    const T* vb = v + ((long long)b * Hkv + hk) * L * d;
    float qv[HDMAX], dov[HDMAX], acc[HDMAX];
    for (int e = 0; e < HDMAX; ++e) {
        qv[e] = e < d ? ld_scalar<T>(q + row * d + e) : 0.0f;
        dov[e] = e < d ? ld_scalar<T>(dO + row * d + e) : 0.0f;
        acc[e] = 0.0f;
    }
    const float l2 = lse[row] * kLog2e, Di = Dv[row];
    const int jend = causal ? i + 1 : L;
    for (int j = 0; j < jend; ++j) {
        float s = 0.0f, dp = 0.0f;
        for (int e = 0; e < d; ++e) {
            s = fmaf(qv[e], ld_scalar<T>(kb + (long long)j * d + e), s);
            dp = fmaf(dov[e], ld_scalar<T>(vb + (long long)j * d + e), dp);
        }
        const float bias = cs != nullptr ? cs[((long long)b * Hq + hq) * L + j] * kLog2e : 0.0f;
        const float p = exp2f(s * scale * kLog2e - l2 - bias);
        const float ds = p * (dp - Di) * scale;
        for (int e = 0; e < d; ++e) acc[e] = fmaf(ds, ld_scalar<T>(kb + (long long)j * d + e), acc[e]);
    }
    for (int e = 0; e < d; ++e) st_scalar<T>(dq + row * d + e, acc[e]);
}

template <typename T, int HDMAX>
__global__ void attn_bwd_dkdv_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                          const T* __restrict__ v, const T* __restrict__ dO,
                                          const float* __restrict__ lse,
                                          const float* __restrict__ Dv, T* __restrict__ dk,
                                          T* __restrict__ dvo, int L, int Hq, int Hkv, int d,
                                          int causal, float scale,
                                          const float* __restrict__ cs = nullptr,
                                          float* __restrict__ cs_part = nullptr) {
    const int hk = blockIdx.y, b = blockIdx.z;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= L) return;
    const int G = Hq / Hkv;
    const long long krow = ((long long)b * Hkv + hk) * L + j;
    float kv[HDMAX], vv[HDMAX], ak[HDMAX], av[HDMAX];
    for (int e = 0; e < HDMAX; ++e) {
        kv[e] = e < d ? ld_scalar<T>(k + krow * d + e) : 0.0f;
        vv[e] = e < d ? ld_scalar<T>(v + krow * d + e) : 0.0f;
        ak[e] = 0.0f;
        av[e] = 0.0f;
    }
    for (int g = 0; g < G; ++g) {
        const long long bh = (long long)b * Hq + hk * G + g;
        const float bias = cs != nullptr ? cs[bh * L + j] * kLog2e : 0.0f;
        float dssum = 0.0f;
        for (int i = causal ? j : 0; i < L; ++i) {
            const long long row = bh * L + i;
            float s = 0.0f, dp = 0.0f;
            for (int e = 0; e < d; ++e) {
                s = fmaf(ld_scalar<T>(q + row * d + e), kv[e], s);
                dp = fmaf(ld_scalar<T>(dO + row * d + e), vv[e], dp);
            }
            const float p = exp2f(s * scale * kLog2e - lse[row] * kLog2e - bias);
            const float ds = p * (dp - Dv[row]) * scale;
            dssum += ds;
            for (int e = 0; e < d; ++e) {
                ak[e] = fmaf(ds, ld_scalar<T>(q + row * d + e), ak[e]);
                av[e] = fmaf(p, ld_scalar<T>(dO + row * d + e), av[e]);
            }
        }
        if (cs_part != nullptr) {  // one writer per (bh, j): the second half is zero
            const long long bhq = (long long)gridDim.z * Hq;
            cs_part[bh * L + j] = dssum;
            cs_part[(bhq + bh) * L + j] = 0.0f;
        }
    }
    for (int e = 0; e < d; ++e) {
        st_scalar<T>(dk + krow * d + e, ak[e]);
        st_scalar<T>(dvo + krow * d + e, av[e]);
    }
}

// grad_cs = -(part[0] + part[1]) / scale: the two halves' column sums of dS (which
// carry the softmax scale) for the key side; the query side (row sums of dS) is zero.
__global__ void fox_dcs_kernel(const float* __restrict__ part, float* __restrict__ dcs, long long n,
                               float inv_scale) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dcs[i] = -(part[i] + part[n + i]) * inv_scale;
}

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

bool tc_shape(int dtype, int head_dim) {
    return dtype == EDB_BF16 && (head_dim == 64 || head_dim == 128);
}

template <int HD, bool CAUSAL, bool FOX = false>
int launch_bwd_tc(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                  const float* D, float* dq_acc, void* dk, void* dv, int B, int Hq, int Hkv, int L,
                  float scale, cudaStream_t st, const float* cs = nullptr,
                  float* cs_part = nullptr) {
    BwdMaps maps;
    int s;
    if ((s = tc::make_attn_map(&maps.q, q, HD, L, B * Hq, BQ))) return s;
    if ((s = tc::make_attn_map(&maps.dO, dO, HD, L, B * Hq, BQ))) return s;
    if ((s = tc::make_attn_map(&maps.k, k, HD, L, B * Hkv, BKV))) return s;
    if ((s = tc::make_attn_map(&maps.v, v, HD, L, B * Hkv, BKV))) return s;
    if ((s = tc::make_attn_map_f32(&maps.dq, dq_acc, HD, L, B * Hq, BQ))) return s;
    auto kern = attn_bwd_tc_kernel<HD, CAUSAL, FOX>;
    const int smem = BwdSmem<HD>::TOTAL;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    dim3 grid((L + BKV - 1) / BKV, Hkv, B);
    kern<<<grid, kBwdThreads, smem, st>>>(maps, lse, D, dq_acc, (__nv_bfloat16*)dk,
                                          (__nv_bfloat16*)dv, L, Hq, Hkv, scale,
                                          edb::device_error_word(), cs, cs_part);
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T>
int launch_bwd_simt(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                    const float* D, void* dq, void* dk, void* dv, int B, int Hq, int Hkv, int L,
                    int d, int causal, float scale, cudaStream_t st, const float* cs = nullptr,
                    float* cs_part = nullptr) {
    dim3 gq((L + 63) / 64, Hq, B), gk((L + 63) / 64, Hkv, B);
#define EDB_SIMT_BWD(HDM)                                                                        \
    attn_bwd_dq_simt_kernel<T, HDM><<<gq, 64, 0, st>>>((const T*)q, (const T*)k, (const T*)v,   \
                                                       (const T*)dO, lse, D, (T*)dq, L, Hq, Hkv, \
                                                       d, causal, scale, cs);                    \
    attn_bwd_dkdv_simt_kernel<T, HDM><<<gk, 64, 0, st>>>((const T*)q, (const T*)k, (const T*)v, \
                                                         (const T*)dO, lse, D, (T*)dk, (T*)dv,  \
                                                         L, Hq, Hkv, d, causal, scale, cs,      \
                                                         cs_part);
    if (d <= 32) {
        EDB_SIMT_BWD(32)
    } else if (d <= 64) {
        EDB_SIMT_BWD(64)
    } else {
        EDB_SIMT_BWD(128)
    }
#undef EDB_SIMT_BWD
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T>
int launch_lse_simt(const void* q, const void* k, float* lse, int B, int Hq, int Hkv, int L, int d,
                    int causal, float scale, cudaStream_t st) {
    dim3 g((L + 63) / 64, Hq, B);
    if (d <= 32)
        attn_lse_simt_kernel<T, 32><<<g, 64, 0, st>>>((const T*)q, (const T*)k, lse, L, Hq, Hkv, d,
                                                      causal, scale);
    else if (d <= 64)
        attn_lse_simt_kernel<T, 64><<<g, 64, 0, st>>>((const T*)q, (const T*)k, lse, L, Hq, Hkv, d,
                                                      causal, scale);
    else
        attn_lse_simt_kernel<T, 128><<<g, 64, 0, st>>>((const T*)q, (const T*)k, lse, L, Hq, Hkv,
                                                       d, causal, scale);
    return edb::status_from_cuda(cudaGetLastError());
}

}  // namespace

// forward entry with the row log-sum-exp only (flash_attn.cu)
int edb_attn_fwd_lse_only(int head_dim, int causal, const void* q, const void* k, float* lse,
                          int B, int Hq, int Hkv, int L, float scale, cudaStream_t st);

extern "C" size_t edb_flash_attention_bwd_workspace(int dtype, int batch, int q_heads,
                                                    int kv_heads, int seq_len, int head_dim,
                                                    int have_lse) {
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || seq_len <= 0 || head_dim <= 0) return 0;
    const size_t rows = (size_t)batch * q_heads * seq_len;
    size_t ws = a256(rows * 4);                      // D
    if (!have_lse) ws += a256(rows * 4);             // lse
    if (tc_shape(dtype, head_dim)) ws += a256(rows * head_dim * 4);  // f32 dQ accumulator
    return ws;
}

extern "C" int edb_flash_attention_bwd(int dtype, const void* q, const void* k, const void* v,
                                       const void* o, const void* dO, const float* lse, void* dq,
                                       void* dk, void* dv, int batch, int q_heads, int kv_heads,
                                       int seq_len, int head_dim, int causal, float scale,
                                       void* workspace, size_t workspace_bytes, void* stream) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || seq_len <= 0 || head_dim <= 0)
        return EDB_ERR_BAD_SHAPE;
    if (q_heads % kv_heads != 0) return EDB_ERR_BAD_SHAPE;
    if (head_dim > 128) return EDB_ERR_UNSUPPORTED;
    if (!q || !k || !v || !o || !dO || !dq || !dk || !dv) return EDB_ERR_NULL_POINTER;
    const size_t need = edb_flash_attention_bwd_workspace(dtype, batch, q_heads, kv_heads,
                                                          seq_len, head_dim, lse != nullptr);
    if (workspace_bytes < need || !workspace) return EDB_ERR_WORKSPACE_TOO_SMALL;
    if (!edb::aligned16(workspace)) return EDB_ERR_MISALIGNED;
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)head_dim);
    cudaStream_t st = (cudaStream_t)stream;
    const size_t rows = (size_t)batch * q_heads * seq_len;
    char* w = static_cast<char*>(workspace);
    float* D = reinterpret_cast<float*>(w);
    w += a256(rows * 4);
    const float* L_ = lse;
    float* lse_ws = nullptr;
    if (!lse) {
        lse_ws = reinterpret_cast<float*>(w);
        w += a256(rows * 4);
        L_ = lse_ws;
    }
    const bool use_tc = tc_shape(dtype, head_dim) && edb::aligned16(q) && edb::aligned16(k) &&
                        edb::aligned16(v) && edb::aligned16(dO) && edb::aligned16(dk) &&
                        edb::aligned16(dv);
    // D = rowsum(dO * O)
    {
        dim3 blk(32, 4);
        const unsigned nb = (unsigned)((rows + 3) / 4);
        if (dtype == EDB_BF16)
            attn_bwd_rowdot_kernel<__nv_bfloat16><<<nb, blk, 0, st>>>(
                (const __nv_bfloat16*)o, (const __nv_bfloat16*)dO, D, (long long)rows, head_dim);
        else
            attn_bwd_rowdot_kernel<float><<<nb, blk, 0, st>>>((const float*)o, (const float*)dO, D,
                                                              (long long)rows, head_dim);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return (int)e;
    }
    if (lse_ws) {
        int s;
        if (use_tc)
            s = edb_attn_fwd_lse_only(head_dim, causal, q, k, lse_ws, batch, q_heads, kv_heads,
                                      seq_len, scale, st);
        else
            s = dtype == EDB_BF16
                    ? launch_lse_simt<__nv_bfloat16>(q, k, lse_ws, batch, q_heads, kv_heads,
                                                     seq_len, head_dim, causal, scale, st)
                    : launch_lse_simt<float>(q, k, lse_ws, batch, q_heads, kv_heads, seq_len,
                                             head_dim, causal, scale, st);
        if (s) return s;
    }
    if (use_tc) {
        float* acc = reinterpret_cast<float*>(w);
        const size_t nel = rows * head_dim;
        cudaError_t e = cudaMemsetAsync(acc, 0, nel * 4, st);
        if (e != cudaSuccess) return (int)e;
        int s;
        if (head_dim == 128)
            s = causal ? launch_bwd_tc<128, true>(q, k, v, dO, L_, D, acc, dk, dv, batch, q_heads,
                                                  kv_heads, seq_len, scale, st)
                       : launch_bwd_tc<128, false>(q, k, v, dO, L_, D, acc, dk, dv, batch, q_heads,
                                                   kv_heads, seq_len, scale, st);
        else
            s = causal ? launch_bwd_tc<64, true>(q, k, v, dO, L_, D, acc, dk, dv, batch, q_heads,
                                                 kv_heads, seq_len, scale, st)
                       : launch_bwd_tc<64, false>(q, k, v, dO, L_, D, acc, dk, dv, batch, q_heads,
                                                  kv_heads, seq_len, scale, st);
        if (s) return s;
        const unsigned nb = (unsigned)((nel / 4 + 255) / 256);
        dq_convert_kernel<__nv_bfloat16><<<nb, 256, 0, st>>>(acc, (__nv_bfloat16*)dq,
                                                            (long long)nel);
        return edb::status_from_cuda(cudaGetLastError());
    }
    return dtype == EDB_BF16
               ? launch_bwd_simt<__nv_bfloat16>(q, k, v, dO, L_, D, dq, dk, dv, batch, q_heads,
                                                kv_heads, seq_len, head_dim, causal, scale, st)
               : launch_bwd_simt<float>(q, k, v, dO, L_, D, dq, dk, dv, batch, q_heads, kv_heads,
                                        seq_len, head_dim, causal, scale, st);
}

// ------------------------------------------------------------ FoX attention backward
extern "C" size_t edb_fox_attention_bwd_workspace(int dtype, int batch, int q_heads,
                                                  int kv_heads, int seq_len, int head_dim) {
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || seq_len <= 0 || head_dim <= 0) return 0;
    const size_t rows = (size_t)batch * q_heads * seq_len;
    size_t ws = a256(rows * 4) + a256(2 * rows * 4);  // D, the two cs partial halves
    if (tc_shape(dtype, head_dim)) ws += a256(rows * head_dim * 4);  // f32 dQ accumulator
    return ws;
}

extern "C" int edb_fox_attention_bwd(int dtype, const void* q, const void* k, const void* v,
                                     const float* cs, const void* o, const void* dO,
                                     const float* lse, void* dq, void* dk, void* dv, float* dcs,
                                     int batch, int q_heads, int kv_heads, int seq_len,
                                     int head_dim, float scale, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || seq_len <= 0 || head_dim <= 0)
        return EDB_ERR_BAD_SHAPE;
    if (q_heads % kv_heads != 0) return EDB_ERR_BAD_SHAPE;
    if (head_dim > 128) return EDB_ERR_UNSUPPORTED;
    if (!q || !k || !v || !cs || !o || !dO || !lse || !dq || !dk || !dv || !dcs)
        return EDB_ERR_NULL_POINTER;
    const size_t need = edb_fox_attention_bwd_workspace(dtype, batch, q_heads, kv_heads, seq_len,
                                                        head_dim);
    if (workspace_bytes < need || !workspace) return EDB_ERR_WORKSPACE_TOO_SMALL;
    if (!edb::aligned16(workspace)) return EDB_ERR_MISALIGNED;
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)head_dim);
    cudaStream_t st = (cudaStream_t)stream;
    const size_t rows = (size_t)batch * q_heads * seq_len;
    char* w = static_cast<char*>(workspace);
    float* D = reinterpret_cast<float*>(w);
    w += a256(rows * 4);
    float* part = reinterpret_cast<float*>(w);
    w += a256(2 * rows * 4);
    {
        dim3 blk(32, 4);
        const unsigned nb = (unsigned)((rows + 3) / 4);
        if (dtype == EDB_BF16)
            attn_bwd_rowdot_kernel<__nv_bfloat16><<<nb, blk, 0, st>>>(
                (const __nv_bfloat16*)o, (const __nv_bfloat16*)dO, D, (long long)rows, head_dim);
        else
            attn_bwd_rowdot_kernel<float><<<nb, blk, 0, st>>>((const float*)o, (const float*)dO, D,
                                                              (long long)rows, head_dim);
        if (cudaError_t e = cudaGetLastError()) return (int)e;
    }
    if (tc_shape(dtype, head_dim) && edb::aligned16(q) && edb::aligned16(k) &&
        edb::aligned16(v) && edb::aligned16(dO) && edb::aligned16(dk) && edb::aligned16(dv)) {
        // the tcgen05 kernel with the per-key-row bias and the dS column sums
        float* acc = reinterpret_cast<float*>(w);
        const size_t nel = rows * head_dim;
        cudaError_t e = cudaMemsetAsync(acc, 0, nel * 4, st);
        if (e != cudaSuccess) return (int)e;
        const int s = head_dim == 128
                          ? launch_bwd_tc<128, true, true>(q, k, v, dO, lse, D, acc, dk, dv, batch,
                                                           q_heads, kv_heads, seq_len, scale, st,
                                                           cs, part)
                          : launch_bwd_tc<64, true, true>(q, k, v, dO, lse, D, acc, dk, dv, batch,
                                                          q_heads, kv_heads, seq_len, scale, st,
                                                          cs, part);
        if (s) return s;
        const unsigned nb = (unsigned)((nel / 4 + 255) / 256);
        dq_convert_kernel<__nv_bfloat16><<<nb, 256, 0, st>>>(acc, (__nv_bfloat16*)dq,
                                                            (long long)nel);
        if ((e = cudaGetLastError()) != cudaSuccess) return (int)e;
        fox_dcs_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(part, dcs, (long long)rows,
                                                                     1.0f / scale);
        return edb::status_from_cuda(cudaGetLastError());
    }
    // SIMT kernels: other dtypes and head dims
    const int s =
        dtype == EDB_BF16
            ? launch_bwd_simt<__nv_bfloat16>(q, k, v, dO, lse, D, dq, dk, dv, batch, q_heads,
                                             kv_heads, seq_len, head_dim, 1, scale, st, cs, part)
            : launch_bwd_simt<float>(q, k, v, dO, lse, D, dq, dk, dv, batch, q_heads, kv_heads,
                                     seq_len, head_dim, 1, scale, st, cs, part);
    if (s) return s;
    fox_dcs_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(part, dcs, (long long)rows,
                                                                 1.0f / scale);
    return edb::status_from_cuda(cudaGetLastError());
}
