// flash_attn.cu -- scaled-dot-product attention forward (causal or full, GQA).
//
// Reference semantics (edifice project paths):
//   lib/edifice/cuda/fused_scan.ex:3476-3508 (flash_attention_fallback):
//     O = softmax(Q K^T * scale, -inf above the diagonal when causal) V
//   native/cuda/fused_flash_attention.cu:52-191 (equal heads, scale rsqrt(d)).
// GQA (new capability): q head h reads kv head h / (Hq / Hkv), the K/V repeat
// of lib/edifice/attention/gqa.ex:257-271.
//
// B200 path (bf16, head_dim 64 or 128): tcgen05 tensor cores with TMEM
// accumulators, TMA (SWIZZLE_128B, 3D tensor maps so rows past L are zero
// filled on load and clipped on store), warp-specialised CTA:
//   warps 0-3  softmax: thread r owns query row r = TMEM lane r; reads S with
//              tcgen05.ld, online softmax in the log2 domain (one ex2.approx per
//              score), lazy O rescale (only when the running max grows by more
//              than 8, i.e. P <= 256; decided per warp, since the TMEM load and
//              store need the whole warp), writes P (bf16, swizzled) to shared
//              memory, and at the end normalises O and stores it with TMA;
//   warp 4     TMA producer: Q once, then K_j / V_j through a 2-stage ring;
//   warp 5     MMA issuer (one thread): S_{j+1} = Q K_{j+1}^T is issued as soon
//              as the softmax has read S_j, so it overlaps the softmax of tile
//              j; O += P_j V_j after P_j lands.
// Tiles: 128 query rows x 64 kv rows; TMEM: S 64 columns + O head_dim
// columns (256 allocated), two CTAs per SM so one CTA's MMAs overlap the
// other's softmax.  Causal: kv tiles past the diagonal are never loaded; the
// grid runs the longest query tiles first.
//
// Other shapes (f32 io, other head dims) run a SIMT kernel with the same math.
#include <math.h>

#include "tc_common.cuh"

namespace {

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 64;   // kv rows per tile
constexpr int KV_STAGES = 2;
constexpr int kFwdThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnMaps {
    CUtensorMap q, k, v, o;
};

template <int HD>
struct FwdSmem {
    static constexpr int NB = HD / 64;                 // 64-column (128 B) boxes per row
    static constexpr int Q_BYTES = BM * HD * 2;        // also the O staging tile
    static constexpr int KV_BYTES = BN * HD * 2;       // one K or V tile
    static constexpr int P_BYTES = BM * BN * 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + KV_STAGES * KV_BYTES;
    static constexpr int OFF_P = OFF_V + KV_STAGES * KV_BYTES;
    static constexpr int OFF_BAR = OFF_P + P_BYTES;
    // barriers: q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full, s_free,
    // p_full, pv_done, mma_done.  K and V rings are separate: K_j is free once
    // S_j has been computed, V_j only after P_j V_j.
    static constexpr int NBAR = 1 + 4 * KV_STAGES + 5;
    static constexpr int TOTAL = OFF_BAR + NBAR * 8 + 16;
    static constexpr int TMEM_COLS = HD == 128 ? 256 : 128;
    static constexpr int TMEM_S = 0;
    static constexpr int TMEM_O = HD == 128 ? 128 : 64;
};

// ------------------------------------------------------------ tcgen05 forward
// STORE_O = false: only the row log-sum-exp is written (the backward's
// recompute when the caller has no lse from the forward).
// FOX: FoX attention (lib/edifice/cuda/fused_scan.ex:3796-3870), the score of
// key j less cs[b, h, j] (the cs_i of the query row cancels in the softmax and
// is left out of lse as well).  The bias is register arithmetic on values the
// softmax threads read with plain loads; the pipeline and its waits are the
// same as without it.
template <int HD, bool CAUSAL, bool STORE_O = true, bool FOX = false>
__global__ void __launch_bounds__(kFwdThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ AttnMaps maps, float* __restrict__ lse, int L,
                       int Hq, int Hkv, float scale_log2, unsigned* err,
                       const float* __restrict__ cs = nullptr) {
    using S = FwdSmem<HD>;
    constexpr int NB = S::NB;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sQ = smem + S::OFF_Q;
    uint8_t* sK = smem + S::OFF_K;
    uint8_t* sV = smem + S::OFF_V;
    uint8_t* sP = smem + S::OFF_P;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + KV_STAGES;
    uint64_t* v_full = k_empty + KV_STAGES;
    uint64_t* v_empty = v_full + KV_STAGES;
    uint64_t* s_full = bars + 1 + 4 * KV_STAGES;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_full + 2;
    uint64_t* pv_done = s_full + 3;
    uint64_t* mma_done = s_full + 4;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + S::NBAR);
    int* s_abort = reinterpret_cast<int*>(s_tmem + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nq = (L + BM - 1) / BM;
    // longest causal query tiles first within each (head, batch); taking the query
    // tile as the grid's slowest index instead (longest first across all heads)
    // measured no faster
    const int qt = CAUSAL ? nq - 1 - (int)blockIdx.x : (int)blockIdx.x;
    const int hq = blockIdx.y, b = blockIdx.z;
    const int hk = hq / (Hq / Hkv);
    const int bh = b * Hq + hq, bhk = b * Hkv + hk;
    const int q0 = qt * BM;
    const int nkv_all = (L + BN - 1) / BN;
    const int nkv = CAUSAL ? min(nkv_all, (q0 + BM + BN - 1) / BN) : nkv_all;

    if ((smem_u32(smem) & 1023u) != 0) {  // SWIZZLE_128B tiles need 1 KB alignment
        if (tid == 0) edb_flag_error(err, EDB_DEVERR_ATTN_PIPE);
        return;
    }
    if (warp == 5) {
        tc::tmem_alloc(s_tmem, S::TMEM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 128) {
        mbar_init(q_full, 1);
        for (int s = 0; s < KV_STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(p_full, 4);
        mbar_init(pv_done, 1);
        mbar_init(mma_done, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *s_tmem;

    if (warp == 4) {
        // ------------------------------------------------ TMA producer
        // lane 0: Q, then the K ring; lane 1: the V ring (independent waits)
        if (lane < 2) {
            const bool is_k = lane == 0;
            const CUtensorMap* map = is_k ? &maps.k : &maps.v;
            uint8_t* ring = is_k ? sK : sV;
            uint64_t* full = is_k ? k_full : v_full;
            uint64_t* empty = is_k ? k_empty : v_empty;
            prefetch_tmap(map);
            if (is_k) {
                prefetch_tmap(&maps.q);
                mbar_arrive_expect_tx(q_full, S::Q_BYTES);
                for (int bx = 0; bx < NB; ++bx)
                    tma_load_3d(sQ + bx * (BM * 128), &maps.q, q_full, bx * 64, q0, bh);
            }
            int issued = 0;
            for (int j = 0; j < nkv; ++j) {
                const int s = j % KV_STAGES;
                if (j >= KV_STAGES) {
                    if (*(volatile int*)s_abort) break;
                    if (!mbar_wait_bounded(&empty[s], ((j / KV_STAGES) - 1) & 1, err,
                                           EDB_DEVERR_ATTN_PIPE)) {
                        *(volatile int*)s_abort = 1;
                        break;
                    }
                }
                mbar_arrive_expect_tx(&full[s], S::KV_BYTES);
                for (int bx = 0; bx < NB; ++bx)
                    tma_load_3d(ring + s * S::KV_BYTES + bx * (BN * 128), map, &full[s], bx * 64,
                                (FOX ? nkv - 1 - j : j) * BN, bhk);
                issued = j + 1;
            }
            // make sure no copy is still landing when the CTA leaves (bounded)
            for (int j = max(0, issued - KV_STAGES); j < issued; ++j)
                mbar_wait_bounded(&full[j % KV_STAGES], (j / KV_STAGES) & 1, err,
                                  EDB_DEVERR_ATTN_PIPE);
            if (is_k) mbar_wait_bounded(q_full, 0, err, EDB_DEVERR_ATTN_PIPE);
        }
    } else if (warp == 5) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = tc::idesc_bf16(BM, BN, 0, 0);
            constexpr uint32_t idO = tc::idesc_bf16(BM, HD, 0, 1);
            const uint32_t tS = tmem + S::TMEM_S, tO = tmem + S::TMEM_O;
            auto issue_S = [&](int j) {
                const int s = j % KV_STAGES;
                const uint8_t* kb = sK + s * S::KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint64_t ad = tc::sdesc_sw128(sQ + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
                    const uint64_t bd = tc::sdesc_sw128(kb + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
                    tc::mma_bf16_ss(tS, ad, bd, idS, kk > 0);
                }
                tc::commit(s_full);
                tc::commit(&k_empty[s]);  // K_j may be reloaded once S_j is done
            };
            bool ok = mbar_wait_bounded(q_full, 0, err, EDB_DEVERR_ATTN_PIPE) &&
                      mbar_wait_bounded(&k_full[0], 0, err, EDB_DEVERR_ATTN_PIPE);
            if (ok) {
                tc::fence_after_sync();
                issue_S(0);
            }
            for (int j = 0; ok && j < nkv; ++j) {
                if (j + 1 < nkv) {
                    const int s1 = (j + 1) % KV_STAGES;
                    ok = mbar_wait_bounded(&k_full[s1], ((j + 1) / KV_STAGES) & 1, err,
                                           EDB_DEVERR_ATTN_PIPE) &&
                         mbar_wait_bounded(s_free, j & 1, err, EDB_DEVERR_ATTN_PIPE);
                    if (!ok) break;
                    tc::fence_after_sync();
                    issue_S(j + 1);
                }
                ok = mbar_wait_bounded(p_full, j & 1, err, EDB_DEVERR_ATTN_PIPE) &&
                     mbar_wait_bounded(&v_full[j % KV_STAGES], (j / KV_STAGES) & 1, err,
                                       EDB_DEVERR_ATTN_PIPE);
                if (!ok) break;
                tc::fence_after_sync();
                const uint8_t* vb = sV + (j % KV_STAGES) * S::KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    const uint64_t ad = tc::sdesc_sw128(sP + kk * 32, 16, 1024);
                    const uint64_t bd = tc::sdesc_sw128(vb + kk * 16 * 128, BN * 128, 1024);
                    tc::mma_bf16_ss(tO, ad, bd, idO, (j > 0 || kk > 0));
                }
                tc::commit(pv_done);
                tc::commit(&v_empty[j % KV_STAGES]);
            }
            if (!ok) *(volatile int*)s_abort = 1;
            // every MMA issued above has completed before TMEM is released
            tc::commit(mma_done);
            mbar_wait_bounded(mma_done, 0, err, EDB_DEVERR_ATTN_PIPE);
        }
    } else {
        // ------------------------------------------------ softmax warps 0-3
        const int row = warp * 32 + lane;  // TMEM lane == query row in the tile
        const int qrow = q0 + row;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        const uint32_t tS = tmem + S::TMEM_S + lane_base;
        const uint32_t tO = tmem + S::TMEM_O + lane_base;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        // Every go / give-up decision below is taken by the whole warp (__all_sync):
        // a lane that left the loop alone would leave the others in tcgen05.ld.
        for (int j = 0; j < nkv; ++j) {
            const bool got = !*(volatile int*)s_abort &&
                             mbar_wait_bounded(s_full, j & 1, err, EDB_DEVERR_ATTN_PIPE);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            uint32_t sr[2][32];
            tc::tmem_ld32(tS, sr[0]);
            tc::tmem_ld32(tS + 32, sr[1]);
            tc::tmem_wait_ld();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);

            // FoX visits the kv tiles newest first: its bias -cs_j grows with j, so
            // the first tile sets each row's max and later tiles rarely raise it
            // (oldest first, every tile would rescale O)
            const int kv0 = (FOX ? nkv - 1 - j : j) * BN;
            // x: the raw scores (FoX: s scale - cs_j, natural units); xs scales x
            // into the log2 domain inside the exponent's FFMA, so the max runs on x
            // and no separate multiply is spent per score
            float x[BN];
            const float xs = FOX ? kLog2e : scale_log2;
            // only the diagonal tiles and a ragged last tile need a mask (CTA-uniform)
            const bool need_mask = (kv0 + BN > L) || (CAUSAL && kv0 + BN - 1 > q0);
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < BN; ++c) {
                    const int kv = kv0 + c;
                    const bool masked = kv >= L || (CAUSAL && kv > qrow);
                    x[c] = masked ? -INFINITY : __uint_as_float(sr[c >> 5][c & 31]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < BN; ++c) x[c] = __uint_as_float(sr[c >> 5][c & 31]);
            }
            if (FOX) {
                // x_j = s_j scale - cs_j, one FFMA per score; 16-byte loads when the
                // row is aligned and the tile lies inside L (the same addresses for
                // every thread: broadcast).  Masked scores stay -inf.
                const float sc = scale_log2 * kLn2;
                const float* cr = cs + (long long)bh * L + kv0;
                // the next tile's 256 bytes of cs into L1 ahead of use
                if (lane < 2 && kv0 >= BN)
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(cr - BN + 32 * lane));
                if (kv0 + BN <= L && ((reinterpret_cast<uintptr_t>(cr) & 15) == 0)) {
                    const float2 sc2 = dup2(sc);
#pragma unroll
                    for (int c4 = 0; c4 < BN / 4; ++c4) {
                        const float4 v = __ldg(reinterpret_cast<const float4*>(cr) + c4);
                        const float2 lo = fma2(make_float2(x[4 * c4], x[4 * c4 + 1]), sc2,
                                               make_float2(-v.x, -v.y));
                        const float2 hi = fma2(make_float2(x[4 * c4 + 2], x[4 * c4 + 3]), sc2,
                                               make_float2(-v.z, -v.w));
                        x[4 * c4] = lo.x;
                        x[4 * c4 + 1] = lo.y;
                        x[4 * c4 + 2] = hi.x;
                        x[4 * c4 + 3] = hi.y;
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < BN; ++c)
                        x[c] = kv0 + c < L ? fmaf(x[c], sc, -__ldg(cr + c)) : -INFINITY;
                }
            }
            // 4 independent max chains, two scores per three-input max
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < BN; c += 2) mx4[(c >> 1) & 3] = tc::fmax3(mx4[(c >> 1) & 3], x[c], x[c + 1]);
            const float mt = tc::fmax3(fmaxf(mx4[0], mx4[1]), mx4[2], mx4[3]) * xs;
            const float m_new = fmaxf(m_used, mt);
            // Each row decides for itself whether its max grew by more than 8; the
            // O rescale below is tcgen05.ld/st, which the whole warp must execute
            // together (.sync.aligned), so the warp rescales when any of its rows
            // needs it and the other rows multiply by alpha = 1.  A lane-divergent
            // rescale leaves the warp stalled in tcgen05.ld.
            float alpha = 1.0f;
            bool grow = false;
            if (j == 0) {
                m_used = m_new;
            } else if (m_new > m_used + 8.0f) {
                alpha = tc::ex2(m_used - m_new);
                m_used = m_new;
                grow = true;
            }
            const bool rescale = __any_sync(0xffffffffu, grow);
            // P_j in registers first: its exps overlap P_{j-1} V_{j-1} on the tensor
            // core; only the O rescale and the P stores wait for that product
            const float nmu = m_used == -INFINITY ? 0.0f : -m_used;
            // exponent arguments and row sums in packed f32x2 arithmetic
            const float2 xs2 = dup2(xs), nmu2 = dup2(nmu);
            float2 rs2[2] = {dup2(0.0f), dup2(0.0f)};
            uint4 pv[BN / 8];
#pragma unroll
            for (int ch = 0; ch < BN / 8; ++ch) {
                float p[8];
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const float2 a = fma2(make_float2(x[ch * 8 + e], x[ch * 8 + e + 1]), xs2, nmu2);
                    p[e] = tc::ex2(a.x);
                    p[e + 1] = tc::ex2(a.y);
                    rs2[(e >> 1) & 1] = add2(rs2[(e >> 1) & 1], make_float2(p[e], p[e + 1]));
                }
                pv[ch] = make_uint4(tc::pack_bf16x2(p[0], p[1]), tc::pack_bf16x2(p[2], p[3]),
                                    tc::pack_bf16x2(p[4], p[5]), tc::pack_bf16x2(p[6], p[7]));
            }
            // P buffer and O are free once PV_{j-1} has completed
            if (j > 0 && !__all_sync(0xffffffffu, mbar_wait_bounded(pv_done, (j - 1) & 1, err,
                                                                    EDB_DEVERR_ATTN_PIPE))) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            if (rescale) {
                l *= alpha;
#pragma unroll
                for (int cc = 0; cc < HD / 32; ++cc) {
                    uint32_t o[32];
                    tc::tmem_ld32(tO + cc * 32, o);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tc::tmem_st32(tO + cc * 32, o);
                }
                tc::tmem_wait_st();
            }
            uint8_t* prow = sP;
#pragma unroll
            for (int ch = 0; ch < BN / 8; ++ch)
                *reinterpret_cast<uint4*>(prow + tc::sw128_off(row, ch)) = pv[ch];
            l += (rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y);
            fence_proxy_async();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        // ---- epilogue: O / l -> bf16 -> smem (Q tile region, swizzled) -> TMA store
        if (__all_sync(0xffffffffu,
                       ok && mbar_wait_bounded(pv_done, (nkv - 1) & 1, err, EDB_DEVERR_ATTN_PIPE))) {
            tc::fence_after_sync();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
            for (int cc = 0; cc < (STORE_O ? HD / 32 : 0); ++cc) {
                uint32_t o[32];
                tc::tmem_ld32(tO + cc * 32, o);
                tc::tmem_wait_ld();
                uint8_t* box = sQ + (cc >> 1) * (BM * 128);
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    const int chunk = (cc & 1) * 4 + ch;
                    const uint4 v = make_uint4(
                        tc::pack_bf16x2(__uint_as_float(o[ch * 8 + 0]) * inv, __uint_as_float(o[ch * 8 + 1]) * inv),
                        tc::pack_bf16x2(__uint_as_float(o[ch * 8 + 2]) * inv, __uint_as_float(o[ch * 8 + 3]) * inv),
                        tc::pack_bf16x2(__uint_as_float(o[ch * 8 + 4]) * inv, __uint_as_float(o[ch * 8 + 5]) * inv),
                        tc::pack_bf16x2(__uint_as_float(o[ch * 8 + 6]) * inv, __uint_as_float(o[ch * 8 + 7]) * inv));
                    *reinterpret_cast<uint4*>(box + tc::sw128_off(row, chunk)) = v;
                }
            }
            if (lse != nullptr && qrow < L)
                lse[(long long)bh * L + qrow] = (m_used + log2f(l)) * kLn2;
            fence_proxy_async();
        } else {
            *(volatile int*)s_abort = 1;
        }
        // every softmax warp reaches this barrier, whether or not its waits succeeded
        // (a warp that gave up must not leave the others waiting); the tile is stored
        // only when none gave up
        tc::named_bar(1, 128);
        if (STORE_O && tid == 0 && *(volatile int*)s_abort == 0) {
            prefetch_tmap(&maps.o);
            for (int bx = 0; bx < NB; ++bx)
                tc::tma_store_3d(&maps.o, sQ + bx * (BM * 128), bx * 64, q0, bh);
            tc::tma_store_commit();
            tc::tma_store_wait_all();
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 5) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

// ------------------------------------------------------------ SIMT forward
// One thread per query row; K/V tiles of 32 rows staged in shared memory (f32).
template <typename T, int HDMAX>
__global__ void __launch_bounds__(128)
    attn_fwd_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                         T* __restrict__ o, float* __restrict__ lse, int L, int Hq, int Hkv, int d,
                         int causal, float scale, const float* __restrict__ cs = nullptr) {
    constexpr int TK = 32;
    __shared__ float sk[TK][HDMAX];
    __shared__ float sv[TK][HDMAX];
    const int hq = blockIdx.y, b = blockIdx.z;
    const int hk = hq / (Hq / Hkv);
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = i < L;
    const T* qi = q + (((long long)b * Hq + hq) * L + (live ? i : 0)) * d;
    const T* kb = k + ((long long)b * Hkv + hk) * L * d;
    const T* vb = v + ((long long)b * Hkv + hk) * L * d;
    float qv[HDMAX], acc[HDMAX];
    for (int e = 0; e < HDMAX; ++e) {
        qv[e] = (live && e < d) ? ld_scalar<T>(qi + e) * scale * kLog2e : 0.0f;
        acc[e] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const int blk_last = blockIdx.x * blockDim.x + blockDim.x - 1;
    const int jend = causal ? min(L, blk_last + 1) : L;
    for (int j0 = 0; j0 < jend; j0 += TK) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < TK * HDMAX; idx += blockDim.x) {
            const int r = idx / HDMAX, e = idx % HDMAX;
            const bool okr = j0 + r < L && e < d;
            sk[r][e] = okr ? ld_scalar<T>(kb + (long long)(j0 + r) * d + e) : 0.0f;
            sv[r][e] = okr ? ld_scalar<T>(vb + (long long)(j0 + r) * d + e) : 0.0f;
        }
        __syncthreads();
        if (!live) continue;
        const int rmax = min(TK, L - j0);
        for (int r = 0; r < rmax; ++r) {
            const int j = j0 + r;
            if (causal && j > i) break;
            float s = 0.0f;
            for (int e = 0; e < HDMAX; ++e) s = fmaf(qv[e], sk[r][e], s);
            if (cs != nullptr) s = fmaf(-cs[((long long)b * Hq + hq) * L + j], kLog2e, s);
            const float mn = fmaxf(m, s);
            const float a = exp2f(m - mn), p = exp2f(s - mn);
            l = l * a + p;
            for (int e = 0; e < HDMAX; ++e) acc[e] = fmaf(acc[e], a, p * sv[r][e]);
            m = mn;
        }
    }
    if (!live) return;
    T* oi = o + (((long long)b * Hq + hq) * L + i) * d;
    const float inv = 1.0f / l;
    for (int e = 0; e < d; ++e) st_scalar<T>(oi + e, acc[e] * inv);
    if (lse) lse[((long long)b * Hq + hq) * L + i] = (m + log2f(l)) * kLn2;
}

// ------------------------------------------------------------ launch
int make_map3(CUtensorMap* m, const void* p, int d, int L, int nbh, int box_rows) {
    return tc::make_attn_map(m, p, d, L, nbh, box_rows);
}

template <int HD, bool CAUSAL, bool STORE_O = true, bool FOX = false>
int launch_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                  int Hkv, int L, float scale, cudaStream_t st, const float* cs = nullptr) {
    AttnMaps maps;
    int s;
    if ((s = make_map3(&maps.q, q, HD, L, B * Hq, BM))) return s;
    if ((s = make_map3(&maps.k, k, HD, L, B * Hkv, BN))) return s;
    if ((s = make_map3(&maps.v, v, HD, L, B * Hkv, BN))) return s;
    if ((s = make_map3(&maps.o, o, HD, L, B * Hq, BM))) return s;
    auto kern = attn_fwd_tc_kernel<HD, CAUSAL, STORE_O, FOX>;
    const int smem = FwdSmem<HD>::TOTAL;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    dim3 grid((L + BM - 1) / BM, Hq, B);
    kern<<<grid, kFwdThreads, smem, st>>>(maps, lse, L, Hq, Hkv, scale * kLog2e,
                                          edb::device_error_word(), cs);
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T>
int launch_fwd_simt(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                    int Hq, int Hkv, int L, int d, int causal, float scale, cudaStream_t st,
                    const float* cs = nullptr) {
    dim3 grid((L + 127) / 128, Hq, B);
    if (d <= 32)
        attn_fwd_simt_kernel<T, 32><<<grid, 128, 0, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                          (T*)o, lse, L, Hq, Hkv, d, causal, scale,
                                                          cs);
    else if (d <= 64)
        attn_fwd_simt_kernel<T, 64><<<grid, 128, 0, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                          (T*)o, lse, L, Hq, Hkv, d, causal, scale,
                                                          cs);
    else
        attn_fwd_simt_kernel<T, 128><<<grid, 128, 0, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                           (T*)o, lse, L, Hq, Hkv, d, causal, scale,
                                                           cs);
    return edb::status_from_cuda(cudaGetLastError());
}

}  // namespace

// Row log-sum-exp only (bf16, head_dim 64/128), for the backward when the
// caller did not keep the forward's lse.  Library-internal.
int edb_attn_fwd_lse_only(int head_dim, int causal, const void* q, const void* k, float* lse,
                          int B, int Hq, int Hkv, int L, float scale, cudaStream_t st) {
    // the V operand is read by the PV MMAs; K stands in for it (O is not stored)
    if (head_dim == 128)
        return causal ? launch_fwd_tc<128, true, false>(q, k, k, const_cast<void*>(q), lse, B, Hq,
                                                        Hkv, L, scale, st)
                      : launch_fwd_tc<128, false, false>(q, k, k, const_cast<void*>(q), lse, B,
                                                         Hq, Hkv, L, scale, st);
    return causal ? launch_fwd_tc<64, true, false>(q, k, k, const_cast<void*>(q), lse, B, Hq, Hkv,
                                                   L, scale, st)
                  : launch_fwd_tc<64, false, false>(q, k, k, const_cast<void*>(q), lse, B, Hq,
                                                    Hkv, L, scale, st);
}

extern "C" int edb_flash_attention_fwd(int dtype, const void* q, const void* k, const void* v,
                                       void* o, float* lse, int batch, int q_heads, int kv_heads,
                                       int seq_len, int head_dim, int causal, float scale,
                                       void* stream) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || seq_len <= 0 || head_dim <= 0)
        return EDB_ERR_BAD_SHAPE;
    if (q_heads % kv_heads != 0) return EDB_ERR_BAD_SHAPE;
    if (head_dim > 128) return EDB_ERR_UNSUPPORTED;
    if (!q || !k || !v || !o) return EDB_ERR_NULL_POINTER;
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)head_dim);
    cudaStream_t st = (cudaStream_t)stream;
    const bool tc_ok = dtype == EDB_BF16 && (head_dim == 64 || head_dim == 128) &&
                       edb::aligned16(q) && edb::aligned16(k) && edb::aligned16(v) &&
                       edb::aligned16(o) && (long long)batch * q_heads < (1LL << 31);
    if (tc_ok) {
        if (head_dim == 128)
            return causal ? launch_fwd_tc<128, true>(q, k, v, o, lse, batch, q_heads, kv_heads,
                                                     seq_len, scale, st)
                          : launch_fwd_tc<128, false>(q, k, v, o, lse, batch, q_heads, kv_heads,
                                                      seq_len, scale, st);
        return causal ? launch_fwd_tc<64, true>(q, k, v, o, lse, batch, q_heads, kv_heads, seq_len,
                                                scale, st)
                      : launch_fwd_tc<64, false>(q, k, v, o, lse, batch, q_heads, kv_heads,
                                                 seq_len, scale, st);
    }
    return dtype == EDB_BF16
               ? launch_fwd_simt<__nv_bfloat16>(q, k, v, o, lse, batch, q_heads, kv_heads, seq_len,
                                                head_dim, causal, scale, st)
               : launch_fwd_simt<float>(q, k, v, o, lse, batch, q_heads, kv_heads, seq_len,
                                        head_dim, causal, scale, st);
}

// ------------------------------------------------------------ FoX attention forward
// The shapes FoX runs on tensor cores (the plain flash kernels' condition).
static bool fox_tc_shape(int dtype, int d, const void* q, const void* k, const void* v,
                         const void* o) {
    return dtype == EDB_BF16 && (d == 64 || d == 128) && edb::aligned16(q) && edb::aligned16(k) &&
           edb::aligned16(v) && edb::aligned16(o);
}

extern "C" int edb_fox_attention_fwd(int dtype, const void* q, const void* k, const void* v,
                                     const float* cs, void* o, float* lse, int B, int Hq, int Hkv,
                                     int L, int d, float scale, void* stream) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || L <= 0 || d <= 0) return EDB_ERR_BAD_SHAPE;
    if (Hq % Hkv != 0) return EDB_ERR_BAD_SHAPE;
    if (d > 128) return EDB_ERR_UNSUPPORTED;
    if (!q || !k || !v || !cs || !o || !lse) return EDB_ERR_NULL_POINTER;
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)d);
    cudaStream_t st = (cudaStream_t)stream;
    // bf16, head_dim 64/128: the tcgen05 kernel with the bias in its softmax warps
    if (fox_tc_shape(dtype, d, q, k, v, o)) {
        return d == 128 ? launch_fwd_tc<128, true, true, true>(q, k, v, o, lse, B, Hq, Hkv, L,
                                                               scale, st, cs)
                        : launch_fwd_tc<64, true, true, true>(q, k, v, o, lse, B, Hq, Hkv, L,
                                                              scale, st, cs);
    }
    return dtype == EDB_BF16
               ? launch_fwd_simt<__nv_bfloat16>(q, k, v, o, lse, B, Hq, Hkv, L, d, 1, scale, st,
                                                cs)
               : launch_fwd_simt<float>(q, k, v, o, lse, B, Hq, Hkv, L, d, 1, scale, st, cs);
}
