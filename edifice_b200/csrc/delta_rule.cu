// delta_rule.cu -- DeltaNet delta rule, forward + backward (recurrent path).
//
// Reference semantics (edifice project paths):
//   forward   lib/edifice/cuda/fused_scan.ex:2212-2236 (delta_net_scan_fallback)
//             == lib/edifice/recurrent/delta_net.ex:231-273:
//             r = S_{t-1} k_t;  S_t = S_{t-1} + (beta_t (.) (v_t - r)) k_t^T;  o_t = S_t q_t
//   backward  fused_scan.ex:1257-1326 (delta_rule_backward_fallback), with the
//             through-retrieval key gradient taken as S_{t-1}^T (beta (.) dS k) --
//             the exact gradient, as in native/cuda/fused_delta_rule_scan_backward.cu
//             and torch autograd of test/fixtures/numerical/delta_net_random; the Nx
//             fallback scales S_{t-1}^T dS k by beta over the key index instead,
//             which only agrees when beta is the same for every row.
// q, k, v, o: [B, L, H, d]; beta: [B, L, H, d] (per element, the model's form,
// delta_net.ex:285-297) or [B, L, H] (one gate per token and head).
//
// GatedDeltaNet (fused_scan.ex:2256-2284, 1347-1431; gated_delta_net.ex:300-350)
// adds a decay alpha [B, L, H] per token and head: S_d = alpha_t S_{t-1},
// r = S_d k_t, S_t = S_d + (beta_t (.) (v_t - r)) k_t^T; its gradients add
// dalpha_t = <dS_d, S_{t-1}> and dS_{t-1} = alpha_t dS_d.
//
// This file is the general path (any d <= 128, either beta form, f32 or bf16
// io; the chunked tensor-core form in delta_chunked*.cu takes bf16, d = 128 and
// one beta per token of the ungated rule).  Forward and backward are
// row-parallel: each row of S (and of dS) evolves on its own, so a row lives in
// the registers of 4 lanes, and only the gradients that sum over rows (gq, gk,
// galpha, a per-token gbeta) couple them.  The forward can write S at the start
// of every CK-token chunk (plus the final state); the backward rebuilds the
// states it needs from those checkpoints by recomputing forward, never by
// undoing an update (that divides by alpha_t in the gated rule, which amplifies
// rounding by 1/alpha per token).
#include <math.h>

#include "edb_common.cuh"

namespace {

constexpr int CK = 64;   // tokens per forward staging chunk
constexpr int CKP = 16;  // tokens between the state checkpoints the forward writes

template <typename T>
static __device__ __forceinline__ float ldv(const T* p) {
    return ld_scalar<T>(p);
}

// Forward, row-parallel.  Each row i of S (value index) evolves on its own in
// the forward: S[i] <- alpha S[i] + beta_i (v_i - alpha S[i].k) k^T,
// o_i = S[i].q, so a row lives in the registers of LPR lanes (CPL columns each:
// 8 x 16 for d > 32, 4 x 8 for d <= 32) and no block barrier is needed per token;
// k, q and the CTA's rows of v, beta (and alpha) are staged in shared memory one
// CK-token chunk at a time.  grid (H, B, ceil(d / 32)), 32 rows x LPR lanes per CTA.
// Shared memory (dynamic): k, q [CK][LPR][CPL + 4] (a pad of 4 floats per lane's
// slice puts the slices of one token on different banks) | v, beta, o [CK][32] |
// alpha [CK].
constexpr int kRowsPerCta = 32;

template <int CPL, int LPR>
constexpr size_t fwd_rows_smem() {
    return ((size_t)2 * CK * LPR * (CPL + 4) + 3 * CK * kRowsPerCta + CK) * sizeof(float);
}

template <typename T, int CPL, int LPR, bool GATED>
__global__ void __launch_bounds__(32 * LPR)
    delta_fwd_rows_kernel(const T* __restrict__ q, const T* __restrict__ k,
                          const T* __restrict__ v, const T* __restrict__ beta,
                          const T* __restrict__ alpha, T* __restrict__ o,
                          float* __restrict__ ckpt, int L, int H, int d, int beta_scalar) {
    constexpr int NT = 32 * LPR;      // threads
    constexpr int W = LPR * CPL;      // columns per CTA
    constexpr int SP = CPL + 4;       // floats per lane slice (padded)
    constexpr int RP = LPR * SP;      // floats per staged token row
    extern __shared__ __align__(16) float smf[];
    float* sk = smf;                        // [CK][RP]
    float* sq = sk + CK * RP;               // [CK][RP]
    float* sv = sq + CK * RP;               // [CK][32]
    float* sb = sv + CK * kRowsPerCta;      // [CK][32]
    float* so = sb + CK * kRowsPerCta;      // [CK][32]
    float* sa = so + CK * kRowsPerCta;      // [CK]
    const int h = blockIdx.x, b = blockIdx.y, rb = blockIdx.z * kRowsPerCta;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rl = warp * (32 / LPR) + lane / LPR;  // local row
    const int i = rb + rl;                  // value-dim row of S
    const int part = lane % LPR;            // column slice [part CPL, part CPL + CPL)
    const int c0 = part * CPL;
    const bool row_ok = i < d;
    const long long rs = (long long)H * d;  // token stride
    const long long base = (long long)b * L * rs + (long long)h * d;
    const int ncp = (L + CKP - 1) / CKP;
    float* ck_row = ckpt != nullptr && row_ok
                        ? ckpt + ((long long)b * H + h) * (ncp + 1) * d * d + (long long)i * d
                        : nullptr;
    float S[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) S[c] = 0.0f;
    // 16-byte stores when the row slice lies inside d and d % 4 == 0 (so the slice starts
    // on a 16-byte boundary), scalar stores otherwise
    const bool vec_ok = d % 4 == 0 && c0 + CPL <= d;
    auto save_state = [&](int slot) {
        if (ck_row == nullptr) return;
        float* dst = ck_row + (long long)slot * d * d + c0;
        if (vec_ok) {
#pragma unroll
            for (int c = 0; c < CPL; c += 4)
                *reinterpret_cast<float4*>(dst + c) = make_float4(S[c], S[c + 1], S[c + 2], S[c + 3]);
        } else {
#pragma unroll
            for (int c = 0; c < CPL; ++c)
                if (c0 + c < d) dst[c] = S[c];
        }
    };

    for (int t0 = 0; t0 < L; t0 += CK) {
        const int tn = min(CK, L - t0);
        __syncthreads();  // the previous chunk's stage is consumed
        // ---- stage this chunk (loads batched per thread before the stores)
        for (int base_idx = 0; base_idx < CK * W; base_idx += NT * 8) {
            float fk[8], fq[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int idx = base_idx + tid + u * NT;
                const int tt = idx / W, c = idx % W;
                const bool ok = tt < tn && c < d;
                const long long off = base + (long long)(t0 + tt) * rs + c;
                fk[u] = ok ? ldv(k + off) : 0.0f;
                fq[u] = ok ? ldv(q + off) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int idx = base_idx + tid + u * NT;
                const int tt = idx / W, c = idx % W;
                if (tt < CK) {
                    const int so_ = tt * RP + (c / CPL) * SP + c % CPL;
                    sk[so_] = fk[u];
                    sq[so_] = fq[u];
                }
            }
        }
        for (int idx = tid; idx < CK * kRowsPerCta; idx += NT) {
            const int tt = idx / kRowsPerCta, r = idx % kRowsPerCta;
            const bool ok = tt < tn && rb + r < d;
            const long long off = base + (long long)(t0 + tt) * rs + rb + r;
            sv[idx] = ok ? ldv(v + off) : 0.0f;
            sb[idx] = !ok ? 0.0f
                          : beta_scalar ? ldv(beta + ((long long)b * L + t0 + tt) * H + h)
                                        : ldv(beta + off);
        }
        if (GATED)
            for (int tt = tid; tt < CK; tt += NT)
                sa[tt] = tt < tn ? ldv(alpha + ((long long)b * L + t0 + tt) * H + h) : 1.0f;
        __syncthreads();
        // ---- the chunk's tokens, row by row in registers
        for (int tt = 0; tt < tn; ++tt) {
            if (tt % CKP == 0) save_state((t0 + tt) / CKP);
            const float* kr = sk + tt * RP + part * SP;
            const float* qr = sq + tt * RP + part * SP;
            // row dots as packed f32x2 FMAs into two accumulators: short dependency
            // chains ahead of the shuffles (the per-token step is latency-bound)
            float2 ra = make_float2(0.0f, 0.0f), rc = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int c = 0; c < CPL; c += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + c);
                ra = fma2(make_float2(S[c], S[c + 1]), make_float2(k4.x, k4.y), ra);
                rc = fma2(make_float2(S[c + 2], S[c + 3]), make_float2(k4.z, k4.w), rc);
            }
            float r = (ra.x + ra.y) + (rc.x + rc.y);
#pragma unroll
            for (int o2 = 1; o2 < LPR; o2 <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o2);
            const float al = GATED ? sa[tt] : 1.0f;
            const float u = sb[tt * kRowsPerCta + rl] * (sv[tt * kRowsPerCta + rl] - al * r);
            const float2 u2 = make_float2(u, u), al2 = make_float2(al, al);
            float2 oa = make_float2(0.0f, 0.0f), oc = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int c = 0; c < CPL; c += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + c);
                const float4 q4 = *reinterpret_cast<const float4*>(qr + c);
                float2 s0 = make_float2(S[c], S[c + 1]), s1 = make_float2(S[c + 2], S[c + 3]);
                if (GATED) {
                    s0 = mul2(al2, s0);
                    s1 = mul2(al2, s1);
                }
                s0 = fma2(u2, make_float2(k4.x, k4.y), s0);
                s1 = fma2(u2, make_float2(k4.z, k4.w), s1);
                S[c] = s0.x;
                S[c + 1] = s0.y;
                S[c + 2] = s1.x;
                S[c + 3] = s1.y;
                oa = fma2(s0, make_float2(q4.x, q4.y), oa);
                oc = fma2(s1, make_float2(q4.z, q4.w), oc);
            }
            float ov = (oa.x + oa.y) + (oc.x + oc.y);
#pragma unroll
            for (int o2 = 1; o2 < LPR; o2 <<= 1) ov += __shfl_xor_sync(0xffffffffu, ov, o2);
            if (part == 0) so[tt * kRowsPerCta + rl] = ov;
        }
        __syncthreads();
        for (int idx = tid; idx < tn * kRowsPerCta; idx += NT) {
            const int tt = idx / kRowsPerCta, r = idx % kRowsPerCta;
            if (rb + r < d) st_scalar<T>(o + base + (long long)(t0 + tt) * rs + rb + r, so[idx]);
        }
    }
    save_state(ncp);
}

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t ckpt_bytes(int B, int L, int H, int d) {
    const int ncp = (L + CKP - 1) / CKP;
    return (size_t)B * H * (ncp + 1) * d * d * sizeof(float);
}

// ---------------------------------------------------------------- backward, row-parallel
// The rows of S and of dS evolve independently in the backward as well.  For
// row i (value index) and token t, with P = S_{t-1}[i], S = S_t[i]:
//   dS[i] += dO_t[i] q_t;  r_i = P.k_t;  err_i = v_i - alpha_t r_i;  u_i = beta_i err_i
//   dsk_i = dS[i].k_t;  gv_i = beta_i dsk_i;  gbeta_i = err_i dsk_i   (per-element beta)
//   x = dS[i] - beta_i dsk_i k_t;  dS[i] <- alpha_t x  (the gradient w.r.t. S_{t-1}[i])
// Only gq = S_t^T dO_t, gk = dS_t^T u - alpha_t S_{t-1}^T (beta (.) dsk), galpha = <x, P>
// summed over rows, and a per-token beta's gradient, couple the rows.
// grid (H, B, ceil(d / 32)), 32 rows per CTA, LPR lanes of CPL columns per row: 8 lanes
// of 16 columns for d > 32 (256 threads: twice the forward's warps, for latency hiding),
// 4 lanes of 8 columns for d <= 32.  The forward's checkpoints are SB = CKP tokens
// apart; per checkpoint piece, last first: forward over the piece from its checkpoint
// writing every S_{t-1} row slice to a per-CTA scratch (sbuf: 256 KB per CTA at d = 128,
// L2-resident; each thread reads back only what it wrote), then backward over the piece
// reading them back.  Row sums: per token, a lane's 2 CPL partials
// are summed over the rows of its warp that share its column slice by recursive
// halving, the warps' sums meet in shared memory every RB tokens, and one partial per
// (row block, token, head) goes to global memory, where delta_rows_reduce_kernel adds
// the row blocks in a fixed order.
constexpr int SB = CKP;  // tokens per backward piece: one checkpoint interval

// Sums v over the lanes that differ in bits 5 - ROUNDS .. 4 (the rows of a warp that
// share a column slice: 8 rows at 4 lanes per row, 4 rows at 8).  Recursive halving:
// on return v[0 .. NV >> ROUNDS) holds the totals of the values starting at
// halving_base(lane) (bit 4 -> NV/2, bit 3 -> NV/4, bit 2 -> NV/8).
template <int NV, int ROUNDS>
static __device__ __forceinline__ void rows_halving_sum(float (&v)[NV], int lane) {
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
        const int m = 16 >> r;          // lane mask of this round
        const int hn = NV >> (r + 1);   // values kept after this round
        const bool up = (lane & m) != 0;
#pragma unroll
        for (int j = 0; j < hn; ++j) {
            const float send = up ? v[j] : v[j + hn];
            const float keep = up ? v[j + hn] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
    }
}
template <int ROUNDS>
static __device__ __forceinline__ int halving_base(int lane, int nv) {
    int base = 0;
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r)
        if (lane & (16 >> r)) base += nv >> (r + 1);
    return base;
}

// LPR lanes per row of S, CPL columns each; 32 rows per CTA, so LPR warps.
template <int CPL, int LPR>
struct RowsBwdSmem {
    static constexpr int NT = 32 * LPR, NW = LPR;
    static constexpr int ROUNDS = LPR == 4 ? 3 : LPR == 8 ? 2 : 1;  // halving rounds
    static constexpr int SP = CPL + 4, RP = LPR * SP, W = LPR * CPL;  // W: columns per CTA
    // per warp and token: [gq | gk][LPR slices][CPL + 1], the halves LPR (CPL + 1) + 8
    // apart, then galpha and a per-token gbeta: the skews put the 32 lanes' stores of one
    // halving result on 32 different banks
    static constexpr int SLICE = CPL + 1, HALF = LPR * SLICE + 8;
    static constexpr int RED = 2 * HALF + 2;
    // tokens per cross-warp reduction, and 2 RB slots: a token's gq arrives one step
    // after its gk
    static constexpr int RB = LPR == 4 ? 8 : LPR == 8 ? 4 : 2, NSLOT = 2 * RB;
    static constexpr size_t floats = (size_t)2 * SB * RP + 5 * SB * kRowsPerCta + SB +
                                     (size_t)NSLOT * NW * RED;
    static constexpr size_t bytes = floats * sizeof(float);
};

// per-CTA scratch floats: SB token states of 32 rows x W columns
template <int CPL, int LPR>
constexpr size_t rows_scratch_floats() {
    return (size_t)SB * 32 * LPR * CPL;
}

template <typename T, int CPL, int LPR, bool GATED>
__global__ void __launch_bounds__(32 * LPR, 2)
    delta_bwd_rows_kernel(const T* __restrict__ q, const T* __restrict__ k,
                          const T* __restrict__ v, const T* __restrict__ beta,
                          const T* __restrict__ alpha, const T* __restrict__ dO,
                          const float* __restrict__ ckpt, float* scratch,
                          float* __restrict__ part, float* __restrict__ part_s,
                          T* __restrict__ gv, T* __restrict__ gbeta, int B, int L, int H, int d,
                          int beta_scalar) {
    using G = RowsBwdSmem<CPL, LPR>;
    constexpr int NT = G::NT, NW = G::NW, ROUNDS = G::ROUNDS;
    constexpr int SP = G::SP, RP = G::RP, W = G::W, RED = G::RED;
    constexpr int SLICE = G::SLICE, HALF = G::HALF, RB = G::RB, NSLOT = G::NSLOT;
    static_assert(SB % NSLOT == 0, "red slots are indexed by the token's place in its piece");
    constexpr int NV = 2 * CPL;  // gq | gk partials of one lane
    constexpr int NP = CPL / 2;  // packed f32 pairs per row slice
    extern __shared__ __align__(16) float smf[];
    float* sk = smf;                       // [SB][RP]
    float* sq = sk + SB * RP;              // [SB][RP]
    float* sv = sq + SB * RP;              // [SB][32]
    float* sb = sv + SB * kRowsPerCta;     // [SB][32]
    float* sdo = sb + SB * kRowsPerCta;    // [SB][32]
    float* sgv = sdo + SB * kRowsPerCta;   // [SB][32] staged gv
    float* sgb = sgv + SB * kRowsPerCta;   // [SB][32] staged per-element gbeta
    float* sa = sgb + SB * kRowsPerCta;    // [SB]
    float* red = sa + SB;                  // [NSLOT][NW warps][RED]
    const int h = blockIdx.x, b = blockIdx.y, z = blockIdx.z, rb = z * kRowsPerCta;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rl = warp * (32 / LPR) + lane / LPR;
    const int i = rb + rl;
    const int part_ix = lane % LPR;
    const int c0 = part_ix * CPL;
    const bool row_ok = i < d;
    const long long rs = (long long)H * d;
    const long long base = (long long)b * L * rs + (long long)h * d;
    const int ncp = (L + CKP - 1) / CKP;
    const long long cta = ((long long)b * H + h) * gridDim.z + z;
    float* sbuf = scratch + cta * rows_scratch_floats<CPL, LPR>();
    const float* ck_unit = ckpt + ((long long)b * H + h) * (ncp + 1) * d * d;
    const int hb = halving_base<ROUNDS>(lane, NV);

    auto st_slice = [&](float* dst, const float2 (&x)[NP]) {
        float4* p = reinterpret_cast<float4*>(dst + (size_t)tid * CPL);
#pragma unroll
        for (int c = 0; c < NP; c += 2) p[c / 2] = make_float4(x[c].x, x[c].y, x[c + 1].x, x[c + 1].y);
    };
    auto ld_slice = [&](const float* src, float2 (&x)[NP]) {
        const float4* p = reinterpret_cast<const float4*>(src + (size_t)tid * CPL);
#pragma unroll
        for (int c = 0; c < NP; c += 2) {
            const float4 w = p[c / 2];
            x[c] = make_float2(w.x, w.y);
            x[c + 1] = make_float2(w.z, w.w);
        }
    };
    // stage tokens [t0, t0 + n) of the piece; with_q: also q and dO (the backward's)
    auto stage = [&](int t0, int n, bool with_q) {
        __syncthreads();  // the previous piece's stage is consumed
        for (int base_idx = 0; base_idx < SB * W; base_idx += NT * 4) {
            float fk[4], fq[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = base_idx + tid + u * NT;
                const int tt = idx / W, c = idx % W;
                const bool ok = tt < n && c < d;
                const long long off = base + (long long)(t0 + tt) * rs + c;
                fk[u] = ok ? ldv(k + off) : 0.0f;
                fq[u] = (ok && with_q) ? ldv(q + off) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = base_idx + tid + u * NT;
                const int tt = idx / W, c = idx % W;
                if (tt < SB) {
                    const int so = tt * RP + (c / CPL) * SP + c % CPL;
                    sk[so] = fk[u];
                    sq[so] = fq[u];
                }
            }
        }
        for (int idx = tid; idx < SB * kRowsPerCta; idx += NT) {
            const int tt = idx / kRowsPerCta, r = idx % kRowsPerCta;
            const bool ok = tt < n && rb + r < d;
            const long long off = base + (long long)(t0 + tt) * rs + rb + r;
            sv[idx] = ok ? ldv(v + off) : 0.0f;
            sb[idx] = !ok ? 0.0f
                          : beta_scalar ? ldv(beta + ((long long)b * L + t0 + tt) * H + h)
                                        : ldv(beta + off);
            sdo[idx] = (ok && with_q) ? ldv(dO + off) : 0.0f;
        }
        if (GATED)
            for (int tt = tid; tt < SB; tt += NT)
                sa[tt] = tt < n ? ldv(alpha + ((long long)b * L + t0 + tt) * H + h) : 1.0f;
        __syncthreads();
    };
    auto krow = [&](int tt, int p) {  // k pair p of token tt (this lane's slice)
        return *reinterpret_cast<const float2*>(sk + tt * RP + part_ix * SP + 2 * p);
    };
    auto qrow = [&](int tt, int p) {
        return *reinterpret_cast<const float2*>(sq + tt * RP + part_ix * SP + 2 * p);
    };
    // one forward step of this thread's row slice (token tt of the staged piece)
    auto fwd_step = [&](float2 (&S)[NP], int tt) {
        float2 ra = dup2(0.0f), rc = dup2(0.0f);
#pragma unroll
        for (int p = 0; p < NP; p += 2) {
            ra = fma2(S[p], krow(tt, p), ra);
            rc = fma2(S[p + 1], krow(tt, p + 1), rc);
        }
        float r = (ra.x + ra.y) + (rc.x + rc.y);
#pragma unroll
        for (int o = 1; o < LPR; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
        const float al = GATED ? sa[tt] : 1.0f;
        const float2 u2 = dup2(sb[tt * kRowsPerCta + rl] * (sv[tt * kRowsPerCta + rl] - al * r));
#pragma unroll
        for (int p = 0; p < NP; ++p)
            S[p] = fma2(u2, krow(tt, p), GATED ? mul2(dup2(al), S[p]) : S[p]);
    };
    // the 4 warps' row sums of tokens [tt0, tt0 + n) of the piece -> global partials
    auto flush = [&](int pt0, int tt0, int n) {
        __syncthreads();
        for (int idx = tid; idx < n * (2 * W + 2); idx += NT) {
            const int tt = tt0 + idx / (2 * W + 2), e = idx % (2 * W + 2);
            const long long row = ((long long)z * B + b) * L + pt0 + tt;
            if (e < 2 * W) {
                const int which = e / W, col = e % W;
                const float* rr =
                    red + (tt % NSLOT) * NW * RED + which * HALF + (col / CPL) * SLICE + col % CPL;
                float s = 0.0f;
#pragma unroll
                for (int w = 0; w < NW; ++w) s += rr[w * RED];
                if (col < d) part[(row * H + h) * 2 * d + which * d + col] = s;
            } else {
                const float* rr = red + (tt % NSLOT) * NW * RED + 2 * HALF + (e - 2 * W);
                float s = 0.0f;
#pragma unroll
                for (int w = 0; w < NW; ++w) s += rr[w * RED];
                part_s[(row * H + h) * 2 + (e - 2 * W)] = s;
            }
        }
        __syncthreads();
    };
    // w = [gq partial of token tq | gk partial of token tk] (tq < 0 or tk < 0: skip that half)
    auto reduce_rows = [&](float (&w)[NV], int tq, int tk) {
        rows_halving_sum<NV, ROUNDS>(w, lane);
#pragma unroll
        for (int j = 0; j < (NV >> ROUNDS); ++j) {
            const int e = hb + j;  // index into [gq CPL | gk CPL] of slice part_ix
            const int which = e >= CPL;
            const int tt = which ? tk : tq;
            if (tt >= 0)
                red[((tt % NSLOT) * NW + warp) * RED + which * HALF + part_ix * SLICE + e -
                    which * CPL] =
                    w[j];
        }
    };

    float2 dS[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) dS[p] = dup2(0.0f);

    // backward step of token tt; P = S_{t-1} (slot tt), Pn <- slot tt - 1.  Also the gq
    // of token tt - 1, whose state after the update is P.
    auto bstep = [&](const float2 (&P)[NP], float2 (&Pn)[NP], int pt0, int pn, int tt) {
        if (tt > 0) ld_slice(sbuf + (size_t)(tt - 1) * NT * CPL, Pn);
        const float doj = sdo[tt * kRowsPerCta + rl];
        const float dop = tt > 0 ? sdo[(tt - 1) * kRowsPerCta + rl] : 0.0f;
        const float al = GATED ? sa[tt] : 1.0f;
        const float be = sb[tt * kRowsPerCta + rl];
        float w[NV];
        float2 ra = dup2(0.0f), rc = dup2(0.0f), sa2 = dup2(0.0f), sc2 = dup2(0.0f);
        const float2 do2 = dup2(doj), dp2 = dup2(dop);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const float2 kp = krow(tt, p);
            dS[p] = fma2(do2, qrow(tt, p), dS[p]);
            const float2 g = mul2(P[p], dp2);
            w[2 * p] = g.x;
            w[2 * p + 1] = g.y;
            if (p & 1) {
                rc = fma2(P[p], kp, rc);
                sc2 = fma2(dS[p], kp, sc2);
            } else {
                ra = fma2(P[p], kp, ra);
                sa2 = fma2(dS[p], kp, sa2);
            }
        }
        float r = (ra.x + ra.y) + (rc.x + rc.y), dsk = (sa2.x + sa2.y) + (sc2.x + sc2.y);
#pragma unroll
        for (int o = 1; o < LPR; o <<= 1) {
            r += __shfl_xor_sync(0xffffffffu, r, o);
            dsk += __shfl_xor_sync(0xffffffffu, dsk, o);
        }
        const float err = sv[tt * kRowsPerCta + rl] - al * r;
        const float u = be * err;
        const float bd = be * dsk;
        if (part_ix == 0) {
            sgv[tt * kRowsPerCta + rl] = bd;
            sgb[tt * kRowsPerCta + rl] = err * dsk;
        }
        // gk partial: dS u - alpha P (beta dsk); then dS <- alpha (dS - bd k)
        const float2 u2 = dup2(u), nabd = dup2(-al * bd), nbd = dup2(-bd), al2 = dup2(al);
        float2 ga2 = dup2(0.0f);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const float2 g = fma2(dS[p], u2, mul2(nabd, P[p]));
            w[CPL + 2 * p] = g.x;
            w[CPL + 2 * p + 1] = g.y;
            const float2 x = fma2(nbd, krow(tt, p), dS[p]);
            if (GATED) ga2 = fma2(x, P[p], ga2);
            dS[p] = GATED ? mul2(al2, x) : x;
        }
        reduce_rows(w, tt - 1, tt);
        // scalars: galpha (gated only), and a per-token beta's gradient (one lane per
        // row; a per-element beta's goes out per row above)
        float ga = 0.0f, bsum = 0.0f;
        if (GATED) {
            ga = ga2.x + ga2.y;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ga += __shfl_xor_sync(0xffffffffu, ga, o);
        }
        if (beta_scalar) {
            bsum = (part_ix == 0 && row_ok) ? err * dsk : 0.0f;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
        }
        if (lane == 0) {
            red[((tt % NSLOT) * NW + warp) * RED + 2 * HALF] = ga;
            red[((tt % NSLOT) * NW + warp) * RED + 2 * HALF + 1] = bsum;
        }
        if (tt % RB == 0) flush(pt0, tt, min(RB, pn - tt));
    };

    for (int p = ncp - 1; p >= 0; --p) {
        {
            const int pt0 = p * SB, pn = min(SB, L - pt0);
            stage(pt0, pn, true);
            {
                float2 S[NP];
                const float* src = ck_unit + (long long)p * d * d + (long long)i * d + c0;
#pragma unroll
                for (int q2 = 0; q2 < NP; ++q2)
                    S[q2] = make_float2((row_ok && c0 + 2 * q2 < d) ? src[2 * q2] : 0.0f,
                                        (row_ok && c0 + 2 * q2 + 1 < d) ? src[2 * q2 + 1] : 0.0f);
                for (int tt = 0; tt < pn; ++tt) {
                    st_slice(sbuf + (size_t)tt * NT * CPL, S);
                    fwd_step(S, tt);
                }
                // gq of the piece's last token from its state after the update
                float w[NV];
                const float2 dl = dup2(sdo[(pn - 1) * kRowsPerCta + rl]);
#pragma unroll
                for (int p2 = 0; p2 < NP; ++p2) {
                    const float2 g = mul2(S[p2], dl);
                    w[2 * p2] = g.x;
                    w[2 * p2 + 1] = g.y;
                    w[CPL + 2 * p2] = 0.0f;
                    w[CPL + 2 * p2 + 1] = 0.0f;
                }
                reduce_rows(w, pn - 1, -1);
            }
            // walk back; the two state buffers trade roles every token
            float2 A[NP], Bv[NP];
            ld_slice(sbuf + (size_t)(pn - 1) * NT * CPL, A);
            for (int tt = pn - 1; tt >= 0; tt -= 2) {
                bstep(A, Bv, pt0, pn, tt);
                if (tt == 0) break;
                bstep(Bv, A, pt0, pn, tt - 1);
            }
            // this piece's gv and per-element gbeta rows
            for (int idx = tid; idx < pn * kRowsPerCta; idx += NT) {
                const int tt = idx / kRowsPerCta, r = idx % kRowsPerCta;
                if (rb + r < d) {
                    const long long off = base + (long long)(pt0 + tt) * rs + rb + r;
                    st_scalar<T>(gv + off, sgv[idx]);
                    if (!beta_scalar) st_scalar<T>(gbeta + off, sgb[idx]);
                }
            }
        }
    }
}

// gq, gk [B, L, H, d] and galpha, a per-token gbeta [B, L, H]: the row blocks' partials
// added in order.  One block of 128 threads per (b, t, h) row group of 4.
template <typename T, bool GATED>
__global__ void __launch_bounds__(256)
    delta_rows_reduce_kernel(const float* __restrict__ part, const float* __restrict__ part_s,
                             T* __restrict__ gq, T* __restrict__ gk, T* __restrict__ galpha,
                             T* __restrict__ gbeta, long long rows, int d, int nz,
                             int beta_scalar) {
    const long long row = (long long)blockIdx.x * 2 + (threadIdx.x >> 7);
    const int tx = threadIdx.x & 127;
    if (row >= rows) return;
    for (int e = tx; e < 2 * d; e += 128) {
        float s = 0.0f;
        for (int zz = 0; zz < nz; ++zz) s += part[((long long)zz * rows + row) * 2 * d + e];
        if (e < d) st_scalar<T>(gq + row * d + e, s);
        else st_scalar<T>(gk + row * d + e - d, s);
    }
    if (tx < 2) {
        float s = 0.0f;
        for (int zz = 0; zz < nz; ++zz) s += part_s[((long long)zz * rows + row) * 2 + tx];
        if (tx == 0 && GATED) st_scalar<T>(galpha + row, s);
        if (tx == 1 && beta_scalar) st_scalar<T>(gbeta + row, s);
    }
}

template <int CPL, int LPR>
size_t rows_bwd_scratch_bytes(int B, int H, int d) {
    const int nz = (d + kRowsPerCta - 1) / kRowsPerCta;
    return (size_t)B * H * nz * rows_scratch_floats<CPL, LPR>() * sizeof(float);
}
size_t rows_bwd_ws_bytes(int B, int L, int H, int d) {
    const int nz = (d + kRowsPerCta - 1) / kRowsPerCta;
    const size_t rows = (size_t)B * L * H;
    const size_t sc = d <= 32 ? rows_bwd_scratch_bytes<8, 4>(B, H, d)
                              : rows_bwd_scratch_bytes<8, 16>(B, H, d);
    return a256(sc) + a256((size_t)nz * rows * 2 * d * sizeof(float)) +
           a256((size_t)nz * rows * 2 * sizeof(float));
}

template <typename T, int CPL, int LPR, bool GATED>
int launch_bwd_rows_t(const void* q, const void* k, const void* v, const void* beta,
                      const void* alpha, const void* dO, const float* ckpt, void* ws, void* gq,
                      void* gk, void* gv, void* gbeta, void* galpha, int B, int L, int H, int d,
                      int beta_scalar, cudaStream_t st) {
    const int nz = (d + kRowsPerCta - 1) / kRowsPerCta;
    const size_t rows = (size_t)B * L * H;
    char* p = static_cast<char*>(ws);
    float* scratch = reinterpret_cast<float*>(p);
    p += a256(rows_bwd_scratch_bytes<CPL, LPR>(B, H, d));
    float* part = reinterpret_cast<float*>(p);
    p += a256((size_t)nz * rows * 2 * d * sizeof(float));
    float* part_s = reinterpret_cast<float*>(p);
    constexpr size_t smem = RowsBwdSmem<CPL, LPR>::bytes;
    cudaError_t e = cudaFuncSetAttribute(delta_bwd_rows_kernel<T, CPL, LPR, GATED>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    delta_bwd_rows_kernel<T, CPL, LPR, GATED><<<dim3(H, B, nz), 32 * LPR, smem, st>>>(
        (const T*)q, (const T*)k, (const T*)v, (const T*)beta, (const T*)alpha, (const T*)dO,
        ckpt, scratch, part, part_s, (T*)gv, (T*)gbeta, B, L, H, d, beta_scalar);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    delta_rows_reduce_kernel<T, GATED><<<(unsigned)((rows + 1) / 2), 256, 0, st>>>(
        part, part_s, (T*)gq, (T*)gk, (T*)galpha, (T*)gbeta, (long long)rows, d, nz,
        beta_scalar);
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T>
int launch_bwd_rows(const void* q, const void* k, const void* v, const void* beta,
                    const void* alpha, const void* dO, const float* ckpt, void* ws, void* gq,
                    void* gk, void* gv, void* gbeta, void* galpha, int B, int L, int H, int d,
                    int beta_scalar, cudaStream_t st) {
    if (d <= 32)
        return alpha ? launch_bwd_rows_t<T, 8, 4, true>(q, k, v, beta, alpha, dO, ckpt, ws, gq, gk,
                                                     gv, gbeta, galpha, B, L, H, d, beta_scalar,
                                                     st)
                     : launch_bwd_rows_t<T, 8, 4, false>(q, k, v, beta, alpha, dO, ckpt, ws, gq, gk,
                                                      gv, gbeta, galpha, B, L, H, d, beta_scalar,
                                                      st);
    return alpha ? launch_bwd_rows_t<T, 8, 16, true>(q, k, v, beta, alpha, dO, ckpt, ws, gq, gk, gv,
                                                  gbeta, galpha, B, L, H, d, beta_scalar, st)
                 : launch_bwd_rows_t<T, 8, 16, false>(q, k, v, beta, alpha, dO, ckpt, ws, gq, gk,
                                                   gv, gbeta, galpha, B, L, H, d, beta_scalar,
                                                   st);
}


template <typename T, int CPL, int LPR, bool GATED>
int launch_fwd_rows(const void* q, const void* k, const void* v, const void* beta,
                    const void* alpha, void* o, float* ckpt, int B, int L, int H, int d,
                    int beta_scalar, cudaStream_t st) {
    constexpr size_t smem = fwd_rows_smem<CPL, LPR>();
    cudaError_t e = cudaFuncSetAttribute(delta_fwd_rows_kernel<T, CPL, LPR, GATED>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    delta_fwd_rows_kernel<T, CPL, LPR, GATED>
        <<<dim3(H, B, (d + kRowsPerCta - 1) / kRowsPerCta), 32 * LPR, smem, st>>>(
            (const T*)q, (const T*)k, (const T*)v, (const T*)beta, (const T*)alpha, (T*)o, ckpt,
            L, H, d, beta_scalar);
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T>
int launch_fwd(const void* q, const void* k, const void* v, const void* beta, const void* alpha,
               void* o, float* ckpt, int B, int L, int H, int d, int beta_scalar,
               cudaStream_t st) {
    if (d <= 32)
        return alpha != nullptr
                   ? launch_fwd_rows<T, 8, 4, true>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                                 beta_scalar, st)
                   : launch_fwd_rows<T, 8, 4, false>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                                  beta_scalar, st);
    return alpha != nullptr
               ? launch_fwd_rows<T, 16, 8, true>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                              beta_scalar, st)
               : launch_fwd_rows<T, 16, 8, false>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                               beta_scalar, st);
}

int check(int dtype, int B, int L, int H, int d) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || L <= 0 || H <= 0 || d <= 0) return EDB_ERR_BAD_SHAPE;
    if (d > 128) return EDB_ERR_UNSUPPORTED;
    return EDB_OK;
}

}  // namespace

// Chunked tensor-core path (delta_chunked.cu, delta_chunked_bwd.cu).
bool edb_delta_chunked_ok(int dtype, int beta_per_element, int head_dim);
size_t edb_delta_chunked_ckpt_bytes(int B, int L, int H);
size_t edb_delta_chunked_fwd_ws(int B, int L, int H);
size_t edb_delta_chunked_bwd_ws(int B, int L, int H, int gated);
int edb_delta_chunked_fwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* alpha, void* o, float* resid, int B, int L, int H, void* ws,
                          cudaStream_t st);
int edb_delta_chunked_bwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* alpha, const void* dO, const float* resid, void* gq,
                          void* gk, void* gv, void* gbeta, void* galpha, int B, int L, int H,
                          void* ws, cudaStream_t st);

extern "C" size_t edb_delta_rule_ckpt_bytes(int dtype, int beta_per_element, int batch,
                                            int seq_len, int heads, int head_dim) {
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    return edb_delta_chunked_ok(dtype, beta_per_element, head_dim)
               ? edb_delta_chunked_ckpt_bytes(batch, seq_len, heads)
               : ckpt_bytes(batch, seq_len, heads, head_dim);
}

extern "C" size_t edb_delta_rule_fwd_workspace(int dtype, int beta_per_element, int batch,
                                               int seq_len, int heads, int head_dim) {
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    return edb_delta_chunked_ok(dtype, beta_per_element, head_dim)
               ? edb_delta_chunked_fwd_ws(batch, seq_len, heads)
               : 0;
}

extern "C" int edb_delta_rule_fwd(int dtype, const void* q, const void* k, const void* v,
                                  const void* beta, int beta_per_element, void* o, float* s_ckpt,
                                  int batch, int seq_len, int heads, int head_dim,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    if (int s = check(dtype, batch, seq_len, heads, head_dim)) return s;
    if (!q || !k || !v || !beta || !o) return EDB_ERR_NULL_POINTER;
    cudaStream_t st = (cudaStream_t)stream;
    if (edb_delta_chunked_ok(dtype, beta_per_element, head_dim)) {
        const size_t need = edb_delta_chunked_fwd_ws(batch, seq_len, heads);
        if (workspace_bytes < need || !workspace) return EDB_ERR_WORKSPACE_TOO_SMALL;
        if (!edb::aligned16(q) || !edb::aligned16(k) || !edb::aligned16(v) ||
            !edb::aligned16(workspace) ||
            (reinterpret_cast<uintptr_t>(s_ckpt) & 15u))
            return EDB_ERR_MISALIGNED;
        return edb_delta_chunked_fwd(q, k, v, beta, nullptr, o, s_ckpt, batch, seq_len, heads,
                                     workspace, st);
    }
    const int bs = beta_per_element ? 0 : 1;
    return dtype == EDB_BF16
               ? launch_fwd<__nv_bfloat16>(q, k, v, beta, nullptr, o, s_ckpt, batch, seq_len,
                                           heads, head_dim, bs, st)
               : launch_fwd<float>(q, k, v, beta, nullptr, o, s_ckpt, batch, seq_len, heads,
                                   head_dim, bs, st);
}

extern "C" size_t edb_delta_rule_bwd_workspace(int dtype, int beta_per_element, int batch,
                                               int seq_len, int heads, int head_dim,
                                               int have_ckpt) {
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    const size_t ck = have_ckpt ? 0
                                : a256(edb_delta_rule_ckpt_bytes(dtype, beta_per_element, batch,
                                                                 seq_len, heads, head_dim));
    if (edb_delta_chunked_ok(dtype, beta_per_element, head_dim)) {
        // residuals (when not passed), then the forward's or the backward's scratch
        const size_t f = edb_delta_chunked_fwd_ws(batch, seq_len, heads);
        const size_t b = edb_delta_chunked_bwd_ws(batch, seq_len, heads, 0);
        return ck + (have_ckpt ? b : (f > b ? f : b));
    }
    // checkpoints (when not passed), then the row-parallel backward's scratch
    return ck + rows_bwd_ws_bytes(batch, seq_len, heads, head_dim);
}

extern "C" int edb_delta_rule_bwd(int dtype, const void* q, const void* k, const void* v,
                                  const void* beta, int beta_per_element, const void* dO,
                                  const float* s_ckpt, void* gq, void* gk, void* gv, void* gbeta,
                                  int batch, int seq_len, int heads, int head_dim,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    if (int s = check(dtype, batch, seq_len, heads, head_dim)) return s;
    if (!q || !k || !v || !beta || !dO || !gq || !gk || !gv || !gbeta) return EDB_ERR_NULL_POINTER;
    const size_t need = edb_delta_rule_bwd_workspace(dtype, beta_per_element, batch, seq_len,
                                                     heads, head_dim, s_ckpt != nullptr);
    if (workspace_bytes < need || (need && !workspace)) return EDB_ERR_WORKSPACE_TOO_SMALL;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t ckb =
        s_ckpt ? 0
               : a256(edb_delta_rule_ckpt_bytes(dtype, beta_per_element, batch, seq_len, heads,
                                                head_dim));
    if (edb_delta_chunked_ok(dtype, beta_per_element, head_dim)) {
        if (!edb::aligned16(q) || !edb::aligned16(k) || !edb::aligned16(v) ||
            !edb::aligned16(dO) || !edb::aligned16(workspace) ||
            (reinterpret_cast<uintptr_t>(s_ckpt) & 15u))
            return EDB_ERR_MISALIGNED;
        const float* resid = s_ckpt;
        char* scratch = static_cast<char*>(workspace) + ckb;
        if (!resid) {
            // residuals into the workspace; o goes to gq, which the backward overwrites
            float* r = static_cast<float*>(workspace);
            int s = edb_delta_chunked_fwd(q, k, v, beta, nullptr, gq, r, batch, seq_len, heads,
                                          scratch, st);
            if (s) return s;
            resid = r;
        }
        return edb_delta_chunked_bwd(q, k, v, beta, nullptr, dO, resid, gq, gk, gv, gbeta,
                                     nullptr, batch, seq_len, heads, scratch, st);
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return EDB_ERR_MISALIGNED;
    const int bs = beta_per_element ? 0 : 1;
    const float* ck = s_ckpt;
    if (!ck) {
        // states only: the forward writes o into gq, which the backward overwrites
        float* w = static_cast<float*>(workspace);
        int s = edb_delta_rule_fwd(dtype, q, k, v, beta, beta_per_element, gq, w, batch, seq_len,
                                   heads, head_dim, nullptr, 0, stream);
        if (s) return s;
        ck = w;
    }
    void* rows_ws = static_cast<char*>(workspace) + ckb;
    return dtype == EDB_BF16
               ? launch_bwd_rows<__nv_bfloat16>(q, k, v, beta, nullptr, dO, ck, rows_ws, gq, gk,
                                                gv, gbeta, nullptr, batch, seq_len, heads,
                                                head_dim, bs, st)
               : launch_bwd_rows<float>(q, k, v, beta, nullptr, dO, ck, rows_ws, gq, gk, gv,
                                        gbeta, nullptr, batch, seq_len, heads, head_dim, bs, st);
}

// ------------------------------------------------------------------ GatedDeltaNet
// bf16 io, one beta per (token, head), head_dim 128: the chunked tensor-core form
// (delta_chunked*.cu with the decay); every other case the token recurrence.
// The residual (s_ckpt) format follows the path, as for the delta rule.
extern "C" size_t edb_gated_delta_net_ckpt_bytes(int dtype, int beta_per_element, int batch,
                                                 int seq_len, int heads, int head_dim) {
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    return edb_delta_chunked_ok(dtype, beta_per_element, head_dim)
               ? edb_delta_chunked_ckpt_bytes(batch, seq_len, heads)
               : ckpt_bytes(batch, seq_len, heads, head_dim);
}

extern "C" size_t edb_gated_delta_net_fwd_workspace(int dtype, int beta_per_element, int batch,
                                                    int seq_len, int heads, int head_dim) {
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    return edb_delta_chunked_ok(dtype, beta_per_element, head_dim)
               ? edb_delta_chunked_fwd_ws(batch, seq_len, heads)
               : 0;
}

extern "C" int edb_gated_delta_net_fwd_ws(int dtype, const void* q, const void* k, const void* v,
                                          const void* beta, int beta_per_element,
                                          const void* alpha, void* o, float* s_ckpt, int batch,
                                          int seq_len, int heads, int head_dim, void* workspace,
                                          size_t workspace_bytes, void* stream) {
    if (int s = check(dtype, batch, seq_len, heads, head_dim)) return s;
    if (!q || !k || !v || !beta || !alpha || !o) return EDB_ERR_NULL_POINTER;
    cudaStream_t st = (cudaStream_t)stream;
    if (edb_delta_chunked_ok(dtype, beta_per_element, head_dim)) {
        const size_t need = edb_delta_chunked_fwd_ws(batch, seq_len, heads);
        if (workspace_bytes < need || !workspace) return EDB_ERR_WORKSPACE_TOO_SMALL;
        if (!edb::aligned16(q) || !edb::aligned16(k) || !edb::aligned16(v) ||
            !edb::aligned16(workspace) || (reinterpret_cast<uintptr_t>(s_ckpt) & 15u))
            return EDB_ERR_MISALIGNED;
        return edb_delta_chunked_fwd(q, k, v, beta, alpha, o, s_ckpt, batch, seq_len, heads,
                                     workspace, st);
    }
    const int bs = beta_per_element ? 0 : 1;
    return dtype == EDB_BF16
               ? launch_fwd<__nv_bfloat16>(q, k, v, beta, alpha, o, s_ckpt, batch, seq_len,
                                           heads, head_dim, bs, st)
               : launch_fwd<float>(q, k, v, beta, alpha, o, s_ckpt, batch, seq_len, heads,
                                   head_dim, bs, st);
}

extern "C" int edb_gated_delta_net_fwd(int dtype, const void* q, const void* k, const void* v,
                                       const void* beta, int beta_per_element, const void* alpha,
                                       void* o, float* s_ckpt, int batch, int seq_len, int heads,
                                       int head_dim, void* stream) {
    if (int s = check(dtype, batch, seq_len, heads, head_dim)) return s;
    if (!q || !k || !v || !beta || !alpha || !o) return EDB_ERR_NULL_POINTER;
    const size_t wsb = edb_gated_delta_net_fwd_workspace(dtype, beta_per_element, batch,
                                                         seq_len, heads, head_dim);
    if (wsb == 0)
        return edb_gated_delta_net_fwd_ws(dtype, q, k, v, beta, beta_per_element, alpha, o,
                                          s_ckpt, batch, seq_len, heads, head_dim, nullptr, 0,
                                          stream);
    // the chunked form's scratch, taken stream-ordered (no workspace argument here)
    cudaStream_t st = (cudaStream_t)stream;
    void* ws = nullptr;
    cudaError_t e = cudaMallocAsync(&ws, wsb, st);
    if (e != cudaSuccess) return (int)e;
    const int s = edb_gated_delta_net_fwd_ws(dtype, q, k, v, beta, beta_per_element, alpha, o,
                                             s_ckpt, batch, seq_len, heads, head_dim, ws, wsb,
                                             stream);
    cudaFreeAsync(ws, st);
    return s;
}

extern "C" size_t edb_gated_delta_net_bwd_workspace(int dtype, int beta_per_element, int batch,
                                                    int seq_len, int heads, int head_dim,
                                                    int have_ckpt) {
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    const size_t ck = have_ckpt ? 0
                                : a256(edb_gated_delta_net_ckpt_bytes(dtype, beta_per_element,
                                                                      batch, seq_len, heads,
                                                                      head_dim));
    if (edb_delta_chunked_ok(dtype, beta_per_element, head_dim)) {
        const size_t f = edb_delta_chunked_fwd_ws(batch, seq_len, heads);
        const size_t b = edb_delta_chunked_bwd_ws(batch, seq_len, heads, 1);
        return ck + (have_ckpt ? b : (f > b ? f : b));
    }
    return ck + rows_bwd_ws_bytes(batch, seq_len, heads, head_dim);
}

extern "C" int edb_gated_delta_net_bwd(int dtype, const void* q, const void* k, const void* v,
                                       const void* beta, int beta_per_element, const void* alpha,
                                       const void* dO, const float* s_ckpt, void* gq, void* gk,
                                       void* gv, void* gbeta, void* galpha, int batch,
                                       int seq_len, int heads, int head_dim, void* workspace,
                                       size_t workspace_bytes, void* stream) {
    if (int s = check(dtype, batch, seq_len, heads, head_dim)) return s;
    if (!q || !k || !v || !beta || !alpha || !dO || !gq || !gk || !gv || !gbeta || !galpha)
        return EDB_ERR_NULL_POINTER;
    const size_t need = edb_gated_delta_net_bwd_workspace(dtype, beta_per_element, batch,
                                                          seq_len, heads, head_dim,
                                                          s_ckpt != nullptr);
    if (workspace_bytes < need || !workspace) return EDB_ERR_WORKSPACE_TOO_SMALL;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return EDB_ERR_MISALIGNED;
    cudaStream_t st = (cudaStream_t)stream;
    char* p = static_cast<char*>(workspace);
    const size_t ckb = s_ckpt ? 0
                              : a256(edb_gated_delta_net_ckpt_bytes(dtype, beta_per_element,
                                                                    batch, seq_len, heads,
                                                                    head_dim));
    if (edb_delta_chunked_ok(dtype, beta_per_element, head_dim)) {
        if (!edb::aligned16(q) || !edb::aligned16(k) || !edb::aligned16(v) ||
            !edb::aligned16(dO) || (reinterpret_cast<uintptr_t>(s_ckpt) & 15u))
            return EDB_ERR_MISALIGNED;
        const float* resid = s_ckpt;
        char* scratch = p + ckb;
        if (!resid) {
            // residuals into the workspace; o goes to gq, which the backward overwrites
            float* r = reinterpret_cast<float*>(p);
            int s = edb_delta_chunked_fwd(q, k, v, beta, alpha, gq, r, batch, seq_len, heads,
                                          scratch, st);
            if (s) return s;
            resid = r;
        }
        return edb_delta_chunked_bwd(q, k, v, beta, alpha, dO, resid, gq, gk, gv, gbeta, galpha,
                                     batch, seq_len, heads, scratch, st);
    }
    const float* ck = s_ckpt;
    if (!ck) {
        // states only: the forward writes o into gq, which the backward overwrites
        float* w = reinterpret_cast<float*>(p);
        int s = edb_gated_delta_net_fwd_ws(dtype, q, k, v, beta, beta_per_element, alpha, gq, w,
                                           batch, seq_len, heads, head_dim, nullptr, 0, stream);
        if (s) return s;
        ck = w;
    }
    p += ckb;
    const int bs = beta_per_element ? 0 : 1;
    return dtype == EDB_BF16
               ? launch_bwd_rows<__nv_bfloat16>(q, k, v, beta, alpha, dO, ck, p, gq, gk, gv,
                                                gbeta, galpha, batch, seq_len, heads, head_dim,
                                                bs, st)
               : launch_bwd_rows<float>(q, k, v, beta, alpha, dO, ck, p, gq, gk, gv, gbeta,
                                        galpha, batch, seq_len, heads, head_dim, bs, st);
}
