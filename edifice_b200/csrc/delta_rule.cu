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
// io): one CTA per (b, h) holding S (and dS) in shared memory as f32, token
// order.  The forward can write S at the start of every CK-token chunk (plus
// the final state); the delta-rule backward walks chunks in reverse, recomputes
// each chunk's retrievals r_t from its checkpoint, and undoes the updates
// (S_{t-1} = S_t - u_t k_t^T with the stored r_t) instead of storing every state.
// The gated backward cannot undo an update (that divides by alpha_t, which
// amplifies rounding by 1/alpha per token): it recomputes each chunk's states
// S_{t-1} forward from the checkpoint into a global buffer and reads them back
// in reverse.
#include <math.h>

#include "edb_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int CK = 64;  // tokens per checkpoint chunk

template <typename T>
static __device__ __forceinline__ float ldv(const T* p) {
    return ld_scalar<T>(p);
}

// Forward, row-parallel.  Each row i of S (value index) evolves on its own in
// the forward: S[i] <- alpha S[i] + beta_i (v_i - alpha S[i].k) k^T,
// o_i = S[i].q, so a row lives in the registers of 4 lanes (CPL columns each)
// and no block barrier is needed per token; k, q and the CTA's rows of v,
// beta (and alpha) are staged in shared memory one CK-token chunk at a time.
// grid (H, B, ceil(d / 32)), 128 threads = 32 rows x 4 lanes.  Shared memory
// (dynamic): k, q [CK][4][CPL + 4] (a pad of 4 floats per lane's slice puts
// the 4 slices of one token on different banks) | v, beta, o [CK][32] | alpha [CK].
constexpr int kRowThreads = 128, kRowsPerCta = 32;

template <int CPL>
constexpr size_t fwd_rows_smem() {
    return ((size_t)2 * CK * 4 * (CPL + 4) + 3 * CK * kRowsPerCta + CK) * sizeof(float);
}

template <typename T, int CPL, bool GATED>
__global__ void __launch_bounds__(kRowThreads)
    delta_fwd_rows_kernel(const T* __restrict__ q, const T* __restrict__ k,
                          const T* __restrict__ v, const T* __restrict__ beta,
                          const T* __restrict__ alpha, T* __restrict__ o,
                          float* __restrict__ ckpt, int L, int H, int d, int beta_scalar) {
    constexpr int SP = CPL + 4;  // floats per lane slice (padded)
    constexpr int RP = 4 * SP;   // floats per staged token row
    extern __shared__ __align__(16) float smf[];
    float* sk = smf;                        // [CK][RP]
    float* sq = sk + CK * RP;               // [CK][RP]
    float* sv = sq + CK * RP;               // [CK][32]
    float* sb = sv + CK * kRowsPerCta;      // [CK][32]
    float* so = sb + CK * kRowsPerCta;      // [CK][32]
    float* sa = so + CK * kRowsPerCta;      // [CK]
    const int h = blockIdx.x, b = blockIdx.y, rb = blockIdx.z * kRowsPerCta;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rl = warp * 8 + (lane >> 2);  // local row
    const int i = rb + rl;                  // value-dim row of S
    const int part = lane & 3;              // column slice [part CPL, part CPL + CPL)
    const int c0 = part * CPL;
    const bool row_ok = i < d;
    const long long rs = (long long)H * d;  // token stride
    const long long base = (long long)b * L * rs + (long long)h * d;
    const int nck = (L + CK - 1) / CK;
    float* ck_row = ckpt != nullptr && row_ok
                        ? ckpt + ((long long)b * H + h) * (nck + 1) * d * d + (long long)i * d
                        : nullptr;
    float S[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) S[c] = 0.0f;
    auto save_state = [&](int slot) {
        if (ck_row == nullptr) return;
        float* dst = ck_row + (long long)slot * d * d;
#pragma unroll
        for (int c = 0; c < CPL; ++c)
            if (c0 + c < d) dst[c0 + c] = S[c];
    };

    for (int t0 = 0; t0 < L; t0 += CK) {
        const int tn = min(CK, L - t0);
        save_state(t0 / CK);
        __syncthreads();  // the previous chunk's stage is consumed
        // ---- stage this chunk (loads batched per thread before the stores)
        for (int base_idx = 0; base_idx < CK * 4 * CPL; base_idx += kRowThreads * 8) {
            float fk[8], fq[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int idx = base_idx + tid + u * kRowThreads;
                const int tt = idx / (4 * CPL), c = idx % (4 * CPL);
                const bool ok = tt < tn && c < d;
                const long long off = base + (long long)(t0 + tt) * rs + c;
                fk[u] = ok ? ldv(k + off) : 0.0f;
                fq[u] = ok ? ldv(q + off) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int idx = base_idx + tid + u * kRowThreads;
                const int tt = idx / (4 * CPL), c = idx % (4 * CPL);
                if (tt < CK) {
                    const int so_ = tt * RP + (c / CPL) * SP + c % CPL;
                    sk[so_] = fk[u];
                    sq[so_] = fq[u];
                }
            }
        }
        for (int idx = tid; idx < CK * kRowsPerCta; idx += kRowThreads) {
            const int tt = idx / kRowsPerCta, r = idx % kRowsPerCta;
            const bool ok = tt < tn && rb + r < d;
            const long long off = base + (long long)(t0 + tt) * rs + rb + r;
            sv[idx] = ok ? ldv(v + off) : 0.0f;
            sb[idx] = !ok ? 0.0f
                          : beta_scalar ? ldv(beta + ((long long)b * L + t0 + tt) * H + h)
                                        : ldv(beta + off);
        }
        if (GATED)
            for (int tt = tid; tt < CK; tt += kRowThreads)
                sa[tt] = tt < tn ? ldv(alpha + ((long long)b * L + t0 + tt) * H + h) : 1.0f;
        __syncthreads();
        // ---- the chunk's tokens, row by row in registers
        for (int tt = 0; tt < tn; ++tt) {
            const float* kr = sk + tt * RP + part * SP;
            const float* qr = sq + tt * RP + part * SP;
            float r = 0.0f;
#pragma unroll
            for (int c = 0; c < CPL; c += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + c);
                r = fmaf(S[c], k4.x, fmaf(S[c + 1], k4.y, fmaf(S[c + 2], k4.z, fmaf(S[c + 3], k4.w, r))));
            }
            r += __shfl_xor_sync(0xffffffffu, r, 1);
            r += __shfl_xor_sync(0xffffffffu, r, 2);
            const float al = GATED ? sa[tt] : 1.0f;
            const float u = sb[tt * kRowsPerCta + rl] * (sv[tt * kRowsPerCta + rl] - al * r);
            float ov = 0.0f;
#pragma unroll
            for (int c = 0; c < CPL; c += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + c);
                const float4 q4 = *reinterpret_cast<const float4*>(qr + c);
                const float kv[4] = {k4.x, k4.y, k4.z, k4.w}, qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float sn = fmaf(u, kv[e], GATED ? al * S[c + e] : S[c + e]);
                    S[c + e] = sn;
                    ov = fmaf(sn, qv[e], ov);
                }
            }
            ov += __shfl_xor_sync(0xffffffffu, ov, 1);
            ov += __shfl_xor_sync(0xffffffffu, ov, 2);
            if (part == 0) so[tt * kRowsPerCta + rl] = ov;
        }
        __syncthreads();
        for (int idx = tid; idx < tn * kRowsPerCta; idx += kRowThreads) {
            const int tt = idx / kRowsPerCta, r = idx % kRowsPerCta;
            if (rb + r < d) st_scalar<T>(o + base + (long long)(t0 + tt) * rs + rb + r, so[idx]);
        }
    }
    save_state(nck);
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    delta_bwd_rec_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                         const T* __restrict__ beta, const T* __restrict__ dO,
                         const float* __restrict__ ckpt, T* __restrict__ gq, T* __restrict__ gk,
                         T* __restrict__ gv, T* __restrict__ gbeta, int L, int H, int d,
                         int beta_scalar) {
    extern __shared__ float sm[];
    const int sd = d + 1;
    float* S = sm;                 // [d][sd]
    float* dS = S + d * sd;        // [d][sd]
    float* rbuf = dS + d * sd;     // [CK][d] retrievals of the current chunk
    float* sq = rbuf + CK * d;
    float* sk = sq + d;
    float* sdo = sk + d;
    float* su = sdo + d;           // beta (.) err
    float* sbd = su + d;           // beta (.) dS k
    float* red = sbd + d;          // [kThreads] scratch for the scalar-beta sum
    const int h = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x;
    const int nck = (L + CK - 1) / CK;
    const long long rs = (long long)H * d;
    const long long base = (long long)b * L * rs + (long long)h * d;
    for (int i = tid; i < d * sd; i += kThreads) dS[i] = 0.0f;

    for (int c = nck - 1; c >= 0; --c) {
        const int t0 = c * CK, t1 = min(L, t0 + CK);
        const float* cp = ckpt + (((long long)b * H + h) * (nck + 1) + c) * d * d;
        __syncthreads();
        for (int i = tid; i < d * d; i += kThreads) S[(i / d) * sd + i % d] = cp[i];
        __syncthreads();
        // ---- forward over the chunk: retrievals r_t, S ends as S_{t1-1}
        for (int t = t0; t < t1; ++t) {
            const long long off = base + (long long)t * rs;
            for (int i = tid; i < d; i += kThreads) sk[i] = ldv(k + off + i);
            __syncthreads();
            for (int i = tid; i < d; i += kThreads) {
                float r = 0.0f;
                for (int j = 0; j < d; ++j) r = fmaf(S[i * sd + j], sk[j], r);
                rbuf[(t - t0) * d + i] = r;
                const float be = beta_scalar ? ldv(beta + ((long long)b * L + t) * H + h)
                                             : ldv(beta + off + i);
                const float u = be * (ldv(v + off + i) - r);
                for (int j = 0; j < d; ++j) S[i * sd + j] = fmaf(u, sk[j], S[i * sd + j]);
            }
            __syncthreads();
        }
        // ---- reverse over the chunk
        for (int t = t1 - 1; t >= t0; --t) {
            const long long off = base + (long long)t * rs;
            const long long boff = ((long long)b * L + t) * H + h;
            for (int i = tid; i < d; i += kThreads) {
                sq[i] = ldv(q + off + i);
                sk[i] = ldv(k + off + i);
                sdo[i] = ldv(dO + off + i);
            }
            __syncthreads();
            // rows: dS += dO q^T ; u = beta (v - r)
            for (int i = tid; i < d; i += kThreads) {
                const float doi = sdo[i];
                for (int j = 0; j < d; ++j) dS[i * sd + j] = fmaf(doi, sq[j], dS[i * sd + j]);
                const float be = beta_scalar ? ldv(beta + boff) : ldv(beta + off + i);
                su[i] = be * (ldv(v + off + i) - rbuf[(t - t0) * d + i]);
            }
            __syncthreads();
            // columns: dq = S_t^T dO
            for (int j = tid; j < d; j += kThreads) {
                float acc = 0.0f;
                for (int i = 0; i < d; ++i) acc = fmaf(S[i * sd + j], sdo[i], acc);
                st_scalar<T>(gq + off + j, acc);
            }
            // rows: dsk = dS k; dv = beta dsk; dbeta = err dsk
            float bsum = 0.0f;
            for (int i = tid; i < d; i += kThreads) {
                float dsk = 0.0f;
                for (int j = 0; j < d; ++j) dsk = fmaf(dS[i * sd + j], sk[j], dsk);
                const float be = beta_scalar ? ldv(beta + boff) : ldv(beta + off + i);
                const float err = ldv(v + off + i) - rbuf[(t - t0) * d + i];
                st_scalar<T>(gv + off + i, be * dsk);
                if (beta_scalar) bsum = fmaf(err, dsk, bsum);
                else st_scalar<T>(gbeta + off + i, err * dsk);
                sbd[i] = be * dsk;
            }
            if (beta_scalar) {
                red[tid] = bsum;
            }
            __syncthreads();
            if (beta_scalar && tid < 32) {
                float s = 0.0f;
                for (int i = tid; i < kThreads; i += 32) s += red[i];
                for (int off2 = 16; off2 >= 1; off2 >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off2);
                if (tid == 0) st_scalar<T>(gbeta + boff, s);
            }
            // rows: S_{t-1} = S_t - u k^T  (undo the update)
            for (int i = tid; i < d; i += kThreads) {
                const float u = su[i];
                for (int j = 0; j < d; ++j) S[i * sd + j] = fmaf(-u, sk[j], S[i * sd + j]);
            }
            __syncthreads();
            // columns: dk = dS^T u - S_{t-1}^T (beta dsk)
            for (int j = tid; j < d; j += kThreads) {
                float acc = 0.0f;
                for (int i = 0; i < d; ++i)
                    acc += dS[i * sd + j] * su[i] - S[i * sd + j] * sbd[i];
                st_scalar<T>(gk + off + j, acc);
            }
            __syncthreads();
            // rows: dS_{t-1} = dS - (beta dsk) k^T
            for (int i = tid; i < d; i += kThreads) {
                const float bd = sbd[i];
                for (int j = 0; j < d; ++j) dS[i * sd + j] = fmaf(-bd, sk[j], dS[i * sd + j]);
            }
            __syncthreads();
        }
    }
}

// Gated backward.  sbuf: [B*H][CK][d][d] f32 scratch for one chunk's states
// S_{t-1} (written by the chunk's forward recompute, read back in reverse).
// shared: Sa, Sb, dS [d][d+1] | q k dO u beta-dsk err [6][d] | red [kThreads]
template <typename T>
__global__ void __launch_bounds__(kThreads)
    gated_bwd_rec_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                         const T* __restrict__ beta, const T* __restrict__ alpha,
                         const T* __restrict__ dO, const float* __restrict__ ckpt,
                         float* __restrict__ sbuf, T* __restrict__ gq, T* __restrict__ gk,
                         T* __restrict__ gv, T* __restrict__ gbeta, T* __restrict__ galpha,
                         int L, int H, int d, int beta_scalar) {
    extern __shared__ float sm[];
    const int sd = d + 1;
    float* Sa = sm;                // S_t (after the token's update)
    float* Sb = Sa + d * sd;       // S_{t-1}
    float* dS = Sb + d * sd;       // gradient w.r.t. S_t
    float* sq = dS + d * sd;
    float* sk = sq + d;
    float* sdo = sk + d;
    float* su = sdo + d;           // beta (.) err
    float* sbd = su + d;           // beta (.) dS k
    float* ser = sbd + d;          // err = v - alpha S_{t-1} k
    float* red = ser + d;          // [kThreads]
    const int h = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nck = (L + CK - 1) / CK;
    const long long rs = (long long)H * d;
    const long long base = (long long)b * L * rs + (long long)h * d;
    float* buf = sbuf + ((long long)b * H + h) * CK * d * d;
    for (int i = tid; i < d * sd; i += kThreads) dS[i] = 0.0f;

    // block sum of one value per thread; every thread gets the total
    auto block_sum = [&](float x) {
        for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        __syncthreads();  // red is free
        if (lane == 0) red[warp] = x;
        __syncthreads();
        float s = 0.0f;
        for (int w = 0; w < kThreads / 32; ++w) s += red[w];
        return s;
    };

    for (int c = nck - 1; c >= 0; --c) {
        const int t0 = c * CK, t1 = min(L, t0 + CK);
        const float* cp = ckpt + (((long long)b * H + h) * (nck + 1) + c) * d * d;
        __syncthreads();
        for (int i = tid; i < d * d; i += kThreads) Sa[(i / d) * sd + i % d] = cp[i];
        __syncthreads();
        // ---- forward over the chunk: S_{t-1} -> buf[t - t0]; Sa ends as S_{t1-1}
        for (int t = t0; t < t1; ++t) {
            const long long off = base + (long long)t * rs;
            float* dst = buf + (long long)(t - t0) * d * d;
            for (int i = tid; i < d * d; i += kThreads) dst[i] = Sa[(i / d) * sd + i % d];
            for (int i = tid; i < d; i += kThreads) sk[i] = ldv(k + off + i);
            __syncthreads();
            const float al = ldv(alpha + ((long long)b * L + t) * H + h);
            for (int i = tid; i < d; i += kThreads) {
                float r = 0.0f;
                for (int j = 0; j < d; ++j) r = fmaf(Sa[i * sd + j], sk[j], r);
                const float be = beta_scalar ? ldv(beta + ((long long)b * L + t) * H + h)
                                             : ldv(beta + off + i);
                const float u = be * (ldv(v + off + i) - al * r);
                for (int j = 0; j < d; ++j) Sa[i * sd + j] = fmaf(u, sk[j], al * Sa[i * sd + j]);
            }
            __syncthreads();
        }
        // ---- reverse over the chunk (Sa = S_t, Sb = S_{t-1})
        for (int t = t1 - 1; t >= t0; --t) {
            const long long off = base + (long long)t * rs;
            const long long boff = ((long long)b * L + t) * H + h;
            const float al = ldv(alpha + boff);
            const float* srcb = buf + (long long)(t - t0) * d * d;
            for (int i = tid; i < d * d; i += kThreads) Sb[(i / d) * sd + i % d] = srcb[i];
            for (int i = tid; i < d; i += kThreads) {
                sq[i] = ldv(q + off + i);
                sk[i] = ldv(k + off + i);
                sdo[i] = ldv(dO + off + i);
            }
            __syncthreads();
            // rows: dS += dO q^T ; u = beta (v - alpha S_{t-1} k)
            for (int i = tid; i < d; i += kThreads) {
                const float doi = sdo[i];
                float r = 0.0f;
                for (int j = 0; j < d; ++j) {
                    dS[i * sd + j] = fmaf(doi, sq[j], dS[i * sd + j]);
                    r = fmaf(Sb[i * sd + j], sk[j], r);
                }
                const float be = beta_scalar ? ldv(beta + boff) : ldv(beta + off + i);
                const float err = ldv(v + off + i) - al * r;
                ser[i] = err;
                su[i] = be * err;
            }
            __syncthreads();
            // columns: dq = S_t^T dO
            for (int j = tid; j < d; j += kThreads) {
                float acc = 0.0f;
                for (int i = 0; i < d; ++i) acc = fmaf(Sa[i * sd + j], sdo[i], acc);
                st_scalar<T>(gq + off + j, acc);
            }
            // rows: dsk = dS k; dv = beta dsk; dbeta = err dsk
            float bsum = 0.0f;
            for (int i = tid; i < d; i += kThreads) {
                float dsk = 0.0f;
                for (int j = 0; j < d; ++j) dsk = fmaf(dS[i * sd + j], sk[j], dsk);
                const float be = beta_scalar ? ldv(beta + boff) : ldv(beta + off + i);
                const float err = ser[i];
                st_scalar<T>(gv + off + i, be * dsk);
                if (beta_scalar) bsum = fmaf(err, dsk, bsum);
                else st_scalar<T>(gbeta + off + i, err * dsk);
                sbd[i] = be * dsk;
            }
            if (beta_scalar) {
                const float s = block_sum(bsum);
                if (tid == 0) st_scalar<T>(gbeta + boff, s);
            }
            __syncthreads();
            // columns: dk = dS^T u - alpha S_{t-1}^T (beta dsk)
            for (int j = tid; j < d; j += kThreads) {
                float acc = 0.0f;
                for (int i = 0; i < d; ++i)
                    acc += dS[i * sd + j] * su[i] - al * Sb[i * sd + j] * sbd[i];
                st_scalar<T>(gk + off + j, acc);
            }
            __syncthreads();
            // rows: dS_d = dS - (beta dsk) k^T; dalpha = <dS_d, S_{t-1}>; dS_{t-1} = alpha dS_d
            float ga = 0.0f;
            for (int i = tid; i < d; i += kThreads) {
                const float bd = sbd[i];
                for (int j = 0; j < d; ++j) {
                    const float x = fmaf(-bd, sk[j], dS[i * sd + j]);
                    ga = fmaf(x, Sb[i * sd + j], ga);
                    dS[i * sd + j] = al * x;
                }
            }
            const float gas = block_sum(ga);
            if (tid == 0) st_scalar<T>(galpha + boff, gas);
            // S_{t-1} becomes the next step's S_t
            float* tmp = Sa;
            Sa = Sb;
            Sb = tmp;
            __syncthreads();
        }
    }
}

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t ckpt_bytes(int B, int L, int H, int d) {
    const int nck = (L + CK - 1) / CK;
    return (size_t)B * H * (nck + 1) * d * d * sizeof(float);
}

size_t gated_bwd_smem(int d) {
    return ((size_t)3 * d * (d + 1) + 6 * d + kThreads) * sizeof(float);
}
size_t gated_state_buf_bytes(int B, int H, int d) {
    return (size_t)B * H * CK * d * d * sizeof(float);
}
size_t bwd_smem(int d) {
    return ((size_t)2 * d * (d + 1) + (size_t)CK * d + 5 * d + kThreads) * sizeof(float);
}

template <typename T, int CPL, bool GATED>
int launch_fwd_rows(const void* q, const void* k, const void* v, const void* beta,
                    const void* alpha, void* o, float* ckpt, int B, int L, int H, int d,
                    int beta_scalar, cudaStream_t st) {
    constexpr size_t smem = fwd_rows_smem<CPL>();
    cudaError_t e = cudaFuncSetAttribute(delta_fwd_rows_kernel<T, CPL, GATED>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    delta_fwd_rows_kernel<T, CPL, GATED>
        <<<dim3(H, B, (d + kRowsPerCta - 1) / kRowsPerCta), kRowThreads, smem, st>>>(
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
                   ? launch_fwd_rows<T, 8, true>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                                 beta_scalar, st)
                   : launch_fwd_rows<T, 8, false>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                                  beta_scalar, st);
    return alpha != nullptr
               ? launch_fwd_rows<T, 32, true>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                              beta_scalar, st)
               : launch_fwd_rows<T, 32, false>(q, k, v, beta, alpha, o, ckpt, B, L, H, d,
                                               beta_scalar, st);
}

template <typename T>
int launch_gated_bwd(const void* q, const void* k, const void* v, const void* beta,
                     const void* alpha, const void* dO, const float* ckpt, float* sbuf, void* gq,
                     void* gk, void* gv, void* gbeta, void* galpha, int B, int L, int H, int d,
                     int beta_scalar, cudaStream_t st) {
    const size_t smem = gated_bwd_smem(d);
    cudaError_t e = cudaFuncSetAttribute(gated_bwd_rec_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    gated_bwd_rec_kernel<T><<<dim3(H, B), kThreads, smem, st>>>(
        (const T*)q, (const T*)k, (const T*)v, (const T*)beta, (const T*)alpha, (const T*)dO,
        ckpt, sbuf, (T*)gq, (T*)gk, (T*)gv, (T*)gbeta, (T*)galpha, L, H, d, beta_scalar);
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T>
int launch_bwd(const void* q, const void* k, const void* v, const void* beta, const void* dO,
               const float* ckpt, void* gq, void* gk, void* gv, void* gbeta, int B, int L, int H,
               int d, int beta_scalar, cudaStream_t st) {
    const size_t smem = bwd_smem(d);
    cudaError_t e = cudaFuncSetAttribute(delta_bwd_rec_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    delta_bwd_rec_kernel<T><<<dim3(H, B), kThreads, smem, st>>>(
        (const T*)q, (const T*)k, (const T*)v, (const T*)beta, (const T*)dO, ckpt, (T*)gq, (T*)gk,
        (T*)gv, (T*)gbeta, L, H, d, beta_scalar);
    return edb::status_from_cuda(cudaGetLastError());
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
size_t edb_delta_chunked_bwd_ws(int B, int L, int H);
int edb_delta_chunked_fwd(const void* q, const void* k, const void* v, const void* beta, void* o,
                          float* resid, int B, int L, int H, void* ws, cudaStream_t st);
int edb_delta_chunked_bwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* dO, const float* resid, void* gq, void* gk, void* gv,
                          void* gbeta, int B, int L, int H, void* ws, cudaStream_t st);

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
        return edb_delta_chunked_fwd(q, k, v, beta, o, s_ckpt, batch, seq_len, heads, workspace,
                                     st);
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
        const size_t b = edb_delta_chunked_bwd_ws(batch, seq_len, heads);
        return ck + (have_ckpt ? b : (f > b ? f : b));
    }
    return ck;
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
            int s = edb_delta_chunked_fwd(q, k, v, beta, gq, r, batch, seq_len, heads, scratch,
                                          st);
            if (s) return s;
            resid = r;
        }
        return edb_delta_chunked_bwd(q, k, v, beta, dO, resid, gq, gk, gv, gbeta, batch, seq_len,
                                     heads, scratch, st);
    }
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
    return dtype == EDB_BF16
               ? launch_bwd<__nv_bfloat16>(q, k, v, beta, dO, ck, gq, gk, gv, gbeta, batch,
                                           seq_len, heads, head_dim, bs, st)
               : launch_bwd<float>(q, k, v, beta, dO, ck, gq, gk, gv, gbeta, batch, seq_len,
                                   heads, head_dim, bs, st);
}

// ------------------------------------------------------------------ GatedDeltaNet
// Token recurrence only (the chunked tensor-core form serves the ungated rule).
extern "C" size_t edb_gated_delta_net_ckpt_bytes(int dtype, int beta_per_element, int batch,
                                                 int seq_len, int heads, int head_dim) {
    (void)beta_per_element;
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    return ckpt_bytes(batch, seq_len, heads, head_dim);
}

extern "C" int edb_gated_delta_net_fwd(int dtype, const void* q, const void* k, const void* v,
                                       const void* beta, int beta_per_element, const void* alpha,
                                       void* o, float* s_ckpt, int batch, int seq_len, int heads,
                                       int head_dim, void* stream) {
    if (int s = check(dtype, batch, seq_len, heads, head_dim)) return s;
    if (!q || !k || !v || !beta || !alpha || !o) return EDB_ERR_NULL_POINTER;
    const int bs = beta_per_element ? 0 : 1;
    cudaStream_t st = (cudaStream_t)stream;
    return dtype == EDB_BF16
               ? launch_fwd<__nv_bfloat16>(q, k, v, beta, alpha, o, s_ckpt, batch, seq_len,
                                           heads, head_dim, bs, st)
               : launch_fwd<float>(q, k, v, beta, alpha, o, s_ckpt, batch, seq_len, heads,
                                   head_dim, bs, st);
}

extern "C" size_t edb_gated_delta_net_bwd_workspace(int dtype, int beta_per_element, int batch,
                                                    int seq_len, int heads, int head_dim,
                                                    int have_ckpt) {
    if (check(dtype, batch, seq_len, heads, head_dim)) return 0;
    const size_t ck = have_ckpt ? 0
                                : a256(edb_gated_delta_net_ckpt_bytes(dtype, beta_per_element,
                                                                      batch, seq_len, heads,
                                                                      head_dim));
    return ck + gated_state_buf_bytes(batch, heads, head_dim);
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
    if (reinterpret_cast<uintptr_t>(workspace) & 15u) return EDB_ERR_MISALIGNED;
    cudaStream_t st = (cudaStream_t)stream;
    char* p = static_cast<char*>(workspace);
    const float* ck = s_ckpt;
    if (!ck) {
        // states only: the forward writes o into gq, which the backward overwrites
        float* w = reinterpret_cast<float*>(p);
        p += a256(edb_gated_delta_net_ckpt_bytes(dtype, beta_per_element, batch, seq_len, heads,
                                                 head_dim));
        int s = edb_gated_delta_net_fwd(dtype, q, k, v, beta, beta_per_element, alpha, gq, w,
                                        batch, seq_len, heads, head_dim, stream);
        if (s) return s;
        ck = w;
    }
    const int bs = beta_per_element ? 0 : 1;
    float* sbuf = reinterpret_cast<float*>(p);
    return dtype == EDB_BF16
               ? launch_gated_bwd<__nv_bfloat16>(q, k, v, beta, alpha, dO, ck, sbuf, gq, gk, gv,
                                                 gbeta, galpha, batch, seq_len, heads, head_dim,
                                                 bs, st)
               : launch_gated_bwd<float>(q, k, v, beta, alpha, dO, ck, sbuf, gq, gk, gv, gbeta,
                                         galpha, batch, seq_len, heads, head_dim, bs, st);
}
