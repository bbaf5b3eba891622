// selective_scan.cu -- Mamba selective scan, forward + backward (kernel semantics).
//
// Reference semantics (edifice project paths):
//   forward   native/cuda/fused_selective_scan.cu:41-98 ==
//             test/edifice/cuda/backward_kernels_test.exs:1563-1586
//   backward  lib/edifice/cuda/fused_scan.ex:1453-1531 (A gets no gradient;
//             gdt is zero where dt lies outside [dt_min, dt_max]; gB, gC f32)
// per (b, d):  dtc = clip(dt, dt_min, dt_max)
//              h_n = exp(dtc A[d,n]) h_n + dtc B[b,t,n] x       (h_{-1} = 0)
//              y   = sum_n C[b,t,n] h_n
//
// Design (B200): the work is exponential/issue-bound (one exp per (t,d,n)),
// the parallelism is batch x channel (262k channels at config 4), so every
// thread owns one channel and walks the sequence in order with its N states in
// registers; B/C rows (shared by every channel of a batch row) are staged in
// shared memory per time tile; exp(dtc A) is one ex2.approx of dtc * (A log2 e).
//
// Backward (recompute, never the reference's [B,D,L,N] workspace):
//   * the forward can write h at the start of every CK-step chunk
//     (ckpt [B, L/CK, D, N] f32); without it the backward computes them first;
//   * per chunk, in reverse: a pass rebuilds sub-chunk states (every TS steps)
//     into shared memory, then each sub-chunk is recomputed into registers and
//     walked in reverse accumulating dh, gx, gdt;
//   * gB, gC (sums over channels) are reduced deterministically: warp
//     transpose-reduce, cross-warp sum in shared memory, one partial per
//     (channel block, b, t, n) to the workspace, then a second kernel sums the
//     channel-block partials in a fixed order.  No atomics.
#include <type_traits>

#include "edb_common.cuh"
#include "tc_common.cuh"

namespace {

constexpr int kThreads = 128;  // channels per CTA
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

static __device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

static __device__ __forceinline__ float2 ex2_2(float2 x) { return make_float2(ex2(x.x), ex2(x.y)); }

// Decays of the model's fixed A[d, n] = -(n + 1) (lib/edifice/ssm/common.ex:409):
// exp(-dtc (n + 1)) = r^(n+1), r = exp(-dtc).  pw starts at (r, r^2) for the pair
// n = (0, 1); next_power returns the current pair and steps it by r^2.
static __device__ __forceinline__ void fixa_powers(float dtc, float2& pw, float2& rr2) {
    const float r = ex2(-dtc * 1.4426950408889634f);
    pw = make_float2(r, r * r);
    rr2 = make_float2(r * r, r * r);
}
// As fixa_powers for the states of one half of 16: half 1 starts at the pair
// n = (8, 9), i.e. (r^9, r^10) = (r, r^2) r^8.
static __device__ __forceinline__ void fixa_powers_half(float dtc, int half, float2& pw,
                                                        float2& rr2) {
    fixa_powers(dtc, pw, rr2);
    if (half) {
        const float r4 = rr2.x * rr2.x;
        pw = mul2(pw, make_float2(r4 * r4, r4 * r4));
    }
}
static __device__ __forceinline__ float2 next_power(float2& pw, float2 rr2) {
    const float2 a = pw;
    pw = mul2(pw, rr2);
    return a;
}

// chunk / sub-chunk lengths per padded state count: TS*NS = 64 state values in
// registers per sub-chunk.  Checkpoints every CK steps: 8 for 16 states (the
// tensor-core-reduce backward rebuilds one sub-chunk start per chunk, so 1.5
// exps per (t, d, n) instead of 2), 8 sub-chunks for 8 states.
template <int NS>
struct SsmTiling {
    static constexpr int TS = 64 / NS;
    static constexpr int CK = NS == 16 ? 2 * TS : 8 * TS;
};

template <typename T>
static __device__ __forceinline__ float ldf(const T* p) {
    return ld_scalar<T>(p);
}

// A[d, n]; in model mode a NULL A is the fixed diagonal -(n + 1) of
// lib/edifice/ssm/common.ex:409 (discretize_ssm).
template <bool MODEL, typename T>
static __device__ __forceinline__ float a_at(const T* A, int d, int n, int N) {
    if (MODEL && A == nullptr) return -(float)(n + 1);
    return ldf(A + (long long)d * N + n);
}

// ------------------------------------------------------------------ forward
// grid (ceil(D/128), B), block 128.  TB time steps of B/C per smem tile.
template <typename T, int NS, bool STATES_ONLY, bool MODEL>
__global__ void __launch_bounds__(kThreads)
    ssm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ dt, const T* __restrict__ A,
                   const T* __restrict__ Bm, const T* __restrict__ Cm, T* __restrict__ y,
                   float* __restrict__ ckpt, const float* __restrict__ dtm, int L, int D, int N,
                   float dt_min, float dt_max) {
    constexpr int TB = 32;
    constexpr int CK = SsmTiling<NS>::CK;
    __shared__ float sB[TB][NS];
    __shared__ float sC[TB][NS];
    __shared__ float sDm[TB];  // model mode: channel-mean of the clamped dt per step
    const int tid = threadIdx.x;
    const int d = blockIdx.x * kThreads + tid;
    const int b = blockIdx.y;
    const bool live = d < D;
    const int nck = (L + CK - 1) / CK;

    float A2[NS], h[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        A2[n] = (live && n < N) ? a_at<MODEL>(A, d, n, N) * kLog2e : 0.0f;
        h[n] = 0.0f;
    }
    const long long row0 = (long long)b * L;
    for (int t0 = 0; t0 < L; t0 += TB) {
        const int tn = min(TB, L - t0);
        __syncthreads();
        for (int i = tid; i < TB * NS; i += kThreads) {
            const int tt = i / NS, n = i % NS;
            const bool ok = tt < tn && n < N;
            const long long o = (row0 + t0 + tt) * N + n;
            sB[tt][n] = ok ? ldf(Bm + o) : 0.0f;
            if (!STATES_ONLY) sC[tt][n] = ok ? ldf(Cm + o) : 0.0f;
        }
        if (MODEL)
            for (int i = tid; i < TB; i += kThreads) sDm[i] = i < tn ? dtm[row0 + t0 + i] : 0.0f;
        __syncthreads();
        if (!live) continue;
        for (int tt = 0; tt < tn; ++tt) {
            const int t = t0 + tt;
            if (ckpt != nullptr && (t % CK) == 0) {
                float* cp = ckpt + (((long long)b * nck + t / CK) * D + d) * NS;
#pragma unroll
                for (int n = 0; n < NS; n += 4)
                    *reinterpret_cast<float4*>(cp + n) = make_float4(h[n], h[n + 1], h[n + 2], h[n + 3]);
            }
            const long long o = (row0 + t) * D + d;
            const float dtc = fminf(fmaxf(ldf(dt + o), dt_min), dt_max);
            const float dtx = (MODEL ? sDm[tt] : dtc) * ldf(x + o);
            float acc = 0.0f;
#pragma unroll
            for (int n = 0; n < NS; ++n) {
                const float ab = ex2(dtc * A2[n]);
                h[n] = fmaf(ab, h[n], dtx * sB[tt][n]);
                if (!STATES_ONLY) acc = fmaf(sC[tt][n], h[n], acc);
            }
            if (!STATES_ONLY) st_scalar<T>(y + o, acc);
        }
    }
}

// ------------------------------------------------------------------ backward
// Sum V = 2*NS per-lane values over the 32 lanes of a warp.  On return lane l
// holds the warp total of value index (l % V) (for V < 32 several lanes hold
// the same total).  Recursive halving: 31 shuffles for V = 32.
template <int V>
static __device__ __forceinline__ float warp_transpose_reduce(float (&v)[V], int lane) {
    static_assert(V == 16 || V == 32, "V");
    if constexpr (V == 16) {
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], 16);
    }
    // halving: for lane bit V/2 .. 1, a lane whose bit is set keeps the upper
    // half of its remaining values and receives the partner's upper half.
#pragma unroll
    for (int bit = V / 2; bit >= 1; bit >>= 1) {
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int i = 0; i < bit; ++i) {
            const float send = upper ? v[i] : v[i + bit];
            const float keep = upper ? v[i + bit] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
        }
    }
    return v[0];
}

// Value index held by lane l after warp_transpose_reduce<V>.
template <int V>
static __device__ __forceinline__ int reduced_index(int lane) {
    // after halving over bits V/2..1, lane keeps the upper half whenever its bit is set
    return lane & (V - 1);
}

// grid (ceil(D/128), B), block 128.
// gpart: [2][nblk][B][L][NS] f32 partial sums over this CTA's 128 channels
template <typename T, int NS, bool MODEL>
__global__ void __launch_bounds__(kThreads)
    ssm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ dt, const T* __restrict__ A,
                   const T* __restrict__ Bm, const T* __restrict__ Cm, const T* __restrict__ dy,
                   const float* __restrict__ ckpt, const float* __restrict__ dtm,
                   T* __restrict__ gx, T* __restrict__ gdt, float* __restrict__ gpart, int Bsz,
                   int L, int D, int N, float dt_min, float dt_max) {
    constexpr int TS = SsmTiling<NS>::TS;
    constexpr int CK = SsmTiling<NS>::CK;
    constexpr int V = 2 * NS;  // gB and gC values per step
    static_assert(V <= 32, "NS <= 16 in this kernel");
    __shared__ float sB[CK][NS];
    __shared__ float sC[CK][NS];
    __shared__ float sDm[CK];                        // model mode: mean clamped dt per step
    __shared__ float sRed[kThreads / 32][TS][32];    // per-warp reduced gB|gC
    extern __shared__ float sSubFlat[];              // [SUBS][NS][kThreads] sub-chunk states
    auto sSub = reinterpret_cast<float(*)[NS][kThreads]>(sSubFlat);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d = blockIdx.x * kThreads + tid;
    const int b = blockIdx.y;
    const bool live = d < D;
    const int nck = (L + CK - 1) / CK;
    const int nblk = gridDim.x;
    const long long row0 = (long long)b * L;

    float A2[NS], dh[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        A2[n] = (live && n < N) ? a_at<MODEL>(A, d, n, N) * kLog2e : 0.0f;
        dh[n] = 0.0f;
    }
    const int ridx = reduced_index<V>(lane);

    for (int c = nck - 1; c >= 0; --c) {
        const int t0 = c * CK;
        const int tn = min(CK, L - t0);
        __syncthreads();
        for (int i = tid; i < CK * NS; i += kThreads) {
            const int tt = i / NS, n = i % NS;
            const bool ok = tt < tn && n < N;
            const long long o = (row0 + t0 + tt) * N + n;
            sB[tt][n] = ok ? ldf(Bm + o) : 0.0f;
            sC[tt][n] = ok ? ldf(Cm + o) : 0.0f;
        }
        if (MODEL)
            for (int i = tid; i < CK; i += kThreads) sDm[i] = i < tn ? dtm[row0 + t0 + i] : 0.0f;
        __syncthreads();
        // ---- sub-chunk start states
        float h[NS];
        if (live) {
            const float* cp = ckpt + (((long long)b * nck + c) * D + d) * NS;
#pragma unroll
            for (int n = 0; n < NS; ++n) h[n] = cp[n];
        } else {
#pragma unroll
            for (int n = 0; n < NS; ++n) h[n] = 0.0f;
        }
        for (int tt = 0; tt < tn; ++tt) {
            if (tt % TS == 0) {
#pragma unroll
                for (int n = 0; n < NS; ++n) sSub[tt / TS][n][tid] = h[n];
            }
            if (live) {
                const long long o = (row0 + t0 + tt) * D + d;
                const float dtc = fminf(fmaxf(ldf(dt + o), dt_min), dt_max);
                const float dtx = (MODEL ? sDm[tt] : dtc) * ldf(x + o);
#pragma unroll
                for (int n = 0; n < NS; ++n)
                    h[n] = fmaf(ex2(dtc * A2[n]), h[n], dtx * sB[tt][n]);
            }
        }
        // ---- sub-chunks in reverse
        const int nsub = (tn + TS - 1) / TS;
        for (int s = nsub - 1; s >= 0; --s) {
            const int u0 = s * TS;                // offset in chunk
            const int un = min(TS, tn - u0);
            float hs[TS][NS];
#pragma unroll
            for (int n = 0; n < NS; ++n) h[n] = sSub[s][n][tid];
#pragma unroll
            for (int j = 0; j < TS; ++j) {
                if (j < un && live) {
                    const long long o = (row0 + t0 + u0 + j) * D + d;
                    const float dtc = fminf(fmaxf(ldf(dt + o), dt_min), dt_max);
                    const float dtx = (MODEL ? sDm[u0 + j] : dtc) * ldf(x + o);
#pragma unroll
                    for (int n = 0; n < NS; ++n)
                        h[n] = fmaf(ex2(dtc * A2[n]), h[n], dtx * sB[u0 + j][n]);
                }
#pragma unroll
                for (int n = 0; n < NS; ++n) hs[j][n] = h[n];
            }
#pragma unroll
            for (int j = TS - 1; j >= 0; --j) {
                float red[V];
#pragma unroll
                for (int i = 0; i < V; ++i) red[i] = 0.0f;
                const bool act = j < un && live;
                if (act) {
                    const int tt = u0 + j;
                    const long long o = (row0 + t0 + tt) * D + d;
                    const float draw = ldf(dt + o);
                    const float dtc = fminf(fmaxf(draw, dt_min), dt_max);
                    const float xv = ldf(x + o);
                    const float dyv = ldf(dy + o);
                    const float dti = MODEL ? sDm[tt] : dtc;  // dt of the input term
                    const float dtx = dti * xv;
                    float gxa = 0.0f, gda = 0.0f;
#pragma unroll
                    for (int n = 0; n < NS; ++n) {
                        const float Bn = sB[tt][n], Cn = sC[tt][n];
                        const float ab = ex2(dtc * A2[n]);
                        const float hc = hs[j][n];
                        const float dht = fmaf(dyv, Cn, dh[n]);   // dh_state += dy * C
                        red[NS + n] = dyv * hc;                     // gC partial
                        red[n] = dht * dtx;                         // gB partial (dh x dt)
                        gxa = fmaf(dht, Bn, gxa);                   // gx = dt * sum dh B
                        // ddt = dh * (A_bar h_prev A + B x), A_bar h_prev = hc - dtx B
                        const float abhp = fmaf(-dtx, Bn, hc);
                        gda = fmaf(dht, fmaf(abhp, A2[n] * kLn2, MODEL ? 0.0f : Bn * xv), gda);
                        dh[n] = dht * ab;
                    }
                    st_scalar<T>(gx + o, gxa * dti);
                    const bool inr = draw >= dt_min && draw <= dt_max;
                    st_scalar<T>(gdt + o, inr ? gda : 0.0f);
                }
                const float r = warp_transpose_reduce<V>(red, lane);
                if (lane < V) sRed[warp][j][ridx] = r;
            }
            __syncthreads();
            // cross-warp sum and write this CTA's partials for the sub-chunk
            for (int i = tid; i < TS * V; i += kThreads) {
                const int j = i / V, vi = i % V;
                if (j < un) {
                    float sum = 0.0f;
#pragma unroll
                    for (int w = 0; w < kThreads / 32; ++w) sum += sRed[w][j][vi];
                    const int which = vi >= NS;       // 0: gB, 1: gC
                    const int n = vi - which * NS;
                    const long long o =
                        ((((long long)which * nblk + blockIdx.x) * Bsz + b) * L + t0 + u0 + j) *
                            NS + n;
                    gpart[o] = sum;
                }
            }
            __syncthreads();
        }
    }
}

// gB/gC[b,t,n] = sum over channel blocks of the partials (fixed order)
template <int NS>
__global__ void ssm_reduce_kernel(const float* __restrict__ gpart, float* __restrict__ gB,
                                  float* __restrict__ gC, int nblk, long long BL, int N) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = BL * N;
    if (i >= total) return;
    const long long bl = i / N;
    const int n = (int)(i % N);
    float sb = 0.0f, sc = 0.0f;
    for (int k = 0; k < nblk; ++k) {
        sb += gpart[((long long)k * BL + bl) * NS + n];
        sc += gpart[((long long)(nblk + k) * BL + bl) * NS + n];
    }
    gB[i] = sb;
    gC[i] = sc;
}

// ------------------------------------------------------------------ staged kernels
// The same recurrences with every per-step read of x / dt (/ dy) served from
// shared memory: [steps][128 channels] tiles arrive by 16-byte cp.async
// (zero-filled past L and D), so a step never waits on HBM latency.  Used when
// D is a multiple of 16 / sizeof(T) and x, dt (, dy) are 16-byte aligned.
template <typename T>
struct StageGeom {
    static constexpr int ROWB = kThreads * (int)sizeof(T);  // bytes of one tile row
    static constexpr int CPR = ROWB / 16;                    // 16-byte copies per row
    static constexpr int EPC = 16 / (int)sizeof(T);          // elements per copy
};

// Copies rows t0 .. t0 + rows - 1, channels d0 .. d0 + 127 of a [B*L][D]
// array (row0 = b * L) into dst[rows][128].
template <typename T, int ROWS>
static __device__ __forceinline__ void stage_rows(unsigned char* dst, const T* src, long long row0,
                                                  int t0, int L, int d0, int D) {
    using G = StageGeom<T>;
    constexpr int CPT = ROWS * G::CPR / kThreads;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
        const int idx = threadIdx.x + i * kThreads;
        const int r = idx / G::CPR, c16 = idx % G::CPR;
        const int t = t0 + r, dd = d0 + c16 * G::EPC;
        const bool ok = t < L && dd < D;
        cp_async16(dst + r * G::ROWB + c16 * 16, src + (ok ? (row0 + t) * D + dd : 0),
                   ok ? 16u : 0u);
    }
}

// grid (ceil(D/128), B), block 128; two x/dt tiles of TB steps in flight.
// FIXA (model semantics with A = NULL): A[d, n] = -(n + 1), so the decays of one
// (t, d) are the powers r^(n+1) of r = exp(-dtc): one ex2 and NS/2 packed
// multiplies instead of NS ex2 (relative error ~(n+1) ulp of r, ~4e-6 at n = 15).
template <typename T, int NS, bool STATES_ONLY, bool MODEL, bool FIXA = false>
__global__ void __launch_bounds__(kThreads)
    ssm_fwd_staged_kernel(const T* __restrict__ x, const T* __restrict__ dt,
                          const T* __restrict__ A, const T* __restrict__ Bm,
                          const T* __restrict__ Cm, T* __restrict__ y, float* __restrict__ ckpt,
                          const float* __restrict__ dtm, int L, int D, int N, float dt_min,
                          float dt_max) {
    constexpr int TB = 32;
    constexpr int CK = SsmTiling<NS>::CK;
    static_assert(CK % TB == 0 || TB % CK == 0, "checkpoints fall on tile starts or inside");
    constexpr int TILEB = TB * StageGeom<T>::ROWB;
    constexpr int BCV = TB * NS / kThreads;  // B (and C) values per thread and tile
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char* sX = smem;                                 // [2][TB][128] T
    unsigned char* sDt = smem + 2 * TILEB;                    // [2][TB][128] T
    float* sB = reinterpret_cast<float*>(smem + 4 * TILEB);  // [2][TB][NS]
    float* sC = sB + 2 * TB * NS;                             // [2][TB][NS]
    float* sDm = sC + 2 * TB * NS;                            // [2][TB] (model mode)
    const int tid = threadIdx.x;
    const int d0 = blockIdx.x * kThreads, d = d0 + tid;
    const int b = blockIdx.y;
    const bool live = d < D;
    const int nck = (L + CK - 1) / CK;
    const int ntiles = (L + TB - 1) / TB;
    const long long row0 = (long long)b * L;

    constexpr int NP = NS / 2;  // state pairs for the packed f32x2 instructions
    float2 A2[NP], h[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int n = 2 * p;
        A2[p].x = (live && n < N) ? a_at<MODEL>(A, d, n, N) * kLog2e : 0.0f;
        A2[p].y = (live && n + 1 < N) ? a_at<MODEL>(A, d, n + 1, N) * kLog2e : 0.0f;
        h[p] = dup2(0.0f);
    }
    float rb[BCV], rc[BCV], rdm = 0.0f;
    auto load_bc = [&](int k) {
        if (MODEL) {
            const int t = k * TB + tid;
            rdm = (tid < TB && t < L) ? dtm[row0 + t] : 0.0f;
        }
#pragma unroll
        for (int v = 0; v < BCV; ++v) {
            const int idx = tid + v * kThreads, tt = idx / NS, n = idx % NS;
            const int t = k * TB + tt;
            const bool ok = t < L && n < N;
            const long long o = (row0 + (ok ? t : 0)) * N + (ok ? n : 0);
            rb[v] = ok ? ldf(Bm + o) : 0.0f;
            rc[v] = (ok && !STATES_ONLY) ? ldf(Cm + o) : 0.0f;
        }
    };
    auto store_bc = [&](int k) {
#pragma unroll
        for (int v = 0; v < BCV; ++v) {
            sB[(k & 1) * TB * NS + tid + v * kThreads] = rb[v];
            sC[(k & 1) * TB * NS + tid + v * kThreads] = rc[v];
        }
        if (MODEL && tid < TB) sDm[(k & 1) * TB + tid] = rdm;
    };
    auto issue = [&](int k) {
        stage_rows<T, TB>(sX + (k & 1) * TILEB, x, row0, k * TB, L, d0, D);
        stage_rows<T, TB>(sDt + (k & 1) * TILEB, dt, row0, k * TB, L, d0, D);
        cp_async_commit();
    };
    issue(0);
    load_bc(0);
    store_bc(0);
    for (int k = 0; k < ntiles; ++k) {
        if (k + 1 < ntiles) {
            issue(k + 1);
            load_bc(k + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (live) {
            const T* xs = reinterpret_cast<const T*>(sX + (k & 1) * TILEB) + tid;
            const T* dts = reinterpret_cast<const T*>(sDt + (k & 1) * TILEB) + tid;
            const float* bk = sB + (k & 1) * TB * NS;
            const float* ckc = sC + (k & 1) * TB * NS;
            const int t0 = k * TB, tn = min(TB, L - t0);
            for (int tt = 0; tt < tn; ++tt) {
                if (ckpt != nullptr && (t0 + tt) % CK == 0) {
                    float* cp = ckpt + (((long long)b * nck + (t0 + tt) / CK) * D + d) * NS;
#pragma unroll
                    for (int p = 0; p < NP; p += 2)
                        *reinterpret_cast<float4*>(cp + 2 * p) =
                            make_float4(h[p].x, h[p].y, h[p + 1].x, h[p + 1].y);
                }
                const float dtc = fminf(fmaxf(ldf(dts + tt * kThreads), dt_min), dt_max);
                const float dti = MODEL ? sDm[(k & 1) * TB + tt] : dtc;
                const float2 dtc2 = dup2(dtc), dtx2 = dup2(dti * ldf(xs + tt * kThreads));
                float2 acc = dup2(0.0f);
                float2 pw, rr2;
                if (FIXA) fixa_powers(dtc, pw, rr2);
#pragma unroll
                for (int p = 0; p < NP; p += 2) {
                    const float4 b4 = *reinterpret_cast<const float4*>(bk + tt * NS + 2 * p);
                    float4 c4 = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (!STATES_ONLY) c4 = *reinterpret_cast<const float4*>(ckc + tt * NS + 2 * p);
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const float2 bq = q ? make_float2(b4.z, b4.w) : make_float2(b4.x, b4.y);
                        const float2 a = FIXA ? next_power(pw, rr2) : ex2_2(mul2(dtc2, A2[p + q]));
                        h[p + q] = fma2(a, h[p + q], mul2(dtx2, bq));
                        if (!STATES_ONLY) {
                            const float2 cq = q ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
                            acc = fma2(cq, h[p + q], acc);
                        }
                    }
                }
                if (!STATES_ONLY) st_scalar<T>(y + (row0 + t0 + tt) * D + d, acc.x + acc.y);
            }
        }
        if (k + 1 < ntiles) store_bc(k + 1);
        __syncthreads();
    }
}

template <typename T, int NS>
constexpr size_t fwd_staged_smem() {
    return (size_t)4 * 32 * StageGeom<T>::ROWB + (size_t)4 * 32 * NS * sizeof(float) +
           (size_t)2 * 32 * sizeof(float);
}

// grid (ceil(D/128), B), block 128: ssm_bwd_kernel with the chunk's x, dt, dy
// rows staged in shared memory (one chunk at a time; two CTAs share an SM).
template <typename T, int NS, bool MODEL, bool FIXA = false>
__global__ void __launch_bounds__(kThreads)
    ssm_bwd_staged_kernel(const T* __restrict__ x, const T* __restrict__ dt,
                          const T* __restrict__ A, const T* __restrict__ Bm,
                          const T* __restrict__ Cm, const T* __restrict__ dy,
                          const float* __restrict__ ckpt, const float* __restrict__ dtm,
                          T* __restrict__ gx, T* __restrict__ gdt, float* __restrict__ gpart,
                          int Bsz, int L, int D, int N, float dt_min, float dt_max) {
    constexpr int TS = SsmTiling<NS>::TS;
    constexpr int CK = SsmTiling<NS>::CK;
    constexpr int SUBS = CK / TS;
    constexpr int V = 2 * NS;
    static_assert(V <= 32, "NS <= 16 in this kernel");
    constexpr int TILEB = CK * StageGeom<T>::ROWB;
    constexpr int BCV = CK * NS / kThreads;
    extern __shared__ __align__(16) unsigned char smem[];
    auto sSub = reinterpret_cast<float(*)[NS][kThreads]>(smem);  // [SUBS][NS][128]
    unsigned char* tiles = smem + SUBS * NS * kThreads * sizeof(float);  // x | dt | dy
    float* sB = reinterpret_cast<float*>(tiles + 3 * TILEB);             // [CK][NS]
    float* sC = sB + CK * NS;                                             // [CK][NS]
    // per-warp gB|gC sums of every step of the chunk; summed across warps once
    // per chunk, so the warps run out of phase between the chunk barriers
    auto sRed = reinterpret_cast<float(*)[CK][V]>(sC + CK * NS);         // [4][CK][V]
    float* sDm = &sRed[kThreads / 32][0][0];  // [CK] model mode: mean clamped dt per step
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d0 = blockIdx.x * kThreads, d = d0 + tid;
    const int b = blockIdx.y;
    const bool live = d < D;
    const int nck = (L + CK - 1) / CK;
    const int nblk = gridDim.x;
    const long long row0 = (long long)b * L;
    const T* sx = reinterpret_cast<const T*>(tiles) + tid;
    const T* sdt = reinterpret_cast<const T*>(tiles + TILEB) + tid;
    const T* sdy = reinterpret_cast<const T*>(tiles + 2 * TILEB) + tid;

    // state pairs (n, n+1) go through the packed f32x2 instructions
    constexpr int NP = NS / 2;
    float2 A2[NP], A2ln[NP], dh[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int n = 2 * p;
        A2[p].x = (live && n < N) ? a_at<MODEL>(A, d, n, N) * kLog2e : 0.0f;
        A2[p].y = (live && n + 1 < N) ? a_at<MODEL>(A, d, n + 1, N) * kLog2e : 0.0f;
        A2ln[p] = mul2(A2[p], dup2(kLn2));
        dh[p] = dup2(0.0f);
    }
    const int ridx = reduced_index<V>(lane);

    for (int c = nck - 1; c >= 0; --c) {
        const int t0 = c * CK;
        const int tn = min(CK, L - t0);
        __syncthreads();  // the previous chunk is done with the tiles
        stage_rows<T, CK>(tiles, x, row0, t0, L, d0, D);
        stage_rows<T, CK>(tiles + TILEB, dt, row0, t0, L, d0, D);
        stage_rows<T, CK>(tiles + 2 * TILEB, dy, row0, t0, L, d0, D);
        cp_async_commit();
        {
            float rb[BCV], rc[BCV];
#pragma unroll
            for (int v = 0; v < BCV; ++v) {
                const int idx = tid + v * kThreads, tt = idx / NS, n = idx % NS;
                const bool ok = tt < tn && n < N;
                const long long o = (row0 + t0 + (ok ? tt : 0)) * N + (ok ? n : 0);
                rb[v] = ok ? ldf(Bm + o) : 0.0f;
                rc[v] = ok ? ldf(Cm + o) : 0.0f;
            }
#pragma unroll
            for (int v = 0; v < BCV; ++v) {
                sB[tid + v * kThreads] = rb[v];
                sC[tid + v * kThreads] = rc[v];
            }
            if (MODEL)
                for (int i = tid; i < CK; i += kThreads)
                    sDm[i] = i < tn ? dtm[row0 + t0 + i] : 0.0f;
        }
        float2 h[NP];
        if (live) {
            const float* cp = ckpt + (((long long)b * nck + c) * D + d) * NS;
#pragma unroll
            for (int p = 0; p < NP; p += 2) {
                const float4 v4 = *reinterpret_cast<const float4*>(cp + 2 * p);
                h[p] = make_float2(v4.x, v4.y);
                h[p + 1] = make_float2(v4.z, v4.w);
            }
        } else {
#pragma unroll
            for (int p = 0; p < NP; ++p) h[p] = dup2(0.0f);
        }
        cp_async_wait<0>();
        __syncthreads();
        // ---- sub-chunk start states
        for (int tt = 0; tt < tn; ++tt) {
            if (tt % TS == 0) {
#pragma unroll
                for (int p = 0; p < NP; ++p) {
                    sSub[tt / TS][2 * p][tid] = h[p].x;
                    sSub[tt / TS][2 * p + 1][tid] = h[p].y;
                }
            }
            const float dtc = fminf(fmaxf(ldf(sdt + tt * kThreads), dt_min), dt_max);
            const float2 dtc2 = dup2(dtc),
                         dtx2 = dup2((MODEL ? sDm[tt] : dtc) * ldf(sx + tt * kThreads));
            float2 pw, rr2;
            if (FIXA) fixa_powers(dtc, pw, rr2);
#pragma unroll
            for (int p = 0; p < NP; p += 2) {
                const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * NS + 2 * p);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const float2 bq = q ? make_float2(b4.z, b4.w) : make_float2(b4.x, b4.y);
                    const float2 a = FIXA ? next_power(pw, rr2) : ex2_2(mul2(dtc2, A2[p + q]));
                    h[p + q] = fma2(a, h[p + q], mul2(dtx2, bq));
                }
            }
        }
        // ---- sub-chunks in reverse: recompute h and exp(dt A) into registers,
        // then walk back
        const int nsub = (tn + TS - 1) / TS;
        for (int s = nsub - 1; s >= 0; --s) {
            const int u0 = s * TS;
            const int un = min(TS, tn - u0);
            float2 hs[TS][NP], as[TS][NP];
#pragma unroll
            for (int p = 0; p < NP; ++p) h[p] = make_float2(sSub[s][2 * p][tid], sSub[s][2 * p + 1][tid]);
#pragma unroll
            for (int j = 0; j < TS; ++j) {
                const int tt = min(u0 + j, tn - 1);  // steps past tn are never read back
                const float dtc = fminf(fmaxf(ldf(sdt + tt * kThreads), dt_min), dt_max);
                const float2 dtc2 = dup2(dtc),
                             dtx2 = dup2((MODEL ? sDm[tt] : dtc) * ldf(sx + tt * kThreads));
                float2 pw, rr2;
                if (FIXA) fixa_powers(dtc, pw, rr2);
#pragma unroll
                for (int p = 0; p < NP; p += 2) {
                    const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * NS + 2 * p);
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const float2 bq = q ? make_float2(b4.z, b4.w) : make_float2(b4.x, b4.y);
                        as[j][p + q] =
                            FIXA ? next_power(pw, rr2) : ex2_2(mul2(dtc2, A2[p + q]));
                        h[p + q] = fma2(as[j][p + q], h[p + q], mul2(dtx2, bq));
                        hs[j][p + q] = h[p + q];
                    }
                }
            }
#pragma unroll
            for (int j = TS - 1; j >= 0; --j) {
                float red[V];
                if (j < un && live) {
                    const int tt = u0 + j;
                    const float draw = ldf(sdt + tt * kThreads);
                    const float dtc = fminf(fmaxf(draw, dt_min), dt_max);
                    const float xv = ldf(sx + tt * kThreads);
                    const float dyv = ldf(sdy + tt * kThreads);
                    const float dti = MODEL ? sDm[tt] : dtc;  // dt of the input term
                    const float dtx = dti * xv;
                    const float2 dy2 = dup2(dyv), dtx2 = dup2(dtx), ndtx2 = dup2(-dtx);
                    float2 gxa = dup2(0.0f), gda = dup2(0.0f);
#pragma unroll
                    for (int p = 0; p < NP; p += 2) {
                        const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * NS + 2 * p);
                        const float4 c4 = *reinterpret_cast<const float4*>(sC + tt * NS + 2 * p);
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int m = p + q;
                            const float2 bq = q ? make_float2(b4.z, b4.w) : make_float2(b4.x, b4.y);
                            const float2 cq = q ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
                            const float2 hc = hs[j][m];
                            const float2 dht = fma2(dy2, cq, dh[m]);
                            const float2 gc = mul2(dy2, hc);
                            const float2 gb = mul2(dht, dtx2);
                            red[NS + 2 * m] = gc.x;
                            red[NS + 2 * m + 1] = gc.y;
                            red[2 * m] = gb.x;
                            red[2 * m + 1] = gb.y;
                            gxa = fma2(dht, bq, gxa);
                            // d h_t / d dtc = A (a h_{t-1}) + B x, a h_{t-1} = h_t - dtc x B;
                            // the B x part is summed once below (x gxa)
                            gda = fma2(mul2(dht, A2ln[m]), fma2(ndtx2, bq, hc), gda);
                            dh[m] = mul2(dht, as[j][m]);
                        }
                    }
                    const float gxs = gxa.x + gxa.y;
                    // model mode: the input term's dt is the channel mean, whose
                    // gradient ssm_model_gdt_kernel adds afterwards
                    const float gds = MODEL ? gda.x + gda.y : fmaf(xv, gxs, gda.x + gda.y);
                    const long long o = (row0 + t0 + tt) * D + d;
                    st_scalar<T>(gx + o, gxs * dti);
                    const bool inr = draw >= dt_min && draw <= dt_max;
                    st_scalar<T>(gdt + o, inr ? gds : 0.0f);
                } else {
#pragma unroll
                    for (int i = 0; i < V; ++i) red[i] = 0.0f;
                }
                const float r = warp_transpose_reduce<V>(red, lane);
                if (lane < V) sRed[warp][u0 + j][ridx] = r;
            }
        }
        __syncthreads();
        // this CTA's partial gB|gC of every step of the chunk (fixed warp order)
        for (int i = tid; i < CK * V; i += kThreads) {
            const int j = i / V, vi = i % V;
            if (j < tn) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kThreads / 32; ++w) sum += sRed[w][j][vi];
                const int which = vi >= NS;
                const int n = vi - which * NS;
                const long long o =
                    ((((long long)which * nblk + blockIdx.x) * Bsz + b) * L + t0 + j) * NS + n;
                gpart[o] = sum;
            }
        }
    }
}

template <typename T, int NS>
constexpr size_t bwd_staged_smem() {
    constexpr int TS = SsmTiling<NS>::TS, CK = SsmTiling<NS>::CK;
    return (size_t)(CK / TS) * NS * kThreads * sizeof(float) +
           (size_t)3 * CK * StageGeom<T>::ROWB + (size_t)2 * CK * NS * sizeof(float) +
           (size_t)(kThreads / 32) * CK * 2 * NS * sizeof(float) + (size_t)CK * sizeof(float);
}

// ------------------------------------------------ backward, tensor-core reduce
// bf16 io, 16 states: the same recompute-not-store backward (one thread per
// channel, its 16 states in registers) with the two sums over channels
// (gB = sum_d dh x dtc, gC = sum_d dY h) taken by the tensor core.  Each step's
// per-channel products go to shared memory as bf16 and tcgen05.mma.kind::f16
// adds them up, 16 channels per instruction:
//   D[m][*] = sum_k P[k][m] * 1,  m = (step j of a 4-step sub-chunk, gB|gC, n)
// with P (128 values x 128 channels, MN-major: a channel's values contiguous,
// so a thread stores its own products with 16-byte vectors) as operand A and a
// tile of ones as operand B; D (128 TMEM lanes x 16 columns, all columns
// equal) is read back one value per thread.  That replaces the warp
// transpose-reduce (~7.75 instructions per (t, d, n)) with ~0.5 (bf16x2
// converts and 16-byte stores).  Each product is rounded to bf16 (relative
// error <= 2^-9, unbiased) before the f32 sum, so gB/gC carry ~1e-3 relative
// error; the f32-io path keeps the exact SIMT reduce.  (The tensor core reads
// no MN-major tf32 operand, so f32 products would need one scalar store each.)
// Chunks of CK = 8 steps run last to first; the x/dt/dY tiles and the chunk
// checkpoint arrive by cp.async one chunk ahead.  Per chunk: rebuild the
// second sub-chunk's start state from the checkpoint, then per 4-step
// sub-chunk recompute h and exp(dt A) into registers and walk back writing P
// (all 8 steps of the chunk: 256 values), gx and gdt.  A warp that has written
// its P rows counts itself in with one shared-memory atomic and the last of
// the four issues the chunk's two MMAs (steps 0-3 and 4-7, into TMEM columns
// 0-15 and 16-31); the sums are read once per chunk,
// after the next chunk's first recompute, so the MMA latency stays hidden and
// no CTA barrier runs inside a chunk.
namespace sstc {
constexpr int THREADS = kThreads;       // one thread per channel
constexpr int WARPS = THREADS / 32;
constexpr int NS = 16, NP = 8;          // states, state pairs per thread
constexpr int TS = 4, CK = 8;
constexpr int ROWB = kThreads * 2;      // bytes of one bf16 tile row (128 channels)
constexpr int TILEB = CK * ROWB;        // one [CK][128] bf16 tile
constexpr int CHS = 20;                 // floats per channel of a state row (16 + bank skew)
constexpr int P_BYTES = 64 * 1024;      // 16 K-groups x 4 M-blocks x 1 KB atoms
constexpr int OFF_P = 0;                // the chunk's products
constexpr int OFF_ONES = OFF_P + P_BYTES;  // B: 2 KB of bf16 1.0 (16 rows x 128 B)
constexpr int OFF_CK = OFF_ONES + 2048;           // [2][128][CHS] f32 chunk checkpoints
constexpr int OFF_S1 = OFF_CK + 2 * kThreads * CHS * 4;  // [128][CHS] sub-chunk 1 start
constexpr int OFF_TILE = OFF_S1 + kThreads * CHS * 4;    // [2][x|dt|dy][CK][128] bf16
constexpr int OFF_BC = OFF_TILE + 2 * 3 * TILEB;         // [2][B|C][CK][NS] f32
constexpr int OFF_DM = OFF_BC + 2 * 2 * CK * NS * 4;     // [2][CK] f32 (model mode)
constexpr int OFF_BAR = OFF_DM + 2 * CK * 4;  // mbarrier, TMEM address, arrival counter
constexpr int SMEM = OFF_BAR + 32;
constexpr int SMEM_ALLOC = SMEM;  // the dynamic base is 1 KB aligned (checked in the kernel)
static_assert(2 * (SMEM_ALLOC + 1024) <= 228 * 1024, "two CTAs per SM");
constexpr int TMEM_COLS = 32;            // D: columns 0-15 = steps 0-3, 16-31 = steps 4-7
// kind::f16, bf16 x bf16 -> f32, M = 128, N = 16, A MN-major, B K-major
constexpr uint32_t IDESC = tc::idesc_bf16(128, 16, 1, 0);

// Byte offset of the 16-byte chunk holding values m8..m8+7 (m8 % 8 == 0) of
// channel k in P: K-group k/8 (4 KB), M-block m8/64 (1 KB atom of 8 channel
// rows x 128 B), row k%8, chunk (m8%64)/8 swizzled by the row (SWIZZLE_128B).
static __device__ __forceinline__ uint32_t p_off(int k, int m8) {
    return (uint32_t)(k >> 3) * 4096u + (uint32_t)(m8 >> 6) * 1024u +
           tc::sw128_off((uint32_t)(k & 7), (uint32_t)((m8 & 63) >> 3));
}

static __device__ __forceinline__ float bf16_at(const unsigned char* tile, int row, int ch) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(tile + row * ROWB)[ch]);
}
static __device__ __forceinline__ uint4 pack8(float2 a, float2 b, float2 c, float2 d) {
    return make_uint4(tc::pack_bf16x2(a.x, a.y), tc::pack_bf16x2(b.x, b.y),
                      tc::pack_bf16x2(c.x, c.y), tc::pack_bf16x2(d.x, d.y));
}
static __device__ __forceinline__ void load16(const float* p, float2 (&h)[NP]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(p + 4 * q);
        h[2 * q] = make_float2(v.x, v.y);
        h[2 * q + 1] = make_float2(v.z, v.w);
    }
}
static __device__ __forceinline__ void bq16(const float* p, float2 (&v)[NP]) { load16(p, v); }
}  // namespace sstc

// grid (ceil(D/128), B), block 128, two CTAs per SM.  D % 8 == 0 and x, dt, dy
// 16-byte aligned (the staged geometry).  gpart as ssm_bwd_kernel's.
template <bool MODEL, bool FIXA>
__global__ void __launch_bounds__(sstc::THREADS, 2)
    ssm_bwd_tc_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dt,
                      const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ Bm,
                      const __nv_bfloat16* __restrict__ Cm, const __nv_bfloat16* __restrict__ dy,
                      const float* __restrict__ ckpt, const float* __restrict__ dtm,
                      __nv_bfloat16* __restrict__ gx, __nv_bfloat16* __restrict__ gdt,
                      float* __restrict__ gpart, int Bsz, int L, int D, int N, float dt_min,
                      float dt_max, unsigned* err) {
    using namespace sstc;
    using T = __nv_bfloat16;
    extern __shared__ __align__(1024) unsigned char smem[];
    float* sCk = reinterpret_cast<float*>(smem + OFF_CK);
    float* sS1 = reinterpret_cast<float*>(smem + OFF_S1);
    float* sBC = reinterpret_cast<float*>(smem + OFF_BC);
    float* sDm = reinterpret_cast<float*>(smem + OFF_DM);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 8);
    unsigned* arrivals = reinterpret_cast<unsigned*>(smem + OFF_BAR + 12);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d0 = blockIdx.x * kThreads, d = d0 + tid;
    const int b = blockIdx.y;
    const bool live = d < D;
    const int nck = (L + CK - 1) / CK;
    const int nblk = gridDim.x;
    const long long row0 = (long long)b * L;
    if ((smem_u32(smem) & 1023u) != 0) {  // SWIZZLE_128B operands need 1 KB alignment
        if (tid == 0) edb_flag_error(err, EDB_DEVERR_SSM_PIPE);
        return;
    }

    // ---- set-up: TMEM columns for D, the MMA barriers, the ones tile
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, TMEM_COLS);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(mbar, 1);
        fence_mbar_init();
        *arrivals = 0;
    }
    for (int i = tid; i < 512; i += THREADS)  // 1024 bf16 ones = 512 words of 0x3F80 pairs
        reinterpret_cast<uint32_t*>(smem + OFF_ONES)[i] = 0x3F803F80u;
    fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    // exp(dtc A) = 2^(dtc A log2 e); the ln 2 of d/d dtc is applied to the sum
    float2 A2[NP], dh[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int n = 2 * p;
        A2[p].x = (live && n < N) ? a_at<MODEL>(A, d, n, N) * kLog2e : 0.0f;
        A2[p].y = (live && n + 1 < N) ? a_at<MODEL>(A, d, n + 1, N) * kLog2e : 0.0f;
        dh[p] = dup2(0.0f);
    }

    // staging of chunk c into buffer c & 1: x | dt | dy rows and the chunk's
    // checkpoint (zeros for channels past D), one cp.async group
    auto issue_chunk = [&](int c) {
        unsigned char* base = smem + OFF_TILE + (c & 1) * 3 * TILEB;
        const T* src[3] = {x, dt, dy};
        constexpr int PER = CK * (ROWB / 16);  // 16-byte copies per tile
        static_assert(PER == THREADS, "one copy per thread and tile");
        const int r = tid / (ROWB / 16), c16 = tid % (ROWB / 16);
        const int t = c * CK + r, dd = d0 + c16 * 8;
        const bool ok = t < L && dd < D;
#pragma unroll
        for (int q = 0; q < 3; ++q)
            cp_async16(base + q * TILEB + r * ROWB + c16 * 16,
                       src[q] + (ok ? (row0 + t) * D + dd : 0), ok ? 16u : 0u);
        float* ck_dst = sCk + (c & 1) * kThreads * CHS;
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // 4 x 16 bytes per channel
            const int i = tid + k * THREADS, ch = i >> 2, q4 = i & 3;
            const bool okc = d0 + ch < D;
            cp_async16(ck_dst + ch * CHS + q4 * 4,
                       ckpt + (okc ? (((long long)b * nck + c) * D + d0 + ch) * NS + q4 * 4 : 0),
                       okc ? 16u : 0u);
        }
        cp_async_commit();
    };
    // B, C (and the mean dt) of chunk c: two values per thread, to registers
    float rbc0 = 0.0f, rbc1 = 0.0f, rdm = 0.0f;
    auto load_bc = [&](int c) {
        const int t = c * CK + tid / NS, n = tid % NS;  // tid < CK * NS = 128
        const bool ok = t < L && n < N;
        rbc0 = ok ? ldf(Bm + (row0 + t) * N + n) : 0.0f;
        rbc1 = ok ? ldf(Cm + (row0 + t) * N + n) : 0.0f;
        if (MODEL && tid < CK) {
            const int tt = c * CK + tid;
            rdm = tt < L ? dtm[row0 + tt] : 0.0f;
        }
    };
    auto store_bc = [&](int c) {
        sBC[(c & 1) * 2 * CK * NS + tid] = rbc0;
        sBC[(c & 1) * 2 * CK * NS + CK * NS + tid] = rbc1;
        if (MODEL && tid < CK) sDm[(c & 1) * CK + tid] = rdm;
    };

    issue_chunk(nck - 1);
    load_bc(nck - 1);
    store_bc(nck - 1);

    int n_mma = 0;            // chunks handed to the tensor core
    int pend_t = 0, pend_tn = 0;  // first step and step count of the last one
    bool failed = false, wfailed = false;  // CTA-wide (at chunk starts) / this warp's
    // Waits for the last chunk's MMAs (P is then free) and reads its sums (two
    // values per thread: steps warp and 4 + warp) into gpart.  Returns false if
    // the wait gave up.
    auto drain = [&]() -> bool {
        bool ok = mbar_wait_bounded(mbar, (unsigned)((n_mma - 1) & 1), err, EDB_DEVERR_SSM_PIPE);
        // warp-uniform, so that the .sync.aligned TMEM load below runs on whole warps
        if (!__all_sync(0xffffffffu, ok)) return false;
        tc::fence_after_sync();
        uint32_t v0, v1;
        const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16);
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v0) : "r"(ta));
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v1) : "r"(ta + 16));
        tc::tmem_wait_ld();
        const int which = lane >> 4, n = lane & 15;  // value 32 warp + lane of each half
        const long long o = (((long long)which * nblk + blockIdx.x) * Bsz + b) * L + pend_t;
        if (warp < pend_tn) gpart[(o + warp) * NS + n] = __uint_as_float(v0);
        if (4 + warp < pend_tn) gpart[(o + 4 + warp) * NS + n] = __uint_as_float(v1);
        return true;
    };

    for (int c = nck - 1; c >= 0; --c) {
        const int t0 = c * CK, tn = min(CK, L - t0);
        const unsigned char* tx = smem + OFF_TILE + (c & 1) * 3 * TILEB;
        const unsigned char* tdt = tx + TILEB;
        const unsigned char* tdy = tx + 2 * TILEB;
        const float* sB = sBC + (c & 1) * 2 * CK * NS;
        const float* sC = sB + CK * NS;
        const float* dm = sDm + (c & 1) * CK;
        const float* ck0 = sCk + (c & 1) * kThreads * CHS + tid * CHS;
        float* s1 = sS1 + tid * CHS;

        cp_async_wait<0>();
        // chunk c's tiles, checkpoint, B/C visible; every warp is done with chunk c+1
        failed = __syncthreads_or(wfailed) != 0;
        if (failed) break;
        if (c > 0) {
            issue_chunk(c - 1);
            load_bc(c - 1);
        }

        // ---- start state of sub-chunk 1: TS steps on from the checkpoint.  Rows
        // past L were staged as zeros, so the walk needs no bound on the step.
        const int nsub = (tn + TS - 1) / TS;
        float2 h[NP];
        if (nsub > 1) {
            load16(ck0, h);
#pragma unroll
            for (int tt = 0; tt < TS; ++tt) {
                const float dtc = fminf(fmaxf(bf16_at(tdt, tt, tid), dt_min), dt_max);
                const float2 dtc2 = dup2(dtc),
                             dtx2 = dup2((MODEL ? dm[tt] : dtc) * bf16_at(tx, tt, tid));
                float2 pw, rr2;
                if (FIXA) fixa_powers(dtc, pw, rr2);
                float2 bq[NP];
                bq16(sB + tt * NS, bq);
#pragma unroll
                for (int p = 0; p < NP; ++p) {
                    const float2 a = FIXA ? next_power(pw, rr2) : ex2_2(mul2(dtc2, A2[p]));
                    h[p] = fma2(a, h[p], mul2(dtx2, bq[p]));
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
                *reinterpret_cast<float4*>(s1 + 4 * q) =
                    make_float4(h[2 * q].x, h[2 * q].y, h[2 * q + 1].x, h[2 * q + 1].y);
        }

#pragma unroll
        for (int s = 1; s >= 0; --s) {  // sub-chunks of the chunk, last first
            if (s >= nsub) continue;
            const int u0 = s * TS, un = min(TS, tn - u0);
            float2 hs[TS][NP], as[TS][NP];
            load16(s ? s1 : ck0, h);
#pragma unroll
            for (int j = 0; j < TS; ++j) {
                const int tt = u0 + j;
                const float dtc = fminf(fmaxf(bf16_at(tdt, tt, tid), dt_min), dt_max);
                const float2 dtc2 = dup2(dtc),
                             dtx2 = dup2((MODEL ? dm[tt] : dtc) * bf16_at(tx, tt, tid));
                float2 pw, rr2;
                if (FIXA) fixa_powers(dtc, pw, rr2);
                float2 bq[NP];
                bq16(sB + tt * NS, bq);
#pragma unroll
                for (int p = 0; p < NP; ++p) {
                    as[j][p] = FIXA ? next_power(pw, rr2) : ex2_2(mul2(dtc2, A2[p]));
                    h[p] = fma2(as[j][p], h[p], mul2(dtx2, bq[p]));
                    hs[j][p] = h[p];
                }
            }
            // P is free once the previous chunk's MMAs are done and read
            if (s == nsub - 1 && n_mma > 0 && !drain()) wfailed = true;
            unsigned char* P = smem + OFF_P;
#pragma unroll
            for (int j = TS - 1; j >= 0; --j) {
                if (j >= un) continue;
                const int tt = u0 + j;
                const float draw = bf16_at(tdt, tt, tid);
                const float dtc = fminf(fmaxf(draw, dt_min), dt_max);
                const float xv = bf16_at(tx, tt, tid);
                const float dyv = live ? bf16_at(tdy, tt, tid) : 0.0f;
                const float dti = MODEL ? dm[tt] : dtc;  // dt of the input term
                const float dtx = dti * xv;
                const float2 dy2 = dup2(dyv), dtx2 = dup2(dtx), ndtx2 = dup2(-dtx);
                float2 bq[NP], cq[NP];
                bq16(sB + tt * NS, bq);
                bq16(sC + tt * NS, cq);
                // two partial sums each (even / odd pairs): shorter dependency chains
                float2 gxa[2] = {dup2(0.0f), dup2(0.0f)}, gda[2] = {dup2(0.0f), dup2(0.0f)};
                float2 pb[NP], pc[NP];
#pragma unroll
                for (int p = 0; p < NP; ++p) {
                    const float2 hc = hs[j][p];
                    const float2 dht = fma2(dy2, cq[p], dh[p]);
                    pc[p] = mul2(dy2, hc);
                    pb[p] = mul2(dht, dtx2);
                    gxa[p & 1] = fma2(dht, bq[p], gxa[p & 1]);
                    // d h_t / d dtc = A (a h_{t-1}) + B x with a h_{t-1} = h_t - dtc x B
                    // (A in log2 units here; the B x part is summed once below)
                    gda[p & 1] = fma2(mul2(dht, A2[p]), fma2(ndtx2, bq[p], hc), gda[p & 1]);
                    dh[p] = mul2(dht, as[j][p]);
                }
                const int m0 = tt * 32;  // this step's values: {gB 0..15 | gC 16..31}
                *reinterpret_cast<uint4*>(P + p_off(tid, m0)) = pack8(pb[0], pb[1], pb[2], pb[3]);
                *reinterpret_cast<uint4*>(P + p_off(tid, m0 + 8)) = pack8(pb[4], pb[5], pb[6], pb[7]);
                *reinterpret_cast<uint4*>(P + p_off(tid, m0 + 16)) = pack8(pc[0], pc[1], pc[2], pc[3]);
                *reinterpret_cast<uint4*>(P + p_off(tid, m0 + 24)) = pack8(pc[4], pc[5], pc[6], pc[7]);
                const float gxs = (gxa[0].x + gxa[0].y) + (gxa[1].x + gxa[1].y);
                const float gdl = kLn2 * ((gda[0].x + gda[0].y) + (gda[1].x + gda[1].y));
                // model mode: the input term's dt is the channel mean, whose
                // gradient ssm_model_gdt_kernel adds afterwards
                const float gds = MODEL ? gdl : fmaf(xv, gxs, gdl);
                if (live) {
                    const long long o = (row0 + t0 + tt) * D + d;
                    st_scalar<T>(gx + o, gxs * dti);
                    st_scalar<T>(gdt + o, (draw >= dt_min && draw <= dt_max) ? gds : 0.0f);
                }
            }
        }
        // Hand P to the tensor core: each warp makes its stores visible to the
        // async proxy and counts itself in; the warp that arrives last issues
        // the chunk's MMAs.  The counter only grows (WARPS per chunk): a warp
        // writes the next chunk's P only after draining these MMAs.
        tc::fence_before_sync();  // this warp's TMEM reads of D before the count
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            const unsigned prev = atomicAdd(arrivals, 1u);
            if (prev % WARPS == WARPS - 1) {
                __threadfence_block();
                tc::fence_after_sync();
                const uint64_t bdesc = tc::sdesc_sw128(smem + OFF_ONES, 16, 1024);
                // steps 0-3 (M-blocks 0, 1) into columns 0-15, steps 4-7 (M-blocks 2, 3)
                // into columns 16-31
#pragma unroll
                for (int hf = 0; hf < 2; ++hf)
#pragma unroll
                    for (int kk = 0; kk < kThreads / 16; ++kk)
                        tc::mma_bf16_ss(tmem + (uint32_t)(hf * 16),
                                        tc::sdesc_sw128(smem + OFF_P + kk * 8192 + hf * 2048, 1024,
                                                        4096),
                                        bdesc, IDESC, kk > 0);
                tc::commit(mbar);
            }
        }
        __syncwarp();
        pend_t = t0;
        pend_tn = tn;
        ++n_mma;
        if (c > 0) store_bc(c - 1);
    }
    cp_async_wait<0>();  // nothing may land after the CTA has left
    if (!failed && !wfailed && n_mma > 0) drain();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ------------------------------------------------------------ model semantics
// lib/edifice/ssm/common.ex:402-444 (discretize_ssm): B_bar = mean_d(clip(dt)) B.
// dtm[row] = mean over d_inner of the clamped dt, one warp per (b, t) row, summed
// in a fixed order (deterministic).
template <typename T>
__global__ void __launch_bounds__(256)
    ssm_dt_mean_kernel(const T* __restrict__ dt, float* __restrict__ dtm, long long rows, int D,
                       float dt_min, float dt_max) {
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const T* p = dt + row * D;
    float acc = 0.0f;
    constexpr int EPV = 16 / (int)sizeof(T);
    if (D % EPV == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        for (int i = lane * EPV; i < D; i += 32 * EPV) {
            float f[EPV];
            Vec16<T>::unpack(*reinterpret_cast<const uint4*>(p + i), f);
#pragma unroll
            for (int j = 0; j < EPV; ++j) acc += fminf(fmaxf(f[j], dt_min), dt_max);
        }
    } else {
        for (int i = lane; i < D; i += 32) acc += fminf(fmaxf(ldf(p + i), dt_min), dt_max);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) dtm[row] = acc / (float)D;
}

// gdt[b,t,d] += [dt in range] * g_m / D with g_m = sum_{d,n} dh B x
// = sum_n B[b,t,n] gB[b,t,n] / dtm[b,t] (gB = dtm sum_d dh x).  One warp per row.
template <typename T>
__global__ void __launch_bounds__(256)
    ssm_model_gdt_kernel(const T* __restrict__ dt, const T* __restrict__ Bm,
                         const float* __restrict__ gB, const float* __restrict__ dtm,
                         T* __restrict__ gdt, long long rows, int D, int N, float dt_min,
                         float dt_max) {
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float gm = lane < N ? ldf(Bm + row * N + lane) * gB[row * N + lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gm += __shfl_xor_sync(0xffffffffu, gm, o);
    const float add = gm / dtm[row] / (float)D;
    const T* p = dt + row * D;
    T* g = gdt + row * D;
    constexpr int EPV = 16 / (int)sizeof(T);
    if (D % EPV == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
        for (int i = lane * EPV; i < D; i += 32 * EPV) {
            float fd[EPV], fg[EPV];
            Vec16<T>::unpack(*reinterpret_cast<const uint4*>(p + i), fd);
            Vec16<T>::unpack(*reinterpret_cast<const uint4*>(g + i), fg);
#pragma unroll
            for (int j = 0; j < EPV; ++j)
                if (fd[j] >= dt_min && fd[j] <= dt_max) fg[j] += add;
            *reinterpret_cast<uint4*>(g + i) = Vec16<T>::pack(fg);
        }
    } else {
        for (int i = lane; i < D; i += 32) {
            const float draw = ldf(p + i);
            if (draw >= dt_min && draw <= dt_max) st_scalar<T>(g + i, ldf(g + i) + add);
        }
    }
}

int pad_states(int N) {
    if (N <= 8) return 8;
    if (N <= 16) return 16;
    return 0;
}

int ck_of(int NS) { return NS == 8 ? SsmTiling<8>::CK : SsmTiling<16>::CK; }

size_t ckpt_bytes(int B, int L, int D, int NS) {
    const int CK = ck_of(NS);
    return (size_t)B * ((L + CK - 1) / CK) * D * NS * sizeof(float);
}

size_t part_bytes(int B, int L, int D, int NS) {
    const int nblk = (D + kThreads - 1) / kThreads;
    return (size_t)2 * nblk * B * L * NS * sizeof(float);
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

template <typename T, int NS, bool MODEL>
int launch_fwd(const void* x, const void* dt, const void* A, const void* Bm, const void* Cm,
               void* y, float* ckpt, const float* dtm, int B, int L, int D, int N, float lo,
               float hi, bool states_only, cudaStream_t st) {
    dim3 grid((D + kThreads - 1) / kThreads, B);
    if (D % StageGeom<T>::EPC == 0 && edb::aligned16(x) && edb::aligned16(dt)) {
        constexpr size_t sm = fwd_staged_smem<T, NS>();
        auto kern = states_only ? ssm_fwd_staged_kernel<T, NS, true, MODEL>
                                : ssm_fwd_staged_kernel<T, NS, false, MODEL>;
        if (MODEL && A == nullptr)  // the model's fixed A: decays as powers
            kern = states_only ? ssm_fwd_staged_kernel<T, NS, true, MODEL, MODEL>
                               : ssm_fwd_staged_kernel<T, NS, false, MODEL, MODEL>;
        cudaError_t ea =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (ea != cudaSuccess) return (int)ea;
        kern<<<grid, kThreads, sm, st>>>((const T*)x, (const T*)dt, (const T*)A, (const T*)Bm,
                                         (const T*)Cm, (T*)y, ckpt, dtm, L, D, N, lo, hi);
        return edb::status_from_cuda(cudaGetLastError());
    }
    auto kern = states_only ? ssm_fwd_kernel<T, NS, true, MODEL> : ssm_fwd_kernel<T, NS, false, MODEL>;
    kern<<<grid, kThreads, 0, st>>>((const T*)x, (const T*)dt, (const T*)A, (const T*)Bm,
                                    (const T*)Cm, (T*)y, ckpt, dtm, L, D, N, lo, hi);
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T, int NS, bool MODEL>
int launch_bwd(const void* x, const void* dt, const void* A, const void* Bm, const void* Cm,
               const void* dy, const float* ckpt, const float* dtm, void* gx, void* gdt,
               float* gB, float* gC, float* gpart, int B, int L, int D, int N, float lo, float hi,
               cudaStream_t st) {
    const int nblk = (D + kThreads - 1) / kThreads;
    dim3 grid(nblk, B);
    bool tc_done = false;
    if constexpr (std::is_same<T, __nv_bfloat16>::value && NS == 16) {
        // bf16 io, 16 states: the tensor-core channel reduce (gx/gdt leave in
        // 16-byte rows, so they must be 16-byte aligned as well)
        if (D % 8 == 0 && edb::aligned16(x) && edb::aligned16(dt) && edb::aligned16(dy) &&
            edb::aligned16(gx) && edb::aligned16(gdt)) {
            auto kern = ssm_bwd_tc_kernel<MODEL, false>;
            if (MODEL && A == nullptr) kern = ssm_bwd_tc_kernel<MODEL, MODEL>;
            cudaError_t ea = cudaFuncSetAttribute(
                kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sstc::SMEM_ALLOC);
            if (ea != cudaSuccess) return (int)ea;
            kern<<<grid, sstc::THREADS, sstc::SMEM_ALLOC, st>>>(
                (const T*)x, (const T*)dt, (const T*)A, (const T*)Bm, (const T*)Cm,
                (const T*)dy, ckpt, dtm, (T*)gx, (T*)gdt, gpart, B, L, D, N, lo, hi,
                edb::device_error_word());
            tc_done = true;
        }
    }
    if (tc_done) {
    } else if (D % StageGeom<T>::EPC == 0 && edb::aligned16(x) && edb::aligned16(dt) &&
               edb::aligned16(dy)) {
        constexpr size_t sm = bwd_staged_smem<T, NS>();
        auto kern = ssm_bwd_staged_kernel<T, NS, MODEL>;
        if (MODEL && A == nullptr) kern = ssm_bwd_staged_kernel<T, NS, MODEL, MODEL>;
        cudaError_t ea =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (ea != cudaSuccess) return (int)ea;
        kern<<<grid, kThreads, sm, st>>>(
            (const T*)x, (const T*)dt, (const T*)A, (const T*)Bm, (const T*)Cm, (const T*)dy,
            ckpt, dtm, (T*)gx, (T*)gdt, gpart, B, L, D, N, lo, hi);
    } else {
        constexpr int SUBS = SsmTiling<NS>::CK / SsmTiling<NS>::TS;
        const size_t dsmem = (size_t)SUBS * NS * kThreads * sizeof(float);
        cudaError_t ea = cudaFuncSetAttribute(ssm_bwd_kernel<T, NS, MODEL>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)dsmem);
        if (ea != cudaSuccess) return (int)ea;
        ssm_bwd_kernel<T, NS, MODEL><<<grid, kThreads, dsmem, st>>>(
            (const T*)x, (const T*)dt, (const T*)A, (const T*)Bm, (const T*)Cm, (const T*)dy,
            ckpt, dtm, (T*)gx, (T*)gdt, gpart, B, L, D, N, lo, hi);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    const long long total = (long long)B * L * N;
    const int thr = 256;
    ssm_reduce_kernel<NS><<<(unsigned)((total + thr - 1) / thr), thr, 0, st>>>(
        gpart, gB, gC, nblk, (long long)B * L, N);
    e = cudaGetLastError();
    if (e != cudaSuccess || !MODEL) return edb::status_from_cuda(e);
    // model mode: the gradient through the channel mean of dt
    const long long rows = (long long)B * L;
    ssm_model_gdt_kernel<T><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
        (const T*)dt, (const T*)Bm, gB, dtm, (T*)gdt, rows, D, N, lo, hi);
    return edb::status_from_cuda(cudaGetLastError());
}

// Runs F<T, NS>::run(args...) for the dtype / padded state count.
template <template <typename, int> class F, typename... Args>
int dispatch(int dtype, int NS, Args... args) {
    if (dtype == EDB_BF16)
        return NS == 8 ? F<__nv_bfloat16, 8>::run(args...) : F<__nv_bfloat16, 16>::run(args...);
    return NS == 8 ? F<float, 8>::run(args...) : F<float, 16>::run(args...);
}

template <typename T, int NS>
struct FwdKernelMode {
    template <typename... A>
    static int run(A... a) { return launch_fwd<T, NS, false>(a...); }
};
template <typename T, int NS>
struct FwdModelMode {
    template <typename... A>
    static int run(A... a) { return launch_fwd<T, NS, true>(a...); }
};
template <typename T, int NS>
struct BwdKernelMode {
    template <typename... A>
    static int run(A... a) { return launch_bwd<T, NS, false>(a...); }
};
template <typename T, int NS>
struct BwdModelMode {
    template <typename... A>
    static int run(A... a) { return launch_bwd<T, NS, true>(a...); }
};

int check_args(int dtype, int B, int L, int D, int N, float lo, float hi) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || L <= 0 || D <= 0 || N <= 0) return EDB_ERR_BAD_SHAPE;
    if (!(lo <= hi)) return EDB_ERR_BAD_SHAPE;
    if (pad_states(N) == 0) return EDB_ERR_UNSUPPORTED;
    if ((long long)B * L * D >= (1LL << 40)) return EDB_ERR_BAD_SHAPE;
    return EDB_OK;
}

}  // namespace

extern "C" size_t edb_selective_scan_ckpt_bytes(int batch, int seq_len, int d_inner, int d_state) {
    const int NS = pad_states(d_state);
    if (batch <= 0 || seq_len <= 0 || d_inner <= 0 || NS == 0) return 0;
    return ckpt_bytes(batch, seq_len, d_inner, NS);
}

extern "C" int edb_selective_scan_fwd(int dtype, const void* x, const void* dt, const void* A,
                                      const void* B, const void* C, void* y, float* h_ckpt,
                                      int batch, int seq_len, int d_inner, int d_state,
                                      float dt_min, float dt_max, void* stream) {
    if (int s = check_args(dtype, batch, seq_len, d_inner, d_state, dt_min, dt_max)) return s;
    if (!x || !dt || !A || !B || !C || !y) return EDB_ERR_NULL_POINTER;
    if (h_ckpt && !edb::aligned16(h_ckpt)) return EDB_ERR_MISALIGNED;
    return dispatch<FwdKernelMode>(dtype, pad_states(d_state), x, dt, A, B, C, y, h_ckpt,
                                   (const float*)nullptr, batch, seq_len, d_inner, d_state,
                                   dt_min, dt_max, false, (cudaStream_t)stream);
}

extern "C" size_t edb_selective_scan_bwd_workspace(int batch, int seq_len, int d_inner,
                                                   int d_state, int have_ckpt) {
    const int NS = pad_states(d_state);
    if (batch <= 0 || seq_len <= 0 || d_inner <= 0 || NS == 0) return 0;
    size_t ws = align256(part_bytes(batch, seq_len, d_inner, NS));
    if (!have_ckpt) ws += align256(ckpt_bytes(batch, seq_len, d_inner, NS));
    return ws;
}

namespace {

// Shared body of the kernel-mode and model-mode backward (dtm != nullptr: model).
int ssm_bwd(int dtype, const void* x, const void* dt, const void* A, const void* B,
            const void* C, const void* dy, const float* dtm, const float* h_ckpt, void* gx,
            void* gdt, float* gB, float* gC, int batch, int seq_len, int d_inner, int d_state,
            float dt_min, float dt_max, void* workspace, size_t workspace_bytes, void* stream) {
    const bool model = dtm != nullptr;
    const size_t need =
        edb_selective_scan_bwd_workspace(batch, seq_len, d_inner, d_state, h_ckpt != nullptr);
    if (workspace_bytes < need || (need && !workspace)) return EDB_ERR_WORKSPACE_TOO_SMALL;
    if (!edb::aligned16(workspace) || (h_ckpt && !edb::aligned16(h_ckpt)))
        return EDB_ERR_MISALIGNED;
    const int NS = pad_states(d_state);
    cudaStream_t st = (cudaStream_t)stream;
    float* gpart = static_cast<float*>(workspace);
    const float* ck = h_ckpt;
    if (!ck) {
        float* ckw = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                              align256(part_bytes(batch, seq_len, d_inner, NS)));
        const int s =
            model ? dispatch<FwdModelMode>(dtype, NS, x, dt, A, B, C, (void*)nullptr, ckw, dtm,
                                           batch, seq_len, d_inner, d_state, dt_min, dt_max, true,
                                           st)
                  : dispatch<FwdKernelMode>(dtype, NS, x, dt, A, B, C, (void*)nullptr, ckw, dtm,
                                            batch, seq_len, d_inner, d_state, dt_min, dt_max, true,
                                            st);
        if (s) return s;
        ck = ckw;
    }
    return model ? dispatch<BwdModelMode>(dtype, NS, x, dt, A, B, C, dy, ck, dtm, gx, gdt, gB, gC,
                                          gpart, batch, seq_len, d_inner, d_state, dt_min, dt_max,
                                          st)
                 : dispatch<BwdKernelMode>(dtype, NS, x, dt, A, B, C, dy, ck, dtm, gx, gdt, gB, gC,
                                           gpart, batch, seq_len, d_inner, d_state, dt_min, dt_max,
                                           st);
}

}  // namespace

extern "C" int edb_selective_scan_bwd(int dtype, const void* x, const void* dt, const void* A,
                                      const void* B, const void* C, const void* dy,
                                      const float* h_ckpt, void* gx, void* gdt, float* gB,
                                      float* gC, int batch, int seq_len, int d_inner,
                                      int d_state, float dt_min, float dt_max, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    if (int s = check_args(dtype, batch, seq_len, d_inner, d_state, dt_min, dt_max)) return s;
    if (!x || !dt || !A || !B || !C || !dy || !gx || !gdt || !gB || !gC)
        return EDB_ERR_NULL_POINTER;
    return ssm_bwd(dtype, x, dt, A, B, C, dy, nullptr, h_ckpt, gx, gdt, gB, gC, batch, seq_len,
                   d_inner, d_state, dt_min, dt_max, workspace, workspace_bytes, stream);
}

// ------------------------------------------------------------- model semantics
extern "C" int edb_selective_scan_model_fwd(int dtype, const void* x, const void* dt,
                                            const void* A, const void* B, const void* C, void* y,
                                            float* dt_mean, float* h_ckpt, int batch,
                                            int seq_len, int d_inner, int d_state, float dt_min,
                                            float dt_max, void* stream) {
    if (int s = check_args(dtype, batch, seq_len, d_inner, d_state, dt_min, dt_max)) return s;
    if (!x || !dt || !B || !C || !y || !dt_mean) return EDB_ERR_NULL_POINTER;
    if (h_ckpt && !edb::aligned16(h_ckpt)) return EDB_ERR_MISALIGNED;
    cudaStream_t st = (cudaStream_t)stream;
    const long long rows = (long long)batch * seq_len;
    if (dtype == EDB_BF16)
        ssm_dt_mean_kernel<__nv_bfloat16><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
            (const __nv_bfloat16*)dt, dt_mean, rows, d_inner, dt_min, dt_max);
    else
        ssm_dt_mean_kernel<float><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
            (const float*)dt, dt_mean, rows, d_inner, dt_min, dt_max);
    if (cudaError_t e = cudaGetLastError()) return (int)e;
    return dispatch<FwdModelMode>(dtype, pad_states(d_state), x, dt, A, B, C, y, h_ckpt,
                                  (const float*)dt_mean, batch, seq_len, d_inner, d_state, dt_min,
                                  dt_max, false, st);
}

extern "C" int edb_selective_scan_model_bwd(int dtype, const void* x, const void* dt,
                                            const void* A, const void* B, const void* C,
                                            const void* dy, const float* dt_mean,
                                            const float* h_ckpt, void* gx, void* gdt, float* gB,
                                            float* gC, int batch, int seq_len, int d_inner,
                                            int d_state, float dt_min, float dt_max,
                                            void* workspace, size_t workspace_bytes,
                                            void* stream) {
    if (int s = check_args(dtype, batch, seq_len, d_inner, d_state, dt_min, dt_max)) return s;
    if (!x || !dt || !B || !C || !dy || !dt_mean || !gx || !gdt || !gB || !gC)
        return EDB_ERR_NULL_POINTER;
    return ssm_bwd(dtype, x, dt, A, B, C, dy, dt_mean, h_ckpt, gx, gdt, gB, gC, batch, seq_len,
                   d_inner, d_state, dt_min, dt_max, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------- no-alloc variant
// Scratch of edb_selective_scan_bwd_noalloc: a fixed array inside the library,
// one per device, so that callers which must not allocate device memory can
// still run the backward.  Host code cannot use the symbol itself as a device
// address (on the host it names a host-side stand-in): the address comes from
// cudaGetSymbolAddress with the device current, on the first call in each
// context (edb::symbol_address caches it per device, keyed on the context's
// unique id, so a device reset is noticed and the address looked up again).
static __device__ __align__(256) unsigned char g_ssm_noalloc_scratch[EDB_SSM_NOALLOC_SCRATCH_BYTES];

namespace {

edb::SymbolCache g_ssm_noalloc_cache;

int ssm_noalloc_scratch(void** out) {
    return edb::symbol_address(g_ssm_noalloc_scratch, g_ssm_noalloc_cache, out);
}

}  // namespace

extern "C" int edb_selective_scan_bwd_noalloc(int dtype, const void* x, const void* dt,
                                              const void* A, const void* B, const void* C,
                                              const void* dy, const float* h_ckpt, void* gx,
                                              void* gdt, float* gB, float* gC, int batch,
                                              int seq_len, int d_inner, int d_state, float dt_min,
                                              float dt_max, void* stream) {
    if (int s = check_args(dtype, batch, seq_len, d_inner, d_state, dt_min, dt_max)) return s;
    if (!x || !dt || !A || !B || !C || !dy || !gx || !gdt || !gB || !gC)
        return EDB_ERR_NULL_POINTER;
    const size_t need =
        edb_selective_scan_bwd_workspace(batch, seq_len, d_inner, d_state, h_ckpt != nullptr);
    if (need > (size_t)EDB_SSM_NOALLOC_SCRATCH_BYTES) return EDB_ERR_WORKSPACE_TOO_SMALL;
    void* ws = nullptr;
    if (int s = ssm_noalloc_scratch(&ws)) return s;
    return edb_selective_scan_bwd(dtype, x, dt, A, B, C, dy, h_ckpt, gx, gdt, gB, gC, batch,
                                  seq_len, d_inner, d_state, dt_min, dt_max, ws,
                                  (size_t)EDB_SSM_NOALLOC_SCRATCH_BYTES, stream);
}
