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
#include <atomic>

#include "edb_common.cuh"

namespace {

constexpr int kThreads = 128;  // channels per CTA
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

static __device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// chunk / sub-chunk lengths per padded state count: TS*NS = 64 state values in
// registers per sub-chunk, CK/TS = 8 sub-checkpoints (8*NS floats) in smem.
template <int NS>
struct SsmTiling {
    static constexpr int TS = 64 / NS;
    static constexpr int CK = 8 * TS;
};

template <typename T>
static __device__ __forceinline__ float ldf(const T* p) {
    return ld_scalar<T>(p);
}

// ------------------------------------------------------------------ forward
// grid (ceil(D/128), B), block 128.  TB time steps of B/C per smem tile.
template <typename T, int NS, bool STATES_ONLY>
__global__ void __launch_bounds__(kThreads)
    ssm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ dt, const T* __restrict__ A,
                   const T* __restrict__ Bm, const T* __restrict__ Cm, T* __restrict__ y,
                   float* __restrict__ ckpt, int L, int D, int N, float dt_min, float dt_max) {
    constexpr int TB = 32;
    constexpr int CK = SsmTiling<NS>::CK;
    __shared__ float sB[TB][NS];
    __shared__ float sC[TB][NS];
    const int tid = threadIdx.x;
    const int d = blockIdx.x * kThreads + tid;
    const int b = blockIdx.y;
    const bool live = d < D;
    const int nck = (L + CK - 1) / CK;

    float A2[NS], h[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        A2[n] = (live && n < N) ? ldf(A + (long long)d * N + n) * kLog2e : 0.0f;
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
            const float dtx = dtc * ldf(x + o);
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
template <typename T, int NS>
__global__ void __launch_bounds__(kThreads)
    ssm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ dt, const T* __restrict__ A,
                   const T* __restrict__ Bm, const T* __restrict__ Cm, const T* __restrict__ dy,
                   const float* __restrict__ ckpt, T* __restrict__ gx, T* __restrict__ gdt,
                   float* __restrict__ gpart, int Bsz, int L, int D, int N, float dt_min,
                   float dt_max) {
    constexpr int TS = SsmTiling<NS>::TS;
    constexpr int CK = SsmTiling<NS>::CK;
    constexpr int SUBS = CK / TS;
    constexpr int V = 2 * NS;  // gB and gC values per step
    static_assert(V <= 32, "NS <= 16 in this kernel");
    __shared__ float sB[CK][NS];
    __shared__ float sC[CK][NS];
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
        A2[n] = (live && n < N) ? ldf(A + (long long)d * N + n) * kLog2e : 0.0f;
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
                const float dtx = dtc * ldf(x + o);
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
                    const float dtx = dtc * ldf(x + o);
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
                    const float dtx = dtc * xv;
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
                        gda = fmaf(dht, fmaf(abhp, A2[n] * kLn2, Bn * xv), gda);
                        dh[n] = dht * ab;
                    }
                    st_scalar<T>(gx + o, gxa * dtc);
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

template <typename T, int NS>
int launch_fwd(const void* x, const void* dt, const void* A, const void* Bm, const void* Cm,
               void* y, float* ckpt, int B, int L, int D, int N, float lo, float hi,
               bool states_only, cudaStream_t st) {
    dim3 grid((D + kThreads - 1) / kThreads, B);
    if (states_only)
        ssm_fwd_kernel<T, NS, true><<<grid, kThreads, 0, st>>>(
            (const T*)x, (const T*)dt, (const T*)A, (const T*)Bm, (const T*)Cm, (T*)y, ckpt, L, D,
            N, lo, hi);
    else
        ssm_fwd_kernel<T, NS, false><<<grid, kThreads, 0, st>>>(
            (const T*)x, (const T*)dt, (const T*)A, (const T*)Bm, (const T*)Cm, (T*)y, ckpt, L, D,
            N, lo, hi);
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T, int NS>
int launch_bwd(const void* x, const void* dt, const void* A, const void* Bm, const void* Cm,
               const void* dy, const float* ckpt, void* gx, void* gdt, float* gB, float* gC,
               float* gpart, int B, int L, int D, int N, float lo, float hi, cudaStream_t st) {
    const int nblk = (D + kThreads - 1) / kThreads;
    dim3 grid(nblk, B);
    constexpr int SUBS = SsmTiling<NS>::CK / SsmTiling<NS>::TS;
    const size_t dsmem = (size_t)SUBS * NS * kThreads * sizeof(float);
    cudaError_t ea = cudaFuncSetAttribute(ssm_bwd_kernel<T, NS>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsmem);
    if (ea != cudaSuccess) return (int)ea;
    ssm_bwd_kernel<T, NS><<<grid, kThreads, dsmem, st>>>(
        (const T*)x, (const T*)dt, (const T*)A, (const T*)Bm, (const T*)Cm, (const T*)dy, ckpt,
        (T*)gx, (T*)gdt, gpart, B, L, D, N, lo, hi);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    const long long total = (long long)B * L * N;
    const int thr = 256;
    ssm_reduce_kernel<NS><<<(unsigned)((total + thr - 1) / thr), thr, 0, st>>>(
        gpart, gB, gC, nblk, (long long)B * L, N);
    return edb::status_from_cuda(cudaGetLastError());
}

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
    const int NS = pad_states(d_state);
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == EDB_BF16)
        return NS == 8 ? launch_fwd<__nv_bfloat16, 8>(x, dt, A, B, C, y, h_ckpt, batch, seq_len,
                                                      d_inner, d_state, dt_min, dt_max, false, st)
                       : launch_fwd<__nv_bfloat16, 16>(x, dt, A, B, C, y, h_ckpt, batch, seq_len,
                                                       d_inner, d_state, dt_min, dt_max, false, st);
    return NS == 8 ? launch_fwd<float, 8>(x, dt, A, B, C, y, h_ckpt, batch, seq_len, d_inner,
                                          d_state, dt_min, dt_max, false, st)
                   : launch_fwd<float, 16>(x, dt, A, B, C, y, h_ckpt, batch, seq_len, d_inner,
                                           d_state, dt_min, dt_max, false, st);
}

extern "C" size_t edb_selective_scan_bwd_workspace(int batch, int seq_len, int d_inner,
                                                   int d_state, int have_ckpt) {
    const int NS = pad_states(d_state);
    if (batch <= 0 || seq_len <= 0 || d_inner <= 0 || NS == 0) return 0;
    size_t ws = align256(part_bytes(batch, seq_len, d_inner, NS));
    if (!have_ckpt) ws += align256(ckpt_bytes(batch, seq_len, d_inner, NS));
    return ws;
}

extern "C" int edb_selective_scan_bwd(int dtype, const void* x, const void* dt, const void* A,
                                      const void* B, const void* C, const void* dy,
                                      const float* h_ckpt, void* gx, void* gdt, float* gB,
                                      float* gC, int batch, int seq_len, int d_inner,
                                      int d_state, float dt_min, float dt_max, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    if (int s = check_args(dtype, batch, seq_len, d_inner, d_state, dt_min, dt_max)) return s;
    if (!x || !dt || !A || !B || !C || !dy || !gx || !gdt || !gB || !gC)
        return EDB_ERR_NULL_POINTER;
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
        int s;
        if (dtype == EDB_BF16)
            s = NS == 8 ? launch_fwd<__nv_bfloat16, 8>(x, dt, A, B, C, nullptr, ckw, batch,
                                                       seq_len, d_inner, d_state, dt_min, dt_max,
                                                       true, st)
                        : launch_fwd<__nv_bfloat16, 16>(x, dt, A, B, C, nullptr, ckw, batch,
                                                        seq_len, d_inner, d_state, dt_min, dt_max,
                                                        true, st);
        else
            s = NS == 8 ? launch_fwd<float, 8>(x, dt, A, B, C, nullptr, ckw, batch, seq_len,
                                               d_inner, d_state, dt_min, dt_max, true, st)
                        : launch_fwd<float, 16>(x, dt, A, B, C, nullptr, ckw, batch, seq_len,
                                                d_inner, d_state, dt_min, dt_max, true, st);
        if (s) return s;
        ck = ckw;
    }
    if (dtype == EDB_BF16)
        return NS == 8 ? launch_bwd<__nv_bfloat16, 8>(x, dt, A, B, C, dy, ck, gx, gdt, gB, gC,
                                                      gpart, batch, seq_len, d_inner, d_state,
                                                      dt_min, dt_max, st)
                       : launch_bwd<__nv_bfloat16, 16>(x, dt, A, B, C, dy, ck, gx, gdt, gB, gC,
                                                       gpart, batch, seq_len, d_inner, d_state,
                                                       dt_min, dt_max, st);
    return NS == 8 ? launch_bwd<float, 8>(x, dt, A, B, C, dy, ck, gx, gdt, gB, gC, gpart, batch,
                                          seq_len, d_inner, d_state, dt_min, dt_max, st)
                   : launch_bwd<float, 16>(x, dt, A, B, C, dy, ck, gx, gdt, gB, gC, gpart, batch,
                                           seq_len, d_inner, d_state, dt_min, dt_max, st);
}

// ---------------------------------------------------------------- no-alloc variant
// Scratch of edb_selective_scan_bwd_noalloc: a fixed array inside the library,
// one per device, so that callers which must not allocate device memory can
// still run the backward.  Host code cannot use the symbol itself as a device
// address (on the host it names a host-side stand-in); the address is looked
// up once per device with cudaGetSymbolAddress, the device being current.
static __device__ __align__(256) unsigned char g_ssm_noalloc_scratch[EDB_SSM_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::atomic<void*> g_ssm_noalloc_addr[kMaxDevices];

int ssm_noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kMaxDevices) return EDB_ERR_UNSUPPORTED;
    void* p = g_ssm_noalloc_addr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        e = cudaGetSymbolAddress(&p, g_ssm_noalloc_scratch);
        if (e != cudaSuccess) return (int)e;
        if (p == nullptr) return EDB_ERR_UNSUPPORTED;
        g_ssm_noalloc_addr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return EDB_OK;
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
