// delta_chunked_post.cu -- last stage of the chunked DeltaNet backward: the
// per-chunk C x C chain and the final dQ, dK, dV, dbeta (SIMT f32).
//
// Inputs per chunk (f32 scratch from the earlier stages of
// delta_chunked_bwd.cu): dQa = dO S_0, dW = -dU~ S_0, dK1 = U~ dS_C,
// dM = tril(dO U~^T), dU~, T, K K^T; plus q, k, v, beta (bf16).
//   dQ   = dQa + dM K
//   dV   = T_b^T dU~
//   dT_b = dW K^T + dU~ V^T,   dbeta_s  = sum_t dT_b[t][s] T[t][s]
//   dT   = dT_b diag(beta),    dA = -(T^T dT) T^T  (strictly lower)
//   dbeta_t += sum_{s<t} dA[t][s] (K K^T)[t][s]
//   E    = dG + dG^T,  dG = diag(beta) dA
//   dK   = dK1 + dM^T Q + T_b^T dW + E K
// One CTA (256 threads) per chunk; tiles live in shared memory (202 KB).
#include <math.h>

#include "delta_chunked.cuh"

using namespace dchunk;

namespace {

constexpr int kThreads = 256;
constexpr size_t kSmem = (size_t)(4 * C * PP + 5 * C * PC + 2 * C) * sizeof(float);

// sum over a row of 64: 4 threads per row (quad of consecutive lanes), 16
// columns each, then a quad reduction; returns the sum to all 4 lanes.
static __device__ __forceinline__ float quad_sum(float x) {
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    return x;
}

// Loaders issue every global load of the thread before the first shared
// store, so the load latencies overlap.
static __device__ __forceinline__ void load_f32_rows(float* dst, const float* src) {
    constexpr int N = C * (D / 4) / kThreads;
    float4 v[N];
#pragma unroll
    for (int n = 0; n < N; ++n) v[n] = ld4(src + 4 * (threadIdx.x + n * kThreads));
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const int idx = threadIdx.x + n * kThreads;
        st4(dst + (idx / (D / 4)) * PP + (idx % (D / 4)) * 4, v[n]);
    }
}

static __device__ __forceinline__ void load_cc(float* dst, const float* src) {
    constexpr int N = C * C / 4 / kThreads;
    float4 v[N];
#pragma unroll
    for (int n = 0; n < N; ++n) v[n] = ld4(src + 4 * (threadIdx.x + n * kThreads));
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const int idx = 4 * (threadIdx.x + n * kThreads);
        float* d = dst + (idx / C) * PC + idx % C;
        d[0] = v[n].x;
        d[1] = v[n].y;
        d[2] = v[n].z;
        d[3] = v[n].w;
    }
}

// A thread's [4][8] tile (rows ty + 16 r, columns 4 tx + 64 c + e) of a
// [C][D] f32 array in HBM.
static __device__ __forceinline__ void tile_from_rows(float (&v)[4][8], const float* src) {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const float4 f = ld4(src + (ty + 16 * r) * D + 64 * c + 4 * tx);
            v[r][4 * c] = f.x;
            v[r][4 * c + 1] = f.y;
            v[r][4 * c + 2] = f.z;
            v[r][4 * c + 3] = f.w;
        }
}

// bf16 row segment of 4: dst[0..3] = v[0..3] (+ add[0..3] when add != nullptr)
static __device__ __forceinline__ void put_bf16x4(__nv_bfloat16* dst, const float* v,
                                                  const float* add) {
    float4 a = add != nullptr ? ld4(add) : make_float4(0.f, 0.f, 0.f, 0.f);
    uint2 p;
    p.x = Vec16<__nv_bfloat16>::pack2(v[0] + a.x, v[1] + a.y);
    p.y = Vec16<__nv_bfloat16>::pack2(v[2] + a.z, v[3] + a.w);
    *reinterpret_cast<uint2*>(dst) = p;
}

__global__ void __launch_bounds__(kThreads, 1)
    delta_post2_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                       const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ beta,
                       const float* __restrict__ dQa, const float* __restrict__ dWg,
                       const float* __restrict__ dK1, const float* __restrict__ dMg,
                       const float* __restrict__ Tg, const float* __restrict__ Gg,
                       const float* __restrict__ dUg, __nv_bfloat16* __restrict__ gq,
                       __nv_bfloat16* __restrict__ gk, __nv_bfloat16* __restrict__ gv,
                       __nv_bfloat16* __restrict__ gbeta, int L, int H, int NC) {
    extern __shared__ float sm[];
    float* Ks = sm;                // [C][PP]  K
    float* Ws = Ks + C * PP;       // [C][PP]  dW
    float* Us = Ws + C * PP;       // [C][PP]  dU~, then Q
    float* Vs = Us + C * PP;       // [C][PP]  V
    float* dMs = Vs + C * PP;      // [C][PC]  dM
    float* Ts = dMs + C * PC;      // [C][PC]  T
    float* Xa = Ts + C * PC;       // [C][PC]  dT_b -> dT -> dA
    float* Xb = Xa + C * PC;       // [C][PC]  X = T^T dT -> E
    float* bs = Xb + C * PC;       // [C]
    float* dbs = bs + C;           // [C]
    float* Gs = dbs + C;           // [C][PC]  K K^T
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const long long ch = ((long long)b * H + h) * NC + c;
    const int t0 = c * C, nvalid = min(C, L - t0);
    const long long ts = (long long)H * D;
    const long long row0 = (((long long)b * L + t0) * H + h) * D;

    load_chunk_rows(Ks, k, row0, ts, nvalid, nullptr);
    load_chunk_rows(Vs, v, row0, ts, nvalid, nullptr);
    load_f32_rows(Ws, dWg + ch * C * D);
    load_f32_rows(Us, dUg + ch * C * D);
    load_cc(dMs, dMg + ch * C * C);
    load_cc(Ts, Tg + ch * C * C);
    load_cc(Gs, Gg + ch * C * C);
    if (tid < C)
        bs[tid] = tid < nvalid ? __bfloat162float(beta[((long long)b * L + t0 + tid) * H + h])
                               : 0.0f;
    __syncthreads();

    // dQ = dQa + dM K ;  dV = T_b^T dU~   (rows ty + 16 r, columns 4 tx + 64 cc + e)
    {
        float aq[4][8], av[4][8];
        tile_from_rows(aq, dQa + ch * C * D);  // padded rows of dQa are zero
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int e = 0; e < 8; ++e) av[r][e] = 0.0f;
        for (int kk = 0; kk < C; ++kk) {
            float am[4], at[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int row = ty + 16 * r;
                am[r] = dMs[row * PC + kk];                 // dM[row][kk]
                at[r] = Ts[kk * PC + row] * bs[row];        // T_b[kk][row]
            }
            const float4 k0 = ld4(Ks + kk * PP + 4 * tx), k1 = ld4(Ks + kk * PP + 64 + 4 * tx);
            const float4 u0 = ld4(Us + kk * PP + 4 * tx), u1 = ld4(Us + kk * PP + 64 + 4 * tx);
            const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
            const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    aq[r][e] = fmaf(am[r], kv[e], aq[r][e]);
                    av[r][e] = fmaf(at[r], uv[e], av[r][e]);
                }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int row = ty + 16 * r;
            if (row < nvalid) {
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int col = 64 * cc + 4 * tx;
                    put_bf16x4(gq + row0 + row * ts + col, &aq[r][4 * cc], nullptr);
                    put_bf16x4(gv + row0 + row * ts + col, &av[r][4 * cc], nullptr);
                }
            }
        }
    }
    // dT_b = dW K^T + dU~ V^T   (rows ty + 16 r, columns tx + 16 cc)
    {
        float a[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) a[r][cc] = 0.0f;
        for (int j = 0; j < D; j += 4) {
            float4 aw[4], au[4], bk[4], bv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                aw[r] = ld4(Ws + (ty + 16 * r) * PP + j);
                au[r] = ld4(Us + (ty + 16 * r) * PP + j);
            }
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                bk[cc] = ld4(Ks + (tx + 16 * cc) * PP + j);
                bv[cc] = ld4(Vs + (tx + 16 * cc) * PP + j);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                    a[r][cc] = dot4(aw[r], bk[cc], dot4(au[r], bv[cc], a[r][cc]));
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) Xa[(ty + 16 * r) * PC + tx + 16 * cc] = a[r][cc];
    }
    __syncthreads();
    // dbeta (through T_b), then dT = dT_b diag(beta)
    {
        const int s = tid >> 2, qd = tid & 3;
        float acc = 0.0f;
#pragma unroll 4
        for (int t = qd; t < C; t += 4) acc = fmaf(Xa[t * PC + s], Ts[t * PC + s], acc);
        acc = quad_sum(acc);
        if (qd == 0) dbs[s] = acc;
    }
    __syncthreads();
    for (int idx = tid; idx < C * C; idx += kThreads) {
        const int t = idx / C, s = idx % C;
        Xa[t * PC + s] *= bs[s];
    }
    __syncthreads();
    // X = T^T dT
    {
        float a[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) a[r][cc] = 0.0f;
        for (int t = 0; t < C; ++t) {
            float at[4], bd[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) at[r] = Ts[t * PC + ty + 16 * r];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) bd[cc] = Xa[t * PC + tx + 16 * cc];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) a[r][cc] = fmaf(at[r], bd[cc], a[r][cc]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) Xb[(ty + 16 * r) * PC + tx + 16 * cc] = a[r][cc];
    }
    __syncthreads();
    // dA = -X T^T, strictly lower (into Xa: dT is no longer needed)
    {
        float a[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) a[r][cc] = 0.0f;
        for (int s = 0; s < C; ++s) {
            float ax[4], bt[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) ax[r] = Xb[(ty + 16 * r) * PC + s];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) bt[cc] = Ts[(tx + 16 * cc) * PC + s];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) a[r][cc] = fmaf(ax[r], bt[cc], a[r][cc]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int row = ty + 16 * r, col = tx + 16 * cc;
                Xa[row * PC + col] = col < row ? -a[r][cc] : 0.0f;
            }
    }
    __syncthreads();
    // dbeta (through A) ; E = dG + dG^T with dG = diag(beta) dA (into Xb)
    {
        const int t = tid >> 2, qd = tid & 3;
        float acc = 0.0f;  // dA is strictly lower: columns s >= t add 0
#pragma unroll 4
        for (int s = qd; s < C; s += 4) acc = fmaf(Xa[t * PC + s], Gs[t * PC + s], acc);
        acc = quad_sum(acc) + dbs[t];
        if (qd == 0 && t < nvalid)
            gbeta[((long long)b * L + t0 + t) * H + h] = __float2bfloat16(acc);
    }
    for (int idx = tid; idx < C * C; idx += kThreads) {
        const int t = idx / C, s = idx % C;
        Xb[t * PC + s] = bs[t] * Xa[t * PC + s] + bs[s] * Xa[s * PC + t];
    }
    // Q replaces dU~ (last read by the dT_b products, before two barriers)
    load_chunk_rows(Us, q, row0, ts, nvalid, nullptr);
    __syncthreads();
    // dK = dK1 + dM^T Q + T_b^T dW + E K   (rows ty + 16 r, columns 4 tx + 64 cc + e)
    {
        float a[4][8];
        tile_from_rows(a, dK1 + ch * C * D);
        for (int t = 0; t < C; ++t) {
            float am[4], at[4], ae[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int s = ty + 16 * r;
                am[r] = dMs[t * PC + s];
                at[r] = Ts[t * PC + s] * bs[s];
                ae[r] = Xb[t * PC + s];
            }
            const float4 q0 = ld4(Us + t * PP + 4 * tx), q1 = ld4(Us + t * PP + 64 + 4 * tx);
            const float4 w0 = ld4(Ws + t * PP + 4 * tx), w1 = ld4(Ws + t * PP + 64 + 4 * tx);
            const float4 k0 = ld4(Ks + t * PP + 4 * tx), k1 = ld4(Ks + t * PP + 64 + 4 * tx);
            const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    a[r][e] = fmaf(am[r], qv[e], fmaf(at[r], wv[e], fmaf(ae[r], kv[e], a[r][e])));
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int row = ty + 16 * r;
            if (row < nvalid) {
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int col = 64 * cc + 4 * tx;
                    put_bf16x4(gk + row0 + row * ts + col, &a[r][4 * cc], nullptr);
                }
            }
        }
    }
}

}  // namespace

// Library-internal launcher (called by edb_delta_chunked_bwd).
int edb_delta_chunked_post2(const void* q, const void* k, const void* v, const void* beta,
                            const float* dQa, const float* dW, const float* dK1, const float* dM,
                            const float* T, const float* G, const float* dU, void* gq, void* gk,
                            void* gv, void* gbeta, int B, int L, int H, cudaStream_t st) {
    const int NC = (L + C - 1) / C;
    cudaError_t e = cudaFuncSetAttribute(delta_post2_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) return (int)e;
    delta_post2_kernel<<<dim3(NC, H, B), kThreads, kSmem, st>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
        (const __nv_bfloat16*)beta, dQa, dW, dK1, dM, T, G, dU, (__nv_bfloat16*)gq,
        (__nv_bfloat16*)gk, (__nv_bfloat16*)gv, (__nv_bfloat16*)gbeta, L, H, NC);
    return edb::status_from_cuda(cudaGetLastError());
}
