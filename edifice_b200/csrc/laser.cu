// laser.cu -- LASER attention (attention in the exponentiated value space),
// forward + backward, on top of the flash-attention kernels.
//
// Reference semantics (edifice project paths):
//   forward   lib/edifice/cuda/fused_scan.ex:3593-3611 (v_max = max over the sequence
//             of v), :3667-3703 (laser_attention_fallback):
//             A = softmax(Q K^T scale (+ causal mask)) exp(V - v_max)
//             O = log(max(A, 1e-7)) + v_max
//   backward  fused_scan.ex:3723-3766: dR = dO exp(v_max - O) = dO / max(A, 1e-7);
//             dV = (P^T dR) (.) exp(V - v_max); dS = P (.) (dR exp(V - v_max)^T - D);
//             dQ = dS K scale, dK = dS^T Q scale, with D = rowsum(dR (.) A).  v_max gets
//             no gradient (the reference captures it as a constant).
// replacing native/cuda/fused_laser_attention{,_backward}.cu.
//
// Design: the contraction work is exactly flash attention with exp(V - v_max) as the
// values, so both directions run the library's flash kernels (tcgen05 for bf16,
// head_dim 64/128) on V' = exp(V - v_max), with HBM-bound element-wise kernels around
// them: v_max (a column max over the sequence), V', the output's log, dR, and dV = dV' V'.
// The residual the backward reads: V' [B, Hkv, L, d] and the attention output before the
// log A [B, Hq, L, d] (both in the io dtype), lse [B, Hq, L] f32, v_max [B, Hkv, d] f32.
#include <math.h>

#include "edb_common.cuh"

namespace {

constexpr int kThreads = 256;

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

struct LaserResid {
    void* vexp;    // [B, Hkv, L, d] io dtype
    void* attn;    // [B, Hq, L, d] io dtype
    float* lse;    // [B, Hq, L]
    float* vmax;   // [B, Hkv, d]
};

LaserResid carve(void* base, int es, int B, int Hq, int Hkv, int L, int d) {
    char* p = static_cast<char*>(base);
    LaserResid r;
    r.vexp = p;
    p += a256((size_t)B * Hkv * L * d * es);
    r.attn = p;
    p += a256((size_t)B * Hq * L * d * es);
    r.lse = reinterpret_cast<float*>(p);
    p += a256((size_t)B * Hq * L * sizeof(float));
    r.vmax = reinterpret_cast<float*>(p);
    return r;
}

size_t resid_bytes(int es, int B, int Hq, int Hkv, int L, int d) {
    return a256((size_t)B * Hkv * L * d * es) + a256((size_t)B * Hq * L * d * es) +
           a256((size_t)B * Hq * L * sizeof(float)) + a256((size_t)B * Hkv * d * sizeof(float));
}

// v_max[bh, c] = max over t of v[bh, t, c], in two passes: grid (B*Hkv, ns),
// block (128, kSliceRows): each block takes a 1/ns slice of the sequence (ns <= min(64, L)) and
// writes its column maxima to part[bh][split][c]; laser_vmax_final takes the max over
// the splits (or converts the caller's v_max).
constexpr int kMaxSplit = 64;
constexpr int kSliceRows = kThreads / 128;  // block (128, kSliceRows)

template <typename T>
__global__ void __launch_bounds__(kThreads)
    laser_vmax_part_kernel(const T* __restrict__ v, float* __restrict__ part, int L, int d,
                           int ns) {
    __shared__ float sm[kSliceRows][128];
    const long long bh = blockIdx.x;
    const int c = threadIdx.x, sl = threadIdx.y;
    const int t0 = (int)((long long)L * blockIdx.y / ns);
    const int t1 = (int)((long long)L * (blockIdx.y + 1) / ns);
    float m = -INFINITY;
    if (c < d)
        for (int t = t0 + sl; t < t1; t += kSliceRows)
            m = fmaxf(m, ld_scalar<T>(v + (bh * L + t) * d + c));
    sm[sl][c] = m;
    __syncthreads();
    if (sl == 0 && c < d) {
        for (int s = 1; s < kSliceRows; ++s) m = fmaxf(m, sm[s][c]);
        part[(bh * ns + blockIdx.y) * d + c] = m;
    }
}

template <typename T>
__global__ void laser_vmax_final_kernel(const float* __restrict__ part,
                                        const T* __restrict__ vmax_in, float* __restrict__ vmax,
                                        long long n_bh, int d, int ns) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_bh * d) return;
    if (vmax_in != nullptr) {
        vmax[i] = ld_scalar<T>(vmax_in + i);
        return;
    }
    const long long bh = i / d;
    const int c = (int)(i % d);
    float m = -INFINITY;
    for (int s = 0; s < ns; ++s) m = fmaxf(m, part[(bh * ns + s) * d + c]);
    vmax[i] = m;
}

// element-wise passes over [B, H, L, d] with a per-(b, kv head, c) value vm:
//   MODE 0: out = exp(x - vm)                       (V' from V)
//   MODE 1: out = log(max(x, 1e-7)) + vm            (O from A)
//   MODE 2: out = x / max(y, 1e-7)                  (dR from dO and A)
//   MODE 3: out = x * y                             (dV from dV' and V')
// Each thread takes one 16-byte vector (d is a multiple of the vector length and the
// tensors are 16-byte aligned; laser_ew_kernel_scalar covers the rest).
template <int MODE>
static __device__ __forceinline__ float ew_op(float x, float y, float m) {
    if (MODE == 0) return expf(x - m);
    if (MODE == 1) return logf(fmaxf(x, 1e-7f)) + m;
    if (MODE == 2) return x / fmaxf(y, 1e-7f);
    return x * y;
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads)
    laser_ew_kernel(const T* __restrict__ x, const T* __restrict__ y, const float* __restrict__ vm,
                    T* __restrict__ out, long long nvec, int L, int d, int H, int group) {
    using V = Vec16<T>;
    constexpr int N = V::N;
    const long long iv = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (iv >= nvec) return;
    const long long i = iv * N;
    float xs[N], ys[N], ms[N];
    V::unpack(*reinterpret_cast<const uint4*>(x + i), xs);
    if (MODE >= 2) V::unpack(*reinterpret_cast<const uint4*>(y + i), ys);
    if (MODE <= 1) {
        const int c = (int)(i % d);
        const long long bh = i / ((long long)L * d);  // b * H + h
        const long long b = bh / H, h = bh % H;
        const float* mp = vm + (b * (H / group) + h / group) * d + c;
#pragma unroll
        for (int e = 0; e < N; ++e) ms[e] = mp[e];
    }
    float r[N];
#pragma unroll
    for (int e = 0; e < N; ++e) r[e] = ew_op<MODE>(xs[e], MODE >= 2 ? ys[e] : 0.0f, MODE <= 1 ? ms[e] : 0.0f);
    st_global_v4(out + i, V::pack(r));
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads)
    laser_ew_kernel_scalar(const T* __restrict__ x, const T* __restrict__ y,
                           const float* __restrict__ vm, T* __restrict__ out, long long n, int L,
                           int d, int H, int group) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float m = 0.0f;
    if (MODE <= 1) {
        const int c = (int)(i % d);
        const long long bh = i / ((long long)L * d);
        const long long b = bh / H, h = bh % H;
        m = vm[(b * (H / group) + h / group) * d + c];
    }
    st_scalar<T>(out + i, ew_op<MODE>(ld_scalar<T>(x + i), MODE >= 2 ? ld_scalar<T>(y + i) : 0.0f,
                                      m));
}

template <typename T, int MODE>
int launch_ew(const void* x, const void* y, const float* vm, void* out, long long n, int L, int d,
              int H, int group, cudaStream_t st) {
    constexpr int N = Vec16<T>::N;
    if (d % N == 0 && edb::aligned16(x) && edb::aligned16(out) && (y == nullptr || edb::aligned16(y))) {
        const long long nvec = n / N;
        laser_ew_kernel<T, MODE><<<(unsigned)((nvec + kThreads - 1) / kThreads), kThreads, 0, st>>>(
            (const T*)x, (const T*)y, vm, (T*)out, nvec, L, d, H, group);
    } else {
        laser_ew_kernel_scalar<T, MODE><<<(unsigned)((n + kThreads - 1) / kThreads), kThreads, 0,
                                          st>>>((const T*)x, (const T*)y, vm, (T*)out, n, L, d, H,
                                                group);
    }
    return edb::status_from_cuda(cudaGetLastError());
}

template <typename T>
int laser_fwd(const void* q, const void* k, const void* v, const void* vmax_in, void* o,
              LaserResid r, int dtype, int B, int Hq, int Hkv, int L, int d, int causal,
              float scale, cudaStream_t st) {
    // the split maxima go to the start of the residual (V' and A, not yet written:
    // together at least 2 B Hkv L d io elements >= B Hkv ns d floats for ns <= L)
    float* part = static_cast<float*>(r.vexp);
    const int ns = L < kMaxSplit ? L : kMaxSplit;
    if (vmax_in == nullptr) {
        laser_vmax_part_kernel<T><<<dim3(B * Hkv, ns), dim3(128, kSliceRows), 0, st>>>(
            (const T*)v, part, L, d, ns);
        if (cudaError_t e = cudaGetLastError()) return (int)e;
    }
    const long long nbh = (long long)B * Hkv;
    laser_vmax_final_kernel<T><<<(unsigned)((nbh * d + 255) / 256), 256, 0, st>>>(
        part, (const T*)vmax_in, r.vmax, nbh, d, ns);
    if (cudaError_t e = cudaGetLastError()) return (int)e;
    const long long nkv = (long long)B * Hkv * L * d, nq = (long long)B * Hq * L * d;
    if (int s = launch_ew<T, 0>(v, nullptr, r.vmax, r.vexp, nkv, L, d, Hkv, 1, st)) return s;
    if (int s = edb_flash_attention_fwd(dtype, q, k, r.vexp, r.attn, r.lse, B, Hq, Hkv, L, d,
                                        causal, scale, st))
        return s;
    return launch_ew<T, 1>(r.attn, nullptr, r.vmax, o, nq, L, d, Hq, Hq / Hkv, st);
}

template <typename T>
int laser_bwd(const void* q, const void* k, const void* dO, LaserResid r, void* dq, void* dk,
              void* dv, int dtype, int B, int Hq, int Hkv, int L, int d, int causal, float scale,
              void* ws, size_t ws_bytes, cudaStream_t st) {
    const long long nkv = (long long)B * Hkv * L * d, nq = (long long)B * Hq * L * d;
    const int es = sizeof(T);
    void* dR = ws;
    char* fws = static_cast<char*>(ws) + a256((size_t)nq * es);
    const size_t fws_bytes = ws_bytes - a256((size_t)nq * es);
    if (int s = launch_ew<T, 2>(dO, r.attn, nullptr, dR, nq, L, d, Hq, 1, st)) return s;
    // flash backward with V' as the values, A as the output and dR as its gradient
    if (int s = edb_flash_attention_bwd(dtype, q, k, r.vexp, r.attn, dR, r.lse, dq, dk, dv, B, Hq,
                                        Hkv, L, d, causal, scale, fws, fws_bytes, st))
        return s;
    return launch_ew<T, 3>(dv, r.vexp, nullptr, dv, nkv, L, d, Hkv, 1, st);
}

int check(int dtype, int B, int Hq, int Hkv, int L, int d) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || L <= 0 || d <= 0) return EDB_ERR_BAD_SHAPE;
    if (Hq % Hkv != 0) return EDB_ERR_BAD_SHAPE;
    if (d > 128) return EDB_ERR_UNSUPPORTED;
    return EDB_OK;
}

}  // namespace

extern "C" size_t edb_laser_attention_resid_bytes(int dtype, int batch, int q_heads, int kv_heads,
                                                  int seq_len, int head_dim) {
    if (check(dtype, batch, q_heads, kv_heads, seq_len, head_dim)) return 0;
    return resid_bytes(dtype == EDB_BF16 ? 2 : 4, batch, q_heads, kv_heads, seq_len, head_dim);
}

extern "C" int edb_laser_attention_fwd(int dtype, const void* q, const void* k, const void* v,
                                       const void* v_max, void* o, void* resid, int batch,
                                       int q_heads, int kv_heads, int seq_len, int head_dim,
                                       int causal, float scale, void* stream) {
    if (int s = check(dtype, batch, q_heads, kv_heads, seq_len, head_dim)) return s;
    if (!q || !k || !v || !o || !resid) return EDB_ERR_NULL_POINTER;
    if (reinterpret_cast<uintptr_t>(resid) & 255u) return EDB_ERR_MISALIGNED;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const LaserResid r = carve(resid, es, batch, q_heads, kv_heads, seq_len, head_dim);
    cudaStream_t st = (cudaStream_t)stream;
    return dtype == EDB_BF16
               ? laser_fwd<__nv_bfloat16>(q, k, v, v_max, o, r, dtype, batch, q_heads, kv_heads,
                                          seq_len, head_dim, causal, scale, st)
               : laser_fwd<float>(q, k, v, v_max, o, r, dtype, batch, q_heads, kv_heads, seq_len,
                                  head_dim, causal, scale, st);
}

extern "C" size_t edb_laser_attention_bwd_workspace(int dtype, int batch, int q_heads,
                                                    int kv_heads, int seq_len, int head_dim) {
    if (check(dtype, batch, q_heads, kv_heads, seq_len, head_dim)) return 0;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    return a256((size_t)batch * q_heads * seq_len * head_dim * es) +
           edb_flash_attention_bwd_workspace(dtype, batch, q_heads, kv_heads, seq_len, head_dim,
                                             1);
}

extern "C" int edb_laser_attention_bwd(int dtype, const void* q, const void* k, const void* dO,
                                       const void* resid, void* dq, void* dk, void* dv, int batch,
                                       int q_heads, int kv_heads, int seq_len, int head_dim,
                                       int causal, float scale, void* workspace,
                                       size_t workspace_bytes, void* stream) {
    if (int s = check(dtype, batch, q_heads, kv_heads, seq_len, head_dim)) return s;
    if (!q || !k || !dO || !resid || !dq || !dk || !dv) return EDB_ERR_NULL_POINTER;
    const size_t need = edb_laser_attention_bwd_workspace(dtype, batch, q_heads, kv_heads,
                                                          seq_len, head_dim);
    if (workspace_bytes < need || !workspace) return EDB_ERR_WORKSPACE_TOO_SMALL;
    if ((reinterpret_cast<uintptr_t>(resid) & 255u) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return EDB_ERR_MISALIGNED;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const LaserResid r = carve(const_cast<void*>(resid), es, batch, q_heads, kv_heads, seq_len,
                               head_dim);
    cudaStream_t st = (cudaStream_t)stream;
    return dtype == EDB_BF16
               ? laser_bwd<__nv_bfloat16>(q, k, dO, r, dq, dk, dv, dtype, batch, q_heads,
                                          kv_heads, seq_len, head_dim, causal, scale, workspace,
                                          workspace_bytes, st)
               : laser_bwd<float>(q, k, dO, r, dq, dk, dv, dtype, batch, q_heads, kv_heads,
                                  seq_len, head_dim, causal, scale, workspace, workspace_bytes,
                                  st);
}
