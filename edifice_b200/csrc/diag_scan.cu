// diag_scan.cu -- diagonal linear-recurrence scans (linear scan, MinGRU), fwd + bwd.
//
// Reference semantics (edifice project paths):
//   linear fwd  lib/edifice/cuda/fused_scan.ex:4429-4444, :869-882
//   linear bwd  fused_scan.ex:884-916
//   MinGRU fwd  fused_scan.ex:516-528 (lib/edifice/recurrent/min_gru.ex:305-326)
//   MinGRU bwd  fused_scan.ex:548-581
// replacing native/cuda/fused_{linear,mingru}_scan{,_backward}.cu.
//
// Design (B200, HBM-bound):
//   * Every step is an affine map of the carried state s <- A_t s + B_t:
//       linear fwd (a, b)          MinGRU fwd (1-z, z c)
//       linear bwd (a, a dY)       MinGRU bwd (1-z, (1-z) dY)    [s = dh_acc]
//     so one engine serves all four; the backward runs time in reverse.
//   * A CTA owns one channel block of one batch row -- 256 bytes (128 bf16 / 64
//     f32 channels, 512 threads) when that still gives at least 96 CTAs, else
//     128 bytes (256 threads) -- and streams the whole sequence through shared
//     memory in tiles of ROWS time steps, staged by 2D TMA loads in a
//     STAGES-deep mbarrier ring.  The wide blocks read two full 128-byte lines
//     per row, which DRAM serves measurably better than one (config 1: 88 % /
//     93 % of the measured copy bandwidth against 77 % / 81 %); narrower 64-byte
//     blocks measured slower still.
//   * Inside a tile: thread (seg, g) owns the 16-byte chunk g (8 bf16 channels)
//     of ROWS/32 consecutive steps.  Per-thread sequential composition, a warp
//     shuffle scan over the segments a warp holds, and a cross-warp prefix done
//     by one thread per channel that also carries the state from tile to tile.  Inputs stay in registers between the composition and the
//     apply pass, so every input byte is read from HBM once and every output
//     byte written once (16-byte stores, 128 contiguous bytes per 8 lanes).
//   * The backward needs h_{t-1}: its tile of the forward output is loaded by
//     TMA one row up (y - 1); row t = 0 takes h0 instead.
//   * Shapes the TMA path cannot take (hidden * elem_size not a multiple of 16,
//     unaligned pointers) run a plain one-thread-per-channel kernel.
#include <algorithm>

#include "edb_common.cuh"

namespace {

// OP_ELUGRU / OP_REALGRU / OP_DIAGLIN: the native-recurrence scans
// (lib/edifice/recurrent/native_recurrence.ex:125-230), forward only, with the
// activation applied to the raw inputs on load as native/cuda/fused_native_rec_scan.cu
// does; their backwards are the MinGRU / linear ones on the activated values.
enum { OP_LINEAR = 0, OP_MINGRU = 1, OP_ELUGRU = 2, OP_REALGRU = 3, OP_DIAGLIN = 4 };

// logistic sigmoid from one ex2 and one reciprocal
static __device__ __forceinline__ float sigmoid_fast(float x) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-1.4426950408889634f * x));
    return __frcp_rn(1.0f + e);
}
// 1 + elu(x): x + 1 for x >= 0, exp(x) for x < 0
static __device__ __forceinline__ float one_plus_elu(float x) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(1.4426950408889634f * fminf(x, 0.0f)));
    return x >= 0.0f ? x + 1.0f : e;
}

template <int OP, bool BWD>
struct StepMap;

// forward: x0 = a | z, x1 = b | c
template <>
struct StepMap<OP_LINEAR, false> {
    static __device__ __forceinline__ void map(float x0, float x1, float& A, float& B) {
        A = x0;
        B = x1;
    }
};
template <>
struct StepMap<OP_MINGRU, false> {
    static __device__ __forceinline__ void map(float x0, float x1, float& A, float& B) {
        A = 1.0f - x0;
        B = x0 * x1;
    }
};
// x0 = raw gate, x1 = raw candidate: z = sigmoid(x0), c = 1 + elu(x1)
template <>
struct StepMap<OP_ELUGRU, false> {
    static __device__ __forceinline__ void map(float x0, float x1, float& A, float& B) {
        const float z = sigmoid_fast(x0);
        A = 1.0f - z;
        B = z * one_plus_elu(x1);
    }
};
// x0 = raw gate, x1 = candidate: z = sigmoid(x0)
template <>
struct StepMap<OP_REALGRU, false> {
    static __device__ __forceinline__ void map(float x0, float x1, float& A, float& B) {
        const float z = sigmoid_fast(x0);
        A = 1.0f - z;
        B = z * x1;
    }
};
// x0 = raw a, x1 = b: h = sigmoid(a) h + b
template <>
struct StepMap<OP_DIAGLIN, false> {
    static __device__ __forceinline__ void map(float x0, float x1, float& A, float& B) {
        A = sigmoid_fast(x0);
        B = x1;
    }
};
// backward: x0 = a | z, x1 = dY
template <>
struct StepMap<OP_LINEAR, true> {
    static __device__ __forceinline__ void map(float x0, float x1, float& A, float& B) {
        A = x0;
        B = x0 * x1;
    }
};
template <>
struct StepMap<OP_MINGRU, true> {
    static __device__ __forceinline__ void map(float x0, float x1, float& A, float& B) {
        A = 1.0f - x0;
        B = A * x1;
    }
};

struct ScanMaps {
    CUtensorMap m[4];
};

// NIN inputs:  fwd: [x0, x1]   bwd: [x0, dY, h (shifted -1)] (+ c for MinGRU)
// CW: 16-byte chunks per channel-block row (8: 128-byte blocks, 256 threads;
// 16: 256-byte blocks, 512 threads).
template <typename T, int OP, bool BWD, int ROWS, int STAGES, int CW>
__global__ void __launch_bounds__(32 * CW, CW >= 16 ? 1 : 2)
    diag_scan_tma_kernel(const __grid_constant__ ScanMaps maps, const T* __restrict__ h0,
                         T* __restrict__ out0, T* __restrict__ out1, T* __restrict__ gh0, int L,
                         int H, unsigned* err, unsigned long long wait_ns) {
    using V = Vec16<T>;
    constexpr int VEC = V::N;
    constexpr int NW = CW;             // warps per CTA (32 segments of CW threads)
    constexpr int RB = 16 * CW;        // bytes per channel-block row
    constexpr int NCH = CW * VEC;      // channels per CTA
    constexpr int RPS = ROWS / 32;
    constexpr int NIN = BWD ? (OP == OP_MINGRU ? 4 : 3) : 2;
    constexpr int TILE = ROWS * RB;
    constexpr int SPW = 32 / CW;       // segments per warp

    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stage_base = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * NIN * TILE);
    float* aggA = reinterpret_cast<float*>(full + STAGES);
    float* aggB = aggA + NW * NCH;
    float* cinw = aggB + NW * NCH;
    int* s_abort = reinterpret_cast<int*>(cinw + NW * NCH);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = tid % CW, seg = tid / CW;
    const int cb = blockIdx.x, b = blockIdx.y;
    const int ch0 = cb * NCH + g * VEC;  // first channel of this thread
    const bool ch_ok = ch0 < H;
    const int ntiles = (L + ROWS - 1) / ROWS;
    const long long row_base = (long long)b * L;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
        *s_abort = 0;
        fence_mbar_init();
        for (int k = 0; k < NIN; ++k) prefetch_tmap(&maps.m[k]);
    }
    __syncthreads();

    auto issue = [&](int i) {
        const int pt = BWD ? ntiles - 1 - i : i;
        const int t0 = pt * ROWS;
        const int s = i % STAGES;
        mbar_arrive_expect_tx(&full[s], NIN * TILE);
#pragma unroll
        for (int k = 0; k < NIN; ++k) {
            const int shift = (BWD && k == 2) ? -1 : 0;
            tma_load_2d(stage_base + (s * NIN + k) * TILE, &maps.m[k], &full[s], cb * NCH,
                        (int)(row_base + t0 + shift));
        }
    };
    if (tid == 0)
        for (int i = 0; i < STAGES && i < ntiles; ++i) issue(i);

    // tile-to-tile carry, owned by thread `tid` for channel `tid` (tid < NCH)
    float carry = 0.0f;
    if (!BWD && tid < NCH && h0 != nullptr && cb * NCH + tid < H)
        carry = ld_scalar<T>(h0 + (long long)b * H + cb * NCH + tid);

    // h0 values of this thread's channels (backward: h_{-1} for row t = 0)
    float h0v[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) h0v[c] = 0.0f;
    if (BWD && h0 != nullptr && ch_ok) {
        uint4 v = *reinterpret_cast<const uint4*>(h0 + (long long)b * H + ch0);
        V::unpack(v, h0v);
    }

    int abort_tile = -1;
    for (int i = 0; i < ntiles; ++i) {
        const int s = i % STAGES;
        const unsigned par = (unsigned)(i / STAGES) & 1u;
        const int pt = BWD ? ntiles - 1 - i : i;
        const int t0 = pt * ROWS;

        if (!mbar_wait_limited(&full[s], par, err, EDB_DEVERR_SCAN_PIPE, wait_ns)) *s_abort = 1;

        // ---- registers <- this thread's RPS rows of every input
        uint4 rin[NIN][RPS];
        const uint8_t* sb = stage_base + s * NIN * TILE;
#pragma unroll
        for (int j = 0; j < RPS; ++j) {
            const int p = seg * RPS + j;               // logical (processing-order) row
            const int r = BWD ? ROWS - 1 - p : p;      // physical row in the tile
#pragma unroll
            for (int k = 0; k < NIN; ++k)
                rin[k][j] = *reinterpret_cast<const uint4*>(sb + k * TILE + r * RB + g * 16);
        }

        // ---- per-thread composition over its RPS steps
        float A[VEC], Bc[VEC];
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
            A[c] = 1.0f;
            Bc[c] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < RPS; ++j) {
            const int p = seg * RPS + j;
            const int r = BWD ? ROWS - 1 - p : p;
            if (t0 + r < L) {
                float x0[VEC], x1[VEC];
                V::unpack(rin[0][j], x0);
                V::unpack(rin[1][j], x1);
#pragma unroll
                for (int c = 0; c < VEC; ++c) {
                    if (OP == OP_MINGRU && !BWD) {
                        // (1 - z, z c) composed as A - z A, B + z (c - B): 3 instructions
                        A[c] = fmaf(-x0[c], A[c], A[c]);
                        Bc[c] = fmaf(x0[c], x1[c] - Bc[c], Bc[c]);
                    } else {
                        float a, bb;
                        StepMap<OP, BWD>::map(x0[c], x1[c], a, bb);
                        Bc[c] = fmaf(a, Bc[c], bb);
                        A[c] *= a;
                    }
                }
            }
        }

        // ---- warp scan over the SPW segments of this warp (lanes CW apart)
#pragma unroll
        for (int off = CW; off <= 16; off <<= 1) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) {
                const float Ap = __shfl_up_sync(0xffffffffu, A[c], off);
                const float Bp = __shfl_up_sync(0xffffffffu, Bc[c], off);
                if (lane >= off) {
                    Bc[c] = fmaf(A[c], Bp, Bc[c]);
                    A[c] *= Ap;
                }
            }
        }
        // exclusive prefix within the warp
        float Ae[VEC], Be[VEC];
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
            Ae[c] = __shfl_up_sync(0xffffffffu, A[c], CW);
            Be[c] = __shfl_up_sync(0xffffffffu, Bc[c], CW);
            if (lane < CW) {
                Ae[c] = 1.0f;
                Be[c] = 0.0f;
            }
        }
        if (lane / CW == SPW - 1) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) {
                aggA[warp * NCH + g * VEC + c] = A[c];
                aggB[warp * NCH + g * VEC + c] = Bc[c];
            }
        }
        __syncthreads();
        if (*s_abort) {
            abort_tile = i;
            break;
        }
        // every thread has moved this stage into registers: refill it
        if (tid == 0 && i + STAGES < ntiles) issue(i + STAGES);

        // ---- cross-warp prefix + tile carry, one thread per channel
        if (tid < NCH) {
            float st = carry;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                cinw[w * NCH + tid] = st;
                st = fmaf(aggA[w * NCH + tid], st, aggB[w * NCH + tid]);
            }
            carry = st;
        }
        __syncthreads();

        // ---- apply: rerun this thread's steps from its carry-in, store outputs
        float sv[VEC];
#pragma unroll
        for (int c = 0; c < VEC; ++c) sv[c] = fmaf(Ae[c], cinw[warp * NCH + g * VEC + c], Be[c]);

#pragma unroll
        for (int j = 0; j < RPS; ++j) {
            const int p = seg * RPS + j;
            const int r = BWD ? ROWS - 1 - p : p;
            const int t = t0 + r;
            if (t < L) {
                float x0[VEC], x1[VEC];
                V::unpack(rin[0][j], x0);
                V::unpack(rin[1][j], x1);
                const long long off = (row_base + t) * (long long)H + ch0;
                if (!BWD) {
#pragma unroll
                    for (int c = 0; c < VEC; ++c) {
                        if (OP == OP_MINGRU) {
                            sv[c] = fmaf(x0[c], x1[c] - sv[c], sv[c]);  // h + z (c - h)
                        } else {
                            float a, bb;
                            StepMap<OP, BWD>::map(x0[c], x1[c], a, bb);
                            sv[c] = fmaf(a, sv[c], bb);
                        }
                    }
                    if (ch_ok) st_global_v4(out0 + off, V::pack(sv));
                } else {
                    float hp[VEC], o0[VEC], o1[VEC];
                    V::unpack(rin[2][j], hp);
                    if (t == 0) {
#pragma unroll
                        for (int c = 0; c < VEC; ++c) hp[c] = h0v[c];
                    }
                    float cc[VEC];
                    if (OP == OP_MINGRU) V::unpack(rin[NIN - 1][j], cc);
#pragma unroll
                    for (int c = 0; c < VEC; ++c) {
                        const float gdh = x1[c] + sv[c];  // dY_t + acc
                        if (OP == OP_LINEAR) {
                            o0[c] = gdh * hp[c];             // da
                            o1[c] = gdh;                     // db
                            sv[c] = gdh * x0[c];
                        } else {
                            o0[c] = gdh * (cc[c] - hp[c]);  // dz
                            o1[c] = gdh * x0[c];             // dc
                            sv[c] = gdh * (1.0f - x0[c]);
                        }
                    }
                    if (ch_ok) {
                        st_global_v4(out0 + off, V::pack(o0));
                        st_global_v4(out1 + off, V::pack(o1));
                    }
                }
            }
        }
    }

    if (abort_tile >= 0) {
        // drain the copies this CTA still has in flight (tiles abort_tile ..
        // abort_tile + STAGES - 1), each wait bounded by EDB_WAIT_NS whatever the
        // host's limit (the copies are real and land), then leave
        if (tid == 0) {
            const int last = abort_tile + STAGES < ntiles ? abort_tile + STAGES : ntiles;
            for (int i = abort_tile; i < last; ++i)
                mbar_wait_bounded(&full[i % STAGES], (unsigned)(i / STAGES) & 1u, err,
                                  EDB_DEVERR_SCAN_PIPE);
        }
        return;
    }
    if (BWD && gh0 != nullptr && tid < NCH && cb * NCH + tid < H)
        st_scalar<T>(gh0 + (long long)b * H + cb * NCH + tid, carry);
}

// ---------------------------------------------------------------- generic path
// One thread per (batch, channel), sequential over time.  Used only for shapes
// the TMA path does not take (odd hidden sizes, unaligned pointers).
template <typename T, int OP, bool BWD>
__global__ void diag_scan_simple_kernel(const T* __restrict__ x0p, const T* __restrict__ x1p,
                                        const T* __restrict__ hprevp, const T* __restrict__ cp,
                                        const T* __restrict__ h0, T* __restrict__ out0,
                                        T* __restrict__ out1, T* __restrict__ gh0, int B, int L,
                                        int H) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)B * H) return;
    const int b = (int)(idx / H), h = (int)(idx % H);
    const float hinit = h0 ? ld_scalar<T>(h0 + (long long)b * H + h) : 0.0f;
    if (!BWD) {
        float s = hinit;
        for (int t = 0; t < L; ++t) {
            const long long o = ((long long)b * L + t) * H + h;
            float a, bb;
            StepMap<OP, false>::map(ld_scalar<T>(x0p + o), ld_scalar<T>(x1p + o), a, bb);
            s = fmaf(a, s, bb);
            st_scalar<T>(out0 + o, s);
        }
    } else {
        float acc = 0.0f;
        for (int t = L - 1; t >= 0; --t) {
            const long long o = ((long long)b * L + t) * H + h;
            const float x0 = ld_scalar<T>(x0p + o);
            const float gdh = ld_scalar<T>(x1p + o) + acc;
            const float hp = t == 0 ? hinit : ld_scalar<T>(hprevp + o - H);
            if (OP == OP_LINEAR) {
                st_scalar<T>(out0 + o, gdh * hp);
                st_scalar<T>(out1 + o, gdh);
                acc = gdh * x0;
            } else {
                st_scalar<T>(out0 + o, gdh * (ld_scalar<T>(cp + o) - hp));
                st_scalar<T>(out1 + o, gdh * x0);
                acc = gdh * (1.0f - x0);
            }
        }
        if (gh0) st_scalar<T>(gh0 + (long long)b * H + h, acc);
    }
}

// ---------------------------------------------------------------- launch
template <typename T, int OP, bool BWD, int ROWS, int STAGES, int CW>
size_t tma_smem_bytes() {
    constexpr int NIN = BWD ? (OP == OP_MINGRU ? 4 : 3) : 2;
    constexpr int NCH = CW * Vec16<T>::N;
    return (size_t)STAGES * NIN * ROWS * 16 * CW + STAGES * 8 + 3 * CW * NCH * 4 + 16;
}

template <typename T>
CUtensorMapDataType tmap_dtype();
template <>
CUtensorMapDataType tmap_dtype<float>() {
    return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}
template <>
CUtensorMapDataType tmap_dtype<__nv_bfloat16>() {
    return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

template <typename T>
int make_scan_map(CUtensorMap* m, const void* p, int B, int L, int H, int rows, int row_bytes) {
    const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)B * (cuuint64_t)L};
    const cuuint64_t strides[1] = {(cuuint64_t)H * sizeof(T)};
    const cuuint32_t box[2] = {(cuuint32_t)(row_bytes / sizeof(T)), (cuuint32_t)rows};
    CUresult r = edb::encode_tiled(m, tmap_dtype<T>(), 2, const_cast<void*>(p), dims, strides,
                                   box, CU_TENSOR_MAP_SWIZZLE_NONE);
    return r == CUDA_SUCCESS ? EDB_OK : EDB_ERR_UNSUPPORTED;
}

template <typename T, int OP, bool BWD, int ROWS, int STAGES, int CW>
int launch_tma_cw(const void* const* ins, int nin, const T* h0, T* o0, T* o1, T* gh0, int B,
                  int L, int H, cudaStream_t stream) {
    ScanMaps maps;
    for (int k = 0; k < nin; ++k) {
        int st = make_scan_map<T>(&maps.m[k], ins[k], B, L, H, ROWS, 16 * CW);
        if (st) return st;
    }
    for (int k = nin; k < 4; ++k) maps.m[k] = maps.m[0];
    auto kern = diag_scan_tma_kernel<T, OP, BWD, ROWS, STAGES, CW>;
    const size_t smem = tma_smem_bytes<T, OP, BWD, ROWS, STAGES, CW>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return (int)e;
    constexpr int NCH = CW * Vec16<T>::N;
    dim3 grid((H + NCH - 1) / NCH, B);
    kern<<<grid, 32 * CW, smem, stream>>>(maps, h0, o0, o1, gh0, L, H, edb::device_error_word(),
                                          edb::wait_limit_ns());
    return edb::status_from_cuda(cudaGetLastError());
}

// 256-byte channel blocks (one 512-thread CTA per SM) when there are enough of
// them to cover most SMs and the ring fits; 128-byte blocks otherwise.
template <typename T, int OP, bool BWD, int ROWS, int STAGES>
int launch_tma(const void* const* ins, int nin, const T* h0, T* o0, T* o1, T* gh0, int B, int L,
               int H, cudaStream_t stream) {
    constexpr int NCH16 = 16 * Vec16<T>::N;
    if ((long long)B * ((H + NCH16 - 1) / NCH16) >= 96 &&
        tma_smem_bytes<T, OP, BWD, ROWS, STAGES, 16>() <= 227 * 1024)
        return launch_tma_cw<T, OP, BWD, ROWS, STAGES, 16>(ins, nin, h0, o0, o1, gh0, B, L, H,
                                                           stream);
    return launch_tma_cw<T, OP, BWD, ROWS, STAGES, 8>(ins, nin, h0, o0, o1, gh0, B, L, H, stream);
}

template <typename T, int OP, bool BWD>
int launch_simple(const T* x0, const T* x1, const T* hprev, const T* c, const T* h0, T* o0,
                  T* o1, T* gh0, int B, int L, int H, cudaStream_t stream) {
    const long long n = (long long)B * H;
    const int threads = 128;
    const long long blocks = (n + threads - 1) / threads;
    diag_scan_simple_kernel<T, OP, BWD><<<(unsigned)blocks, threads, 0, stream>>>(
        x0, x1, hprev, c, h0, o0, o1, gh0, B, L, H);
    return edb::status_from_cuda(cudaGetLastError());
}

bool tma_ok(int esize, int H, std::initializer_list<const void*> ptrs) {
    if (((long long)H * esize) % 16 != 0) return false;
    for (const void* p : ptrs)
        if (p && !edb::aligned16(p)) return false;
    return true;
}

template <typename T, int OP>
int scan_fwd(const void* x0, const void* x1, const void* h0, void* h, int B, int L, int H,
             cudaStream_t stream) {
    if (tma_ok(sizeof(T), H, {x0, x1, h0, h})) {
        const void* ins[2] = {x0, x1};
        return launch_tma<T, OP, false, 128, 3>(ins, 2, (const T*)h0, (T*)h, nullptr, nullptr, B,
                                                L, H, stream);
    }
    return launch_simple<T, OP, false>((const T*)x0, (const T*)x1, nullptr, nullptr,
                                       (const T*)h0, (T*)h, nullptr, nullptr, B, L, H, stream);
}

template <typename T, int OP>
int scan_bwd(const void* x0, const void* c, const void* h0, const void* h, const void* dy,
             void* g0, void* g1, void* gh0, int B, int L, int H, cudaStream_t stream) {
    if (tma_ok(sizeof(T), H, {x0, c, h0, h, dy, g0, g1})) {
        if (OP == OP_MINGRU) {
            const void* ins[4] = {x0, dy, h, c};
            return launch_tma<T, OP, true, 64, 3>(ins, 4, (const T*)h0, (T*)g0, (T*)g1, (T*)gh0,
                                                  B, L, H, stream);
        } else {
            const void* ins[3] = {x0, dy, h};
            return launch_tma<T, OP, true, 64, 4>(ins, 3, (const T*)h0, (T*)g0, (T*)g1, (T*)gh0,
                                                  B, L, H, stream);
        }
    }
    return launch_simple<T, OP, true>((const T*)x0, (const T*)dy, (const T*)h, (const T*)c,
                                      (const T*)h0, (T*)g0, (T*)g1, (T*)gh0, B, L, H, stream);
}

int check_common(int dtype, int B, int L, int H) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || L <= 0 || H <= 0) return EDB_ERR_BAD_SHAPE;
    if ((long long)B * L > 0x7fffffffLL) return EDB_ERR_BAD_SHAPE;
    return EDB_OK;
}

}  // namespace

extern "C" int edb_linear_scan_fwd(int dtype, const void* a, const void* b, const void* h0,
                                   void* h, int batch, int seq_len, int hidden, void* stream) {
    if (int st = check_common(dtype, batch, seq_len, hidden)) return st;
    if (!a || !b || !h) return EDB_ERR_NULL_POINTER;
    cudaStream_t s = (cudaStream_t)stream;
    return dtype == EDB_BF16
               ? scan_fwd<__nv_bfloat16, OP_LINEAR>(a, b, h0, h, batch, seq_len, hidden, s)
               : scan_fwd<float, OP_LINEAR>(a, b, h0, h, batch, seq_len, hidden, s);
}

extern "C" int edb_linear_scan_bwd(int dtype, const void* a, const void* h0, const void* h,
                                   const void* dy, void* ga, void* gb, void* gh0, int batch,
                                   int seq_len, int hidden, void* stream) {
    if (int st = check_common(dtype, batch, seq_len, hidden)) return st;
    if (!a || !h || !dy || !ga || !gb) return EDB_ERR_NULL_POINTER;
    cudaStream_t s = (cudaStream_t)stream;
    return dtype == EDB_BF16
               ? scan_bwd<__nv_bfloat16, OP_LINEAR>(a, nullptr, h0, h, dy, ga, gb, gh0, batch,
                                                     seq_len, hidden, s)
               : scan_bwd<float, OP_LINEAR>(a, nullptr, h0, h, dy, ga, gb, gh0, batch, seq_len,
                                            hidden, s);
}

extern "C" int edb_mingru_fwd(int dtype, const void* z, const void* c, const void* h0, void* h,
                              int batch, int seq_len, int hidden, void* stream) {
    if (int st = check_common(dtype, batch, seq_len, hidden)) return st;
    if (!z || !c || !h) return EDB_ERR_NULL_POINTER;
    cudaStream_t s = (cudaStream_t)stream;
    return dtype == EDB_BF16
               ? scan_fwd<__nv_bfloat16, OP_MINGRU>(z, c, h0, h, batch, seq_len, hidden, s)
               : scan_fwd<float, OP_MINGRU>(z, c, h0, h, batch, seq_len, hidden, s);
}

extern "C" int edb_native_rec_fwd(int kind, int dtype, const void* x0, const void* x1,
                                  const void* h0, void* h, int batch, int seq_len, int hidden,
                                  void* stream) {
    if (int st = check_common(dtype, batch, seq_len, hidden)) return st;
    if (!x0 || !x1 || !h) return EDB_ERR_NULL_POINTER;
    cudaStream_t s = (cudaStream_t)stream;
    const bool bf = dtype == EDB_BF16;
    switch (kind) {
        case EDB_NATIVE_ELU_GRU:
            return bf ? scan_fwd<__nv_bfloat16, OP_ELUGRU>(x0, x1, h0, h, batch, seq_len, hidden, s)
                      : scan_fwd<float, OP_ELUGRU>(x0, x1, h0, h, batch, seq_len, hidden, s);
        case EDB_NATIVE_REAL_GRU:
            return bf ? scan_fwd<__nv_bfloat16, OP_REALGRU>(x0, x1, h0, h, batch, seq_len, hidden, s)
                      : scan_fwd<float, OP_REALGRU>(x0, x1, h0, h, batch, seq_len, hidden, s);
        case EDB_NATIVE_DIAG_LINEAR:
            return bf ? scan_fwd<__nv_bfloat16, OP_DIAGLIN>(x0, x1, h0, h, batch, seq_len, hidden, s)
                      : scan_fwd<float, OP_DIAGLIN>(x0, x1, h0, h, batch, seq_len, hidden, s);
        default:
            return EDB_ERR_UNSUPPORTED;
    }
}

extern "C" int edb_mingru_bwd(int dtype, const void* z, const void* c, const void* h0,
                              const void* h, const void* dy, void* gz, void* gc, void* gh0,
                              int batch, int seq_len, int hidden, void* stream) {
    if (int st = check_common(dtype, batch, seq_len, hidden)) return st;
    if (!z || !c || !h || !dy || !gz || !gc) return EDB_ERR_NULL_POINTER;
    cudaStream_t s = (cudaStream_t)stream;
    return dtype == EDB_BF16
               ? scan_bwd<__nv_bfloat16, OP_MINGRU>(z, c, h0, h, dy, gz, gc, gh0, batch,
                                                     seq_len, hidden, s)
               : scan_bwd<float, OP_MINGRU>(z, c, h0, h, dy, gz, gc, gh0, batch, seq_len, hidden,
                                            s);
}
