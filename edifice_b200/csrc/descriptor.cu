// descriptor.cu -- the descriptor form of the C ABI (edb_<op>_{fwd,bwd}_desc):
// per-op argument structs whose tensors carry pointer, dtype, shape and element
// strides.  Each entry point validates the struct on the host, gathers every
// input that is not a dense, 16-byte-aligned row-major array into a dense copy
// inside the caller's workspace, runs the positional entry point on dense
// operands (the rest of the workspace is its scratch), and scatters each
// non-dense output back through its strides.  Dense aligned tensors are used in
// place, so a caller with contiguous buffers pays nothing for the form.
//
// The boundary this serves is the reference's in-graph tier: the XLA FFI
// handlers "exla_fused_<op>_<dtype>" (e.g. native/cuda/fused_selective_scan.cu:
// 185-202) receive buffers with dims and a layout, not bare pointers.
#include <type_traits>

#include "edb_common.cuh"

namespace {

constexpr int kMaxSlots = 16;
constexpr size_t kWsAlign = 256;

size_t align_ws(size_t x) { return (x + kWsAlign - 1) & ~(kWsAlign - 1); }

size_t elem_bytes(int dtype) { return dtype == EDB_BF16 ? 2 : 4; }

// Strides are always the tensor's real element strides: all-zero strides on a
// tensor of more than one element are a broadcast (gathered as an input,
// rejected as an output), never a shorthand for "dense".
bool dense_row_major(const edb_tensor& t) {
    long long expect = 1;
    for (int i = t.ndim - 1; i >= 0; --i) {
        if (t.shape[i] != 1 && t.strides[i] != expect) return false;
        expect *= t.shape[i];
    }
    return true;
}

// 4-D geometry of one copy: leading dimensions of extent 1 pad a lower rank.
struct Geo {
    long long shape[4];
    long long stride[4];
};

// Strided <-> dense copy of raw elements (E = 2 or 4 bytes, no conversion).
// Rows are the flattened outer three dimensions; threads walk the innermost one,
// so the dense side is written (or read) in order.
template <typename E, bool GATHER>
__global__ void __launch_bounds__(256) strided_copy_kernel(const E* __restrict__ src,
                                                           E* __restrict__ dst, Geo g) {
    const long long rows = g.shape[0] * g.shape[1] * g.shape[2];
    const long long inner = g.shape[3];
    for (long long r = blockIdx.y; r < rows; r += gridDim.y) {
        const long long i2 = r % g.shape[2], r1 = r / g.shape[2];
        const long long i1 = r1 % g.shape[1], i0 = r1 / g.shape[1];
        const long long base = i0 * g.stride[0] + i1 * g.stride[1] + i2 * g.stride[2];
        for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < inner;
             i += (long long)gridDim.x * blockDim.x) {
            const long long s = base + i * g.stride[3], d = r * inner + i;
            if (GATHER)
                dst[d] = src[s];
            else
                dst[s] = src[d];
        }
    }
}

int strided_copy(const edb_tensor& t, void* dense, bool gather, cudaStream_t st) {
    Geo g;
    const int pad = 4 - t.ndim;
    for (int i = 0; i < 4; ++i) {
        g.shape[i] = i < pad ? 1 : t.shape[i - pad];
        g.stride[i] = i < pad ? 0 : t.strides[i - pad];
    }
    const long long rows = g.shape[0] * g.shape[1] * g.shape[2];
    long long bx = (g.shape[3] + 255) / 256;
    if (bx > 1024) bx = 1024;
    const dim3 grid((unsigned)bx, (unsigned)(rows < 65535 ? rows : 65535));
    if (t.dtype == EDB_BF16) {
        using E = uint16_t;
        if (gather)
            strided_copy_kernel<E, true><<<grid, 256, 0, st>>>((const E*)t.data, (E*)dense, g);
        else
            strided_copy_kernel<E, false><<<grid, 256, 0, st>>>((const E*)dense, (E*)t.data, g);
    } else {
        using E = uint32_t;
        if (gather)
            strided_copy_kernel<E, true><<<grid, 256, 0, st>>>((const E*)t.data, (E*)dense, g);
        else
            strided_copy_kernel<E, false><<<grid, 256, 0, st>>>((const E*)dense, (E*)t.data, g);
    }
    return edb::status_from_cuda(cudaGetLastError());
}

// The tensors of one call: each is checked against the shape and dtype the op
// expects and either used in place or given a dense copy in the workspace.
class Plan {
  public:
    // Declares a tensor; returns its slot (-1 for an absent optional one).
    // The first failure sticks in status().
    int add(const edb_tensor& t, bool output, bool optional, int dtype, int ndim,
            const long long* shape) {
        if (status_) return -1;
        if (t.data == nullptr) {
            if (!optional) status_ = EDB_ERR_NULL_POINTER;
            return -1;
        }
        if (t.dtype != dtype) return fail(EDB_ERR_BAD_DTYPE);
        if (t.ndim != ndim || ndim < 1 || ndim > EDB_MAX_DIMS) return fail(EDB_ERR_BAD_SHAPE);
        for (int i = 0; i < ndim; ++i) {
            if (t.shape[i] != shape[i]) return fail(EDB_ERR_BAD_SHAPE);
            if (output && t.strides[i] == 0 && t.shape[i] > 1) return fail(EDB_ERR_BAD_SHAPE);
        }
        if (n_ == kMaxSlots) return fail(EDB_ERR_UNSUPPORTED);
        Slot& s = slots_[n_];
        s.t = &t;
        s.output = output;
        s.copy = !dense_row_major(t) || (reinterpret_cast<uintptr_t>(t.data) & 15u) != 0;
        s.offset = bytes_;
        if (s.copy) {
            long long n = 1;
            for (int i = 0; i < ndim; ++i) n *= shape[i];
            bytes_ += align_ws((size_t)n * elem_bytes(dtype));
        }
        return n_++;
    }
    int status() const { return status_; }
    size_t copy_bytes() const { return bytes_; }
    // Binds the copies to the workspace and gathers the inputs that need one.
    int gather(char* ws, cudaStream_t st) {
        for (int i = 0; i < n_; ++i) {
            Slot& s = slots_[i];
            s.ptr = s.copy ? ws + s.offset : s.t->data;
            if (s.copy && !s.output)
                if (int e = strided_copy(*s.t, s.ptr, true, st)) return e;
        }
        return EDB_OK;
    }
    int scatter(cudaStream_t st) {
        for (int i = 0; i < n_; ++i) {
            const Slot& s = slots_[i];
            if (s.copy && s.output)
                if (int e = strided_copy(*s.t, s.ptr, false, st)) return e;
        }
        return EDB_OK;
    }
    void* ptr(int slot) const { return slot < 0 ? nullptr : slots_[slot].ptr; }

  private:
    struct Slot {
        const edb_tensor* t = nullptr;
        bool output = false, copy = false;
        size_t offset = 0;
        void* ptr = nullptr;
    };
    int fail(int st) {
        status_ = st;
        return -1;
    }
    Slot slots_[kMaxSlots];
    int n_ = 0;
    int status_ = EDB_OK;
    size_t bytes_ = 0;
};

bool io_dtype(int d) { return d == EDB_F32 || d == EDB_BF16; }

// Extents of a required tensor of rank `ndim`, each in [1, 2^31).
int dims_of(const edb_tensor& t, int ndim, int* out) {
    if (t.data == nullptr) return EDB_ERR_NULL_POINTER;
    if (t.ndim != ndim) return EDB_ERR_BAD_SHAPE;
    for (int i = 0; i < ndim; ++i) {
        if (t.shape[i] < 1 || t.shape[i] > 0x7fffffffLL) return EDB_ERR_BAD_SHAPE;
        out[i] = (int)t.shape[i];
    }
    return EDB_OK;
}

// Runs one descriptor call: `prepare(plan, inner_ws)` validates and declares the
// tensors, `call(plan, scratch, scratch_bytes)` runs the positional entry point.
template <typename Prepare, typename Call>
int run(Prepare prepare, Call call, void* stream, void* workspace, size_t workspace_bytes) {
    Plan p;
    size_t inner = 0;
    if (int st = prepare(p, inner)) return st;
    const size_t need = p.copy_bytes() + inner;
    if (need > 0) {
        if (workspace == nullptr || workspace_bytes < need) return EDB_ERR_WORKSPACE_TOO_SMALL;
        if (reinterpret_cast<uintptr_t>(workspace) % kWsAlign) return EDB_ERR_MISALIGNED;
    }
    cudaStream_t st = (cudaStream_t)stream;
    char* ws = static_cast<char*>(workspace);
    if (int e = p.gather(ws, st)) return e;
    char* scratch = ws == nullptr ? nullptr : ws + p.copy_bytes();
    if (int e = call(p, inner ? (void*)scratch : nullptr, inner)) return e;
    return p.scatter(st);
}

template <typename Prepare>
size_t workspace_of(Prepare prepare) {
    Plan p;
    size_t inner = 0;
    if (prepare(p, inner)) return 0;
    return p.copy_bytes() + inner;
}

// ------------------------------------------------------------ linear / MinGRU
// The two diagonal scans share their tensor roles: x0 (a or z), x1 (b or c).
struct ScanIdx {
    int x0 = -1, x1 = -1, h0 = -1, h = -1, dy = -1, g0 = -1, g1 = -1, gh0 = -1;
    int B = 0, L = 0, H = 0;
};

template <typename Args>
int prep_scan(const Args* a, const edb_tensor& x0, const edb_tensor& x1, const edb_tensor& h0,
              const edb_tensor& h, const edb_tensor& dy, const edb_tensor& g0,
              const edb_tensor& g1, const edb_tensor& gh0, bool bwd, Plan& p, ScanIdx& ix) {
    if (!io_dtype(a->dtype)) return EDB_ERR_BAD_DTYPE;
    int d[3];
    if (int st = dims_of(x0, 3, d)) return st;
    ix.B = d[0], ix.L = d[1], ix.H = d[2];
    const long long blh[3] = {d[0], d[1], d[2]}, bh[2] = {d[0], d[2]};
    const int dt = a->dtype;
    ix.x0 = p.add(x0, false, false, dt, 3, blh);
    ix.h0 = p.add(h0, false, true, dt, 2, bh);
    if (!bwd) {
        ix.x1 = p.add(x1, false, false, dt, 3, blh);
        ix.h = p.add(h, true, false, dt, 3, blh);
    } else {
        // MinGRU's backward reads c (x1); the linear scan's does not
        ix.x1 = std::is_same<Args, edb_mingru_args>::value ? p.add(x1, false, false, dt, 3, blh)
                                                           : -1;
        ix.h = p.add(h, false, false, dt, 3, blh);
        ix.dy = p.add(dy, false, false, dt, 3, blh);
        ix.g0 = p.add(g0, true, false, dt, 3, blh);
        ix.g1 = p.add(g1, true, false, dt, 3, blh);
        ix.gh0 = p.add(gh0, true, true, dt, 2, bh);
    }
    return p.status();
}

// ------------------------------------------------------------ selective scan
struct SsmIdx {
    int x = -1, dt = -1, A = -1, B = -1, C = -1, y = -1, dy = -1, gx = -1, gdt = -1, gB = -1,
        gC = -1;
    int b = 0, L = 0, D = 0, N = 0;
};

int prep_ssm(const edb_selective_scan_args* a, bool bwd, Plan& p, SsmIdx& ix) {
    if (!a) return EDB_ERR_NULL_POINTER;
    if (!io_dtype(a->dtype)) return EDB_ERR_BAD_DTYPE;
    if (a->semantics != EDB_SSM_KERNEL && a->semantics != EDB_SSM_MODEL)
        return EDB_ERR_UNSUPPORTED;
    const bool model = a->semantics == EDB_SSM_MODEL;
    int d[3], n[3];
    if (int st = dims_of(a->x, 3, d)) return st;
    if (int st = dims_of(a->B, 3, n)) return st;
    ix.b = d[0], ix.L = d[1], ix.D = d[2], ix.N = n[2];
    if (model && a->dt_mean == nullptr) return EDB_ERR_NULL_POINTER;
    const long long bld[3] = {d[0], d[1], d[2]}, bln[3] = {d[0], d[1], n[2]},
                    dn[2] = {d[2], n[2]};
    const int dt = a->dtype;
    ix.x = p.add(a->x, false, false, dt, 3, bld);
    ix.dt = p.add(a->dt, false, false, dt, 3, bld);
    ix.A = p.add(a->A, false, model, dt, 2, dn);
    ix.B = p.add(a->B, false, false, dt, 3, bln);
    ix.C = p.add(a->C, false, false, dt, 3, bln);
    if (!bwd) {
        ix.y = p.add(a->y, true, false, dt, 3, bld);
    } else {
        ix.dy = p.add(a->dy, false, false, dt, 3, bld);
        ix.gx = p.add(a->gx, true, false, dt, 3, bld);
        ix.gdt = p.add(a->gdt, true, false, dt, 3, bld);
        ix.gB = p.add(a->gB, true, false, EDB_F32, 3, bln);
        ix.gC = p.add(a->gC, true, false, EDB_F32, 3, bln);
    }
    return p.status();
}

// ------------------------------------------------------------ delta rule
struct DeltaIdx {
    int q = -1, k = -1, v = -1, beta = -1, alpha = -1, o = -1, dO = -1, gq = -1, gk = -1,
        gv = -1, gbeta = -1, galpha = -1;
    int B = 0, L = 0, H = 0, d = 0;
    bool gated = false, bpe = false;
};

int prep_delta(const edb_delta_rule_args* a, bool bwd, Plan& p, DeltaIdx& ix) {
    if (!a) return EDB_ERR_NULL_POINTER;
    if (!io_dtype(a->dtype)) return EDB_ERR_BAD_DTYPE;
    if (a->beta_mode != EDB_BETA_PER_TOKEN && a->beta_mode != EDB_BETA_PER_ELEMENT)
        return EDB_ERR_UNSUPPORTED;
    int d[4];
    if (int st = dims_of(a->q, 4, d)) return st;
    ix.B = d[0], ix.L = d[1], ix.H = d[2], ix.d = d[3];
    ix.gated = a->alpha.data != nullptr;
    ix.bpe = a->beta_mode == EDB_BETA_PER_ELEMENT;
    const long long blhd[4] = {d[0], d[1], d[2], d[3]}, blh[3] = {d[0], d[1], d[2]};
    const int dt = a->dtype, bnd = ix.bpe ? 4 : 3;
    const long long* bsh = ix.bpe ? blhd : blh;
    ix.q = p.add(a->q, false, false, dt, 4, blhd);
    ix.k = p.add(a->k, false, false, dt, 4, blhd);
    ix.v = p.add(a->v, false, false, dt, 4, blhd);
    ix.beta = p.add(a->beta, false, false, dt, bnd, bsh);
    ix.alpha = p.add(a->alpha, false, true, dt, 3, blh);
    if (!bwd) {
        ix.o = p.add(a->o, true, false, dt, 4, blhd);
    } else {
        ix.dO = p.add(a->dO, false, false, dt, 4, blhd);
        ix.gq = p.add(a->gq, true, false, dt, 4, blhd);
        ix.gk = p.add(a->gk, true, false, dt, 4, blhd);
        ix.gv = p.add(a->gv, true, false, dt, 4, blhd);
        ix.gbeta = p.add(a->gbeta, true, false, dt, bnd, bsh);
        ix.galpha = p.add(a->galpha, true, !ix.gated, dt, 3, blh);
        if (!ix.gated && a->galpha.data != nullptr && p.status() == EDB_OK)
            return EDB_ERR_UNSUPPORTED;  // a decay gradient without a decay
    }
    return p.status();
}

// ------------------------------------------------------------ flash attention
struct AttnIdx {
    int q = -1, k = -1, v = -1, o = -1, dO = -1, dq = -1, dk = -1, dv = -1;
    int B = 0, Hq = 0, Hkv = 0, L = 0, d = 0;
};

int prep_attn(const edb_flash_attention_args* a, bool bwd, Plan& p, AttnIdx& ix) {
    if (!a) return EDB_ERR_NULL_POINTER;
    if (!io_dtype(a->dtype)) return EDB_ERR_BAD_DTYPE;
    int dq[4], dk[4];
    if (int st = dims_of(a->q, 4, dq)) return st;
    if (int st = dims_of(a->k, 4, dk)) return st;
    if (a->num_kv_heads != 0 && a->num_kv_heads != dk[1]) return EDB_ERR_BAD_SHAPE;
    ix.B = dq[0], ix.Hq = dq[1], ix.Hkv = dk[1], ix.L = dq[2], ix.d = dq[3];
    const long long qs[4] = {dq[0], dq[1], dq[2], dq[3]}, ks[4] = {dq[0], dk[1], dq[2], dq[3]};
    const int dt = a->dtype;
    ix.q = p.add(a->q, false, false, dt, 4, qs);
    ix.k = p.add(a->k, false, false, dt, 4, ks);
    ix.v = p.add(a->v, false, false, dt, 4, ks);
    if (!bwd) {
        ix.o = p.add(a->o, true, false, dt, 4, qs);
    } else {
        ix.o = p.add(a->o, false, false, dt, 4, qs);
        ix.dO = p.add(a->dO, false, false, dt, 4, qs);
        ix.dq = p.add(a->dq, true, false, dt, 4, qs);
        ix.dk = p.add(a->dk, true, false, dt, 4, ks);
        ix.dv = p.add(a->dv, true, false, dt, 4, ks);
    }
    return p.status();
}

}  // namespace

// ============================================================ entry points
// linear scan --------------------------------------------------------------
#define PREP_LIN(BWD)                                                                         \
    [&](Plan& p, size_t& inner) {                                                             \
        inner = 0;                                                                            \
        if (!args) return (int)EDB_ERR_NULL_POINTER;                                          \
        return prep_scan(args, args->a, args->b, args->h0, args->h, args->dy, args->ga,       \
                         args->gb, args->gh0, BWD, p, ix);                                    \
    }

extern "C" size_t edb_linear_scan_fwd_desc_workspace(const edb_linear_scan_args* args) {
    ScanIdx ix;
    return workspace_of(PREP_LIN(false));
}
extern "C" int edb_linear_scan_fwd_desc(const edb_linear_scan_args* args, void* stream,
                                        void* workspace, size_t ws_bytes) {
    ScanIdx ix;
    return run(PREP_LIN(false),
               [&](Plan& p, void*, size_t) {
                   return edb_linear_scan_fwd(args->dtype, p.ptr(ix.x0), p.ptr(ix.x1),
                                              p.ptr(ix.h0), p.ptr(ix.h), ix.B, ix.L, ix.H,
                                              stream);
               },
               stream, workspace, ws_bytes);
}
extern "C" size_t edb_linear_scan_bwd_desc_workspace(const edb_linear_scan_args* args) {
    ScanIdx ix;
    return workspace_of(PREP_LIN(true));
}
extern "C" int edb_linear_scan_bwd_desc(const edb_linear_scan_args* args, void* stream,
                                        void* workspace, size_t ws_bytes) {
    ScanIdx ix;
    return run(PREP_LIN(true),
               [&](Plan& p, void*, size_t) {
                   return edb_linear_scan_bwd(args->dtype, p.ptr(ix.x0), p.ptr(ix.h0),
                                              p.ptr(ix.h), p.ptr(ix.dy), p.ptr(ix.g0),
                                              p.ptr(ix.g1), p.ptr(ix.gh0), ix.B, ix.L, ix.H,
                                              stream);
               },
               stream, workspace, ws_bytes);
}

// MinGRU -------------------------------------------------------------------
#define PREP_MG(BWD)                                                                          \
    [&](Plan& p, size_t& inner) {                                                             \
        inner = 0;                                                                            \
        if (!args) return (int)EDB_ERR_NULL_POINTER;                                          \
        return prep_scan(args, args->z, args->c, args->h0, args->h, args->dy, args->gz,       \
                         args->gc, args->gh0, BWD, p, ix);                                    \
    }

extern "C" size_t edb_mingru_fwd_desc_workspace(const edb_mingru_args* args) {
    ScanIdx ix;
    return workspace_of(PREP_MG(false));
}
extern "C" int edb_mingru_fwd_desc(const edb_mingru_args* args, void* stream, void* workspace,
                                   size_t ws_bytes) {
    ScanIdx ix;
    return run(PREP_MG(false),
               [&](Plan& p, void*, size_t) {
                   return edb_mingru_fwd(args->dtype, p.ptr(ix.x0), p.ptr(ix.x1), p.ptr(ix.h0),
                                         p.ptr(ix.h), ix.B, ix.L, ix.H, stream);
               },
               stream, workspace, ws_bytes);
}
extern "C" size_t edb_mingru_bwd_desc_workspace(const edb_mingru_args* args) {
    ScanIdx ix;
    return workspace_of(PREP_MG(true));
}
extern "C" int edb_mingru_bwd_desc(const edb_mingru_args* args, void* stream, void* workspace,
                                   size_t ws_bytes) {
    ScanIdx ix;
    return run(PREP_MG(true),
               [&](Plan& p, void*, size_t) {
                   return edb_mingru_bwd(args->dtype, p.ptr(ix.x0), p.ptr(ix.x1), p.ptr(ix.h0),
                                         p.ptr(ix.h), p.ptr(ix.dy), p.ptr(ix.g0), p.ptr(ix.g1),
                                         p.ptr(ix.gh0), ix.B, ix.L, ix.H, stream);
               },
               stream, workspace, ws_bytes);
}

// selective scan -----------------------------------------------------------
#define PREP_SSM(BWD)                                                                         \
    [&](Plan& p, size_t& inner) {                                                             \
        int st = prep_ssm(args, BWD, p, ix);                                                  \
        inner = (st == EDB_OK && BWD) ? edb_selective_scan_bwd_workspace(                     \
                                            ix.b, ix.L, ix.D, ix.N, args->h_ckpt != nullptr)  \
                                      : 0;                                                    \
        return st;                                                                            \
    }

extern "C" size_t edb_selective_scan_fwd_desc_workspace(const edb_selective_scan_args* args) {
    SsmIdx ix;
    return workspace_of(PREP_SSM(false));
}
extern "C" int edb_selective_scan_fwd_desc(const edb_selective_scan_args* args, void* stream,
                                           void* workspace, size_t ws_bytes) {
    SsmIdx ix;
    return run(PREP_SSM(false),
               [&](Plan& p, void*, size_t) {
                   if (args->semantics == EDB_SSM_MODEL)
                       return edb_selective_scan_model_fwd(
                           args->dtype, p.ptr(ix.x), p.ptr(ix.dt), p.ptr(ix.A), p.ptr(ix.B),
                           p.ptr(ix.C), p.ptr(ix.y), args->dt_mean, args->h_ckpt, ix.b, ix.L,
                           ix.D, ix.N, args->dt_min, args->dt_max, stream);
                   return edb_selective_scan_fwd(args->dtype, p.ptr(ix.x), p.ptr(ix.dt),
                                                 p.ptr(ix.A), p.ptr(ix.B), p.ptr(ix.C),
                                                 p.ptr(ix.y), args->h_ckpt, ix.b, ix.L, ix.D,
                                                 ix.N, args->dt_min, args->dt_max, stream);
               },
               stream, workspace, ws_bytes);
}
extern "C" size_t edb_selective_scan_bwd_desc_workspace(const edb_selective_scan_args* args) {
    SsmIdx ix;
    return workspace_of(PREP_SSM(true));
}
extern "C" int edb_selective_scan_bwd_desc(const edb_selective_scan_args* args, void* stream,
                                           void* workspace, size_t ws_bytes) {
    SsmIdx ix;
    return run(PREP_SSM(true),
               [&](Plan& p, void* scratch, size_t scratch_bytes) {
                   if (args->semantics == EDB_SSM_MODEL)
                       return edb_selective_scan_model_bwd(
                           args->dtype, p.ptr(ix.x), p.ptr(ix.dt), p.ptr(ix.A), p.ptr(ix.B),
                           p.ptr(ix.C), p.ptr(ix.dy), args->dt_mean, args->h_ckpt, p.ptr(ix.gx),
                           p.ptr(ix.gdt), (float*)p.ptr(ix.gB), (float*)p.ptr(ix.gC), ix.b,
                           ix.L, ix.D, ix.N, args->dt_min, args->dt_max, scratch,
                           scratch_bytes, stream);
                   return edb_selective_scan_bwd(
                       args->dtype, p.ptr(ix.x), p.ptr(ix.dt), p.ptr(ix.A), p.ptr(ix.B),
                       p.ptr(ix.C), p.ptr(ix.dy), args->h_ckpt, p.ptr(ix.gx), p.ptr(ix.gdt),
                       (float*)p.ptr(ix.gB), (float*)p.ptr(ix.gC), ix.b, ix.L, ix.D, ix.N,
                       args->dt_min, args->dt_max, scratch, scratch_bytes, stream);
               },
               stream, workspace, ws_bytes);
}

// delta rule / GatedDeltaNet -----------------------------------------------
#define PREP_DELTA(BWD)                                                                       \
    [&](Plan& p, size_t& inner) {                                                             \
        int st = prep_delta(args, BWD, p, ix);                                                \
        inner = 0;                                                                            \
        if (st == EDB_OK) {                                                                   \
            const int ck = args->s_ckpt != nullptr;                                           \
            if (BWD)                                                                          \
                inner = ix.gated ? edb_gated_delta_net_bwd_workspace(args->dtype, ix.bpe,     \
                                                                     ix.B, ix.L, ix.H, ix.d,  \
                                                                     ck)                      \
                                 : edb_delta_rule_bwd_workspace(args->dtype, ix.bpe, ix.B,    \
                                                                ix.L, ix.H, ix.d, ck);        \
            else                                                                              \
                inner = ix.gated ? edb_gated_delta_net_fwd_workspace(args->dtype, ix.bpe,     \
                                                                     ix.B, ix.L, ix.H, ix.d)  \
                                 : edb_delta_rule_fwd_workspace(args->dtype, ix.bpe, ix.B,    \
                                                                ix.L, ix.H, ix.d);            \
        }                                                                                     \
        return st;                                                                            \
    }

extern "C" size_t edb_delta_rule_fwd_desc_workspace(const edb_delta_rule_args* args) {
    DeltaIdx ix;
    return workspace_of(PREP_DELTA(false));
}
extern "C" int edb_delta_rule_fwd_desc(const edb_delta_rule_args* args, void* stream,
                                       void* workspace, size_t ws_bytes) {
    DeltaIdx ix;
    return run(PREP_DELTA(false),
               [&](Plan& p, void* scratch, size_t scratch_bytes) {
                   if (ix.gated)
                       return edb_gated_delta_net_fwd_ws(
                           args->dtype, p.ptr(ix.q), p.ptr(ix.k), p.ptr(ix.v), p.ptr(ix.beta),
                           ix.bpe, p.ptr(ix.alpha), p.ptr(ix.o), args->s_ckpt, ix.B, ix.L, ix.H,
                           ix.d, scratch, scratch_bytes, stream);
                   return edb_delta_rule_fwd(args->dtype, p.ptr(ix.q), p.ptr(ix.k), p.ptr(ix.v),
                                             p.ptr(ix.beta), ix.bpe, p.ptr(ix.o), args->s_ckpt,
                                             ix.B, ix.L, ix.H, ix.d, scratch, scratch_bytes,
                                             stream);
               },
               stream, workspace, ws_bytes);
}
extern "C" size_t edb_delta_rule_bwd_desc_workspace(const edb_delta_rule_args* args) {
    DeltaIdx ix;
    return workspace_of(PREP_DELTA(true));
}
extern "C" int edb_delta_rule_bwd_desc(const edb_delta_rule_args* args, void* stream,
                                       void* workspace, size_t ws_bytes) {
    DeltaIdx ix;
    return run(PREP_DELTA(true),
               [&](Plan& p, void* scratch, size_t scratch_bytes) {
                   if (ix.gated)
                       return edb_gated_delta_net_bwd(
                           args->dtype, p.ptr(ix.q), p.ptr(ix.k), p.ptr(ix.v), p.ptr(ix.beta),
                           ix.bpe, p.ptr(ix.alpha), p.ptr(ix.dO), args->s_ckpt, p.ptr(ix.gq),
                           p.ptr(ix.gk), p.ptr(ix.gv), p.ptr(ix.gbeta), p.ptr(ix.galpha), ix.B,
                           ix.L, ix.H, ix.d, scratch, scratch_bytes, stream);
                   return edb_delta_rule_bwd(args->dtype, p.ptr(ix.q), p.ptr(ix.k), p.ptr(ix.v),
                                             p.ptr(ix.beta), ix.bpe, p.ptr(ix.dO), args->s_ckpt,
                                             p.ptr(ix.gq), p.ptr(ix.gk), p.ptr(ix.gv),
                                             p.ptr(ix.gbeta), ix.B, ix.L, ix.H, ix.d, scratch,
                                             scratch_bytes, stream);
               },
               stream, workspace, ws_bytes);
}

// flash attention ----------------------------------------------------------
#define PREP_ATTN(BWD)                                                                        \
    [&](Plan& p, size_t& inner) {                                                             \
        int st = prep_attn(args, BWD, p, ix);                                                 \
        inner = (st == EDB_OK && BWD)                                                         \
                    ? edb_flash_attention_bwd_workspace(args->dtype, ix.B, ix.Hq, ix.Hkv,     \
                                                        ix.L, ix.d, args->lse != nullptr)     \
                    : 0;                                                                      \
        return st;                                                                            \
    }

extern "C" size_t edb_flash_attention_fwd_desc_workspace(const edb_flash_attention_args* args) {
    AttnIdx ix;
    return workspace_of(PREP_ATTN(false));
}
extern "C" int edb_flash_attention_fwd_desc(const edb_flash_attention_args* args, void* stream,
                                            void* workspace, size_t ws_bytes) {
    AttnIdx ix;
    return run(PREP_ATTN(false),
               [&](Plan& p, void*, size_t) {
                   return edb_flash_attention_fwd(args->dtype, p.ptr(ix.q), p.ptr(ix.k),
                                                  p.ptr(ix.v), p.ptr(ix.o), args->lse, ix.B,
                                                  ix.Hq, ix.Hkv, ix.L, ix.d, args->causal,
                                                  args->scale, stream);
               },
               stream, workspace, ws_bytes);
}
extern "C" size_t edb_flash_attention_bwd_desc_workspace(const edb_flash_attention_args* args) {
    AttnIdx ix;
    return workspace_of(PREP_ATTN(true));
}
extern "C" int edb_flash_attention_bwd_desc(const edb_flash_attention_args* args, void* stream,
                                            void* workspace, size_t ws_bytes) {
    AttnIdx ix;
    return run(PREP_ATTN(true),
               [&](Plan& p, void* scratch, size_t scratch_bytes) {
                   return edb_flash_attention_bwd(args->dtype, p.ptr(ix.q), p.ptr(ix.k),
                                                  p.ptr(ix.v), p.ptr(ix.o), p.ptr(ix.dO),
                                                  args->lse, p.ptr(ix.dq), p.ptr(ix.dk),
                                                  p.ptr(ix.dv), ix.B, ix.Hq, ix.Hkv, ix.L, ix.d,
                                                  args->causal, args->scale, scratch,
                                                  scratch_bytes, stream);
               },
               stream, workspace, ws_bytes);
}

// native-recurrence scans (forward) ----------------------------------------
extern "C" size_t edb_native_rec_fwd_desc_workspace(const edb_native_rec_args* args) {
    ScanIdx ix;
    edb_tensor none = {};
    return workspace_of([&](Plan& p, size_t& inner) {
        inner = 0;
        if (!args) return (int)EDB_ERR_NULL_POINTER;
        return prep_scan(args, args->x0, args->x1, args->h0, args->h, none, none, none, none,
                         false, p, ix);
    });
}
extern "C" int edb_native_rec_fwd_desc(const edb_native_rec_args* args, void* stream,
                                       void* workspace, size_t ws_bytes) {
    ScanIdx ix;
    edb_tensor none = {};
    return run(
        [&](Plan& p, size_t& inner) {
            inner = 0;
            if (!args) return (int)EDB_ERR_NULL_POINTER;
            return prep_scan(args, args->x0, args->x1, args->h0, args->h, none, none, none, none,
                             false, p, ix);
        },
        [&](Plan& p, void*, size_t) {
            return edb_native_rec_fwd(args->kind, args->dtype, p.ptr(ix.x0), p.ptr(ix.x1),
                                      p.ptr(ix.h0), p.ptr(ix.h), ix.B, ix.L, ix.H, stream);
        },
        stream, workspace, ws_bytes);
}

// LASER / FoX attention ----------------------------------------------------
namespace {

// Shapes shared by the attention variants: q-like [B, Hq, L, d], kv-like
// [B, Hkv, L, d], per-row [B, Hq, L], per-kv-head [B, Hkv, d].
struct AttnShapes {
    long long qs[4], ks[4], bhl[3], bhd[3];
};

template <typename Args>
int attn_dims(const Args* a, AttnIdx& x, AttnShapes& s) {
    if (!a) return EDB_ERR_NULL_POINTER;
    if (!io_dtype(a->dtype)) return EDB_ERR_BAD_DTYPE;
    int dq[4], dk[4];
    if (int st = dims_of(a->q, 4, dq)) return st;
    if (int st = dims_of(a->k, 4, dk)) return st;
    x.B = dq[0], x.Hq = dq[1], x.Hkv = dk[1], x.L = dq[2], x.d = dq[3];
    const long long qs[4] = {dq[0], dq[1], dq[2], dq[3]}, ks[4] = {dq[0], dk[1], dq[2], dq[3]};
    const long long bhl[3] = {dq[0], dq[1], dq[2]}, bhd[3] = {dq[0], dk[1], dq[3]};
    for (int i = 0; i < 4; ++i) s.qs[i] = qs[i], s.ks[i] = ks[i];
    for (int i = 0; i < 3; ++i) s.bhl[i] = bhl[i], s.bhd[i] = bhd[i];
    return EDB_OK;
}

struct LaserIdx {
    AttnIdx a;
    int vmax = -1;
};

// fwd reads q, k, v, v_max (optional) and writes o; bwd reads q, k, dO and the
// residuals, and writes dq, dk, dv.
int prep_laser(const edb_laser_attention_args* a, bool bwd, Plan& p, LaserIdx& ix) {
    AttnShapes s;
    AttnIdx& x = ix.a;
    if (int st = attn_dims(a, x, s)) return st;
    if (a->resid == nullptr) return EDB_ERR_NULL_POINTER;
    const int dt = a->dtype;
    x.q = p.add(a->q, false, false, dt, 4, s.qs);
    x.k = p.add(a->k, false, false, dt, 4, s.ks);
    if (!bwd) {
        x.v = p.add(a->v, false, false, dt, 4, s.ks);
        ix.vmax = p.add(a->v_max, false, true, dt, 3, s.bhd);
        x.o = p.add(a->o, true, false, dt, 4, s.qs);
    } else {
        x.dO = p.add(a->dO, false, false, dt, 4, s.qs);
        x.dq = p.add(a->dq, true, false, dt, 4, s.qs);
        x.dk = p.add(a->dk, true, false, dt, 4, s.ks);
        x.dv = p.add(a->dv, true, false, dt, 4, s.ks);
    }
    return p.status();
}

struct FoxIdx {
    AttnIdx a;
    int cs = -1, dcs = -1;
};

int prep_fox(const edb_fox_attention_args* a, bool bwd, Plan& p, FoxIdx& ix) {
    AttnShapes s;
    AttnIdx& x = ix.a;
    if (int st = attn_dims(a, x, s)) return st;
    if (a->lse == nullptr) return EDB_ERR_NULL_POINTER;
    const int dt = a->dtype;
    x.q = p.add(a->q, false, false, dt, 4, s.qs);
    x.k = p.add(a->k, false, false, dt, 4, s.ks);
    x.v = p.add(a->v, false, false, dt, 4, s.ks);
    ix.cs = p.add(a->cs, false, false, EDB_F32, 3, s.bhl);
    x.o = p.add(a->o, !bwd, false, dt, 4, s.qs);
    if (bwd) {
        x.dO = p.add(a->dO, false, false, dt, 4, s.qs);
        x.dq = p.add(a->dq, true, false, dt, 4, s.qs);
        x.dk = p.add(a->dk, true, false, dt, 4, s.ks);
        x.dv = p.add(a->dv, true, false, dt, 4, s.ks);
        ix.dcs = p.add(a->dcs, true, false, EDB_F32, 3, s.bhl);
    }
    return p.status();
}

}  // namespace

#define PREP_LASER(BWD)                                                                       \
    [&](Plan& p, size_t& inner) {                                                             \
        int st = prep_laser(args, BWD, p, ix);                                                \
        inner = (st == EDB_OK && BWD)                                                         \
                    ? edb_laser_attention_bwd_workspace(args->dtype, ix.a.B, ix.a.Hq,         \
                                                        ix.a.Hkv, ix.a.L, ix.a.d)             \
                    : 0;                                                                      \
        return st;                                                                            \
    }

extern "C" size_t edb_laser_attention_fwd_desc_workspace(const edb_laser_attention_args* args) {
    LaserIdx ix;
    return workspace_of(PREP_LASER(false));
}
extern "C" int edb_laser_attention_fwd_desc(const edb_laser_attention_args* args, void* stream,
                                            void* workspace, size_t ws_bytes) {
    LaserIdx ix;
    return run(PREP_LASER(false),
               [&](Plan& p, void*, size_t) {
                   const AttnIdx& x = ix.a;
                   return edb_laser_attention_fwd(args->dtype, p.ptr(x.q), p.ptr(x.k),
                                                  p.ptr(x.v), p.ptr(ix.vmax), p.ptr(x.o),
                                                  args->resid, x.B, x.Hq, x.Hkv, x.L, x.d,
                                                  args->causal, args->scale, stream);
               },
               stream, workspace, ws_bytes);
}
extern "C" size_t edb_laser_attention_bwd_desc_workspace(const edb_laser_attention_args* args) {
    LaserIdx ix;
    return workspace_of(PREP_LASER(true));
}
extern "C" int edb_laser_attention_bwd_desc(const edb_laser_attention_args* args, void* stream,
                                            void* workspace, size_t ws_bytes) {
    LaserIdx ix;
    return run(PREP_LASER(true),
               [&](Plan& p, void* scratch, size_t scratch_bytes) {
                   const AttnIdx& x = ix.a;
                   return edb_laser_attention_bwd(args->dtype, p.ptr(x.q), p.ptr(x.k),
                                                  p.ptr(x.dO), args->resid, p.ptr(x.dq),
                                                  p.ptr(x.dk), p.ptr(x.dv), x.B, x.Hq, x.Hkv,
                                                  x.L, x.d, args->causal, args->scale, scratch,
                                                  scratch_bytes, stream);
               },
               stream, workspace, ws_bytes);
}

#define PREP_FOX(BWD)                                                                         \
    [&](Plan& p, size_t& inner) {                                                             \
        int st = prep_fox(args, BWD, p, ix);                                                  \
        inner = (st == EDB_OK && BWD)                                                         \
                    ? edb_fox_attention_bwd_workspace(args->dtype, ix.a.B, ix.a.Hq, ix.a.Hkv, \
                                                      ix.a.L, ix.a.d)                         \
                    : 0;                                                                      \
        return st;                                                                            \
    }

extern "C" size_t edb_fox_attention_fwd_desc_workspace(const edb_fox_attention_args* args) {
    FoxIdx ix;
    return workspace_of(PREP_FOX(false));
}
extern "C" int edb_fox_attention_fwd_desc(const edb_fox_attention_args* args, void* stream,
                                          void* workspace, size_t ws_bytes) {
    FoxIdx ix;
    return run(PREP_FOX(false),
               [&](Plan& p, void*, size_t) {
                   const AttnIdx& x = ix.a;
                   return edb_fox_attention_fwd(args->dtype, p.ptr(x.q), p.ptr(x.k), p.ptr(x.v),
                                                (const float*)p.ptr(ix.cs), p.ptr(x.o),
                                                args->lse, x.B, x.Hq, x.Hkv, x.L, x.d,
                                                args->scale, stream);
               },
               stream, workspace, ws_bytes);
}
extern "C" size_t edb_fox_attention_bwd_desc_workspace(const edb_fox_attention_args* args) {
    FoxIdx ix;
    return workspace_of(PREP_FOX(true));
}
extern "C" int edb_fox_attention_bwd_desc(const edb_fox_attention_args* args, void* stream,
                                          void* workspace, size_t ws_bytes) {
    FoxIdx ix;
    return run(PREP_FOX(true),
               [&](Plan& p, void* scratch, size_t scratch_bytes) {
                   const AttnIdx& x = ix.a;
                   return edb_fox_attention_bwd(args->dtype, p.ptr(x.q), p.ptr(x.k), p.ptr(x.v),
                                                (const float*)p.ptr(ix.cs), p.ptr(x.o),
                                                p.ptr(x.dO), args->lse, p.ptr(x.dq),
                                                p.ptr(x.dk), p.ptr(x.dv),
                                                (float*)p.ptr(ix.dcs), x.B, x.Hq, x.Hkv, x.L,
                                                x.d, args->scale, scratch, scratch_bytes,
                                                stream);
               },
               stream, workspace, ws_bytes);
}
