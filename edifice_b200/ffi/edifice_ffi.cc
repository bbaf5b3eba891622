// edifice_ffi.cc -- XLA FFI handlers for the in-graph (EXLA custom-call) tier of
// Edifice's fused sequence-mixing path, over libedifice_b200.so.
//
// Each handler is registered under the target name the reference registers for
// the same op (native/cuda/fused_*.cu built with -DEXLA_FFI, e.g.
// fused_selective_scan.cu:185-202, fused_flash_attention.cu:257-270):
// "exla_fused_<op>_<f32|bf16>" on platform "CUDA", with the same operands and
// results in the same order, so the custom calls that Edifice.Block.run/5
// (lib/edifice/block.ex:24-49) and the FusedScan.*_custom_call functions emit
// bind to it unchanged.  Two targets have no counterpart there:
// "exla_fused_selective_scan_model[_backward]_<dtype>", the discretize_ssm
// numbers Edifice.build(:mamba) computes (lib/edifice/ssm/common.ex:402-470).
//
// Every handler forwards to the descriptor form of the C ABI
// (include/edifice_b200.h, edb_<op>_{fwd,bwd}_desc): XLA's dense row-major
// buffers become edb_tensor views, the workspace comes from XLA's scratch
// allocator, and what a backward needs but the reference's backward operands do
// not carry (the attention log-sum-exp, LASER's residual, FoX's lse, the Mamba
// dt mean and chunk states) is recomputed into scratch by the forward entry
// point, as the reference's own backward kernels recompute it.  The causal flag
// arrives, as in the reference, as a one-element tensor of the io type; reading
// it synchronises the stream (fused_flash_attention.cu:224-232 does the same).
//
// Build where XLA's FFI headers are available (they are not in this
// repository's build image, so this file is not compiled or tested here), as
// one command:
//   g++ -std=c++17 -O2 -fPIC -shared -I$XLA_INCLUDE -I$REPO/include
//       -I$CUDA_HOME/include edifice_ffi.cc -L$REPO/edifice_b200 -ledifice_b200
//       -L$CUDA_HOME/lib64 -lcudart -Wl,-rpath,$REPO/edifice_b200 -o libedifice_ffi.so
// and load libedifice_ffi.so into the EXLA process before the first custom call
// (the XLA_FFI_REGISTER_HANDLER statics register the targets at load time).

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <optional>
#include <string>

#include "edifice_b200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

// ---------------------------------------------------------------- helpers
template <ffi::DataType DT>
constexpr int edb_dtype() {
    return DT == ffi::DataType::BF16 ? EDB_BF16 : EDB_F32;
}
template <ffi::DataType DT>
constexpr size_t elem_bytes() {
    return DT == ffi::DataType::BF16 ? 2 : 4;
}

ffi::Error status(int st) {
    if (st == 0) return ffi::Error::Success();
    return ffi::Error(ffi::ErrorCode::kInternal,
                      std::string("edifice_b200: ") + edb_status_string(st));
}
ffi::Error no_scratch() {
    return ffi::Error(ffi::ErrorCode::kResourceExhausted,
                      "edifice_b200: the scratch allocator has no room for the workspace");
}
ffi::Error bad_shape(const char* what) {
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, std::string("edifice_b200: ") + what);
}

// A dense row-major view of `ndim` extents.
edb_tensor dense(void* data, int dtype, int ndim, const int64_t* dims) {
    edb_tensor t;
    std::memset(&t, 0, sizeof(t));
    t.data = data;
    t.dtype = dtype;
    t.ndim = ndim;
    long long acc = 1;
    for (int i = ndim - 1; i >= 0; --i) {
        t.shape[i] = dims[i];
        t.strides[i] = acc;
        acc *= dims[i];
    }
    return t;
}

// A buffer's extents (at most EDB_MAX_DIMS; the ABI rejects higher ranks).
template <typename B>
int dims_of(B& buf, int64_t (&dims)[EDB_MAX_DIMS]) {
    auto d = buf.dimensions();
    const int nd = (int)d.size() < EDB_MAX_DIMS ? (int)d.size() : EDB_MAX_DIMS;
    for (int i = 0; i < EDB_MAX_DIMS; ++i) dims[i] = i < nd ? d[i] : 1;
    return nd;
}

template <typename B>
edb_tensor view(B& buf, int dtype) {
    int64_t dims[EDB_MAX_DIMS];
    const int nd = dims_of(buf, dims);
    return dense(buf.untyped_data(), dtype, nd, dims);
}
template <ffi::DataType DT>
edb_tensor view(ffi::Buffer<DT>& b) {
    return view(b, edb_dtype<DT>());
}
template <ffi::DataType DT>
edb_tensor view(ffi::ResultBuffer<DT>& r) {
    return view(*r, edb_dtype<DT>());
}

// Scratch device memory for the duration of the call (256-byte aligned).
std::optional<void*> scratch_bytes(ffi::ScratchAllocator& sa, size_t n) {
    if (n == 0) return std::optional<void*>(nullptr);
    return sa.Allocate(n, 256);
}

// edb_<op>_<dir>_desc with its queried workspace.
template <typename A>
ffi::Error run(size_t (*ws_fn)(const A*), int (*fn)(const A*, void*, void*, size_t), const A& a,
               cudaStream_t s, ffi::ScratchAllocator& sa) {
    const size_t n = ws_fn(&a);
    auto ws = scratch_bytes(sa, n);
    if (!ws) return no_scratch();
    return status(fn(&a, s, *ws, n));
}

// The reference's causal flag: a one-element tensor of the io type.
template <ffi::DataType DT>
ffi::Error read_flag(cudaStream_t s, ffi::Buffer<DT>& b, int* out) {
    uint32_t raw = 0;
    cudaError_t e = cudaMemcpyAsync(&raw, b.untyped_data(), elem_bytes<DT>(),
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return status((int)e);
    float f;
    if (DT == ffi::DataType::BF16) {
        const uint32_t bits = (raw & 0xFFFFu) << 16;
        std::memcpy(&f, &bits, 4);
    } else {
        std::memcpy(&f, &raw, 4);
    }
    *out = f != 0.0f;
    return ffi::Error::Success();
}

#define EDB_ST(x)                          \
    do {                                   \
        ffi::Error e_ = (x);               \
        if (e_.failure()) return e_;       \
    } while (0)

// ---------------------------------------------------------------- diagonal scans
// exla_fused_linear_scan: (a, b, h0) -> h        fused_linear_scan.cu:100-160
template <ffi::DataType DT>
ffi::Error linear_scan(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> a,
                       ffi::Buffer<DT> b, ffi::Buffer<DT> h0, ffi::ResultBuffer<DT> h) {
    edb_linear_scan_args x{};
    x.dtype = edb_dtype<DT>();
    x.a = view(a), x.b = view(b), x.h0 = view(h0), x.h = view(h);
    return run(edb_linear_scan_fwd_desc_workspace, edb_linear_scan_fwd_desc, x, s, sa);
}

// exla_fused_linear_scan_backward: (a, h0, h, dy) -> (ga, gb, gh0)
// fused_linear_scan_backward.cu; also exla_fused_diag_linear_scan_backward
// (fused_diag_linear_scan_backward.cu: the same recurrence on a = sigmoid(x0)).
template <ffi::DataType DT>
ffi::Error linear_scan_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> a,
                           ffi::Buffer<DT> h0, ffi::Buffer<DT> h, ffi::Buffer<DT> dy,
                           ffi::ResultBuffer<DT> ga, ffi::ResultBuffer<DT> gb,
                           ffi::ResultBuffer<DT> gh0) {
    edb_linear_scan_args x{};
    x.dtype = edb_dtype<DT>();
    x.a = view(a), x.h0 = view(h0), x.h = view(h), x.dy = view(dy);
    x.ga = view(ga), x.gb = view(gb), x.gh0 = view(gh0);
    return run(edb_linear_scan_bwd_desc_workspace, edb_linear_scan_bwd_desc, x, s, sa);
}

// exla_fused_mingru_scan: (z, c, h0) -> h   (z after the sigmoid, as the
// reference's custom call passes it: fused_scan.ex:454-481)
template <ffi::DataType DT>
ffi::Error mingru(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> z, ffi::Buffer<DT> c,
                  ffi::Buffer<DT> h0, ffi::ResultBuffer<DT> h) {
    edb_mingru_args x{};
    x.dtype = edb_dtype<DT>();
    x.z = view(z), x.c = view(c), x.h0 = view(h0), x.h = view(h);
    return run(edb_mingru_fwd_desc_workspace, edb_mingru_fwd_desc, x, s, sa);
}

// exla_fused_mingru_scan_backward: (z, c, h0, h, dy) -> (gz, gc, gh0); also the
// elu_gru / real_gru backwards, which take the activated values
// (fused_elu_gru_scan_backward.cu, fused_real_gru_scan_backward.cu).
template <ffi::DataType DT>
ffi::Error mingru_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> z,
                      ffi::Buffer<DT> c, ffi::Buffer<DT> h0, ffi::Buffer<DT> h,
                      ffi::Buffer<DT> dy, ffi::ResultBuffer<DT> gz, ffi::ResultBuffer<DT> gc,
                      ffi::ResultBuffer<DT> gh0) {
    edb_mingru_args x{};
    x.dtype = edb_dtype<DT>();
    x.z = view(z), x.c = view(c), x.h0 = view(h0), x.h = view(h), x.dy = view(dy);
    x.gz = view(gz), x.gc = view(gc), x.gh0 = view(gh0);
    return run(edb_mingru_bwd_desc_workspace, edb_mingru_bwd_desc, x, s, sa);
}

// exla_fused_{elu_gru,real_gru,diag_linear}_scan: (x0, x1, h0) -> h with the
// activations applied in the kernel (fused_native_rec_scan.cu:142-198)
template <int KIND, ffi::DataType DT>
ffi::Error native_rec(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x0,
                      ffi::Buffer<DT> x1, ffi::Buffer<DT> h0, ffi::ResultBuffer<DT> h) {
    edb_native_rec_args x{};
    x.dtype = edb_dtype<DT>();
    x.kind = KIND;
    x.x0 = view(x0), x.x1 = view(x1), x.h0 = view(h0), x.h = view(h);
    return run(edb_native_rec_fwd_desc_workspace, edb_native_rec_fwd_desc, x, s, sa);
}
template <ffi::DataType DT>
ffi::Error elu_gru(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x0,
                   ffi::Buffer<DT> x1, ffi::Buffer<DT> h0, ffi::ResultBuffer<DT> h) {
    return native_rec<EDB_NATIVE_ELU_GRU, DT>(s, sa, x0, x1, h0, h);
}
template <ffi::DataType DT>
ffi::Error real_gru(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x0,
                    ffi::Buffer<DT> x1, ffi::Buffer<DT> h0, ffi::ResultBuffer<DT> h) {
    return native_rec<EDB_NATIVE_REAL_GRU, DT>(s, sa, x0, x1, h0, h);
}
template <ffi::DataType DT>
ffi::Error diag_linear(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x0,
                       ffi::Buffer<DT> x1, ffi::Buffer<DT> h0, ffi::ResultBuffer<DT> h) {
    return native_rec<EDB_NATIVE_DIAG_LINEAR, DT>(s, sa, x0, x1, h0, h);
}

// ---------------------------------------------------------------- selective scan
constexpr float kDtMin = 0.001f, kDtMax = 0.1f;  // lib/edifice/ssm/common.ex:58-63

// exla_fused_selective_scan: (x, dt, A, B, C) -> y, kernel semantics
// (fused_selective_scan.cu:41-98)
template <ffi::DataType DT>
ffi::Error selective_scan(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x,
                          ffi::Buffer<DT> dt, ffi::Buffer<DT> A, ffi::Buffer<DT> B,
                          ffi::Buffer<DT> C, ffi::ResultBuffer<DT> y) {
    edb_selective_scan_args a{};
    a.dtype = edb_dtype<DT>();
    a.semantics = EDB_SSM_KERNEL;
    a.dt_min = kDtMin, a.dt_max = kDtMax;
    a.x = view(x), a.dt = view(dt), a.A = view(A), a.B = view(B), a.C = view(C), a.y = view(y);
    return run(edb_selective_scan_fwd_desc_workspace, edb_selective_scan_fwd_desc, a, s, sa);
}

// exla_fused_selective_scan_backward: (x, dt, A, B, C, dy) -> (gx, gdt, gB f32,
// gC f32) (fused_selective_scan_backward.cu:320-339); the chunk states are
// recomputed inside the call from the workspace
template <ffi::DataType DT>
ffi::Error selective_scan_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x,
                              ffi::Buffer<DT> dt, ffi::Buffer<DT> A, ffi::Buffer<DT> B,
                              ffi::Buffer<DT> C, ffi::Buffer<DT> dy, ffi::ResultBuffer<DT> gx,
                              ffi::ResultBuffer<DT> gdt, ffi::ResultBuffer<ffi::F32> gB,
                              ffi::ResultBuffer<ffi::F32> gC) {
    edb_selective_scan_args a{};
    a.dtype = edb_dtype<DT>();
    a.semantics = EDB_SSM_KERNEL;
    a.dt_min = kDtMin, a.dt_max = kDtMax;
    a.x = view(x), a.dt = view(dt), a.A = view(A), a.B = view(B), a.C = view(C);
    a.dy = view(dy), a.gx = view(gx), a.gdt = view(gdt);
    a.gB = view(*gB, EDB_F32), a.gC = view(*gC, EDB_F32);
    return run(edb_selective_scan_bwd_desc_workspace, edb_selective_scan_bwd_desc, a, s, sa);
}

// exla_fused_selective_scan_model: (x, dt, B, C) -> y, the model semantics with
// the fixed A = -(1..N) (no counterpart in the reference's handlers)
template <ffi::DataType DT>
ffi::Error selective_scan_model(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x,
                                ffi::Buffer<DT> dt, ffi::Buffer<DT> B, ffi::Buffer<DT> C,
                                ffi::ResultBuffer<DT> y) {
    auto d = x.dimensions();
    if (d.size() != 3) return bad_shape("selective_scan_model: x must be [batch, seq, d_inner]");
    auto dtm = scratch_bytes(sa, (size_t)d[0] * d[1] * sizeof(float));
    if (!dtm) return no_scratch();
    edb_selective_scan_args a{};
    a.dtype = edb_dtype<DT>();
    a.semantics = EDB_SSM_MODEL;
    a.dt_min = kDtMin, a.dt_max = kDtMax;
    a.x = view(x), a.dt = view(dt), a.B = view(B), a.C = view(C), a.y = view(y);
    a.dt_mean = static_cast<float*>(*dtm);
    return run(edb_selective_scan_fwd_desc_workspace, edb_selective_scan_fwd_desc, a, s, sa);
}

// exla_fused_selective_scan_model_backward: (x, dt, B, C, dy) -> (gx, gdt, gB,
// gC); the forward runs first into scratch for the dt mean and chunk states
template <ffi::DataType DT>
ffi::Error selective_scan_model_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> x,
                                    ffi::Buffer<DT> dt, ffi::Buffer<DT> B, ffi::Buffer<DT> C,
                                    ffi::Buffer<DT> dy, ffi::ResultBuffer<DT> gx,
                                    ffi::ResultBuffer<DT> gdt, ffi::ResultBuffer<ffi::F32> gB,
                                    ffi::ResultBuffer<ffi::F32> gC) {
    auto d = x.dimensions();
    auto n = B.dimensions();
    if (d.size() != 3 || n.size() != 3)
        return bad_shape("selective_scan_model_backward: x, B must be rank 3");
    const int Bz = (int)d[0], L = (int)d[1], D = (int)d[2], N = (int)n[2];
    auto ysc = scratch_bytes(sa, (size_t)Bz * L * D * elem_bytes<DT>());
    auto dtm = scratch_bytes(sa, (size_t)Bz * L * sizeof(float));
    auto ck = scratch_bytes(sa, edb_selective_scan_ckpt_bytes(Bz, L, D, N));
    if (!ysc || !dtm || !ck) return no_scratch();
    edb_selective_scan_args a{};
    a.dtype = edb_dtype<DT>();
    a.semantics = EDB_SSM_MODEL;
    a.dt_min = kDtMin, a.dt_max = kDtMax;
    a.x = view(x), a.dt = view(dt), a.B = view(B), a.C = view(C);
    int64_t xd[EDB_MAX_DIMS];
    dims_of(x, xd);
    a.y = dense(*ysc, edb_dtype<DT>(), 3, xd);
    a.dt_mean = static_cast<float*>(*dtm);
    a.h_ckpt = static_cast<float*>(*ck);
    EDB_ST(run(edb_selective_scan_fwd_desc_workspace, edb_selective_scan_fwd_desc, a, s, sa));
    a.dy = view(dy), a.gx = view(gx), a.gdt = view(gdt);
    a.gB = view(*gB, EDB_F32), a.gC = view(*gC, EDB_F32);
    return run(edb_selective_scan_bwd_desc_workspace, edb_selective_scan_bwd_desc, a, s, sa);
}

// ---------------------------------------------------------------- delta rule
template <typename B>
int beta_mode(B& beta) {
    return beta.dimensions().size() == 4 ? EDB_BETA_PER_ELEMENT : EDB_BETA_PER_TOKEN;
}

// exla_fused_delta_net_scan: (q, k, v, beta) -> o   (fused_delta_rule_scan.cu:352-363)
template <ffi::DataType DT>
ffi::Error delta_net(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                     ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> beta,
                     ffi::ResultBuffer<DT> o) {
    edb_delta_rule_args a{};
    a.dtype = edb_dtype<DT>();
    a.beta_mode = beta_mode(beta);
    a.q = view(q), a.k = view(k), a.v = view(v), a.beta = view(beta), a.o = view(o);
    return run(edb_delta_rule_fwd_desc_workspace, edb_delta_rule_fwd_desc, a, s, sa);
}

// exla_fused_gated_delta_net_scan: (q, k, v, beta, alpha) -> o  (:365-382)
template <ffi::DataType DT>
ffi::Error gated_delta_net(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                           ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> beta,
                           ffi::Buffer<DT> alpha, ffi::ResultBuffer<DT> o) {
    edb_delta_rule_args a{};
    a.dtype = edb_dtype<DT>();
    a.beta_mode = beta_mode(beta);
    a.q = view(q), a.k = view(k), a.v = view(v), a.beta = view(beta), a.alpha = view(alpha);
    a.o = view(o);
    return run(edb_delta_rule_fwd_desc_workspace, edb_delta_rule_fwd_desc, a, s, sa);
}

// exla_fused_delta_rule_scan_backward: (q, k, v, beta, o, dO) -> (gq, gk, gv,
// gbeta) (fused_delta_rule_scan_backward.cu); the states are recomputed
template <ffi::DataType DT>
ffi::Error delta_rule_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                          ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> beta,
                          ffi::Buffer<DT> o, ffi::Buffer<DT> dO, ffi::ResultBuffer<DT> gq,
                          ffi::ResultBuffer<DT> gk, ffi::ResultBuffer<DT> gv,
                          ffi::ResultBuffer<DT> gbeta) {
    edb_delta_rule_args a{};
    a.dtype = edb_dtype<DT>();
    a.beta_mode = beta_mode(beta);
    a.q = view(q), a.k = view(k), a.v = view(v), a.beta = view(beta), a.o = view(o);
    a.dO = view(dO), a.gq = view(gq), a.gk = view(gk), a.gv = view(gv), a.gbeta = view(gbeta);
    return run(edb_delta_rule_bwd_desc_workspace, edb_delta_rule_bwd_desc, a, s, sa);
}

// exla_fused_gated_delta_net_scan_backward: (q, k, v, beta, alpha, o, dO) ->
// (gq, gk, gv, gbeta, galpha) (fused_gated_delta_net_scan_backward.cu)
template <ffi::DataType DT>
ffi::Error gated_delta_net_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                               ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> beta,
                               ffi::Buffer<DT> alpha, ffi::Buffer<DT> o, ffi::Buffer<DT> dO,
                               ffi::ResultBuffer<DT> gq, ffi::ResultBuffer<DT> gk,
                               ffi::ResultBuffer<DT> gv, ffi::ResultBuffer<DT> gbeta,
                               ffi::ResultBuffer<DT> galpha) {
    edb_delta_rule_args a{};
    a.dtype = edb_dtype<DT>();
    a.beta_mode = beta_mode(beta);
    a.q = view(q), a.k = view(k), a.v = view(v), a.beta = view(beta), a.alpha = view(alpha);
    a.o = view(o), a.dO = view(dO);
    a.gq = view(gq), a.gk = view(gk), a.gv = view(gv), a.gbeta = view(gbeta);
    a.galpha = view(galpha);
    return run(edb_delta_rule_bwd_desc_workspace, edb_delta_rule_bwd_desc, a, s, sa);
}

// ---------------------------------------------------------------- attention
// exla_fused_flash_attention: (q, k, v, causal[1]) -> o  (fused_flash_attention.cu:257-270);
// grouped heads when k, v carry fewer heads than q
template <ffi::DataType DT>
ffi::Error flash_attention(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                           ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> causal,
                           ffi::ResultBuffer<DT> o) {
    edb_flash_attention_args a{};
    a.dtype = edb_dtype<DT>();
    EDB_ST(read_flag(s, causal, &a.causal));
    a.q = view(q), a.k = view(k), a.v = view(v), a.o = view(o);
    return run(edb_flash_attention_fwd_desc_workspace, edb_flash_attention_fwd_desc, a, s, sa);
}

// exla_fused_flash_attention_backward: (q, k, v, o, dO, causal[1]) -> (dq, dk, dv)
// (fused_flash_attention_backward.cu:521-535); the log-sum-exp is recomputed
template <ffi::DataType DT>
ffi::Error flash_attention_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                               ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> o,
                               ffi::Buffer<DT> dO, ffi::Buffer<DT> causal,
                               ffi::ResultBuffer<DT> dq, ffi::ResultBuffer<DT> dk,
                               ffi::ResultBuffer<DT> dv) {
    edb_flash_attention_args a{};
    a.dtype = edb_dtype<DT>();
    EDB_ST(read_flag(s, causal, &a.causal));
    a.q = view(q), a.k = view(k), a.v = view(v), a.o = view(o), a.dO = view(dO);
    a.dq = view(dq), a.dk = view(dk), a.dv = view(dv);
    return run(edb_flash_attention_bwd_desc_workspace, edb_flash_attention_bwd_desc, a, s, sa);
}

// LASER's v_max arrives as [B, H, 1, d]; the ABI takes [B, H, d].
template <ffi::DataType DT>
edb_tensor vmax_view(ffi::Buffer<DT>& vmax) {
    auto d = vmax.dimensions();
    if (d.size() != 4) return view(vmax);
    const int64_t dims[3] = {d[0], d[1], d[3]};
    return dense(vmax.untyped_data(), edb_dtype<DT>(), 3, dims);
}
template <ffi::DataType DT>
size_t laser_resid(ffi::Buffer<DT>& q, ffi::Buffer<DT>& k) {
    auto dq = q.dimensions();
    auto dk = k.dimensions();
    return edb_laser_attention_resid_bytes(edb_dtype<DT>(), (int)dq[0], (int)dq[1], (int)dk[1],
                                           (int)dq[2], (int)dq[3]);
}

// exla_fused_laser_attention: (q, k, v, v_max, causal[1]) -> o
// (fused_laser_attention.cu); the residual goes to scratch
template <ffi::DataType DT>
ffi::Error laser_attention(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                           ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> vmax,
                           ffi::Buffer<DT> causal, ffi::ResultBuffer<DT> o) {
    if (q.dimensions().size() != 4 || k.dimensions().size() != 4)
        return bad_shape("laser_attention: q, k must be [batch, heads, seq, head_dim]");
    auto resid = scratch_bytes(sa, laser_resid(q, k));
    if (!resid) return no_scratch();
    edb_laser_attention_args a{};
    a.dtype = edb_dtype<DT>();
    EDB_ST(read_flag(s, causal, &a.causal));
    a.q = view(q), a.k = view(k), a.v = view(v), a.v_max = vmax_view(vmax), a.o = view(o);
    a.resid = *resid;
    return run(edb_laser_attention_fwd_desc_workspace, edb_laser_attention_fwd_desc, a, s, sa);
}

// exla_fused_laser_attention_backward: (q, k, v, v_max, o, dO, causal[1]) ->
// (dq, dk, dv) (fused_laser_attention_backward.cu); the forward runs first into
// scratch for the residual
template <ffi::DataType DT>
ffi::Error laser_attention_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                               ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> vmax,
                               ffi::Buffer<DT> o, ffi::Buffer<DT> dO, ffi::Buffer<DT> causal,
                               ffi::ResultBuffer<DT> dq, ffi::ResultBuffer<DT> dk,
                               ffi::ResultBuffer<DT> dv) {
    auto dqs = q.dimensions();
    if (dqs.size() != 4 || k.dimensions().size() != 4)
        return bad_shape("laser_attention_backward: q, k must be [batch, heads, seq, head_dim]");
    auto resid = scratch_bytes(sa, laser_resid(q, k));
    auto osc = scratch_bytes(sa, (size_t)dqs[0] * dqs[1] * dqs[2] * dqs[3] * elem_bytes<DT>());
    if (!resid || !osc) return no_scratch();
    edb_laser_attention_args a{};
    a.dtype = edb_dtype<DT>();
    EDB_ST(read_flag(s, causal, &a.causal));
    a.q = view(q), a.k = view(k), a.v = view(v), a.v_max = vmax_view(vmax);
    int64_t qd[EDB_MAX_DIMS];
    dims_of(q, qd);
    a.o = dense(*osc, edb_dtype<DT>(), 4, qd);
    a.resid = *resid;
    EDB_ST(run(edb_laser_attention_fwd_desc_workspace, edb_laser_attention_fwd_desc, a, s, sa));
    a.o = view(o), a.dO = view(dO), a.dq = view(dq), a.dk = view(dk), a.dv = view(dv);
    return run(edb_laser_attention_bwd_desc_workspace, edb_laser_attention_bwd_desc, a, s, sa);
}

// FoX takes cs and returns grad_cs in f32; the reference's operands are io-typed.
template <ffi::DataType DT>
ffi::Error cs_f32(cudaStream_t s, ffi::ScratchAllocator& sa, ffi::Buffer<DT>& cs,
                  edb_tensor* out) {
    if (DT == ffi::DataType::F32) {
        *out = view(cs, EDB_F32);
        return ffi::Error::Success();
    }
    const size_t n = cs.element_count();
    auto p = scratch_bytes(sa, n * sizeof(float));
    if (!p) return no_scratch();
    EDB_ST(status(edb_convert(EDB_BF16, cs.untyped_data(), EDB_F32, *p, n, s)));
    *out = view(cs, EDB_F32);
    out->data = *p;
    return ffi::Error::Success();
}

// exla_fused_fox_attention: (q, k, v, cs) -> o  (fused_fox_attention.cu); causal
template <ffi::DataType DT>
ffi::Error fox_attention(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                         ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> cs,
                         ffi::ResultBuffer<DT> o) {
    auto dqs = q.dimensions();
    if (dqs.size() != 4) return bad_shape("fox_attention: q must be [batch, heads, seq, head_dim]");
    auto lse = scratch_bytes(sa, (size_t)dqs[0] * dqs[1] * dqs[2] * sizeof(float));
    if (!lse) return no_scratch();
    edb_fox_attention_args a{};
    a.dtype = edb_dtype<DT>();
    EDB_ST(cs_f32(s, sa, cs, &a.cs));
    a.q = view(q), a.k = view(k), a.v = view(v), a.o = view(o);
    a.lse = static_cast<float*>(*lse);
    return run(edb_fox_attention_fwd_desc_workspace, edb_fox_attention_fwd_desc, a, s, sa);
}

// exla_fused_fox_attention_backward: (q, k, v, cs, o, dO) -> (dq, dk, dv, grad_cs)
// (fused_fox_attention_backward.cu); the forward runs first into scratch for lse
template <ffi::DataType DT>
ffi::Error fox_attention_bwd(cudaStream_t s, ffi::ScratchAllocator sa, ffi::Buffer<DT> q,
                             ffi::Buffer<DT> k, ffi::Buffer<DT> v, ffi::Buffer<DT> cs,
                             ffi::Buffer<DT> o, ffi::Buffer<DT> dO, ffi::ResultBuffer<DT> dq,
                             ffi::ResultBuffer<DT> dk, ffi::ResultBuffer<DT> dv,
                             ffi::ResultBuffer<DT> dcs) {
    auto dqs = q.dimensions();
    if (dqs.size() != 4)
        return bad_shape("fox_attention_backward: q must be [batch, heads, seq, head_dim]");
    const size_t nrow = (size_t)dqs[0] * dqs[1] * dqs[2];
    auto lse = scratch_bytes(sa, nrow * sizeof(float));
    auto osc = scratch_bytes(sa, nrow * dqs[3] * elem_bytes<DT>());
    if (!lse || !osc) return no_scratch();
    edb_fox_attention_args a{};
    a.dtype = edb_dtype<DT>();
    EDB_ST(cs_f32(s, sa, cs, &a.cs));
    a.q = view(q), a.k = view(k), a.v = view(v);
    int64_t qd[EDB_MAX_DIMS];
    dims_of(q, qd);
    a.o = dense(*osc, edb_dtype<DT>(), 4, qd);
    a.lse = static_cast<float*>(*lse);
    EDB_ST(run(edb_fox_attention_fwd_desc_workspace, edb_fox_attention_fwd_desc, a, s, sa));
    a.o = view(o), a.dO = view(dO), a.dq = view(dq), a.dk = view(dk), a.dv = view(dv);
    void* dcs_f32 = dcs->untyped_data();
    if (DT != ffi::DataType::F32) {
        auto p = scratch_bytes(sa, nrow * sizeof(float));
        if (!p) return no_scratch();
        dcs_f32 = *p;
    }
    a.dcs = view(*dcs, EDB_F32);
    a.dcs.data = dcs_f32;
    EDB_ST(run(edb_fox_attention_bwd_desc_workspace, edb_fox_attention_bwd_desc, a, s, sa));
    if (DT != ffi::DataType::F32)
        return status(edb_convert(EDB_F32, dcs_f32, EDB_BF16, dcs->untyped_data(), nrow, s));
    return ffi::Error::Success();
}

}  // namespace

// ---------------------------------------------------------------- bindings
// Operands and results in the reference's order; the scratch allocator is
// context, not an operand, so the custom calls are unchanged.
#define EDB_CTX(T) \
    ffi::Ffi::Bind().Ctx<ffi::PlatformStream<cudaStream_t>>().Ctx<ffi::ScratchAllocator>()
#define EDB_A(T) .Arg<ffi::Buffer<T>>()
#define EDB_R(T) .Ret<ffi::Buffer<T>>()

#define EDB_BIND_SCAN_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_LINEAR_BWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) EDB_R(T) EDB_R(T)
#define EDB_BIND_MINGRU_BWD(T) \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) EDB_R(T) EDB_R(T)
#define EDB_BIND_SSM_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_SSM_BWD(T)                                                                    \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) EDB_R(T)        \
        EDB_R(ffi::F32) EDB_R(ffi::F32)
#define EDB_BIND_SSM_MODEL_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_SSM_MODEL_BWD(T)                                                              \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) EDB_R(T) EDB_R(ffi::F32) \
        EDB_R(ffi::F32)
#define EDB_BIND_DELTA_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_GATED_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_DELTA_BWD(T)                                                             \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) EDB_R(T) \
        EDB_R(T) EDB_R(T)
#define EDB_BIND_GATED_BWD(T)                                                                 \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)     \
        EDB_R(T) EDB_R(T) EDB_R(T) EDB_R(T)
#define EDB_BIND_FLASH_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_FLASH_BWD(T) \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) EDB_R(T) EDB_R(T)
#define EDB_BIND_LASER_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_LASER_BWD(T)                                                             \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) \
        EDB_R(T) EDB_R(T)
#define EDB_BIND_FOX_FWD(T) EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T)
#define EDB_BIND_FOX_BWD(T)                                                                \
    EDB_CTX(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_A(T) EDB_R(T) EDB_R(T) \
        EDB_R(T) EDB_R(T)

// One symbol per (op, dtype), registered as "exla_fused_<op>_<dtype>" on CUDA.
#define EDB_HANDLERS(OP, FN, BIND)                                                          \
    XLA_FFI_DEFINE_HANDLER_SYMBOL(edb_ffi_##OP##_f32, FN<ffi::F32>, BIND(ffi::F32));         \
    XLA_FFI_DEFINE_HANDLER_SYMBOL(edb_ffi_##OP##_bf16, FN<ffi::BF16>, BIND(ffi::BF16));      \
    XLA_FFI_REGISTER_HANDLER(XLA_FFI_GetApi(), "exla_fused_" #OP "_f32", "CUDA",            \
                             edb_ffi_##OP##_f32);                                            \
    XLA_FFI_REGISTER_HANDLER(XLA_FFI_GetApi(), "exla_fused_" #OP "_bf16", "CUDA",           \
                             edb_ffi_##OP##_bf16)

EDB_HANDLERS(linear_scan, linear_scan, EDB_BIND_SCAN_FWD);
EDB_HANDLERS(linear_scan_backward, linear_scan_bwd, EDB_BIND_LINEAR_BWD);
EDB_HANDLERS(mingru_scan, mingru, EDB_BIND_SCAN_FWD);
EDB_HANDLERS(mingru_scan_backward, mingru_bwd, EDB_BIND_MINGRU_BWD);
EDB_HANDLERS(elu_gru_scan, elu_gru, EDB_BIND_SCAN_FWD);
EDB_HANDLERS(elu_gru_scan_backward, mingru_bwd, EDB_BIND_MINGRU_BWD);
EDB_HANDLERS(real_gru_scan, real_gru, EDB_BIND_SCAN_FWD);
EDB_HANDLERS(real_gru_scan_backward, mingru_bwd, EDB_BIND_MINGRU_BWD);
EDB_HANDLERS(diag_linear_scan, diag_linear, EDB_BIND_SCAN_FWD);
EDB_HANDLERS(diag_linear_scan_backward, linear_scan_bwd, EDB_BIND_LINEAR_BWD);
EDB_HANDLERS(selective_scan, selective_scan, EDB_BIND_SSM_FWD);
EDB_HANDLERS(selective_scan_backward, selective_scan_bwd, EDB_BIND_SSM_BWD);
EDB_HANDLERS(selective_scan_model, selective_scan_model, EDB_BIND_SSM_MODEL_FWD);
EDB_HANDLERS(selective_scan_model_backward, selective_scan_model_bwd, EDB_BIND_SSM_MODEL_BWD);
EDB_HANDLERS(delta_net_scan, delta_net, EDB_BIND_DELTA_FWD);
EDB_HANDLERS(gated_delta_net_scan, gated_delta_net, EDB_BIND_GATED_FWD);
EDB_HANDLERS(delta_rule_scan_backward, delta_rule_bwd, EDB_BIND_DELTA_BWD);
EDB_HANDLERS(gated_delta_net_scan_backward, gated_delta_net_bwd, EDB_BIND_GATED_BWD);
EDB_HANDLERS(flash_attention, flash_attention, EDB_BIND_FLASH_FWD);
EDB_HANDLERS(flash_attention_backward, flash_attention_bwd, EDB_BIND_FLASH_BWD);
EDB_HANDLERS(laser_attention, laser_attention, EDB_BIND_LASER_FWD);
EDB_HANDLERS(laser_attention_backward, laser_attention_bwd, EDB_BIND_LASER_BWD);
EDB_HANDLERS(fox_attention, fox_attention, EDB_BIND_FOX_FWD);
EDB_HANDLERS(fox_attention_backward, fox_attention_bwd, EDB_BIND_FOX_BWD);
