// legacy_shim.cpp -- reference-named launch symbols forwarding to libedifice_b200.
//
// Built twice by edifice_b200/build.py: without EDB_SHIM_BF16 into
// libedifice_cuda_kernels.so (f32 io) and with it into
// libedifice_cuda_kernels_bf16.so (bf16 io), the two file names the
// reference's NIF dlopen()s (c_src/edifice_cuda_nif.c:4052-4230).  The
// concatenated backward outputs keep the reference's layouts.
#include "edifice_b200.h"
#include "edifice_cuda_kernels.h"

namespace {
#ifdef EDB_SHIM_BF16
constexpr int kDtype = EDB_BF16;
#else
constexpr int kDtype = EDB_F32;
#endif
}  // namespace

extern "C" {

int fused_linear_scan_launch(cudaStream_t stream, const edb_io_t* a_vals, const edb_io_t* b_vals,
                             const edb_io_t* h0, edb_io_t* output, int batch, int seq_len,
                             int hidden) {
    return edb_linear_scan_fwd(kDtype, a_vals, b_vals, h0, output, batch, seq_len, hidden,
                               stream);
}

int fused_linear_scan_backward_launch(cudaStream_t stream, const edb_io_t* a_vals,
                                      const edb_io_t* h0, const edb_io_t* forward_out,
                                      const edb_io_t* grad_output, edb_io_t* output_concat,
                                      int batch, int seq_len, int hidden) {
    const long long bth = (long long)batch * seq_len * hidden;
    return edb_linear_scan_bwd(kDtype, a_vals, h0, forward_out, grad_output, output_concat,
                               output_concat + bth, output_concat + 2 * bth, batch, seq_len,
                               hidden, stream);
}

int fused_mingru_scan_launch(cudaStream_t stream, const edb_io_t* gates,
                             const edb_io_t* candidates, const edb_io_t* h0, edb_io_t* output,
                             int batch, int seq_len, int hidden) {
    return edb_mingru_fwd(kDtype, gates, candidates, h0, output, batch, seq_len, hidden, stream);
}

int fused_mingru_scan_backward_launch(cudaStream_t stream, const edb_io_t* z,
                                      const edb_io_t* candidates, const edb_io_t* h0,
                                      const edb_io_t* forward_out, const edb_io_t* grad_output,
                                      edb_io_t* output_concat, int batch, int seq_len,
                                      int hidden) {
    const long long bth = (long long)batch * seq_len * hidden;
    return edb_mingru_bwd(kDtype, z, candidates, h0, forward_out, grad_output, output_concat,
                          output_concat + bth, output_concat + 2 * bth, batch, seq_len, hidden,
                          stream);
}

int fused_elu_gru_scan_launch(cudaStream_t stream, const edb_io_t* gates,
                              const edb_io_t* candidates, const edb_io_t* h0, edb_io_t* output,
                              int batch, int seq_len, int hidden) {
    return edb_native_rec_fwd(EDB_NATIVE_ELU_GRU, kDtype, gates, candidates, h0, output, batch,
                              seq_len, hidden, stream);
}

int fused_real_gru_scan_launch(cudaStream_t stream, const edb_io_t* gates,
                               const edb_io_t* candidates, const edb_io_t* h0, edb_io_t* output,
                               int batch, int seq_len, int hidden) {
    return edb_native_rec_fwd(EDB_NATIVE_REAL_GRU, kDtype, gates, candidates, h0, output, batch,
                              seq_len, hidden, stream);
}

int fused_diag_linear_scan_launch(cudaStream_t stream, const edb_io_t* a_vals,
                                  const edb_io_t* b_vals, const edb_io_t* h0, edb_io_t* output,
                                  int batch, int seq_len, int hidden) {
    return edb_native_rec_fwd(EDB_NATIVE_DIAG_LINEAR, kDtype, a_vals, b_vals, h0, output, batch,
                              seq_len, hidden, stream);
}

// the three backwards are the MinGRU / linear-scan backwards on activated values
int fused_elu_gru_scan_backward_launch(cudaStream_t stream, const edb_io_t* z, const edb_io_t* c,
                                       const edb_io_t* h0, const edb_io_t* forward_out,
                                       const edb_io_t* grad_output, edb_io_t* output_concat,
                                       int batch, int seq_len, int hidden) {
    return fused_mingru_scan_backward_launch(stream, z, c, h0, forward_out, grad_output,
                                             output_concat, batch, seq_len, hidden);
}

int fused_real_gru_scan_backward_launch(cudaStream_t stream, const edb_io_t* z,
                                        const edb_io_t* candidates, const edb_io_t* h0,
                                        const edb_io_t* forward_out, const edb_io_t* grad_output,
                                        edb_io_t* output_concat, int batch, int seq_len,
                                        int hidden) {
    return fused_mingru_scan_backward_launch(stream, z, candidates, h0, forward_out, grad_output,
                                             output_concat, batch, seq_len, hidden);
}

int fused_diag_linear_scan_backward_launch(cudaStream_t stream, const edb_io_t* a,
                                           const edb_io_t* h0, const edb_io_t* forward_out,
                                           const edb_io_t* grad_output, edb_io_t* output_concat,
                                           int batch, int seq_len, int hidden) {
    return fused_linear_scan_backward_launch(stream, a, h0, forward_out, grad_output,
                                             output_concat, batch, seq_len, hidden);
}

int fused_laser_attention_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                 const edb_io_t* v, const edb_io_t* v_max, edb_io_t* output,
                                 int batch, int num_heads, int seq_len, int head_dim,
                                 int causal) {
    const size_t rb = edb_laser_attention_resid_bytes(kDtype, batch, num_heads, num_heads,
                                                      seq_len, head_dim);
    void* resid = nullptr;
    cudaError_t e = cudaMallocAsync(&resid, rb ? rb : 256, stream);
    if (e != cudaSuccess) return (int)e;
    int st = edb_laser_attention_fwd(kDtype, q, k, v, v_max, output, resid, batch, num_heads,
                                     num_heads, seq_len, head_dim, causal, 0.0f, stream);
    cudaFreeAsync(resid, stream);
    return st;
}

int fused_laser_attention_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                          const edb_io_t* k, const edb_io_t* v,
                                          const edb_io_t* v_max, const edb_io_t* o,
                                          const edb_io_t* grad_o, edb_io_t* output_concat,
                                          int batch, int num_heads, int seq_len, int head_dim,
                                          int causal) {
    (void)o;  // the residual is rebuilt by a forward pass; its output lands in dq first
    const long long n = (long long)batch * num_heads * seq_len * head_dim;
    const size_t rb = edb_laser_attention_resid_bytes(kDtype, batch, num_heads, num_heads,
                                                      seq_len, head_dim);
    const size_t wb = edb_laser_attention_bwd_workspace(kDtype, batch, num_heads, num_heads,
                                                        seq_len, head_dim);
    void* buf = nullptr;
    cudaError_t e = cudaMallocAsync(&buf, rb + wb, stream);
    if (e != cudaSuccess) return (int)e;
    int st = edb_laser_attention_fwd(kDtype, q, k, v, v_max, output_concat, buf, batch,
                                     num_heads, num_heads, seq_len, head_dim, causal, 0.0f,
                                     stream);
    if (st == 0)
        st = edb_laser_attention_bwd(kDtype, q, k, grad_o, buf, output_concat, output_concat + n,
                                     output_concat + 2 * n, batch, num_heads, num_heads, seq_len,
                                     head_dim, causal, 0.0f, static_cast<char*>(buf) + rb, wb,
                                     stream);
    cudaFreeAsync(buf, stream);
    return st;
}

int fused_fox_attention_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                               const edb_io_t* v, const edb_io_t* cs, edb_io_t* output,
                               int batch, int num_heads, int seq_len, int head_dim) {
    const size_t rows = (size_t)batch * num_heads * seq_len;
    void* buf = nullptr;  // cs as f32, then lse
    cudaError_t e = cudaMallocAsync(&buf, 2 * rows * sizeof(float), stream);
    if (e != cudaSuccess) return (int)e;
    float* cs32 = static_cast<float*>(buf);
    int st = edb_convert(kDtype, cs, EDB_F32, cs32, rows, stream);
    if (st == 0)
        st = edb_fox_attention_fwd(kDtype, q, k, v, cs32, output, cs32 + rows, batch, num_heads,
                                   num_heads, seq_len, head_dim, 0.0f, stream);
    cudaFreeAsync(buf, stream);
    return st;
}

int fused_fox_attention_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                        const edb_io_t* k, const edb_io_t* v,
                                        const edb_io_t* cs, const edb_io_t* o,
                                        const edb_io_t* grad_o, edb_io_t* output_concat,
                                        int batch, int num_heads, int seq_len, int head_dim) {
    (void)o;  // rebuilt with its lse by a forward pass (into the dq slot, then overwritten)
    const long long n = (long long)batch * num_heads * seq_len * head_dim;
    const size_t rows = (size_t)batch * num_heads * seq_len;
    const size_t wb = edb_fox_attention_bwd_workspace(kDtype, batch, num_heads, num_heads,
                                                      seq_len, head_dim);
    const size_t ob = ((size_t)n * sizeof(edb_io_t) + 255) & ~(size_t)255;
    void* buf = nullptr;  // cs f32 | lse | dcs f32 | o | workspace
    const size_t head = ((3 * rows * sizeof(float)) + 255) & ~(size_t)255;
    cudaError_t e = cudaMallocAsync(&buf, head + ob + wb, stream);
    if (e != cudaSuccess) return (int)e;
    float* cs32 = static_cast<float*>(buf);
    float* lse = cs32 + rows;
    float* dcs = lse + rows;
    edb_io_t* o2 = reinterpret_cast<edb_io_t*>(static_cast<char*>(buf) + head);
    void* ws = static_cast<char*>(buf) + head + ob;
    int st = edb_convert(kDtype, cs, EDB_F32, cs32, rows, stream);
    if (st == 0)
        st = edb_fox_attention_fwd(kDtype, q, k, v, cs32, o2, lse, batch, num_heads, num_heads,
                                   seq_len, head_dim, 0.0f, stream);
    if (st == 0)
        st = edb_fox_attention_bwd(kDtype, q, k, v, cs32, o2, grad_o, lse, output_concat,
                                   output_concat + n, output_concat + 2 * n, dcs, batch,
                                   num_heads, num_heads, seq_len, head_dim, 0.0f, ws, wb, stream);
    if (st == 0) st = edb_convert(EDB_F32, dcs, kDtype, output_concat + 3 * n, rows, stream);
    cudaFreeAsync(buf, stream);
    return st;
}

int fused_selective_scan_launch(cudaStream_t stream, const edb_io_t* x, const edb_io_t* dt,
                                const edb_io_t* A, const edb_io_t* B, const edb_io_t* C,
                                edb_io_t* out, int batch, int seq_len, int hidden, int state) {
    return edb_selective_scan_fwd(kDtype, x, dt, A, B, C, out, nullptr, batch, seq_len, hidden,
                                  state, 0.001f, 0.1f, stream);
}

int fused_selective_scan_backward_launch(cudaStream_t stream, const edb_io_t* x,
                                         const edb_io_t* dt, const edb_io_t* A,
                                         const edb_io_t* B, const edb_io_t* C,
                                         const edb_io_t* grad_output, edb_io_t* output_concat,
                                         int batch, int seq_len, int hidden, int state_size) {
    const long long bth = (long long)batch * seq_len * hidden;
    const long long bts = (long long)batch * seq_len * state_size;
    edb_io_t* gx = output_concat;
    edb_io_t* gdt = output_concat + bth;
    float* gB = reinterpret_cast<float*>(output_concat + 2 * bth);
    float* gC = gB + bts;
    const size_t wsb = edb_selective_scan_bwd_workspace(batch, seq_len, hidden, state_size, 0);
    void* ws = nullptr;
    if (wsb) {
        cudaError_t e = cudaMallocAsync(&ws, wsb, stream);
        if (e != cudaSuccess) return (int)e;
    }
    int st = edb_selective_scan_bwd(kDtype, x, dt, A, B, C, grad_output, nullptr, gx, gdt, gB, gC,
                                    batch, seq_len, hidden, state_size, 0.001f, 0.1f, ws, wsb,
                                    stream);
    if (ws) cudaFreeAsync(ws, stream);
    return st;
}

int fused_delta_net_scan_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                const edb_io_t* v, const edb_io_t* beta, edb_io_t* output,
                                int batch, int seq_len, int num_heads, int head_dim) {
    return edb_delta_rule_fwd(kDtype, q, k, v, beta, 1, output, nullptr, batch, seq_len,
                              num_heads, head_dim, nullptr, 0, stream);
}

int fused_delta_rule_scan_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                          const edb_io_t* k, const edb_io_t* v,
                                          const edb_io_t* beta, const edb_io_t* forward_out,
                                          const edb_io_t* grad_output, edb_io_t* output_concat,
                                          int batch, int seq_len, int num_heads, int head_dim) {
    (void)forward_out;  // the backward recomputes what it needs from q, k, v, beta
    const long long n = (long long)batch * seq_len * num_heads * head_dim;
    const size_t wsb =
        edb_delta_rule_bwd_workspace(kDtype, 1, batch, seq_len, num_heads, head_dim, 0);
    void* ws = nullptr;
    cudaError_t e = cudaMallocAsync(&ws, wsb, stream);
    if (e != cudaSuccess) return (int)e;
    int st = edb_delta_rule_bwd(kDtype, q, k, v, beta, 1, grad_output, nullptr, output_concat,
                                output_concat + n, output_concat + 2 * n, output_concat + 3 * n,
                                batch, seq_len, num_heads, head_dim, ws, wsb, stream);
    cudaFreeAsync(ws, stream);
    return st;
}

int fused_gated_delta_net_scan_launch(cudaStream_t stream, const edb_io_t* q,
                                      const edb_io_t* k, const edb_io_t* v, const edb_io_t* beta,
                                      const edb_io_t* alpha, edb_io_t* output, int batch,
                                      int seq_len, int num_heads, int head_dim) {
    return edb_gated_delta_net_fwd(kDtype, q, k, v, beta, 1, alpha, output, nullptr, batch,
                                   seq_len, num_heads, head_dim, stream);
}

int fused_delta_rule_scan_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                 const edb_io_t* v, const edb_io_t* beta, const edb_io_t* alpha,
                                 edb_io_t* output, int batch, int seq_len, int num_heads,
                                 int head_dim) {
    if (alpha != nullptr)
        return fused_gated_delta_net_scan_launch(stream, q, k, v, beta, alpha, output, batch,
                                                 seq_len, num_heads, head_dim);
    return fused_delta_net_scan_launch(stream, q, k, v, beta, output, batch, seq_len, num_heads,
                                       head_dim);
}

int fused_gated_delta_net_scan_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                               const edb_io_t* k, const edb_io_t* v,
                                               const edb_io_t* beta, const edb_io_t* alpha,
                                               const edb_io_t* forward_out,
                                               const edb_io_t* grad_output,
                                               edb_io_t* output_concat, int batch, int seq_len,
                                               int num_heads, int head_dim) {
    (void)forward_out;  // the backward recomputes what it needs from q, k, v, beta, alpha
    const long long n = (long long)batch * seq_len * num_heads * head_dim;
    const size_t wsb =
        edb_gated_delta_net_bwd_workspace(kDtype, 1, batch, seq_len, num_heads, head_dim, 0);
    void* ws = nullptr;
    cudaError_t e = cudaMallocAsync(&ws, wsb, stream);
    if (e != cudaSuccess) return (int)e;
    int st = edb_gated_delta_net_bwd(kDtype, q, k, v, beta, 1, alpha, grad_output, nullptr,
                                     output_concat, output_concat + n, output_concat + 2 * n,
                                     output_concat + 3 * n, output_concat + 4 * n, batch, seq_len,
                                     num_heads, head_dim, ws, wsb, stream);
    cudaFreeAsync(ws, stream);
    return st;
}

int fused_flash_attention_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                 const edb_io_t* v, edb_io_t* output, int batch, int num_heads,
                                 int seq_len, int head_dim, int causal) {
    return edb_flash_attention_fwd(kDtype, q, k, v, output, nullptr, batch, num_heads, num_heads,
                                   seq_len, head_dim, causal, 0.0f, stream);
}

int fused_flash_attention_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                          const edb_io_t* k, const edb_io_t* v,
                                          const edb_io_t* o, const edb_io_t* grad_o,
                                          edb_io_t* output_concat, int batch, int num_heads,
                                          int seq_len, int head_dim, int causal) {
    const long long n = (long long)batch * num_heads * seq_len * head_dim;
    const size_t wsb = edb_flash_attention_bwd_workspace(kDtype, batch, num_heads, num_heads,
                                                         seq_len, head_dim, 0);
    void* ws = nullptr;
    cudaError_t e = cudaMallocAsync(&ws, wsb, stream);
    if (e != cudaSuccess) return (int)e;
    int st = edb_flash_attention_bwd(kDtype, q, k, v, o, grad_o, nullptr, output_concat,
                                     output_concat + n, output_concat + 2 * n, batch, num_heads,
                                     num_heads, seq_len, head_dim, causal, 0.0f, ws, wsb, stream);
    cudaFreeAsync(ws, stream);
    return st;
}

}  // extern "C"
