// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Re-exports the reference's own C++ CPU references from
// native/cuda/test_kernels.cu (mingru_scan_cpu :68, linear_scan_cpu :166,
// delta_net_scan_cpu :205) under unmangled C names so the parity tests can call
// them through ctypes.  Linked together with test_kernels.cu by oracle/build.py;
// nothing here computes anything itself.

void mingru_scan_cpu(const float* gates, const float* candidates, const float* h0,
                     float* output, int batch, int seq_len, int hidden);
void linear_scan_cpu(const float* a_vals, const float* b_vals, const float* h0,
                     float* output, int batch, int seq_len, int hidden);
void delta_net_scan_cpu(const float* q, const float* k, const float* v, const float* beta,
                        float* output, int batch, int seq_len, int num_heads, int head_dim);

extern "C" {

void ref_mingru_scan_cpu(const float* gates, const float* candidates, const float* h0,
                         float* output, int batch, int seq_len, int hidden) {
    mingru_scan_cpu(gates, candidates, h0, output, batch, seq_len, hidden);
}

void ref_linear_scan_cpu(const float* a_vals, const float* b_vals, const float* h0,
                         float* output, int batch, int seq_len, int hidden) {
    linear_scan_cpu(a_vals, b_vals, h0, output, batch, seq_len, hidden);
}

void ref_delta_net_scan_cpu(const float* q, const float* k, const float* v, const float* beta,
                            float* output, int batch, int seq_len, int num_heads,
                            int head_dim) {
    delta_net_scan_cpu(q, k, v, beta, output, batch, seq_len, num_heads, head_dim);
}

}  // extern "C"
