/*
 * edifice_cuda_kernels.h -- the reference-named launch symbols, exported by the
 * two shim libraries
 *     edifice_b200/shim/libedifice_cuda_kernels.so       (io = f32)
 *     edifice_b200/shim/libedifice_cuda_kernels_bf16.so  (io = bf16)
 * with exactly the names and argument lists that c_src/edifice_cuda_nif.c
 * dlsym()s from priv/cuda/libedifice_cuda_kernels{,_bf16}.so
 * (edifice_cuda_nif.c:4052-4230).  Dropping these two files in place of the
 * reference's libraries switches the NIF to the B200 kernels unchanged.  Each
 * forwards to the edb_* entry point of edifice_b200.h.
 *
 * io pointers are float* in the f32 shim and __nv_bfloat16* in the bf16 shim
 * (same C ABI: a pointer).  Return: cudaError_t as int, or an edb_status.
 */
#ifndef EDIFICE_CUDA_KERNELS_H
#define EDIFICE_CUDA_KERNELS_H

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifdef EDB_SHIM_BF16
typedef unsigned short edb_io_t; /* bit pattern of __nv_bfloat16 */
#else
typedef float edb_io_t;
#endif

/* native/cuda/fused_linear_scan.cu:78-94 */
int fused_linear_scan_launch(cudaStream_t stream, const edb_io_t* a_vals, const edb_io_t* b_vals,
                             const edb_io_t* h0, edb_io_t* output, int batch, int seq_len,
                             int hidden);

/* native/cuda/fused_linear_scan_backward.cu:96-120; output_concat = [ga | gb | gh0] */
int fused_linear_scan_backward_launch(cudaStream_t stream, const edb_io_t* a_vals,
                                      const edb_io_t* h0, const edb_io_t* forward_out,
                                      const edb_io_t* grad_output, edb_io_t* output_concat,
                                      int batch, int seq_len, int hidden);

/* native/cuda/fused_mingru_scan.cu:82-101 */
int fused_mingru_scan_launch(cudaStream_t stream, const edb_io_t* gates,
                             const edb_io_t* candidates, const edb_io_t* h0, edb_io_t* output,
                             int batch, int seq_len, int hidden);

/* native/cuda/fused_mingru_scan_backward.cu:95-120; output_concat = [gz | gc | gh0] */
int fused_mingru_scan_backward_launch(cudaStream_t stream, const edb_io_t* z,
                                      const edb_io_t* candidates, const edb_io_t* h0,
                                      const edb_io_t* forward_out, const edb_io_t* grad_output,
                                      edb_io_t* output_concat, int batch, int seq_len,
                                      int hidden);

/* native/cuda/fused_native_rec_scan.cu:142-198: raw gates / candidates / a,
 * activations applied in the kernel */
int fused_elu_gru_scan_launch(cudaStream_t stream, const edb_io_t* gates,
                              const edb_io_t* candidates, const edb_io_t* h0, edb_io_t* output,
                              int batch, int seq_len, int hidden);
int fused_real_gru_scan_launch(cudaStream_t stream, const edb_io_t* gates,
                               const edb_io_t* candidates, const edb_io_t* h0, edb_io_t* output,
                               int batch, int seq_len, int hidden);
int fused_diag_linear_scan_launch(cudaStream_t stream, const edb_io_t* a_vals,
                                  const edb_io_t* b_vals, const edb_io_t* h0, edb_io_t* output,
                                  int batch, int seq_len, int hidden);

/* native/cuda/fused_elu_gru_scan_backward.cu:97-127, fused_real_gru_scan_backward.cu:94-124
 * (post-activation z, c); output_concat = [gz | gc | gh0] */
int fused_elu_gru_scan_backward_launch(cudaStream_t stream, const edb_io_t* z, const edb_io_t* c,
                                       const edb_io_t* h0, const edb_io_t* forward_out,
                                       const edb_io_t* grad_output, edb_io_t* output_concat,
                                       int batch, int seq_len, int hidden);
int fused_real_gru_scan_backward_launch(cudaStream_t stream, const edb_io_t* z,
                                        const edb_io_t* candidates, const edb_io_t* h0,
                                        const edb_io_t* forward_out, const edb_io_t* grad_output,
                                        edb_io_t* output_concat, int batch, int seq_len,
                                        int hidden);

/* native/cuda/fused_diag_linear_scan_backward.cu:90-120 (post-sigmoid a);
 * output_concat = [ga | gb | gh0] */
int fused_diag_linear_scan_backward_launch(cudaStream_t stream, const edb_io_t* a,
                                           const edb_io_t* h0, const edb_io_t* forward_out,
                                           const edb_io_t* grad_output, edb_io_t* output_concat,
                                           int batch, int seq_len, int hidden);

/* native/cuda/fused_laser_attention.cu:156-178 (equal heads; v_max [B, H, d]) */
int fused_laser_attention_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                 const edb_io_t* v, const edb_io_t* v_max, edb_io_t* output,
                                 int batch, int num_heads, int seq_len, int head_dim, int causal);

/* native/cuda/fused_laser_attention_backward.cu:372-420; output_concat = [dq | dk | dv] */
int fused_laser_attention_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                          const edb_io_t* k, const edb_io_t* v,
                                          const edb_io_t* v_max, const edb_io_t* o,
                                          const edb_io_t* grad_o, edb_io_t* output_concat,
                                          int batch, int num_heads, int seq_len, int head_dim,
                                          int causal);

/* native/cuda/fused_fox_attention.cu:162-190 (causal, equal heads; cs [B, H, L]) */
int fused_fox_attention_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                               const edb_io_t* v, const edb_io_t* cs, edb_io_t* output,
                               int batch, int num_heads, int seq_len, int head_dim);

/* native/cuda/fused_fox_attention_backward.cu:373-420;
 * output_concat = [dq | dk | dv | dcs (B*H*L)] */
int fused_fox_attention_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                        const edb_io_t* k, const edb_io_t* v,
                                        const edb_io_t* cs, const edb_io_t* o,
                                        const edb_io_t* grad_o, edb_io_t* output_concat,
                                        int batch, int num_heads, int seq_len, int head_dim);

/* native/cuda/fused_selective_scan.cu:105-124 (dt clamp [0.001, 0.1]) */
int fused_selective_scan_launch(cudaStream_t stream, const edb_io_t* x, const edb_io_t* dt,
                                const edb_io_t* A, const edb_io_t* B, const edb_io_t* C,
                                edb_io_t* out, int batch, int seq_len, int hidden, int state);

/* native/cuda/fused_selective_scan_backward.cu:198-238;
 * output_concat = [gx io (B*L*H) | gdt io (B*L*H) | gB f32 (B*L*S) | gC f32 (B*L*S)]
 * -- the byte layout the reference kernel writes (the reference NIF under-sizes
 * this buffer in bf16, c_src/edifice_cuda_nif.c:3758; size it per tensor dtype).
 * The workspace is taken stream-ordered (cudaMallocAsync / cudaFreeAsync), as
 * the reference launcher does. */
int fused_selective_scan_backward_launch(cudaStream_t stream, const edb_io_t* x,
                                         const edb_io_t* dt, const edb_io_t* A,
                                         const edb_io_t* B, const edb_io_t* C,
                                         const edb_io_t* grad_output, edb_io_t* output_concat,
                                         int batch, int seq_len, int hidden, int state_size);

/* native/cuda/fused_delta_rule_scan.cu:234-245: q, k, v, beta, output
 * [B, T, H, d] (beta per element). */
int fused_delta_net_scan_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                const edb_io_t* v, const edb_io_t* beta, edb_io_t* output,
                                int batch, int seq_len, int num_heads, int head_dim);

/* native/cuda/fused_delta_rule_scan_backward.cu:277-318;
 * output_concat = [gq | gk | gv | gbeta], each B*T*H*d io elements.  The
 * checkpoint workspace is taken stream-ordered (cudaMallocAsync / cudaFreeAsync). */
int fused_delta_rule_scan_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                          const edb_io_t* k, const edb_io_t* v,
                                          const edb_io_t* beta, const edb_io_t* forward_out,
                                          const edb_io_t* grad_output, edb_io_t* output_concat,
                                          int batch, int seq_len, int num_heads, int head_dim);

/* native/cuda/fused_delta_rule_scan.cu:247-258: GatedDeltaNet, q, k, v, beta,
 * output [B, T, H, d] (beta per element), alpha [B, T, H]. */
int fused_gated_delta_net_scan_launch(cudaStream_t stream, const edb_io_t* q,
                                      const edb_io_t* k, const edb_io_t* v, const edb_io_t* beta,
                                      const edb_io_t* alpha, edb_io_t* output, int batch,
                                      int seq_len, int num_heads, int head_dim);

/* native/cuda/fused_delta_rule_scan.cu:213-232: the delta rule, gated when
 * alpha is not NULL. */
int fused_delta_rule_scan_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                 const edb_io_t* v, const edb_io_t* beta, const edb_io_t* alpha,
                                 edb_io_t* output, int batch, int seq_len, int num_heads,
                                 int head_dim);

/* native/cuda/fused_gated_delta_net_scan_backward.cu:348-394;
 * output_concat = [gq | gk | gv | gbeta | galpha]: four B*T*H*d blocks, then
 * B*T*H io elements.  Scratch is taken stream-ordered (cudaMallocAsync /
 * cudaFreeAsync). */
int fused_gated_delta_net_scan_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                               const edb_io_t* k, const edb_io_t* v,
                                               const edb_io_t* beta, const edb_io_t* alpha,
                                               const edb_io_t* forward_out,
                                               const edb_io_t* grad_output,
                                               edb_io_t* output_concat, int batch, int seq_len,
                                               int num_heads, int head_dim);

/* native/cuda/fused_flash_attention.cu:168-191: q, k, v, output [B, H, T, d],
 * equal heads, scale 1/sqrt(d), causal 0/1. */
int fused_flash_attention_launch(cudaStream_t stream, const edb_io_t* q, const edb_io_t* k,
                                 const edb_io_t* v, edb_io_t* output, int batch, int num_heads,
                                 int seq_len, int head_dim, int causal);

/* native/cuda/fused_flash_attention_backward.cu:355-408;
 * output_concat = [dq | dk | dv], each B*H*T*d io elements.  Scratch is taken
 * stream-ordered (cudaMallocAsync / cudaFreeAsync). */
int fused_flash_attention_backward_launch(cudaStream_t stream, const edb_io_t* q,
                                          const edb_io_t* k, const edb_io_t* v,
                                          const edb_io_t* o, const edb_io_t* grad_o,
                                          edb_io_t* output_concat, int batch, int num_heads,
                                          int seq_len, int head_dim, int causal);

#ifdef __cplusplus
}
#endif

#endif /* EDIFICE_CUDA_KERNELS_H */
