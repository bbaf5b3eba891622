/*
 * edifice_b200.h -- C ABI of libedifice_b200.so, the B200 (sm_100a) kernels for
 * Edifice's fused sequence-mixing path.
 *
 * This ABI replaces the reference's two boundaries for the path:
 *   - the per-op C launch wrappers that c_src/edifice_cuda_nif.c dlsym()s out of
 *     priv/cuda/libedifice_cuda_kernels{,_bf16}.so (edifice_cuda_nif.c:4052-4230);
 *   - the XLA FFI handlers "exla_fused_<op>_{f32,bf16}" registered by
 *     native/cuda/fused_*.cu under -DEXLA_FFI.
 * The reference-named launch symbols themselves (fused_<op>_launch with the
 * reference's exact signatures) are exported by the two shim libraries
 * declared in edifice_cuda_kernels.h; they forward to the entry points below.
 *
 * Conventions
 *   - Every tensor is a plain device pointer to a dense row-major array in the
 *     reference's layout; the caller owns every buffer, outputs included.
 *   - dtype (EDB_F32 / EDB_BF16) selects the storage type of the op's io
 *     tensors; arithmetic is f32 (recurrent state f32) in both cases.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Everything is stream-ordered; no entry point synchronises the
 *     device or allocates memory unless its comment says so.
 *   - Return value: 0 on success; a cudaError_t value (1..999) passes through
 *     unchanged; ABI validation errors are >= 1000 (edb_status).  Nothing
 *     aborts, traps or throws across this boundary.
 *   - Waits inside kernels are bounded.  A wait that gives up sets a bit in a
 *     per-device error word which edb_get_device_errors() returns.
 */
#ifndef EDIFICE_B200_H
#define EDIFICE_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    EDB_OK = 0,
    EDB_ERR_NULL_POINTER = 1000,
    EDB_ERR_BAD_SHAPE = 1001,
    EDB_ERR_BAD_DTYPE = 1002,
    EDB_ERR_MISALIGNED = 1003,
    EDB_ERR_WORKSPACE_TOO_SMALL = 1004,
    EDB_ERR_UNSUPPORTED = 1005,
    EDB_ERR_DEVICE_TIMEOUT = 1006
} edb_status;

typedef enum { EDB_F32 = 0, EDB_BF16 = 1 } edb_dtype;

/* bits of the per-device error word */
#define EDB_DEVERR_SCAN_PIPE 0x1u   /* diagonal-scan TMA pipeline wait gave up */
#define EDB_DEVERR_SSM_PIPE 0x2u    /* selective-scan pipeline wait gave up */
#define EDB_DEVERR_ATTN_PIPE 0x4u   /* attention pipeline wait gave up */
#define EDB_DEVERR_DELTA_PIPE 0x8u  /* delta-rule pipeline wait gave up */

/* Library version string, e.g. "edifice_b200 0.1 sm_100a". */
const char* edb_version(void);

/* Human-readable text for a status returned by any entry point. */
const char* edb_status_string(int status);

/* Read (and, if clear != 0, reset) the current device's error word.
 * Synchronises the current device.  Returns 0 or a cudaError_t. */
int edb_get_device_errors(unsigned int* flags_out, int clear);

/* Wall-clock limit of the waits of the diagonal-scan TMA pipeline (linear scan,
 * MinGRU and the native-recurrence scans), read at each launch.  limit_ns < 0
 * restores the default (2 s); 0 means a wait that finds its copy not yet landed
 * gives up at once -- that is how a test makes the pipeline give up on purpose.
 * A CTA that gives up sets EDB_DEVERR_SCAN_PIPE, writes no outputs from that
 * tile on, waits (2 s at most) for the copies it has in flight, and exits.  Process-wide;
 * returns 0.  No counterpart in the reference (its kernels have no waits). */
int edb_set_wait_limit_ns(long long limit_ns);

/* ------------------------------------------------------------------------
 * Diagonal linear recurrence  h_t = a_t * h_{t-1} + b_t   (h_{-1} = h0)
 * a, b, h: [batch, seq_len, hidden]; h0: [batch, hidden] or NULL (= zeros).
 * Replaces fused_linear_scan_launch (native/cuda/fused_linear_scan.cu:78-94)
 * and the "exla_fused_linear_scan_<dtype>" FFI handler (:100-160); Nx
 * semantics of lib/edifice/cuda/fused_scan.ex:4429-4444 / :869-882.
 * ---------------------------------------------------------------------- */
int edb_linear_scan_fwd(int dtype, const void* a, const void* b, const void* h0, void* h,
                        int batch, int seq_len, int hidden, void* stream);

/* Backward of the above given dY = dL/dh:
 *   g = dY_t + acc;  ga_t = g * h_{t-1};  gb_t = g;  acc = g * a_t;  gh0 = acc.
 * h is the forward output; gh0 may be NULL.
 * Replaces fused_linear_scan_backward_launch
 * (native/cuda/fused_linear_scan_backward.cu:96-120; fused_scan.ex:884-916). */
int edb_linear_scan_bwd(int dtype, const void* a, const void* h0, const void* h, const void* dy,
                        void* ga, void* gb, void* gh0, int batch, int seq_len, int hidden,
                        void* stream);

/* ------------------------------------------------------------------------
 * MinGRU  h_t = (1 - z_t) h_{t-1} + z_t c_t  with z already sigmoided.
 * Replaces fused_mingru_scan_launch (native/cuda/fused_mingru_scan.cu:82-101);
 * Nx semantics fused_scan.ex:516-528 / lib/edifice/recurrent/min_gru.ex:305-326.
 * ---------------------------------------------------------------------- */
int edb_mingru_fwd(int dtype, const void* z, const void* c, const void* h0, void* h,
                   int batch, int seq_len, int hidden, void* stream);

/* Backward: g = dY_t + acc; gz_t = g (c_t - h_{t-1}); gc_t = g z_t; acc = g (1 - z_t).
 * The sigmoid chain rule (fused_scan.ex:477-479) stays with the caller.
 * Replaces fused_mingru_scan_backward_launch
 * (native/cuda/fused_mingru_scan_backward.cu:95-120; fused_scan.ex:548-581). */
int edb_mingru_bwd(int dtype, const void* z, const void* c, const void* h0, const void* h,
                   const void* dy, void* gz, void* gc, void* gh0, int batch, int seq_len,
                   int hidden, void* stream);

/* ------------------------------------------------------------------------
 * Native-recurrence scans (lib/edifice/recurrent/native_recurrence.ex:125-230),
 * forward, activations applied to the raw inputs inside the kernel:
 *   EDB_NATIVE_ELU_GRU:    z = sigmoid(x0), c = 1 + elu(x1), h = (1 - z) h + z c
 *   EDB_NATIVE_REAL_GRU:   z = sigmoid(x0), h = (1 - z) h + z x1
 *   EDB_NATIVE_DIAG_LINEAR: h = sigmoid(x0) h + x1
 * x0, x1, h: [batch, seq_len, hidden]; h0: [batch, hidden] or NULL (zeros).
 * Replaces fused_{elu_gru,real_gru,diag_linear}_scan_launch
 * (native/cuda/fused_native_rec_scan.cu:142-198).  Their backwards
 * (fused_{elu_gru,real_gru}_scan_backward.cu, fused_diag_linear_scan_backward.cu;
 * fused_scan.ex:941-1023) take the activated values and are edb_mingru_bwd
 * (z, c) and edb_linear_scan_bwd (a = sigmoid(x0)).
 * ---------------------------------------------------------------------- */
enum { EDB_NATIVE_ELU_GRU = 0, EDB_NATIVE_REAL_GRU = 1, EDB_NATIVE_DIAG_LINEAR = 2 };

int edb_native_rec_fwd(int kind, int dtype, const void* x0, const void* x1, const void* h0,
                       void* h, int batch, int seq_len, int hidden, void* stream);

/* ------------------------------------------------------------------------
 * Forward + backward of the linear scan / MinGRU over HOST tensors.
 * a, b (z, c), dy, and the outputs h, ga, gb (gz, gc): [batch, seq_len, hidden]
 * in host memory; h0 / gh0: [batch, hidden] host or NULL (h0 = NULL: zeros;
 * gh0 = NULL: not returned).  Batch rows stream through a ring of device slots
 * in `workspace` (edb_scan_train_host_workspace() bytes, 256-byte aligned) so
 * that host->device copies, the kernels above and device->host copies of
 * successive row chunks overlap.  Host buffers should be page-locked
 * (cudaHostAlloc / cudaHostRegister) for the copies to overlap.  Stream-ordered:
 * the results are on the host once `stream` has reached this point; after an
 * error status no copy into or out of the host buffers is left pending once
 * `stream` has reached this point either.
 * Results are those of edb_<op>_fwd followed by edb_<op>_bwd on the whole batch.
 * Replaces the host-side round trip a caller with host-resident Nx tensors makes
 * around fused_linear_scan_launch / fused_mingru_scan_launch (and their
 * backward launches, native/cuda/fused_linear_scan{,_backward}.cu,
 * fused_mingru_scan{,_backward}.cu); the reference has no single entry point
 * for it.
 * ---------------------------------------------------------------------- */
size_t edb_scan_train_host_workspace(int dtype, int batch, int seq_len, int hidden);

int edb_linear_scan_train_host(int dtype, const void* a, const void* b, const void* h0,
                               const void* dy, void* h, void* ga, void* gb, void* gh0, int batch,
                               int seq_len, int hidden, void* workspace, size_t workspace_bytes,
                               void* stream);

int edb_mingru_train_host(int dtype, const void* z, const void* c, const void* h0, const void* dy,
                          void* h, void* gz, void* gc, void* gh0, int batch, int seq_len,
                          int hidden, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Mamba selective scan, kernel semantics (given A, per-channel clamped dt):
 *   dtc = clip(dt, dt_min, dt_max);  h_n = exp(dtc A[d,n]) h_n + dtc B[b,t,n] x;
 *   y = sum_n C[b,t,n] h_n   (h_{-1} = 0).
 * x, dt, y: [batch, seq_len, d_inner]; A: [d_inner, d_state];
 * B, C: [batch, seq_len, d_state]; all in `dtype`.  d_state <= 16.
 * The reference uses dt_min = 0.001, dt_max = 0.1.
 * h_ckpt (optional, f32, edb_selective_scan_ckpt_bytes() bytes, 16-byte
 * aligned): the forward also writes the state at the start of every chunk, so
 * the backward can skip recomputing them.
 * Replaces fused_selective_scan_launch (native/cuda/fused_selective_scan.cu:105-124)
 * and "exla_fused_selective_scan_<dtype>"; Nx semantics
 * test/edifice/cuda/backward_kernels_test.exs:1563-1586.
 * ---------------------------------------------------------------------- */
size_t edb_selective_scan_ckpt_bytes(int batch, int seq_len, int d_inner, int d_state);

int edb_selective_scan_fwd(int dtype, const void* x, const void* dt, const void* A, const void* B,
                           const void* C, void* y, float* h_ckpt, int batch, int seq_len,
                           int d_inner, int d_state, float dt_min, float dt_max, void* stream);

/* Workspace bytes edb_selective_scan_bwd needs (have_ckpt: a forward h_ckpt
 * will be passed). */
size_t edb_selective_scan_bwd_workspace(int batch, int seq_len, int d_inner, int d_state,
                                        int have_ckpt);

/* Backward given dY: gx, gdt in `dtype`; gB, gC f32 [batch, seq_len, d_state]
 * (sums over d_inner, reduced deterministically).  A gets no gradient and gdt
 * is 0 where dt lies outside [dt_min, dt_max], as in
 * lib/edifice/cuda/fused_scan.ex:1453-1531.  The caller provides the workspace
 * (16-byte aligned).  Replaces fused_selective_scan_backward_launch
 * (native/cuda/fused_selective_scan_backward.cu:198-238), whose [B,D,L,N]
 * f32 workspace and atomics are not used. */
int edb_selective_scan_bwd(int dtype, const void* x, const void* dt, const void* A, const void* B,
                           const void* C, const void* dy, const float* h_ckpt, void* gx, void* gdt,
                           float* gB, float* gC, int batch, int seq_len, int d_inner, int d_state,
                           float dt_min, float dt_max, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Forward (with chunk-start states) + backward of the selective scan over HOST
 * tensors, kernel semantics as above: x, dt, dy and the outputs y, gx, gdt
 * [batch, seq_len, d_inner] and B, C [batch, seq_len, d_state] in `dtype`, gB,
 * gC f32 [batch, seq_len, d_state], A [d_inner, d_state] in `dtype`, all in host
 * memory (page-locked for the copies to overlap).  Batch rows stream through a
 * ring of device slots in `workspace`
 * (edb_selective_scan_train_host_workspace() bytes, 256-byte aligned): the
 * host->device copies of one row chunk, the kernels of the previous one and the
 * device->host copies of the one before run at once.  Results equal
 * edb_selective_scan_fwd + edb_selective_scan_bwd on the whole batch.
 * Stream-ordered: the results are on the host once `stream` has reached this
 * point, also after an error status (no copy is left pending).  Replaces the
 * host-side round trip a caller with host-resident Nx tensors makes around
 * fused_selective_scan_launch and fused_selective_scan_backward_launch
 * (native/cuda/fused_selective_scan.cu:105-124, fused_selective_scan_backward.cu:
 * 198-238); the reference has no single entry point for it. */
size_t edb_selective_scan_train_host_workspace(int dtype, int batch, int seq_len, int d_inner,
                                               int d_state);

int edb_selective_scan_train_host(int dtype, const void* x, const void* dt, const void* A,
                                  const void* B, const void* C, const void* dy, void* y, void* gx,
                                  void* gdt, float* gB, float* gC, int batch, int seq_len,
                                  int d_inner, int d_state, float dt_min, float dt_max,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Mamba selective scan, MODEL semantics (what Edifice.build(:mamba) computes:
 * lib/edifice/ssm/common.ex:402-470 discretize_ssm + scan + output, reached
 * through selective_scan_fallback :661-670 and mamba.ex:183-213):
 *   dtc = clip(dt, dt_min, dt_max);  m_t = mean over d_inner of dtc;
 *   h_n = exp(dtc A[d,n]) h_n + m_t B[b,t,n] x;  y = sum_n C[b,t,n] h_n.
 * A = NULL is the model's fixed diagonal A[d,n] = -(n+1) (common.ex:409); a
 * non-NULL A [d_inner, d_state] is used as given.  dt_mean ([batch, seq_len]
 * f32) receives m; the backward reads it back.  h_ckpt as in
 * edb_selective_scan_fwd.
 * ---------------------------------------------------------------------- */
int edb_selective_scan_model_fwd(int dtype, const void* x, const void* dt, const void* A,
                                 const void* B, const void* C, void* y, float* dt_mean,
                                 float* h_ckpt, int batch, int seq_len, int d_inner, int d_state,
                                 float dt_min, float dt_max, void* stream);

/* Backward of the model semantics (the gradient Nx's autodiff takes through
 * common.ex:402-515): gx, gdt in `dtype`, gB, gC f32; A gets no gradient; gdt
 * is 0 where dt lies outside [dt_min, dt_max] and includes the term through the
 * channel mean m.  dt_mean: the forward's.  Workspace:
 * edb_selective_scan_bwd_workspace() bytes, 16-byte aligned. */
int edb_selective_scan_model_bwd(int dtype, const void* x, const void* dt, const void* A,
                                 const void* B, const void* C, const void* dy,
                                 const float* dt_mean, const float* h_ckpt, void* gx, void* gdt,
                                 float* gB, float* gC, int batch, int seq_len, int d_inner,
                                 int d_state, float dt_min, float dt_max, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Forward + backward of the model semantics for host-resident tensors, as
 * edb_selective_scan_train_host (A may be NULL: the fixed -(n+1) diagonal; the
 * dt means stay on the device). */
size_t edb_selective_scan_model_train_host_workspace(int dtype, int batch, int seq_len,
                                                     int d_inner, int d_state);

int edb_selective_scan_model_train_host(int dtype, const void* x, const void* dt, const void* A,
                                        const void* B, const void* C, const void* dy, void* y,
                                        void* gx, void* gdt, float* gB, float* gC, int batch,
                                        int seq_len, int d_inner, int d_state, float dt_min,
                                        float dt_max, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* ------------------------------------------------------------------------
 * Scaled-dot-product attention, causal or full, with grouped KV heads (GQA).
 *   O = softmax(Q K^T * scale [+ -inf above the diagonal if causal]) V
 * q, o: [batch, q_heads, seq_len, head_dim]; k, v: [batch, kv_heads, seq_len,
 * head_dim]; q head h reads kv head h / (q_heads / kv_heads).  head_dim <= 128
 * (bf16 with head_dim 64/128 runs on tcgen05 tensor cores).  scale <= 0 means
 * 1/sqrt(head_dim).  lse (optional, f32 [batch, q_heads, seq_len]): natural-log
 * row log-sum-exp of the scaled scores, for the backward.
 * Replaces fused_flash_attention_launch (native/cuda/fused_flash_attention.cu:
 * 168-191; equal heads only there) and "exla_fused_flash_attention_<dtype>";
 * Nx semantics lib/edifice/cuda/fused_scan.ex:3476-3508.
 * ---------------------------------------------------------------------- */
int edb_flash_attention_fwd(int dtype, const void* q, const void* k, const void* v, void* o,
                            float* lse, int batch, int q_heads, int kv_heads, int seq_len,
                            int head_dim, int causal, float scale, void* stream);

/* Workspace bytes edb_flash_attention_bwd needs (have_lse: the forward's lse
 * will be passed). */
size_t edb_flash_attention_bwd_workspace(int dtype, int batch, int q_heads, int kv_heads,
                                         int seq_len, int head_dim, int have_lse);

/* Backward given o (forward output) and dO: dq [B,Hq,L,d], dk/dv [B,Hkv,L,d]
 * in `dtype` (dk, dv of a kv head sum over its query heads).  lse may be NULL
 * (recomputed).  Caller-provided workspace, 16-byte aligned.
 * Replaces fused_flash_attention_backward_launch
 * (native/cuda/fused_flash_attention_backward.cu:355-408, which cudaMallocs and
 * cudaFrees its scratch synchronously on every call); Nx semantics
 * lib/edifice/cuda/fused_scan.ex:3527-3574. */
int edb_flash_attention_bwd(int dtype, const void* q, const void* k, const void* v, const void* o,
                            const void* dO, const float* lse, void* dq, void* dk, void* dv,
                            int batch, int q_heads, int kv_heads, int seq_len, int head_dim,
                            int causal, float scale, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Forward + backward of flash attention for HOST-resident q, k, v, dO (page-
 * locked for the copies to overlap): returns o, dq, dk, dv in host memory.
 * (batch, kv head) units stream through a ring of device slots in `workspace`
 * (edb_flash_attention_train_host_workspace() bytes, 256-byte aligned): the
 * host->device copies of one chunk of units, the kernels of the previous one and
 * the device->host copies of the one before run at once.  Results equal
 * edb_flash_attention_fwd + edb_flash_attention_bwd on the whole problem.
 * Stream-ordered as edb_selective_scan_train_host.  The reference has no single
 * entry point for it: a caller with host-resident Nx tensors makes the round trip
 * around fused_flash_attention_launch / _backward_launch
 * (native/cuda/fused_flash_attention.cu:168-191, fused_flash_attention_backward.cu:
 * 355-408). */
size_t edb_flash_attention_train_host_workspace(int dtype, int batch, int q_heads,
                                                int kv_heads, int seq_len, int head_dim);

int edb_flash_attention_train_host(int dtype, const void* q, const void* k, const void* v,
                                   const void* dO, void* o, void* dq, void* dk, void* dv,
                                   int batch, int q_heads, int kv_heads, int seq_len,
                                   int head_dim, int causal, float scale, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * LASER attention (attention over exp(V)):
 *   A = softmax(Q K^T scale (+ causal mask)) exp(V - v_max);  O = log(max(A, 1e-7)) + v_max
 * q, o [B, Hq, L, d]; k, v [B, Hkv, L, d] (Hq a multiple of Hkv, grouped heads);
 * v_max [B, Hkv, d] in `dtype` (the reference's argument: the max over the sequence
 * of v), or NULL to have it computed.  scale <= 0 means 1/sqrt(d).  resid
 * (edb_laser_attention_resid_bytes(), 256-byte aligned) receives what the backward
 * reads.  The contractions run the flash-attention kernels above on exp(V - v_max).
 * Replaces fused_laser_attention_launch (native/cuda/fused_laser_attention.cu:156-178);
 * Nx semantics lib/edifice/cuda/fused_scan.ex:3593-3611, 3667-3703.
 * ---------------------------------------------------------------------- */
size_t edb_laser_attention_resid_bytes(int dtype, int batch, int q_heads, int kv_heads,
                                       int seq_len, int head_dim);

int edb_laser_attention_fwd(int dtype, const void* q, const void* k, const void* v,
                            const void* v_max, void* o, void* resid, int batch, int q_heads,
                            int kv_heads, int seq_len, int head_dim, int causal, float scale,
                            void* stream);

size_t edb_laser_attention_bwd_workspace(int dtype, int batch, int q_heads, int kv_heads,
                                         int seq_len, int head_dim);

/* Backward from the forward's resid and dO: dq [B,Hq,L,d], dk/dv [B,Hkv,L,d]; v_max
 * gets no gradient (the reference holds it constant).  Workspace 256-byte aligned.
 * Replaces fused_laser_attention_backward_launch
 * (native/cuda/fused_laser_attention_backward.cu:372-420); fused_scan.ex:3723-3766. */
int edb_laser_attention_bwd(int dtype, const void* q, const void* k, const void* dO,
                            const void* resid, void* dq, void* dk, void* dv, int batch,
                            int q_heads, int kv_heads, int seq_len, int head_dim, int causal,
                            float scale, void* workspace, size_t workspace_bytes, void* stream);

/* Forward + backward of LASER attention for host-resident q, k, v, dO, as
 * edb_flash_attention_train_host (v_max computed per unit, the residual kept on the
 * device): returns o, dq, dk, dv in host memory. */
size_t edb_laser_attention_train_host_workspace(int dtype, int batch, int q_heads,
                                                int kv_heads, int seq_len, int head_dim);

int edb_laser_attention_train_host(int dtype, const void* q, const void* k, const void* v,
                                   const void* dO, void* o, void* dq, void* dk, void* dv,
                                   int batch, int q_heads, int kv_heads, int seq_len,
                                   int head_dim, int causal, float scale, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * FoX attention (forgetting attention), always causal:
 *   S_ij = q_i.k_j scale + cs_i - cs_j (j <= i);  O = softmax(S) V
 * cs [B, Hq, L] f32: the cumulative log forget gates, cumsum(log(sigmoid(f))).
 * q, o [B, Hq, L, d]; k, v [B, Hkv, L, d] (grouped heads).  lse [B, Hq, L] f32
 * (required; the backward reads it) is the row log-sum-exp without the row's own
 * cs_i, which cancels in the softmax.  scale <= 0 means 1/sqrt(d).  tcgen05 kernels
 * for bf16, head_dim 64/128, L % 4 == 0; SIMT kernels otherwise.
 * Replaces fused_fox_attention_launch (native/cuda/fused_fox_attention.cu:162-190);
 * Nx semantics lib/edifice/cuda/fused_scan.ex:3796-3912.
 * ---------------------------------------------------------------------- */
int edb_fox_attention_fwd(int dtype, const void* q, const void* k, const void* v,
                          const float* cs, void* o, float* lse, int batch, int q_heads,
                          int kv_heads, int seq_len, int head_dim, float scale, void* stream);

size_t edb_fox_attention_bwd_workspace(int dtype, int batch, int q_heads, int kv_heads,
                                       int seq_len, int head_dim);

/* Backward: dq [B,Hq,L,d], dk/dv [B,Hkv,L,d] in `dtype`, dcs [B,Hq,L] f32 =
 * rowsum(dS) - colsum(dS) of the unscaled score gradient (the row sums vanish: only
 * the key side is computed).  o and lse are the forward's.  Workspace 16-byte aligned.
 * Replaces fused_fox_attention_backward_launch
 * (native/cuda/fused_fox_attention_backward.cu:373-420); fused_scan.ex:3914-3984. */
int edb_fox_attention_bwd(int dtype, const void* q, const void* k, const void* v,
                          const float* cs, const void* o, const void* dO, const float* lse,
                          void* dq, void* dk, void* dv, float* dcs, int batch, int q_heads,
                          int kv_heads, int seq_len, int head_dim, float scale, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Forward + backward of FoX attention for host-resident q, k, v, cs (f32
 * [B, Hq, L]) and dO, as edb_flash_attention_train_host: returns o, dq, dk, dv and
 * dcs (f32) in host memory. */
size_t edb_fox_attention_train_host_workspace(int dtype, int batch, int q_heads, int kv_heads,
                                              int seq_len, int head_dim);

int edb_fox_attention_train_host(int dtype, const void* q, const void* k, const void* v,
                                 const float* cs, const void* dO, void* o, void* dq, void* dk,
                                 void* dv, float* dcs, int batch, int q_heads, int kv_heads,
                                 int seq_len, int head_dim, float scale, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Element-wise storage conversion of n values (EDB_F32 <-> EDB_BF16, or a copy);
 * the shims use it for the reference's io-typed cs arguments. */
int edb_convert(int src_dtype, const void* src, int dst_dtype, void* dst, size_t n, void* stream);

/* ------------------------------------------------------------------------
 * DeltaNet delta rule.  Per (batch, head), S_0 = 0:
 *   r = S_{t-1} k_t;  S_t = S_{t-1} + (beta_t (.) (v_t - r)) k_t^T;  o_t = S_t q_t
 * q, k, v, o: [batch, seq_len, heads, head_dim] (k L2-normalised by the
 * caller); beta: [batch, seq_len, heads, head_dim] when beta_per_element
 * (Edifice.build(:delta_net)'s form, lib/edifice/recurrent/delta_net.ex:285-297),
 * else [batch, seq_len, heads] (one gate per token and head).  head_dim <= 128.
 * bf16 io with one beta per token and head_dim 128 runs the chunked
 * tensor-core form (WY representation over 64-token chunks, tcgen05 TF32
 * products, f32 state); every other case runs the token recurrence.
 * s_ckpt (optional, f32, edb_delta_rule_ckpt_bytes() bytes): residuals the
 * forward leaves for edb_delta_rule_bwd of the same dtype, beta form and shape.
 * Token recurrence: S ([head_dim][head_dim], value index first) at the start
 * of every 16-token piece and the final S, [batch][heads][npieces + 1][d][d].
 * Chunked form: S^T (key index first) at the start of every 64-token chunk
 * and the final one, [batch * heads][nchunks + 1][d][d], followed by the
 * per-chunk errors U~ = U0 - W S_0^T, [batch * heads][nchunks][64][d].
 * Replaces fused_delta_net_scan_launch / fused_delta_rule_scan_launch with
 * alpha = NULL (native/cuda/fused_delta_rule_scan.cu:213-258); Nx semantics
 * lib/edifice/cuda/fused_scan.ex:2212-2236.
 * ---------------------------------------------------------------------- */
size_t edb_delta_rule_ckpt_bytes(int dtype, int beta_per_element, int batch, int seq_len,
                                 int heads, int head_dim);

/* Workspace bytes edb_delta_rule_fwd needs (0 when the token recurrence serves
 * the call). */
size_t edb_delta_rule_fwd_workspace(int dtype, int beta_per_element, int batch, int seq_len,
                                    int heads, int head_dim);

int edb_delta_rule_fwd(int dtype, const void* q, const void* k, const void* v, const void* beta,
                       int beta_per_element, void* o, float* s_ckpt, int batch, int seq_len,
                       int heads, int head_dim, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Workspace bytes edb_delta_rule_bwd needs; have_ckpt: the forward's s_ckpt
 * will be passed. */
size_t edb_delta_rule_bwd_workspace(int dtype, int beta_per_element, int batch, int seq_len,
                                    int heads, int head_dim, int have_ckpt);

/* Backward given dO: gq, gk, gv (shape of q) and gbeta (shape of beta), in
 * `dtype`.  The key gradient is the exact one (S_{t-1}^T (beta (.) dS k) for the
 * path through the retrieval), as in native/cuda/fused_delta_rule_scan_backward.cu;
 * lib/edifice/cuda/fused_scan.ex:1318-1319 scales that term by beta over the key
 * index, which agrees only for a per-token beta.  Replaces
 * fused_delta_rule_scan_backward_launch
 * (native/cuda/fused_delta_rule_scan_backward.cu:277-318). */
int edb_delta_rule_bwd(int dtype, const void* q, const void* k, const void* v, const void* beta,
                       int beta_per_element, const void* dO, const float* s_ckpt, void* gq,
                       void* gk, void* gv, void* gbeta, int batch, int seq_len, int heads,
                       int head_dim, void* workspace, size_t workspace_bytes, void* stream);

/* ----------------------------------------------------------------------
 * GatedDeltaNet: per token, S_d = alpha_t S_{t-1}; r = S_d k_t;
 * S_t = S_d + (beta_t (.) (v_t - r)) k_t^T; o_t = S_t q_t (S_0 = 0).
 * q, k, v, o, beta as edb_delta_rule_fwd; alpha: [batch, seq_len, heads]
 * (one decay per token and head, Edifice.build(:gated_delta_net)'s form,
 * lib/edifice/recurrent/gated_delta_net.ex:389-394).  head_dim <= 128.
 * bf16 with one beta per (token, head) and head_dim 128 takes the chunked
 * tensor-core form (64-token chunks, the decay folded into the chunk products);
 * every other case the token recurrence.  s_ckpt (optional, f32,
 * edb_gated_delta_net_ckpt_bytes() bytes) follows the path as for
 * edb_delta_rule_fwd: token recurrence, S at the start of every 16-token piece
 * and the final S, [batch][heads][npieces + 1][d][d]; chunked form, S^T at the
 * start of every 64-token chunk and the final one, followed by the per-chunk
 * errors U~.
 * Replaces fused_gated_delta_net_scan_launch / fused_delta_rule_scan_launch
 * with alpha (native/cuda/fused_delta_rule_scan.cu:213-258); Nx semantics
 * lib/edifice/cuda/fused_scan.ex:2256-2284.
 * ---------------------------------------------------------------------- */
size_t edb_gated_delta_net_ckpt_bytes(int dtype, int beta_per_element, int batch, int seq_len,
                                      int heads, int head_dim);

/* Workspace bytes edb_gated_delta_net_fwd_ws needs (0 for the token recurrence). */
size_t edb_gated_delta_net_fwd_workspace(int dtype, int beta_per_element, int batch,
                                         int seq_len, int heads, int head_dim);

/* The forward with a caller-owned workspace (16-byte aligned, at least
 * edb_gated_delta_net_fwd_workspace() bytes): no allocation inside. */
int edb_gated_delta_net_fwd_ws(int dtype, const void* q, const void* k, const void* v,
                               const void* beta, int beta_per_element, const void* alpha, void* o,
                               float* s_ckpt, int batch, int seq_len, int heads, int head_dim,
                               void* workspace, size_t workspace_bytes, void* stream);

/* The same forward without a workspace argument: the chunked form takes its
 * scratch stream-ordered (cudaMallocAsync / cudaFreeAsync on `stream`). */
int edb_gated_delta_net_fwd(int dtype, const void* q, const void* k, const void* v,
                            const void* beta, int beta_per_element, const void* alpha, void* o,
                            float* s_ckpt, int batch, int seq_len, int heads, int head_dim,
                            void* stream);

/* Workspace bytes edb_gated_delta_net_bwd needs (the token recurrence: a buffer
 * of one chunk's 64 states per (batch, head); the chunked form: its per-chunk
 * scratch; plus the residuals when have_ckpt == 0). */
size_t edb_gated_delta_net_bwd_workspace(int dtype, int beta_per_element, int batch,
                                         int seq_len, int heads, int head_dim, int have_ckpt);

/* Backward given dO: gq, gk, gv (shape of q), gbeta (shape of beta), galpha
 * (shape of alpha), in `dtype`.  The key gradient is the exact one
 * (-S_d^T (beta (.) dS k) through the retrieval); lib/edifice/cuda/
 * fused_scan.ex:1405-1407 scales S_d^T dS k by beta over the key index, which
 * agrees only for a per-token beta.  dalpha_t = <dS_t - (beta (.) dS_t k_t) k_t^T,
 * S_{t-1}>.  Replaces fused_gated_delta_net_scan_backward_launch
 * (native/cuda/fused_gated_delta_net_scan_backward.cu:348-394); Nx semantics
 * lib/edifice/cuda/fused_scan.ex:1347-1431. */
int edb_gated_delta_net_bwd(int dtype, const void* q, const void* k, const void* v,
                            const void* beta, int beta_per_element, const void* alpha,
                            const void* dO, const float* s_ckpt, void* gq, void* gk, void* gv,
                            void* gbeta, void* galpha, int batch, int seq_len, int heads,
                            int head_dim, void* workspace, size_t workspace_bytes, void* stream);

/* Forward + backward of the delta rule / GatedDeltaNet for host-resident q, k, v,
 * beta (, alpha) and dO (page-locked for the copies to overlap): returns o, gq, gk,
 * gv, gbeta (, galpha) in host memory.  Batch rows stream through a ring of device
 * slots in `workspace` (edb_{delta_rule,gated_delta_net}_train_host_workspace()
 * bytes, 256-byte aligned) as in edb_selective_scan_train_host; each slot runs its
 * chunk's forward (with residual) and backward on a stream of its own, so the
 * chunks' serial recurrences overlap.  Results equal the device entry points on the
 * whole batch.  The reference has no single entry point for it (a host-resident Nx
 * caller round-trips around fused_delta_rule_scan_launch / _backward_launch,
 * native/cuda/fused_delta_rule_scan.cu:213-258, fused_delta_rule_scan_backward.cu:
 * 277-318). */
size_t edb_delta_rule_train_host_workspace(int dtype, int beta_per_element, int batch,
                                           int seq_len, int heads, int head_dim);

int edb_delta_rule_train_host(int dtype, const void* q, const void* k, const void* v,
                              const void* beta, int beta_per_element, const void* dO, void* o,
                              void* gq, void* gk, void* gv, void* gbeta, int batch, int seq_len,
                              int heads, int head_dim, void* workspace, size_t workspace_bytes,
                              void* stream);

size_t edb_gated_delta_net_train_host_workspace(int dtype, int beta_per_element, int batch,
                                                int seq_len, int heads, int head_dim);

int edb_gated_delta_net_train_host(int dtype, const void* q, const void* k, const void* v,
                                   const void* beta, int beta_per_element, const void* alpha,
                                   const void* dO, void* o, void* gq, void* gk, void* gv,
                                   void* gbeta, void* galpha, int batch, int seq_len, int heads,
                                   int head_dim, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* Capacity of the library's built-in scratch array used by
 * edb_selective_scan_bwd_noalloc (16 MiB; every GPU that loads the library
 * holds it until the process exits). */
#define EDB_SSM_NOALLOC_SCRATCH_BYTES (16u << 20)

/* Same backward as edb_selective_scan_bwd, for callers that must not allocate
 * device memory -- above all an XLA/EXLA custom-call handler: XLA reserves most
 * of the GPU for its own allocator up front, so a cudaMalloc made from inside
 * the handler can fail for lack of memory, and XLA hands these handlers no
 * scratch buffer.  This entry point allocates nothing: its scratch is a
 * fixed-size array inside the library (EDB_SSM_NOALLOC_SCRATCH_BYTES).  The
 * caller still passes every input and output.
 *   - Problems whose workspace (edb_selective_scan_bwd_workspace) exceeds the
 *     array are rejected with EDB_ERR_WORKSPACE_TOO_SMALL before any GPU work.
 *   - The first call on a device looks up the array's device address, with
 *     that device current, and caches it together with the unique id of the
 *     CUDA context it was found in; after a cudaDeviceReset (a new context)
 *     the next call looks it up again.  Make the first call in each context
 *     before any stream capture.
 *   - All calls share the one array per device and it keeps the last call's
 *     contents (every byte this backward reads is written first, so nothing
 *     needs clearing); calls that overlap on the GPU -- different streams, or
 *     different host threads on one device -- race on it and must be ordered
 *     by the caller.
 * No counterpart in the reference. */
int edb_selective_scan_bwd_noalloc(int dtype, const void* x, const void* dt, const void* A,
                                   const void* B, const void* C, const void* dy,
                                   const float* h_ckpt, void* gx, void* gdt, float* gB, float* gC,
                                   int batch, int seq_len, int d_inner, int d_state, float dt_min,
                                   float dt_max, void* stream);

/* ========================================================================
 * Descriptor form of the ABI.  One argument struct per op carries every tensor
 * as an edb_tensor (device pointer, dtype, shape, element strides) next to the
 * op's flags, and each direction has a workspace query and an entry point:
 *   size_t edb_<op>_{fwd,bwd}_desc_workspace(const edb_<op>_args* args);
 *   int    edb_<op>_{fwd,bwd}_desc(const edb_<op>_args* args, void* stream,
 *                                  void* workspace, size_t workspace_bytes);
 * The entry points compute what the positional entry points above compute.
 *   - Strides are the tensor's real element strides (a dense row-major
 *     [B, L, H] tensor has strides {L*H, H, 1}); a zero stride on a dimension
 *     of extent > 1 is a broadcast, even when every stride is zero.
 *   - A tensor is used in place when it is dense row-major and 16-byte
 *     aligned.  Any other input (a transposed or sliced view, a broadcast with
 *     stride 0, a negative stride, an unaligned pointer) is first gathered
 *     into a dense copy inside the workspace; any
 *     other output is computed into a dense copy and scattered back through
 *     its strides.  Outputs may not have a zero stride on a dimension of
 *     extent > 1, and outputs must not overlap inputs.
 *   - The workspace query covers those copies plus the op's own scratch; it
 *     returns 0 when no workspace is needed or the arguments are invalid (the
 *     entry point then returns the reason).  A non-empty workspace must be
 *     256-byte aligned.
 *   - Residuals the backward reads back (lse, dt_mean, checkpoints) are plain
 *     dense f32 buffers, as in the positional entry points.
 *   - Validation (null, dtype, shape, stride, workspace size) happens on the
 *     host before any GPU work; the codes are the edb_status values.
 * This is the in-graph boundary the EXLA custom-call handlers
 * ("exla_fused_<op>_<dtype>", e.g. native/cuda/fused_selective_scan.cu:185-202)
 * bind: an XLA FFI buffer's dims and layout map onto edb_tensor directly.
 * ---------------------------------------------------------------------- */
#define EDB_MAX_DIMS 4

typedef struct {
    void* data;                      /* device pointer; NULL = absent (optional tensors) */
    int dtype;                       /* EDB_F32 / EDB_BF16 */
    int ndim;                        /* 1..EDB_MAX_DIMS */
    long long shape[EDB_MAX_DIMS];   /* extents, outermost first */
    long long strides[EDB_MAX_DIMS]; /* in elements (real strides; 0 = broadcast) */
} edb_tensor;

/* Linear scan (edb_linear_scan_fwd / _bwd).  io tensors in `dtype`:
 * a, b, h, dy, ga, gb [batch, seq_len, hidden]; h0, gh0 [batch, hidden],
 * optional.  fwd reads a, b, h0 and writes h; bwd reads a, h0, h, dy and writes
 * ga, gb, gh0. */
typedef struct {
    int dtype;
    edb_tensor a, b, h0, h;
    edb_tensor dy, ga, gb, gh0;
} edb_linear_scan_args;

/* MinGRU (edb_mingru_fwd / _bwd): z (sigmoided), c as a, b above. */
typedef struct {
    int dtype;
    edb_tensor z, c, h0, h;
    edb_tensor dy, gz, gc, gh0;
} edb_mingru_args;

/* Selective scan.  semantics EDB_SSM_KERNEL: edb_selective_scan_fwd / _bwd
 * (A required); EDB_SSM_MODEL: edb_selective_scan_model_fwd / _bwd (A optional,
 * dt_mean required).  x, dt, y, dy, gx, gdt [batch, seq_len, d_inner] and
 * B, C [batch, seq_len, d_state], A [d_inner, d_state] in `dtype`; gB, gC
 * [batch, seq_len, d_state] f32.  dt_mean: dense f32 [batch, seq_len];
 * h_ckpt: optional, edb_selective_scan_ckpt_bytes() bytes. */
enum { EDB_SSM_KERNEL = 0, EDB_SSM_MODEL = 1 };
typedef struct {
    int dtype;
    int semantics;
    float dt_min, dt_max;
    edb_tensor x, dt, A, B, C, y;
    float* dt_mean;
    float* h_ckpt;
    edb_tensor dy, gx, gdt, gB, gC;
} edb_selective_scan_args;

/* Delta rule: alpha absent = DeltaNet (edb_delta_rule_fwd / _bwd), alpha
 * present = GatedDeltaNet (edb_gated_delta_net_fwd / _bwd).  q, k, v, o, dO,
 * gq, gk, gv [batch, seq_len, heads, head_dim]; beta, gbeta [batch, seq_len,
 * heads] (EDB_BETA_PER_TOKEN) or [batch, seq_len, heads, head_dim]
 * (EDB_BETA_PER_ELEMENT); alpha, galpha [batch, seq_len, heads]; all in
 * `dtype`.  s_ckpt: optional, the positional entry points' checkpoint bytes. */
enum { EDB_BETA_PER_TOKEN = 0, EDB_BETA_PER_ELEMENT = 1 };
typedef struct {
    int dtype;
    int beta_mode;
    edb_tensor q, k, v, beta, alpha, o;
    float* s_ckpt;
    edb_tensor dO, gq, gk, gv, gbeta, galpha;
} edb_delta_rule_args;

/* Flash attention (edb_flash_attention_fwd / _bwd).  q, o, dO, dq [batch,
 * q_heads, seq_len, head_dim]; k, v, dk, dv [batch, kv_heads, seq_len,
 * head_dim]; all in `dtype`.  num_kv_heads: 0 or k's second extent.  lse:
 * optional dense f32 [batch, q_heads, seq_len] (written by fwd, read by bwd). */
typedef struct {
    int dtype;
    int causal;
    int num_kv_heads;
    float scale;
    edb_tensor q, k, v, o;
    float* lse;
    edb_tensor dO, dq, dk, dv;
} edb_flash_attention_args;

/* Native-recurrence scans (edb_native_rec_fwd), forward only (their backwards
 * are the linear-scan / MinGRU backwards on the activated values): kind is
 * EDB_NATIVE_*; x0, x1, h [batch, seq_len, hidden], h0 [batch, hidden] optional. */
typedef struct {
    int dtype;
    int kind;
    edb_tensor x0, x1, h0, h;
} edb_native_rec_args;

/* LASER attention (edb_laser_attention_fwd / _bwd): q, o, dO, dq as flash;
 * k, v, dk, dv [batch, kv_heads, seq_len, head_dim]; v_max [batch, kv_heads,
 * head_dim] optional; resid: dense, edb_laser_attention_resid_bytes() bytes,
 * 256-byte aligned, written by fwd and read by bwd. */
typedef struct {
    int dtype;
    int causal;
    float scale;
    edb_tensor q, k, v, v_max, o;
    void* resid;
    edb_tensor dO, dq, dk, dv;
} edb_laser_attention_args;

/* FoX attention (edb_fox_attention_fwd / _bwd), causal: q, k, v, o, dO, dq,
 * dk, dv as flash; cs, dcs [batch, q_heads, seq_len] f32; lse: dense f32
 * [batch, q_heads, seq_len], required (written by fwd, read by bwd). */
typedef struct {
    int dtype;
    float scale;
    edb_tensor q, k, v, cs, o;
    float* lse;
    edb_tensor dO, dq, dk, dv, dcs;
} edb_fox_attention_args;

size_t edb_linear_scan_fwd_desc_workspace(const edb_linear_scan_args* args);
int edb_linear_scan_fwd_desc(const edb_linear_scan_args* args, void* stream, void* workspace,
                             size_t workspace_bytes);
size_t edb_linear_scan_bwd_desc_workspace(const edb_linear_scan_args* args);
int edb_linear_scan_bwd_desc(const edb_linear_scan_args* args, void* stream, void* workspace,
                             size_t workspace_bytes);

size_t edb_mingru_fwd_desc_workspace(const edb_mingru_args* args);
int edb_mingru_fwd_desc(const edb_mingru_args* args, void* stream, void* workspace,
                        size_t workspace_bytes);
size_t edb_mingru_bwd_desc_workspace(const edb_mingru_args* args);
int edb_mingru_bwd_desc(const edb_mingru_args* args, void* stream, void* workspace,
                        size_t workspace_bytes);

size_t edb_selective_scan_fwd_desc_workspace(const edb_selective_scan_args* args);
int edb_selective_scan_fwd_desc(const edb_selective_scan_args* args, void* stream,
                                void* workspace, size_t workspace_bytes);
size_t edb_selective_scan_bwd_desc_workspace(const edb_selective_scan_args* args);
int edb_selective_scan_bwd_desc(const edb_selective_scan_args* args, void* stream,
                                void* workspace, size_t workspace_bytes);

size_t edb_delta_rule_fwd_desc_workspace(const edb_delta_rule_args* args);
int edb_delta_rule_fwd_desc(const edb_delta_rule_args* args, void* stream, void* workspace,
                            size_t workspace_bytes);
size_t edb_delta_rule_bwd_desc_workspace(const edb_delta_rule_args* args);
int edb_delta_rule_bwd_desc(const edb_delta_rule_args* args, void* stream, void* workspace,
                            size_t workspace_bytes);

size_t edb_flash_attention_fwd_desc_workspace(const edb_flash_attention_args* args);
int edb_flash_attention_fwd_desc(const edb_flash_attention_args* args, void* stream,
                                 void* workspace, size_t workspace_bytes);
size_t edb_flash_attention_bwd_desc_workspace(const edb_flash_attention_args* args);
int edb_flash_attention_bwd_desc(const edb_flash_attention_args* args, void* stream,
                                 void* workspace, size_t workspace_bytes);

size_t edb_native_rec_fwd_desc_workspace(const edb_native_rec_args* args);
int edb_native_rec_fwd_desc(const edb_native_rec_args* args, void* stream, void* workspace,
                            size_t workspace_bytes);

size_t edb_laser_attention_fwd_desc_workspace(const edb_laser_attention_args* args);
int edb_laser_attention_fwd_desc(const edb_laser_attention_args* args, void* stream,
                                 void* workspace, size_t workspace_bytes);
size_t edb_laser_attention_bwd_desc_workspace(const edb_laser_attention_args* args);
int edb_laser_attention_bwd_desc(const edb_laser_attention_args* args, void* stream,
                                 void* workspace, size_t workspace_bytes);

size_t edb_fox_attention_fwd_desc_workspace(const edb_fox_attention_args* args);
int edb_fox_attention_fwd_desc(const edb_fox_attention_args* args, void* stream,
                               void* workspace, size_t workspace_bytes);
size_t edb_fox_attention_bwd_desc_workspace(const edb_fox_attention_args* args);
int edb_fox_attention_bwd_desc(const edb_fox_attention_args* args, void* stream,
                               void* workspace, size_t workspace_bytes);

#ifdef __cplusplus
}
#endif

#endif /* EDIFICE_B200_H */
