/*
 * oracle_body.h -- TEST INFRASTRUCTURE ONLY (the parity checker, never the product).
 *
 * CPU restatement of Edifice's pure-Nx formulation of the fused sequence-mixing
 * hot path.  This file is included twice by oracle.c: once with REAL=double
 * (suffix _f64, the parity oracle) and once with REAL=float (suffix _f32, the
 * timed CPU baseline that mirrors Nx's f32 arithmetic).  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm call it.
 *
 * Inputs are f32 arrays (bf16 inputs are passed already widened, exactly).
 * Outputs are f32 arrays.  Layouts are the reference's:
 *   scans            [B, L, H] row-major, channel fastest
 *   selective scan   x, dt [B, L, D]; A [D, N]; B, C [B, L, N]
 *   delta rule       q, k, v [B, L, H, d]; beta [B, L, H, d] or [B, L, H]
 *   gated delta rule as the delta rule, plus alpha [B, L, H]
 *   attention        q [B, Hq, L, d]; k, v [B, Hkv, L, d]
 *
 * Each function cites the reference file:line it restates (paths relative to
 * the edifice project root).
 */

#define ORC_CAT2(a, b) a##b
#define ORC_CAT(a, b) ORC_CAT2(a, b)
#define FN(name) ORC_CAT(orc_##name, SFX)

static inline REAL ORC_CAT(clampr, SFX)(REAL v, REAL lo, REAL hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

/* ------------------------------------------------------------------------ */
/* Linear recurrence h_t = a_t * h_{t-1} + b_t                                */
/* lib/edifice/cuda/fused_scan.ex:4429-4444 (linear_scan_fallback) and        */
/* :869-882 (linear_scan_cc_fallback, with explicit h0).                      */
/* Time outer, channels inner: the same vectorised-over-(batch,hidden) order  */
/* the Nx Enum.reduce over t uses.                                            */
/* ------------------------------------------------------------------------ */
void FN(linear_scan_fwd)(const float* a, const float* bv, const float* h0, float* out,
                         int B, int L, int H) {
    #pragma omp parallel for schedule(static)
    for (long bh = 0; bh < (long)B * ((H + 255) / 256); bh++) {
        int nblk = (H + 255) / 256;
        int b = (int)(bh / nblk), h_lo = (int)(bh % nblk) * 256;
        int h_hi = h_lo + 256 < H ? h_lo + 256 : H;
        REAL s[256];
        for (int h = h_lo; h < h_hi; h++) s[h - h_lo] = h0 ? (REAL)h0[(size_t)b * H + h] : (REAL)0;
        for (int t = 0; t < L; t++) {
            size_t row = ((size_t)b * L + t) * H;
            for (int h = h_lo; h < h_hi; h++) {
                REAL v = (REAL)a[row + h] * s[h - h_lo] + (REAL)bv[row + h];
                s[h - h_lo] = v;
                out[row + h] = (float)v;
            }
        }
    }
}

/* Backward: fused_scan.ex:884-916 (linear_scan_backward_fallback).
 *   dh = dY_t + acc; da_t = dh * h_{t-1}; db_t = dh; acc = dh * a_t; gh0 = acc. */
void FN(linear_scan_bwd)(const float* a, const float* h0, const float* fwd, const float* dy,
                         float* ga, float* gb, float* gh0, int B, int L, int H) {
    #pragma omp parallel for schedule(static)
    for (long bh = 0; bh < (long)B * ((H + 255) / 256); bh++) {
        int nblk = (H + 255) / 256;
        int b = (int)(bh / nblk), h_lo = (int)(bh % nblk) * 256;
        int h_hi = h_lo + 256 < H ? h_lo + 256 : H;
        REAL acc[256];
        for (int h = h_lo; h < h_hi; h++) acc[h - h_lo] = 0;
        for (int t = L - 1; t >= 0; t--) {
            size_t row = ((size_t)b * L + t) * H;
            for (int h = h_lo; h < h_hi; h++) {
                REAL dh = (REAL)dy[row + h] + acc[h - h_lo];
                REAL hp = t == 0 ? (h0 ? (REAL)h0[(size_t)b * H + h] : (REAL)0)
                                 : (REAL)fwd[row - H + h];
                ga[row + h] = (float)(dh * hp);
                gb[row + h] = (float)dh;
                acc[h - h_lo] = dh * (REAL)a[row + h];
            }
        }
        if (gh0)
            for (int h = h_lo; h < h_hi; h++) gh0[(size_t)b * H + h] = (float)acc[h - h_lo];
    }
}

/* ------------------------------------------------------------------------ */
/* MinGRU h_t = (1 - z_t) h_{t-1} + z_t c_t, z post-sigmoid.                   */
/* fused_scan.ex:516-528 (mingru_scan_fallback) and                           */
/* lib/edifice/recurrent/min_gru.ex:305-326 (sigmoid applied by the caller).  */
/* ------------------------------------------------------------------------ */
void FN(mingru_fwd)(const float* z, const float* c, const float* h0, float* out,
                    int B, int L, int H) {
    #pragma omp parallel for schedule(static)
    for (long bh = 0; bh < (long)B * ((H + 255) / 256); bh++) {
        int nblk = (H + 255) / 256;
        int b = (int)(bh / nblk), h_lo = (int)(bh % nblk) * 256;
        int h_hi = h_lo + 256 < H ? h_lo + 256 : H;
        REAL s[256];
        for (int h = h_lo; h < h_hi; h++) s[h - h_lo] = h0 ? (REAL)h0[(size_t)b * H + h] : (REAL)0;
        for (int t = 0; t < L; t++) {
            size_t row = ((size_t)b * L + t) * H;
            for (int h = h_lo; h < h_hi; h++) {
                REAL zz = (REAL)z[row + h];
                REAL v = ((REAL)1 - zz) * s[h - h_lo] + zz * (REAL)c[row + h];
                s[h - h_lo] = v;
                out[row + h] = (float)v;
            }
        }
    }
}

/* Backward: fused_scan.ex:548-581 (mingru_backward_fallback).
 *   dh = dY_t + acc; dz = dh (c_t - h_{t-1}); dc = dh z_t; acc = dh (1 - z_t). */
void FN(mingru_bwd)(const float* z, const float* c, const float* h0, const float* fwd,
                    const float* dy, float* gz, float* gc, float* gh0, int B, int L, int H) {
    #pragma omp parallel for schedule(static)
    for (long bh = 0; bh < (long)B * ((H + 255) / 256); bh++) {
        int nblk = (H + 255) / 256;
        int b = (int)(bh / nblk), h_lo = (int)(bh % nblk) * 256;
        int h_hi = h_lo + 256 < H ? h_lo + 256 : H;
        REAL acc[256];
        for (int h = h_lo; h < h_hi; h++) acc[h - h_lo] = 0;
        for (int t = L - 1; t >= 0; t--) {
            size_t row = ((size_t)b * L + t) * H;
            for (int h = h_lo; h < h_hi; h++) {
                REAL dh = (REAL)dy[row + h] + acc[h - h_lo];
                REAL hp = t == 0 ? (h0 ? (REAL)h0[(size_t)b * H + h] : (REAL)0)
                                 : (REAL)fwd[row - H + h];
                REAL zz = (REAL)z[row + h];
                gz[row + h] = (float)(dh * ((REAL)c[row + h] - hp));
                gc[row + h] = (float)(dh * zz);
                acc[h - h_lo] = dh * ((REAL)1 - zz);
            }
        }
        if (gh0)
            for (int h = h_lo; h < h_hi; h++) gh0[(size_t)b * H + h] = (float)acc[h - h_lo];
    }
}

/* ------------------------------------------------------------------------ */
/* Mamba selective scan, KERNEL semantics (given A, per-channel dt, clamp):    */
/*   dtc = clip(dt, 1e-3, 0.1); h_n = exp(dtc A[d,n]) h_n + dtc B_n x;         */
/*   y = sum_n C_n h_n.                                                        */
/* test/edifice/cuda/backward_kernels_test.exs:1563-1586                       */
/* (selective_scan_forward) == native/cuda/fused_selective_scan.cu:68-96.      */
/* ------------------------------------------------------------------------ */
void FN(selective_scan_fwd)(const float* x, const float* dt, const float* A, const float* Bm,
                            const float* Cm, float* y, int B, int L, int D, int N,
                            float dt_min, float dt_max) {
    #pragma omp parallel for schedule(static)
    for (long bd = 0; bd < (long)B * ((D + 63) / 64); bd++) {
        int nblk = (D + 63) / 64;
        int b = (int)(bd / nblk), d_lo = (int)(bd % nblk) * 64;
        int d_hi = d_lo + 64 < D ? d_lo + 64 : D;
        REAL h[64 * 64];
        for (int i = 0; i < 64 * N; i++) h[i] = 0;
        for (int t = 0; t < L; t++) {
            size_t row = ((size_t)b * L + t) * D;
            size_t bc = ((size_t)b * L + t) * N;
            for (int d = d_lo; d < d_hi; d++) {
                REAL dtc = ORC_CAT(clampr, SFX)((REAL)dt[row + d], (REAL)dt_min, (REAL)dt_max);
                REAL xv = (REAL)x[row + d];
                REAL acc = 0;
                REAL* hs = h + (size_t)(d - d_lo) * N;
                for (int n = 0; n < N; n++) {
                    REAL abar = exp(dtc * (REAL)A[(size_t)d * N + n]);
                    hs[n] = abar * hs[n] + dtc * (REAL)Bm[bc + n] * xv;
                    acc += (REAL)Cm[bc + n] * hs[n];
                }
                y[row + d] = (float)acc;
            }
        }
    }
}

/* Backward, kernel semantics: fused_scan.ex:1453-1531
 * (selective_scan_backward_fallback).  A receives no gradient.  gB and gC are
 * sums over the channel axis d.  gdt is zero where dt lies outside
 * [dt_min, dt_max] (fused_scan.ex:1510-1511).
 * h_prev is recomputed per time chunk from stored chunk-boundary states
 * (same arithmetic as the forward, so the values are those the fallback
 * stacks in h_prev_list). */
void FN(selective_scan_bwd)(const float* x, const float* dt, const float* A, const float* Bm,
                            const float* Cm, const float* dy, float* gx, float* gdt, float* gB,
                            float* gC, int B, int L, int D, int N, float dt_min, float dt_max) {
    const int CH = 64; /* recompute chunk */
    int nck = (L + CH - 1) / CH;
    for (size_t i = 0; i < (size_t)B * L * N; i++) { gB[i] = 0; gC[i] = 0; }
    for (int b = 0; b < B; b++) {
        #pragma omp parallel
        {
            REAL* pgB = (REAL*)calloc((size_t)L * N, sizeof(REAL));
            REAL* pgC = (REAL*)calloc((size_t)L * N, sizeof(REAL));
            REAL* ck = (REAL*)malloc((size_t)nck * N * sizeof(REAL));
            REAL* hc = (REAL*)malloc((size_t)(CH + 1) * N * sizeof(REAL));
            REAL* dh = (REAL*)malloc((size_t)N * sizeof(REAL));
            #pragma omp for schedule(static)
            for (int d = 0; d < D; d++) {
                const float* Ad = A + (size_t)d * N;
                /* forward: chunk-boundary states */
                for (int n = 0; n < N; n++) hc[n] = 0;
                for (int t = 0; t < L; t++) {
                    if (t % CH == 0)
                        for (int n = 0; n < N; n++) ck[(size_t)(t / CH) * N + n] = hc[n];
                    size_t r = ((size_t)b * L + t) * D + d, bc = ((size_t)b * L + t) * N;
                    REAL dtc = ORC_CAT(clampr, SFX)((REAL)dt[r], (REAL)dt_min, (REAL)dt_max);
                    for (int n = 0; n < N; n++)
                        hc[n] = exp(dtc * (REAL)Ad[n]) * hc[n] + dtc * (REAL)Bm[bc + n] * (REAL)x[r];
                }
                for (int n = 0; n < N; n++) dh[n] = 0;
                for (int c = nck - 1; c >= 0; c--) {
                    int t0 = c * CH, t1 = t0 + CH < L ? t0 + CH : L;
                    /* hc[(t - t0)] = h_{t-1} for t in [t0, t1], hc[t1-t0] = h_{t1-1} */
                    for (int n = 0; n < N; n++) hc[n] = ck[(size_t)c * N + n];
                    for (int t = t0; t < t1; t++) {
                        size_t r = ((size_t)b * L + t) * D + d, bc = ((size_t)b * L + t) * N;
                        REAL dtc = ORC_CAT(clampr, SFX)((REAL)dt[r], (REAL)dt_min, (REAL)dt_max);
                        for (int n = 0; n < N; n++)
                            hc[(size_t)(t - t0 + 1) * N + n] =
                                exp(dtc * (REAL)Ad[n]) * hc[(size_t)(t - t0) * N + n] +
                                dtc * (REAL)Bm[bc + n] * (REAL)x[r];
                    }
                    for (int t = t1 - 1; t >= t0; t--) {
                        size_t r = ((size_t)b * L + t) * D + d, bc = ((size_t)b * L + t) * N;
                        REAL draw = (REAL)dt[r];
                        REAL dtc = ORC_CAT(clampr, SFX)(draw, (REAL)dt_min, (REAL)dt_max);
                        REAL xv = (REAL)x[r], dyv = (REAL)dy[r];
                        REAL gxv = 0, gdv = 0;
                        for (int n = 0; n < N; n++) {
                            REAL hp = hc[(size_t)(t - t0) * N + n];
                            REAL hcur = hc[(size_t)(t - t0 + 1) * N + n];
                            REAL abar = exp(dtc * (REAL)Ad[n]);
                            REAL Bn = (REAL)Bm[bc + n], Cn = (REAL)Cm[bc + n];
                            REAL dtot = dh[n] + dyv * Cn;           /* dh_state += dy * C */
                            pgC[(size_t)t * N + n] += dyv * hcur;    /* dC = sum_d dy h_cur */
                            gxv += dtot * dtc * Bn;                  /* dx = sum_n dh dt B */
                            gdv += dtot * hp * abar * (REAL)Ad[n];   /* through exp(dt A) */
                            gdv += dtot * Bn * xv;                   /* through dt B x */
                            pgB[(size_t)t * N + n] += dtot * xv * dtc; /* dB = sum_d dh x dt */
                            dh[n] = dtot * abar;                     /* carry */
                        }
                        gx[r] = (float)gxv;
                        int inr = draw >= (REAL)dt_min && draw <= (REAL)dt_max;
                        gdt[r] = inr ? (float)gdv : 0.0f;
                    }
                }
            }
            #pragma omp critical
            {
                for (size_t i = 0; i < (size_t)L * N; i++) {
                    gB[(size_t)b * L * N + i] += (float)pgB[i];
                    gC[(size_t)b * L * N + i] += (float)pgC[i];
                }
            }
            free(pgB); free(pgC); free(ck); free(hc); free(dh);
        }
    }
}

/* Mamba selective scan, MODEL semantics (Edifice.build(:mamba) fallback):
 * lib/edifice/ssm/common.ex:661-670 -> discretize_ssm :402-444 (fixed
 * A = -(1..N), B_bar from the channel-mean of the clamped dt), sequential_scan
 * :492-515, compute_ssm_output :462-470.  The fallback does not read its A
 * argument; its caller lib/edifice/ssm/mamba.ex:187-193 hands the fused path the
 * same fixed matrix.  A == NULL here means that fixed diagonal; a non-NULL A
 * [D, N] is used instead (the fused path's contract). */
static REAL ORC_CAT(model_a, SFX)(const float* A, int d, int n, int N) {
    return A ? (REAL)A[(size_t)d * N + n] : -(REAL)(n + 1);
}

void FN(selective_scan_model_fwd)(const float* x, const float* dt, const float* A,
                                  const float* Bm, const float* Cm, float* y, int B, int L, int D,
                                  int N, float dt_min, float dt_max) {
    #pragma omp parallel for schedule(dynamic)
    for (int b = 0; b < B; b++) {
        REAL* h = (REAL*)calloc((size_t)D * N, sizeof(REAL));
        for (int t = 0; t < L; t++) {
            size_t row = ((size_t)b * L + t) * D, bc = ((size_t)b * L + t) * N;
            REAL mean = 0;
            for (int d = 0; d < D; d++)
                mean += ORC_CAT(clampr, SFX)((REAL)dt[row + d], (REAL)dt_min, (REAL)dt_max);
            mean /= (REAL)D;
            for (int d = 0; d < D; d++) {
                REAL dtc = ORC_CAT(clampr, SFX)((REAL)dt[row + d], (REAL)dt_min, (REAL)dt_max);
                REAL acc = 0;
                for (int n = 0; n < N; n++) {
                    REAL abar = exp(dtc * ORC_CAT(model_a, SFX)(A, d, n, N));
                    REAL bx = mean * (REAL)Bm[bc + n] * (REAL)x[row + d];
                    h[(size_t)d * N + n] = abar * h[(size_t)d * N + n] + bx;
                    acc += (REAL)Cm[bc + n] * h[(size_t)d * N + n];
                }
                y[row + d] = (float)acc;
            }
        }
        free(h);
    }
}

/* Backward of the model semantics: the gradient Nx's autodiff takes through
 * discretize_ssm -> sequential_scan -> compute_ssm_output (common.ex:402-515).
 * With m = mean_d(clip(dt)):
 *   dh_tot = dh + dy C;  gC += dy h;  gx = m sum_n dh_tot B;
 *   gB = m sum_d dh_tot x;  g_m = sum_{d,n} dh_tot B x;
 *   gdt = [dt in range] (sum_n dh_tot h_prev abar A + g_m / D);  dh = dh_tot abar.
 * A receives no gradient.  Keeps every state of a batch row (small cases). */
void FN(selective_scan_model_bwd)(const float* x, const float* dt, const float* A,
                                  const float* Bm, const float* Cm, const float* dy, float* gx,
                                  float* gdt, float* gB, float* gC, int B, int L, int D, int N,
                                  float dt_min, float dt_max) {
    #pragma omp parallel for schedule(dynamic)
    for (int b = 0; b < B; b++) {
        REAL* hs = (REAL*)malloc((size_t)(L + 1) * D * N * sizeof(REAL));
        REAL* mean = (REAL*)malloc((size_t)L * sizeof(REAL));
        REAL* dh = (REAL*)malloc((size_t)D * N * sizeof(REAL));
        REAL* gdir = (REAL*)malloc((size_t)D * sizeof(REAL));
        for (size_t i = 0; i < (size_t)D * N; i++) hs[i] = 0;
        for (int t = 0; t < L; t++) {
            size_t row = ((size_t)b * L + t) * D, bc = ((size_t)b * L + t) * N;
            REAL m = 0;
            for (int d = 0; d < D; d++)
                m += ORC_CAT(clampr, SFX)((REAL)dt[row + d], (REAL)dt_min, (REAL)dt_max);
            m /= (REAL)D;
            mean[t] = m;
            REAL* hp = hs + (size_t)t * D * N;
            REAL* hn = hp + (size_t)D * N;
            for (int d = 0; d < D; d++) {
                REAL dtc = ORC_CAT(clampr, SFX)((REAL)dt[row + d], (REAL)dt_min, (REAL)dt_max);
                for (int n = 0; n < N; n++)
                    hn[(size_t)d * N + n] =
                        exp(dtc * ORC_CAT(model_a, SFX)(A, d, n, N)) * hp[(size_t)d * N + n] +
                        m * (REAL)Bm[bc + n] * (REAL)x[row + d];
            }
        }
        for (size_t i = 0; i < (size_t)D * N; i++) dh[i] = 0;
        for (int t = L - 1; t >= 0; t--) {
            size_t row = ((size_t)b * L + t) * D, bc = ((size_t)b * L + t) * N;
            const REAL* hp = hs + (size_t)t * D * N;
            const REAL* hc = hp + (size_t)D * N;
            REAL m = mean[t], gm = 0;
            for (int n = 0; n < N; n++) {
                REAL pb = 0, pc = 0;
                for (int d = 0; d < D; d++) {
                    REAL dtot = dh[(size_t)d * N + n] + (REAL)dy[row + d] * (REAL)Cm[bc + n];
                    pc += (REAL)dy[row + d] * hc[(size_t)d * N + n];
                    pb += dtot * (REAL)x[row + d];
                }
                gB[bc + n] = (float)(m * pb);
                gC[bc + n] = (float)pc;
                gm += pb * (REAL)Bm[bc + n];
            }
            for (int d = 0; d < D; d++) {
                REAL dtc = ORC_CAT(clampr, SFX)((REAL)dt[row + d], (REAL)dt_min, (REAL)dt_max);
                REAL gxv = 0, gdv = 0;
                for (int n = 0; n < N; n++) {
                    REAL a = ORC_CAT(model_a, SFX)(A, d, n, N);
                    REAL abar = exp(dtc * a);
                    REAL dtot = dh[(size_t)d * N + n] + (REAL)dy[row + d] * (REAL)Cm[bc + n];
                    gxv += dtot * m * (REAL)Bm[bc + n];
                    gdv += dtot * hp[(size_t)d * N + n] * abar * a;
                    dh[(size_t)d * N + n] = dtot * abar;
                }
                gdir[d] = gdv;
                gx[row + d] = (float)gxv;
            }
            for (int d = 0; d < D; d++) {
                REAL draw = (REAL)dt[row + d];
                int inr = draw >= (REAL)dt_min && draw <= (REAL)dt_max;
                gdt[row + d] = inr ? (float)(gdir[d] + gm / (REAL)D) : 0.0f;
            }
        }
        free(hs); free(mean); free(dh); free(gdir);
    }
}

/* ------------------------------------------------------------------------ */
/* DeltaNet delta rule.  S_0 = 0; r = S k; S += (beta (.) (v - r)) k^T;       */
/* o = S q.  fused_scan.ex:2212-2236 (delta_net_scan_fallback) ==             */
/* lib/edifice/recurrent/delta_net.ex:231-273.  beta_scalar != 0 means beta   */
/* is [B,L,H] (one gate per token and head, broadcast over rows of S).        */
/* ------------------------------------------------------------------------ */
void FN(delta_net_fwd)(const float* q, const float* k, const float* v, const float* beta,
                       float* o, int B, int L, int H, int d, int beta_scalar) {
    #pragma omp parallel for schedule(dynamic)
    for (long bh = 0; bh < (long)B * H; bh++) {
        int b = (int)(bh / H), hh = (int)(bh % H);
        REAL* S = (REAL*)calloc((size_t)d * d, sizeof(REAL));
        for (int t = 0; t < L; t++) {
            size_t off = (((size_t)b * L + t) * H + hh) * d;
            size_t boff = beta_scalar ? (((size_t)b * L + t) * H + hh) : off;
            for (int i = 0; i < d; i++) {
                REAL r = 0;
                for (int j = 0; j < d; j++) r += S[(size_t)i * d + j] * (REAL)k[off + j];
                REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                REAL se = be * ((REAL)v[off + i] - r);
                for (int j = 0; j < d; j++) S[(size_t)i * d + j] += se * (REAL)k[off + j];
            }
            for (int i = 0; i < d; i++) {
                REAL acc = 0;
                for (int j = 0; j < d; j++) acc += S[(size_t)i * d + j] * (REAL)q[off + j];
                o[off + i] = (float)acc;
            }
        }
        free(S);
    }
}

/* Backward: fused_scan.ex:1257-1326 (delta_rule_backward_fallback).
 *   dS += dO q^T; dq = S_t^T dO; dsk = dS k; dv = beta (.) dsk;
 *   dbeta = (v - r) (.) dsk; dk = dS^T (beta (.) err) - S_{t-1}^T (beta (.) dsk);
 *   dS_prev = dS - (beta (.) dsk) k^T.
 * For scalar beta the per-row dbeta is summed over rows.
 * S_{t-1} is recomputed per chunk from stored chunk-boundary states. */
void FN(delta_net_bwd)(const float* q, const float* k, const float* v, const float* beta,
                       const float* dO, float* gq, float* gk, float* gv, float* gbeta,
                       int B, int L, int H, int d, int beta_scalar) {
    const int CH = 16;
    int nck = (L + CH - 1) / CH;
    #pragma omp parallel for schedule(dynamic)
    for (long bh = 0; bh < (long)B * H; bh++) {
        int b = (int)(bh / H), hh = (int)(bh % H);
        size_t dd = (size_t)d * d;
        REAL* ck = (REAL*)calloc((size_t)nck * dd, sizeof(REAL));
        REAL* Sc = (REAL*)calloc((size_t)(CH + 1) * dd, sizeof(REAL));
        REAL* dS = (REAL*)calloc(dd, sizeof(REAL));
        REAL* r = (REAL*)malloc((size_t)d * sizeof(REAL));
        REAL* dsk = (REAL*)malloc((size_t)d * sizeof(REAL));
        REAL* S = Sc; /* scratch for the boundary pass */
        for (size_t i = 0; i < dd; i++) S[i] = 0;
        for (int t = 0; t < L; t++) {
            if (t % CH == 0) memcpy(ck + (size_t)(t / CH) * dd, S, dd * sizeof(REAL));
            size_t off = (((size_t)b * L + t) * H + hh) * d;
            size_t boff = ((size_t)b * L + t) * H + hh;
            for (int i = 0; i < d; i++) {
                REAL rr = 0;
                for (int j = 0; j < d; j++) rr += S[(size_t)i * d + j] * (REAL)k[off + j];
                REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                REAL se = be * ((REAL)v[off + i] - rr);
                for (int j = 0; j < d; j++) S[(size_t)i * d + j] += se * (REAL)k[off + j];
            }
        }
        for (int c = nck - 1; c >= 0; c--) {
            int t0 = c * CH, t1 = t0 + CH < L ? t0 + CH : L;
            memcpy(Sc, ck + (size_t)c * dd, dd * sizeof(REAL));
            for (int t = t0; t < t1; t++) {
                REAL* Sp = Sc + (size_t)(t - t0) * dd;
                REAL* Sn = Sp + dd;
                size_t off = (((size_t)b * L + t) * H + hh) * d;
                size_t boff = ((size_t)b * L + t) * H + hh;
                for (int i = 0; i < d; i++) {
                    REAL rr = 0;
                    for (int j = 0; j < d; j++) rr += Sp[(size_t)i * d + j] * (REAL)k[off + j];
                    REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                    REAL se = be * ((REAL)v[off + i] - rr);
                    for (int j = 0; j < d; j++)
                        Sn[(size_t)i * d + j] = Sp[(size_t)i * d + j] + se * (REAL)k[off + j];
                }
            }
            for (int t = t1 - 1; t >= t0; t--) {
                REAL* Sp = Sc + (size_t)(t - t0) * dd;
                REAL* Sn = Sp + dd;
                size_t off = (((size_t)b * L + t) * H + hh) * d;
                size_t boff = ((size_t)b * L + t) * H + hh;
                for (int i = 0; i < d; i++) {
                    REAL rr = 0;
                    for (int j = 0; j < d; j++) rr += Sp[(size_t)i * d + j] * (REAL)k[off + j];
                    r[i] = rr;
                }
                /* dS += outer(dO, q) */
                for (int i = 0; i < d; i++)
                    for (int j = 0; j < d; j++)
                        dS[(size_t)i * d + j] += (REAL)dO[off + i] * (REAL)q[off + j];
                /* dq = S_t^T dO */
                for (int j = 0; j < d; j++) {
                    REAL acc = 0;
                    for (int i = 0; i < d; i++) acc += Sn[(size_t)i * d + j] * (REAL)dO[off + i];
                    gq[off + j] = (float)acc;
                }
                /* dsk = dS k */
                for (int i = 0; i < d; i++) {
                    REAL acc = 0;
                    for (int j = 0; j < d; j++) acc += dS[(size_t)i * d + j] * (REAL)k[off + j];
                    dsk[i] = acc;
                }
                REAL gbs = 0;
                for (int i = 0; i < d; i++) {
                    REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                    REAL err = (REAL)v[off + i] - r[i];
                    gv[off + i] = (float)(be * dsk[i]);
                    if (beta_scalar) gbs += err * dsk[i];
                    else gbeta[off + i] = (float)(err * dsk[i]);
                }
                if (beta_scalar) gbeta[boff] = (float)gbs;
                /* dk = dS^T (beta err) - beta * S_prev^T dsk  (per-row beta inside) */
                for (int j = 0; j < d; j++) {
                    REAL a1 = 0, a2 = 0;
                    for (int i = 0; i < d; i++) {
                        REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                        REAL err = (REAL)v[off + i] - r[i];
                        a1 += dS[(size_t)i * d + j] * be * err;
                        a2 += Sp[(size_t)i * d + j] * be * dsk[i];
                    }
                    gk[off + j] = (float)(a1 - a2);
                }
                /* dS_prev = dS - (beta dsk) k^T */
                for (int i = 0; i < d; i++) {
                    REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                    for (int j = 0; j < d; j++)
                        dS[(size_t)i * d + j] -= be * dsk[i] * (REAL)k[off + j];
                }
            }
        }
        free(ck); free(Sc); free(dS); free(r); free(dsk);
    }
}

/* ------------------------------------------------------------------------ */
/* GatedDeltaNet.  S_0 = 0; per token: S_d = alpha_t S; r = S_d k;            */
/* S = S_d + (beta (.) (v - r)) k^T; o = S q.  fused_scan.ex:2256-2284        */
/* (gated_delta_net_scan_fallback) == lib/edifice/recurrent/                  */
/* gated_delta_net.ex:300-350.  alpha [B, L, H] (one decay per token and      */
/* head); beta [B, L, H, d], or [B, L, H] when beta_scalar != 0.              */
/* ------------------------------------------------------------------------ */
void FN(gated_delta_net_fwd)(const float* q, const float* k, const float* v, const float* beta,
                             const float* alpha, float* o, int B, int L, int H, int d,
                             int beta_scalar) {
    #pragma omp parallel for schedule(dynamic)
    for (long bh = 0; bh < (long)B * H; bh++) {
        int b = (int)(bh / H), hh = (int)(bh % H);
        REAL* S = (REAL*)calloc((size_t)d * d, sizeof(REAL));
        for (int t = 0; t < L; t++) {
            size_t off = (((size_t)b * L + t) * H + hh) * d;
            size_t boff = ((size_t)b * L + t) * H + hh;
            REAL al = (REAL)alpha[boff];
            for (int i = 0; i < d; i++) {
                REAL r = 0;
                for (int j = 0; j < d; j++) {
                    S[(size_t)i * d + j] *= al;
                    r += S[(size_t)i * d + j] * (REAL)k[off + j];
                }
                REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                REAL se = be * ((REAL)v[off + i] - r);
                for (int j = 0; j < d; j++) S[(size_t)i * d + j] += se * (REAL)k[off + j];
            }
            for (int i = 0; i < d; i++) {
                REAL acc = 0;
                for (int j = 0; j < d; j++) acc += S[(size_t)i * d + j] * (REAL)q[off + j];
                o[off + i] = (float)acc;
            }
        }
        free(S);
    }
}

/* Backward: fused_scan.ex:1347-1431 (gated_delta_net_backward_fallback):
 *   dS += dO q^T; dq = S_t^T dO; dsk = dS k; dv = beta (.) dsk;
 *   dbeta = err (.) dsk; dk = dS^T (beta (.) err) - S_d^T (beta (.) dsk);
 *   dS_d = dS - (beta (.) dsk) k^T; dalpha = sum(dS_d (.) S_{t-1}); dS_prev = alpha dS_d,
 * with S_d = alpha S_{t-1}.  The through-retrieval key gradient is the exact
 * one, S_d^T (beta (.) dsk) (the fallback scales S_d^T dsk by beta over the key
 * index, equal only when beta is the same for every row).  For scalar beta the
 * per-row dbeta is summed over rows.  S_{t-1} is recomputed per chunk from
 * stored chunk-boundary states. */
void FN(gated_delta_net_bwd)(const float* q, const float* k, const float* v, const float* beta,
                             const float* alpha, const float* dO, float* gq, float* gk,
                             float* gv, float* gbeta, float* galpha, int B, int L, int H, int d,
                             int beta_scalar) {
    const int CH = 16;
    int nck = (L + CH - 1) / CH;
    #pragma omp parallel for schedule(dynamic)
    for (long bh = 0; bh < (long)B * H; bh++) {
        int b = (int)(bh / H), hh = (int)(bh % H);
        size_t dd = (size_t)d * d;
        REAL* ck = (REAL*)calloc((size_t)nck * dd, sizeof(REAL));
        REAL* Sc = (REAL*)calloc((size_t)(CH + 1) * dd, sizeof(REAL));
        REAL* dS = (REAL*)calloc(dd, sizeof(REAL));
        REAL* r = (REAL*)malloc((size_t)d * sizeof(REAL));
        REAL* dsk = (REAL*)malloc((size_t)d * sizeof(REAL));
        /* one step S_prev -> S_next (S_next may alias nothing) */
#define ORC_GATED_STEP(Sp, Sn, t)                                                       \
        do {                                                                             \
            size_t off_ = (((size_t)b * L + (t)) * H + hh) * d;                          \
            size_t boff_ = ((size_t)b * L + (t)) * H + hh;                               \
            REAL al_ = (REAL)alpha[boff_];                                               \
            for (int i = 0; i < d; i++) {                                                \
                REAL rr = 0;                                                             \
                for (int j = 0; j < d; j++) rr += al_ * (Sp)[(size_t)i * d + j] * (REAL)k[off_ + j]; \
                REAL be = (REAL)beta[beta_scalar ? boff_ : off_ + i];                    \
                REAL se = be * ((REAL)v[off_ + i] - rr);                                 \
                for (int j = 0; j < d; j++)                                              \
                    (Sn)[(size_t)i * d + j] = al_ * (Sp)[(size_t)i * d + j] + se * (REAL)k[off_ + j]; \
            }                                                                            \
        } while (0)
        REAL* S = Sc;
        for (size_t i = 0; i < dd; i++) S[i] = 0;
        for (int t = 0; t < L; t++) {
            if (t % CH == 0) memcpy(ck + (size_t)(t / CH) * dd, S, dd * sizeof(REAL));
            ORC_GATED_STEP(Sc, Sc + dd, t);
            memcpy(Sc, Sc + dd, dd * sizeof(REAL));
        }
        for (int c = nck - 1; c >= 0; c--) {
            int t0 = c * CH, t1 = t0 + CH < L ? t0 + CH : L;
            memcpy(Sc, ck + (size_t)c * dd, dd * sizeof(REAL));
            for (int t = t0; t < t1; t++) {
                REAL* Sp = Sc + (size_t)(t - t0) * dd;
                ORC_GATED_STEP(Sp, Sp + dd, t);
            }
            for (int t = t1 - 1; t >= t0; t--) {
                REAL* Sp = Sc + (size_t)(t - t0) * dd;
                REAL* Sn = Sp + dd;
                size_t off = (((size_t)b * L + t) * H + hh) * d;
                size_t boff = ((size_t)b * L + t) * H + hh;
                REAL al = (REAL)alpha[boff];
                for (int i = 0; i < d; i++) {
                    REAL rr = 0;
                    for (int j = 0; j < d; j++) rr += al * Sp[(size_t)i * d + j] * (REAL)k[off + j];
                    r[i] = rr;
                }
                for (int i = 0; i < d; i++)
                    for (int j = 0; j < d; j++)
                        dS[(size_t)i * d + j] += (REAL)dO[off + i] * (REAL)q[off + j];
                for (int j = 0; j < d; j++) {
                    REAL acc = 0;
                    for (int i = 0; i < d; i++) acc += Sn[(size_t)i * d + j] * (REAL)dO[off + i];
                    gq[off + j] = (float)acc;
                }
                for (int i = 0; i < d; i++) {
                    REAL acc = 0;
                    for (int j = 0; j < d; j++) acc += dS[(size_t)i * d + j] * (REAL)k[off + j];
                    dsk[i] = acc;
                }
                REAL gbs = 0;
                for (int i = 0; i < d; i++) {
                    REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                    REAL err = (REAL)v[off + i] - r[i];
                    gv[off + i] = (float)(be * dsk[i]);
                    if (beta_scalar) gbs += err * dsk[i];
                    else gbeta[off + i] = (float)(err * dsk[i]);
                }
                if (beta_scalar) gbeta[boff] = (float)gbs;
                for (int j = 0; j < d; j++) {
                    REAL a1 = 0, a2 = 0;
                    for (int i = 0; i < d; i++) {
                        REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                        REAL err = (REAL)v[off + i] - r[i];
                        a1 += dS[(size_t)i * d + j] * be * err;
                        a2 += al * Sp[(size_t)i * d + j] * be * dsk[i];
                    }
                    gk[off + j] = (float)(a1 - a2);
                }
                /* dS_d = dS - (beta dsk) k^T; dalpha = <dS_d, S_{t-1}>; dS_prev = alpha dS_d */
                REAL ga = 0;
                for (int i = 0; i < d; i++) {
                    REAL be = (REAL)beta[beta_scalar ? boff : off + i];
                    for (int j = 0; j < d; j++) {
                        REAL x = dS[(size_t)i * d + j] - be * dsk[i] * (REAL)k[off + j];
                        ga += x * Sp[(size_t)i * d + j];
                        dS[(size_t)i * d + j] = al * x;
                    }
                }
                galpha[boff] = (float)ga;
            }
        }
#undef ORC_GATED_STEP
        free(ck); free(Sc); free(dS); free(r); free(dsk);
    }
}

/* ------------------------------------------------------------------------ */
/* Scaled dot-product attention, optional causal mask, GQA by head grouping.  */
/* fused_scan.ex:3476-3508 (flash_attention_fallback): scores = q k^T / sqrt(d),*/
/* masked with -inf above the diagonal, softmax, weights v.  GQA: q head hq   */
/* reads kv head hq / (Hq / Hkv), the K/V repeat of                           */
/* lib/edifice/attention/gqa.ex:257-271.  lse (natural log) is optional.      */
/* ------------------------------------------------------------------------ */
void FN(attention_fwd)(const float* q, const float* k, const float* v, float* o, float* lse,
                       int B, int Hq, int Hkv, int L, int d, int causal) {
    int G = Hq / Hkv;
    #pragma omp parallel
    {
        REAL* p = (REAL*)malloc((size_t)L * sizeof(REAL));
        REAL* acc = (REAL*)malloc((size_t)d * sizeof(REAL));
        #pragma omp for schedule(dynamic) collapse(2)
        for (long bh = 0; bh < (long)B * Hq; bh++) {
            for (int i = 0; i < L; i++) {
                int b = (int)(bh / Hq), hq = (int)(bh % Hq), hk = hq / G;
                const float* qi = q + (((size_t)b * Hq + hq) * L + i) * d;
                const float* kb = k + ((size_t)b * Hkv + hk) * L * d;
                const float* vb = v + ((size_t)b * Hkv + hk) * L * d;
                REAL sc = sqrt((REAL)d);
                int jmax = causal ? i + 1 : L;
                REAL m = -INFINITY;
                for (int j = 0; j < jmax; j++) {
                    REAL s = 0;
                    for (int e = 0; e < d; e++) s += (REAL)qi[e] * (REAL)kb[(size_t)j * d + e];
                    s /= sc;
                    p[j] = s;
                    if (s > m) m = s;
                }
                REAL l = 0;
                for (int j = 0; j < jmax; j++) { p[j] = exp(p[j] - m); l += p[j]; }
                for (int e = 0; e < d; e++) acc[e] = 0;
                for (int j = 0; j < jmax; j++) {
                    REAL w = p[j] / l;
                    for (int e = 0; e < d; e++) acc[e] += w * (REAL)vb[(size_t)j * d + e];
                }
                float* oi = o + (((size_t)b * Hq + hq) * L + i) * d;
                for (int e = 0; e < d; e++) oi[e] = (float)acc[e];
                if (lse) lse[((size_t)b * Hq + hq) * L + i] = (float)(m + log(l));
            }
        }
        free(p); free(acc);
    }
}

/* Backward: fused_scan.ex:3527-3574 (flash_attention_backward_fallback).
 *   dV = P^T dO; dP = dO V^T; dS = P (.) (dP - rowsum(dP (.) P)) / sqrt(d);
 *   dQ = dS K; dK = dS^T Q.  GQA: dK, dV of a kv head sum over its q heads. */
void FN(attention_bwd)(const float* q, const float* k, const float* v, const float* dO,
                       float* dq, float* dk, float* dv, int B, int Hq, int Hkv, int L, int d,
                       int causal) {
    int G = Hq / Hkv;
    #pragma omp parallel
    {
        REAL* p = (REAL*)malloc((size_t)L * sizeof(REAL));
        REAL* dp = (REAL*)malloc((size_t)L * sizeof(REAL));
        REAL* gqa = (REAL*)malloc((size_t)d * sizeof(REAL));
        REAL* dka = (REAL*)malloc((size_t)L * d * sizeof(REAL));
        REAL* dva = (REAL*)malloc((size_t)L * d * sizeof(REAL));
        #pragma omp for schedule(dynamic)
        for (long bk = 0; bk < (long)B * Hkv; bk++) {
            int b = (int)(bk / Hkv), hk = (int)(bk % Hkv);
            const float* kb = k + ((size_t)b * Hkv + hk) * L * d;
            const float* vb = v + ((size_t)b * Hkv + hk) * L * d;
            for (size_t e = 0; e < (size_t)L * d; e++) { dka[e] = 0; dva[e] = 0; }
            REAL sc = sqrt((REAL)d);
            for (int hq = hk * G; hq < (hk + 1) * G; hq++) {
                for (int i = 0; i < L; i++) {
                    const float* qi = q + (((size_t)b * Hq + hq) * L + i) * d;
                    const float* doi = dO + (((size_t)b * Hq + hq) * L + i) * d;
                    int jmax = causal ? i + 1 : L;
                    REAL m = -INFINITY;
                    for (int j = 0; j < jmax; j++) {
                        REAL s = 0;
                        for (int e = 0; e < d; e++) s += (REAL)qi[e] * (REAL)kb[(size_t)j * d + e];
                        s /= sc;
                        p[j] = s;
                        if (s > m) m = s;
                    }
                    REAL l = 0;
                    for (int j = 0; j < jmax; j++) { p[j] = exp(p[j] - m); l += p[j]; }
                    REAL Di = 0;
                    for (int j = 0; j < jmax; j++) {
                        p[j] /= l;
                        REAL s = 0;
                        for (int e = 0; e < d; e++) s += (REAL)doi[e] * (REAL)vb[(size_t)j * d + e];
                        dp[j] = s;
                        Di += s * p[j];
                    }
                    for (int e = 0; e < d; e++) gqa[e] = 0;
                    for (int j = 0; j < jmax; j++) {
                        REAL ds = p[j] * (dp[j] - Di) / sc;
                        for (int e = 0; e < d; e++) {
                            gqa[e] += ds * (REAL)kb[(size_t)j * d + e];
                            dka[(size_t)j * d + e] += ds * (REAL)qi[e];
                            dva[(size_t)j * d + e] += p[j] * (REAL)doi[e];
                        }
                    }
                    float* dqi = dq + (((size_t)b * Hq + hq) * L + i) * d;
                    for (int e = 0; e < d; e++) dqi[e] = (float)gqa[e];
                }
            }
            float* dkb = dk + ((size_t)b * Hkv + hk) * L * d;
            float* dvb = dv + ((size_t)b * Hkv + hk) * L * d;
            for (size_t e = 0; e < (size_t)L * d; e++) { dkb[e] = (float)dka[e]; dvb[e] = (float)dva[e]; }
        }
        free(p); free(dp); free(gqa); free(dka); free(dva);
    }
}

#undef FN
