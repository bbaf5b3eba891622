/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Builds liboracle.so: the CPU restatement of Edifice's Nx fallbacks for the
 * fused sequence-mixing path, in two arithmetic widths:
 *   orc_*_f64  f64 accumulation; the parity oracle every GPU result is
 *              checked against.
 *   orc_*_f32  f32 arithmetic, as the Nx host backend computes; the timed CPU
 *              baseline (OpenMP over the host cores).
 * The product library (edifice_b200) never links or calls this file.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define REAL double
#define SFX _f64
#include "oracle_body.h"
#undef REAL
#undef SFX

/* f32 arithmetic: route the libm calls to their float versions */
#define exp(x) expf(x)
#define log(x) logf(x)
#define sqrt(x) sqrtf(x)
#define REAL float
#define SFX _f32
#include "oracle_body.h"
#undef REAL
#undef SFX
#undef exp
#undef log
#undef sqrt

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
