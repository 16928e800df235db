/*
 * Linux stand-in for the three Apple Accelerate routines the SlipStream hot
 * path calls (vDSP_dotpr, vDSP_vadd, cblas_saxpy).  TEST INFRASTRUCTURE ONLY:
 * used to compile the reference CPU path into oracle/_ref.
 *
 * Each routine is a plain strided loop.  vDSP_dotpr sums sequentially in fp32,
 * which fixes the oracle's summation order (Apple's own order is vectorised and
 * unpublished, so parity is unpinned at this boundary).
 */
#ifndef SS_ORACLE_SHIM_ACCELERATE_H
#define SS_ORACLE_SHIM_ACCELERATE_H
typedef long vDSP_Stride;
typedef unsigned long vDSP_Length;

static inline void vDSP_dotpr(const float *a, vDSP_Stride ia, const float *b,
                              vDSP_Stride ib, float *c, vDSP_Length n) {
    float s = 0.0f;
    for (vDSP_Length i = 0; i < n; i++) s += a[i * ia] * b[i * ib];
    *c = s;
}

static inline void vDSP_vadd(const float *a, vDSP_Stride ia, const float *b,
                             vDSP_Stride ib, float *c, vDSP_Stride ic,
                             vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] + b[i * ib];
}

static inline void cblas_saxpy(int n, float alpha, const float *x, int incx,
                               float *y, int incy) {
    for (int i = 0; i < n; i++) y[i * incy] += alpha * x[i * incx];
}
#endif
