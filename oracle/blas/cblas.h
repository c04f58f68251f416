/* Minimal CBLAS declarations for building the reference CPU path against the
 * OpenBLAS that numpy's wheel bundles.  That library exports the ILP64
 * interface under a "scipy_" prefix with a "64_" suffix; cblas_shim.c maps the
 * standard LP64 names used by the reference (libffwd/gemm.c, attn.c, norm.c)
 * onto it.  Enum values are the standard CBLAS ones. Test infrastructure only. */
#ifndef FFWD_ORACLE_CBLAS_H
#define FFWD_ORACLE_CBLAS_H
#ifdef __cplusplus
extern "C" {
#endif
typedef enum { CblasRowMajor = 101, CblasColMajor = 102 } CBLAS_ORDER;
typedef enum { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 } CBLAS_TRANSPOSE;
typedef CBLAS_ORDER CBLAS_LAYOUT;

void cblas_sgemm(CBLAS_ORDER order, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb, int m, int n, int k,
                 float alpha, const float *a, int lda, const float *b, int ldb, float beta, float *c,
                 int ldc);
void cblas_sgemv(CBLAS_ORDER order, CBLAS_TRANSPOSE ta, int m, int n, float alpha, const float *a,
                 int lda, const float *x, int incx, float beta, float *y, int incy);
float cblas_sdot(int n, const float *x, int incx, const float *y, int incy);
void cblas_saxpy(int n, float alpha, const float *x, int incx, float *y, int incy);
void cblas_sscal(int n, float alpha, float *x, int incx);
void openblas_set_num_threads(int n);
int openblas_get_num_threads(void);
#ifdef __cplusplus
}
#endif
#endif
