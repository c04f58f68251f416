/* LP64 CBLAS entry points forwarding to numpy's bundled ILP64 OpenBLAS
 * (exports scipy_cblas_*64_ / scipy_openblas_*64_).  Test infrastructure:
 * only the oracle build under oracle/ links this. */
#include "cblas.h"
#include <stdint.h>

typedef int64_t blasint64;
extern void scipy_cblas_sgemm64_(int, int, int, blasint64, blasint64, blasint64, float,
                                 const float *, blasint64, const float *, blasint64, float,
                                 float *, blasint64);
extern void scipy_cblas_sgemv64_(int, int, blasint64, blasint64, float, const float *, blasint64,
                                 const float *, blasint64, float, float *, blasint64);
extern float scipy_cblas_sdot64_(blasint64, const float *, blasint64, const float *, blasint64);
extern void scipy_cblas_saxpy64_(blasint64, float, const float *, blasint64, float *, blasint64);
extern void scipy_cblas_sscal64_(blasint64, float, float *, blasint64);
extern void scipy_openblas_set_num_threads64_(int);
extern int scipy_openblas_get_num_threads64_(void);

void cblas_sgemm(CBLAS_ORDER o, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb, int m, int n, int k,
                 float alpha, const float *a, int lda, const float *b, int ldb, float beta, float *c,
                 int ldc) {
    scipy_cblas_sgemm64_(o, ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}
void cblas_sgemv(CBLAS_ORDER o, CBLAS_TRANSPOSE ta, int m, int n, float alpha, const float *a,
                 int lda, const float *x, int incx, float beta, float *y, int incy) {
    scipy_cblas_sgemv64_(o, ta, m, n, alpha, a, lda, x, incx, beta, y, incy);
}
float cblas_sdot(int n, const float *x, int incx, const float *y, int incy) {
    return scipy_cblas_sdot64_(n, x, incx, y, incy);
}
void cblas_saxpy(int n, float alpha, const float *x, int incx, float *y, int incy) {
    scipy_cblas_saxpy64_(n, alpha, x, incx, y, incy);
}
void cblas_sscal(int n, float alpha, float *x, int incx) { scipy_cblas_sscal64_(n, alpha, x, incx); }
void openblas_set_num_threads(int n) { scipy_openblas_set_num_threads64_(n); }
int openblas_get_num_threads(void) { return scipy_openblas_get_num_threads64_(); }
