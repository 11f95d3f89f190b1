/*
 * Minimal CBLAS prototype header used only to compile the reference's CPU
 * sources (ops.c, model.c, fast.c) against the LP64 OpenBLAS shipped inside
 * the opencv wheel of this image. It declares exactly the BLAS entry points
 * the reference calls (src/ops.c:113-147,633-638, src/model.c:535-803,
 * src/fast.c:196-294) with the standard CBLAS enum values.
 *
 * Test infrastructure only: nothing in the product links this.
 */
#ifndef ORACLE_SHIM_CBLAS_H
#define ORACLE_SHIM_CBLAS_H
#ifdef __cplusplus
extern "C" {
#endif
typedef enum { CblasRowMajor = 101, CblasColMajor = 102 } CBLAS_ORDER;
typedef enum { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 } CBLAS_TRANSPOSE;
typedef CBLAS_ORDER CBLAS_LAYOUT;
void cblas_sgemm(CBLAS_ORDER order, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb,
                 int M, int N, int K, float alpha, const float *A, int lda,
                 const float *B, int ldb, float beta, float *C, int ldc);
void cblas_saxpy(int n, float alpha, const float *x, int incx, float *y, int incy);
float cblas_snrm2(int n, const float *x, int incx);
void cblas_sscal(int n, float alpha, float *x, int incx);
int openblas_get_num_threads(void);
void openblas_set_num_threads(int n);
#ifdef __cplusplus
}
#endif
#endif
