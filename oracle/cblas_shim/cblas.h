/*
 * Minimal CBLAS declarations so the reference tape runner compiles against
 * an OpenBLAS that ships without headers.  Only the two routines the
 * reference calls (T_MATMUL, _tape_runner.c:755-772) are declared, with the
 * public CBLAS enum values.  Test infrastructure only.
 */
#ifndef KLLM_ORACLE_CBLAS_SHIM_H
#define KLLM_ORACLE_CBLAS_SHIM_H
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemv(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE trans, int m, int n,
                 float alpha, const float *a, int lda, const float *x, int incx,
                 float beta, float *y, int incy);
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float *a, int lda,
                 const float *b, int ldb, float beta, float *c, int ldc);
#endif
