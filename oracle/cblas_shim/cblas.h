/* Minimal CBLAS prototypes so the reference's CPU ops (src/cpu_ops.cpp) can be
 * compiled here against the OpenBLAS shared library shipped in the image,
 * which has no cblas.h.  Test infrastructure only.  The enum values are the
 * ones fixed by the CBLAS standard interface. */
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemv(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE trans, int m, int n,
                 float alpha, const float* a, int lda, const float* x, int incx,
                 float beta, float* y, int incy);
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float* a, int lda,
                 const float* b, int ldb, float beta, float* c, int ldc);
void openblas_set_num_threads(int n);
int openblas_get_num_threads(void);
#ifdef __cplusplus
}
#endif
