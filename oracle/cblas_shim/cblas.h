/* Minimal CBLAS prototypes so the reference's BLAS build (-DUSE_BLAS
 * -DUSE_OPENBLAS) compiles against an OpenBLAS shared object that ships
 * without headers. Only the declarations the reference calls are given. */
#ifndef QDB_CBLAS_SHIM_H
#define QDB_CBLAS_SHIM_H
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float *a, int lda,
                 const float *b, int ldb, float beta, float *c, int ldc);
#endif
