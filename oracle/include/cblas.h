/* Prototype-only CBLAS header for building the reference CPU oracle against the OpenBLAS
 * shared library that ships inside the Python environment (no system cblas.h exists here).
 * Declares only the two entry points the reference's CPU kernels call. Test infrastructure. */
#ifndef ORACLE_CBLAS_PROTO_H
#define ORACLE_CBLAS_PROTO_H
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb, int m, int n, int k,
                 float alpha, const float* a, int lda, const float* b, int ldb, float beta, float* c, int ldc);
void openblas_set_num_threads(int n);
#ifdef __cplusplus
}
#endif
#endif
