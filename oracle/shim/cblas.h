/*
 * Minimal CBLAS declaration used only to build the reference CPU oracle
 * (oracle/_ref) against the OpenBLAS shared object bundled in the Python
 * environment, which ships without headers.  Test infrastructure only.
 *
 * The reference calls exactly one BLAS routine on its hot path:
 * cblas_sgemm (iris_kernels.c:262-265, iris_transformer_flux.c:1734-1769).
 */
#ifndef IRIS_ORACLE_CBLAS_SHIM_H
#define IRIS_ORACLE_CBLAS_SHIM_H

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float *a, int lda,
                 const float *b, int ldb, float beta, float *c, int ldc);
void openblas_set_num_threads(int num_threads);
int openblas_get_num_threads(void);

#endif
