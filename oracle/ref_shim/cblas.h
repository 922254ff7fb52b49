/* Minimal CBLAS prototype so the reference's ds_kernels.c (USE_BLAS) compiles
 * against the OpenBLAS 0.3.15 shared library bundled in this image.
 * Test infrastructure only. */
#ifndef DS_REF_CBLAS_SHIM_H
#define DS_REF_CBLAS_SHIM_H
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int M, int N, int K, float alpha, const float *A, int lda,
                 const float *B, int ldb, float beta, float *C, int ldc);
void openblas_set_num_threads(int n);
#endif
