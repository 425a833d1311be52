/* dnnopt/blas/cblas.h -- CBLAS / Fortran BLAS subset exported by
 * libdnnopt_blas.so (same ABI as the reference's include/dnnopt/blas/cblas.h:
 * enum values 101/102 and 111/112/113, cblas_sgemm, cblas_saxpy, OpenBLAS
 * thread control).  Backed by the B200 GEMM: transposes and column-major
 * order are handled inside the kernels, no transposed copies are made. */
#ifndef DNNOPT_BLAS_CBLAS_H
#define DNNOPT_BLAS_CBLAS_H

#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void cblas_sgemm(enum CBLAS_ORDER Order, enum CBLAS_TRANSPOSE TransA, enum CBLAS_TRANSPOSE TransB,
                 int M, int N, int K, float alpha, const float* A, int lda, const float* B, int ldb,
                 float beta, float* C, int ldc);
void cblas_saxpy(int N, float alpha, const float* X, int incX, float* Y, int incY);

void sgemm_(const char* transa, const char* transb, const int* m, const int* n, const int* k,
            const float* alpha, const float* a, const int* lda, const float* b, const int* ldb,
            const float* beta, float* c, const int* ldc);
void SGEMM(const char* transa, const char* transb, const int* m, const int* n, const int* k,
           const float* alpha, const float* a, const int* lda, const float* b, const int* ldb,
           const float* beta, float* c, const int* ldc);

void openblas_set_num_threads(int num_threads);
int openblas_get_num_threads(void);
void blas_set_num_threads(int num_threads);
void omp_set_num_threads_blas(int num_threads);

#ifdef __cplusplus
}
#endif
#endif
