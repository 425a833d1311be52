// libdnnopt_blas.so: CBLAS / Fortran sgemm ABI (reference src/blas/*.cpp) on
// top of libdnnopt_b200.so.  Column-major order and transposes become flags of
// the row-major GEMM descriptor (kernels read op(A), op(B) in place), so no
// transposed copies are made, unlike the reference's sgemm_row_major
// (src/blas/cblas_sgemm.cpp:67-99).
#include "dnnopt/blas/cblas.h"
#include "dnnopt_b200.h"

extern "C" {

// Reference semantics (src/blas/cblas_sgemm.cpp:105-143): early return on
// M, N or K <= 0 and on alpha == 0 && beta == 1; ColMajor is reduced to
// RowMajor by C^T = op(B)^T op(A)^T (swap A<->B, M<->N, TransA<->TransB).
void cblas_sgemm(enum CBLAS_ORDER Order, enum CBLAS_TRANSPOSE TransA, enum CBLAS_TRANSPOSE TransB,
                 int M, int N, int K, float alpha, const float* A, int lda, const float* B, int ldb,
                 float beta, float* C, int ldc) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    if (alpha == 0.0f && beta == 1.0f) return;
    dnnopt_gemm_desc d;
    d.K = K;
    d.alpha = alpha;
    d.beta = beta;
    d.ldc = ldc;
    if (Order == CblasRowMajor) {
        d.M = M; d.N = N;
        d.lda = lda; d.ldb = ldb;
        d.trans_a = TransA != CblasNoTrans;
        d.trans_b = TransB != CblasNoTrans;
        dnnopt_gemm_f32_desc(&d, A, B, C);
    } else {
        d.M = N; d.N = M;
        d.lda = ldb; d.ldb = lda;
        d.trans_a = TransB != CblasNoTrans;
        d.trans_b = TransA != CblasNoTrans;
        dnnopt_gemm_f32_desc(&d, B, A, C);
    }
}

void cblas_saxpy(int N, float alpha, const float* X, int incX, float* Y, int incY) {
    dnnopt_saxpy(N, alpha, X, incX, Y, incY);
}

static enum CBLAS_TRANSPOSE parse_trans(const char* t) {
    if (*t == 'T' || *t == 't') return CblasTrans;
    if (*t == 'C' || *t == 'c') return CblasConjTrans;
    return CblasNoTrans;
}

// Fortran BLAS (reference src/blas/blas_fortran.cpp:12-42): column-major,
// arguments by pointer.
void sgemm_(const char* transa, const char* transb, const int* m, const int* n, const int* k,
            const float* alpha, const float* a, const int* lda, const float* b, const int* ldb,
            const float* beta, float* c, const int* ldc) {
    cblas_sgemm(CblasColMajor, parse_trans(transa), parse_trans(transb), *m, *n, *k, *alpha, a,
                *lda, b, *ldb, *beta, c, *ldc);
}

void SGEMM(const char* transa, const char* transb, const int* m, const int* n, const int* k,
           const float* alpha, const float* a, const int* lda, const float* b, const int* ldb,
           const float* beta, float* c, const int* ldc) {
    sgemm_(transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}

// OpenBLAS-style thread control (reference src/blas/blas_utils.cpp:10-24).
void openblas_set_num_threads(int num_threads) { dnnopt_gemm_set_num_threads(num_threads); }
int openblas_get_num_threads(void) { return dnnopt_gemm_get_num_threads(); }
void blas_set_num_threads(int num_threads) { dnnopt_gemm_set_num_threads(num_threads); }
void omp_set_num_threads_blas(int num_threads) { dnnopt_gemm_set_num_threads(num_threads); }

}  // extern "C"
