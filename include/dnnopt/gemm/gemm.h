// dnnopt/gemm/gemm.h -- drop-in C++ API (same signatures as the reference's
// include/dnnopt/gemm/gemm.h:10-102), implemented by libdnnopt_b200.so on B200.
//
// All matrices are row-major; C = alpha * A * B + beta * C.  Pointers may be
// host or device memory; every call is synchronous (C holds the result on
// return).  The functions return void like the reference; the status of the
// last call on this thread is available from dnnopt_get_last_error()
// (dnnopt_b200.h).  M, N or K <= 0 returns immediately, as in the reference.
#pragma once

#include "dnnopt/gemm/gemm_types.h"

namespace dnnopt {

void gemm_fp32(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc);
void gemm_fp32(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc, GemmAlgo algo);

// FP32 in/out, operands rounded to bf16, FP32 accumulation.
void gemm_bf16(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc);

// bf16 A (M x K) and B (K x N), FP32 C.
void gemm_bf16_bf16bf16f32(int M, int N, int K, float alpha, const bfloat16_t* A, int lda,
                           const bfloat16_t* B, int ldb, float beta, float* C, int ldc);

// FP32 in/out through per-tensor symmetric int8 quantisation.
void gemm_int8(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc);

// int8 A (M x K) and B read as N x K (K contiguous, ldb >= K, as the reference
// implementation reads it), exact int32 C (overwritten).
void gemm_int8_int8int8int32(int M, int N, int K, const int8_t* A, int lda, const int8_t* B,
                             int ldb, int32_t* C, int ldc);

void gemm_fp8_e4m3(int M, int N, int K, float alpha, const fp8_e4m3_t* A, int lda,
                   const fp8_e5m2_t* B, int ldb, float beta, float* C, int ldc);
void gemm_fp8_e5m2(int M, int N, int K, float alpha, const fp8_e5m2_t* A, int lda,
                   const fp8_e5m2_t* B, int ldb, float beta, float* C, int ldc);
void gemm_fp8(int M, int N, int K, float alpha, const float* A, int lda, const float* B, int ldb,
              float beta, float* C, int ldc);
bool has_fp8_support();

void gemm_set_num_threads(int n);
int gemm_get_num_threads();

}  // namespace dnnopt
