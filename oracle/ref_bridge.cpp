// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// extern "C" bridge over the reference's own C++ entry points, compiled
// together with the reference sources into oracle/_ref/libdnnopt_ref.so.
// Python (tests/golden/make_golden.py and bench.py's reference arm) binds
// these with ctypes.  Every function forwards to the reference unchanged.
#include "dnnopt/gemm/gemm.h"
#include "dnnopt/gemm/gemm_types.h"
#include "dnnopt/blas/cblas.h"
#include "dnnopt/conv/conv3d.h"

#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

extern "C" {

// dnnopt::gemm_fp32 with GemmAlgo::kNaive  (reference src/gemm/gemm.cpp:175-186)
void ref_gemm_fp32_naive(int M, int N, int K, float alpha, const float* A, int lda,
                         const float* B, int ldb, float beta, float* C, int ldc) {
    dnnopt::gemm_fp32(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, dnnopt::GemmAlgo::kNaive);
}

// dnnopt::gemm_fp32 default overload (reference src/gemm/gemm.cpp:168-173).
void ref_gemm_fp32(int M, int N, int K, float alpha, const float* A, int lda,
                   const float* B, int ldb, float beta, float* C, int ldc) {
    dnnopt::gemm_fp32(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

// dnnopt::gemm_int8_int8int8int32 (reference src/gemm/gemm_int8_native.cpp:189-248).
void ref_gemm_int8_int8int8int32(int M, int N, int K, const int8_t* A, int lda,
                                 const int8_t* B, int ldb, int32_t* C, int ldc) {
    dnnopt::gemm_int8_int8int8int32(M, N, K, A, lda, B, ldb, C, ldc);
}

// dnnopt::gemm_bf16 / gemm_int8 FP32-API (reference src/gemm/gemm.cpp:379-455).
void ref_gemm_bf16(int M, int N, int K, float alpha, const float* A, int lda,
                   const float* B, int ldb, float beta, float* C, int ldc) {
    dnnopt::gemm_bf16(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}
void ref_gemm_int8(int M, int N, int K, float alpha, const float* A, int lda,
                   const float* B, int ldb, float beta, float* C, int ldc) {
    dnnopt::gemm_int8(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

// FP8 API (reference src/gemm/gemm_fp8.cpp:32-146).
void ref_gemm_fp8_e4m3(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                       const uint8_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt::gemm_fp8_e4m3(M, N, K, alpha, reinterpret_cast<const dnnopt::fp8_e4m3_t*>(A), lda,
                          reinterpret_cast<const dnnopt::fp8_e5m2_t*>(B), ldb, beta, C, ldc);
}
void ref_gemm_fp8_e5m2(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                       const uint8_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt::gemm_fp8_e5m2(M, N, K, alpha, reinterpret_cast<const dnnopt::fp8_e5m2_t*>(A), lda,
                          reinterpret_cast<const dnnopt::fp8_e5m2_t*>(B), ldb, beta, C, ldc);
}
void ref_gemm_fp8(int M, int N, int K, float alpha, const float* A, int lda,
                  const float* B, int ldb, float beta, float* C, int ldc) {
    dnnopt::gemm_fp8(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}
int ref_has_fp8_support(void) { return dnnopt::has_fp8_support() ? 1 : 0; }

// Scalar codecs of include/dnnopt/gemm/gemm_types.h (header-only in the reference).
uint16_t ref_bf16_from_f32(float f) { return dnnopt::bfloat16_t(f).raw_bits; }
float ref_bf16_to_f32(uint16_t r) { return (float)dnnopt::bfloat16_t(r, true); }
uint8_t ref_e4m3_from_f32(float f) { return dnnopt::fp8_e4m3_t(f).raw_bits; }
float ref_e4m3_to_f32(uint8_t r) { return (float)dnnopt::fp8_e4m3_t(r, true); }
uint8_t ref_e5m2_from_f32(float f) { return dnnopt::fp8_e5m2_t(f).raw_bits; }
float ref_e5m2_to_f32(uint8_t r) { return (float)dnnopt::fp8_e5m2_t(r, true); }

// The reference tests' generator: std::mt19937(seed) + uniform_real(-1,1)
// (reference tests/test_gemm_correctness.cpp:20-24, tests/test_cblas.cpp:22-26).
void ref_fill_random(float* data, size_t n, unsigned seed) {
    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    for (size_t i = 0; i < n; ++i) data[i] = dist(gen);
}

// CPU-baseline helper: run the reference's own kernels on column slices of C
// from `threads` host threads.  Each slice is one unmodified reference call
// (same arithmetic per element), so the result equals the single call's.
void ref_gemm_fp32_naive_mt(int M, int N, int K, float alpha, const float* A, int lda,
                            const float* B, int ldb, float beta, float* C, int ldc,
                            int threads) {
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    int chunk = (N + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        int j0 = t * chunk, j1 = std::min(N, j0 + chunk);
        if (j0 >= j1) break;
        pool.emplace_back([=] {
            dnnopt::gemm_fp32(M, j1 - j0, K, alpha, A, lda, B + j0, ldb, beta, C + j0, ldc,
                              dnnopt::GemmAlgo::kNaive);
        });
    }
    for (auto& th : pool) th.join();
}

void ref_gemm_int8_int8int8int32_mt(int M, int N, int K, const int8_t* A, int lda,
                                    const int8_t* B, int ldb, int32_t* C, int ldc,
                                    int threads) {
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    int chunk = (N + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        int j0 = t * chunk, j1 = std::min(N, j0 + chunk);
        if (j0 >= j1) break;
        // B is [N, K]: a column slice of C is a row slice of B.
        pool.emplace_back([=] {
            dnnopt::gemm_int8_int8int8int32(M, j1 - j0, K, A, lda, B + (size_t)j0 * ldb, ldb,
                                            C + j0, ldc);
        });
    }
    for (auto& th : pool) th.join();
}

// dnnopt::conv3d_fp32 / conv3d_bf16 / conv3d_int8 (reference
// src/conv/conv3d.cpp:151-192, :290-345, :460-525).  p: N, IC, ID, IH, IW, OC,
// KD, KH, KW, stride d/h/w, pad d/h/w.  precision 0/1/2 = fp32/bf16/int8; on
// an x86 host the reference's bf16 and int8 entries fall back to conv3d_fp32.
void ref_conv3d(int precision, const int* p, const float* input, const float* filter,
                const float* bias, float* output, int post_op) {
    dnnopt::Conv3DParams c;
    c.N = p[0]; c.IC = p[1]; c.ID = p[2]; c.IH = p[3]; c.IW = p[4];
    c.OC = p[5]; c.KD = p[6]; c.KH = p[7]; c.KW = p[8];
    c.stride_d = p[9]; c.stride_h = p[10]; c.stride_w = p[11];
    c.pad_d = p[12]; c.pad_h = p[13]; c.pad_w = p[14];
    const auto op = static_cast<dnnopt::Conv3DPostOp>(post_op);
    if (precision == 1) dnnopt::conv3d_bf16(c, input, filter, bias, output, op);
    else if (precision == 2) dnnopt::conv3d_int8(c, input, filter, bias, output, op);
    else dnnopt::conv3d_fp32(c, input, filter, bias, output, op);
}

}  // extern "C"
