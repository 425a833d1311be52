// dnnopt:: C++ API with the reference's signatures (include/dnnopt/gemm/gemm.h),
// forwarding to the C ABI.  Each function returns void like the reference; the
// status is recorded for dnnopt_get_last_error().
#include "dnnopt/gemm/gemm.h"
#include "dnnopt_b200.h"

namespace dnnopt {

void gemm_fp32(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_fp32(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

// Every GemmAlgo runs the GPU plan selector: the reference's algorithm ids name
// ARM micro-kernels that have no meaning on B200 (src/gemm/gemm.cpp:175-377).
void gemm_fp32(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc, GemmAlgo) {
    dnnopt_gemm_fp32(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

void gemm_bf16(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_bf16(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

void gemm_bf16_bf16bf16f32(int M, int N, int K, float alpha, const bfloat16_t* A, int lda,
                           const bfloat16_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_bf16_bf16bf16f32(M, N, K, alpha, reinterpret_cast<const uint16_t*>(A), lda,
                                 reinterpret_cast<const uint16_t*>(B), ldb, beta, C, ldc);
}

void gemm_int8(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
               int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_int8(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

void gemm_int8_int8int8int32(int M, int N, int K, const int8_t* A, int lda, const int8_t* B,
                             int ldb, int32_t* C, int ldc) {
    dnnopt_gemm_int8_int8int8int32(M, N, K, A, lda, B, ldb, C, ldc);
}

void gemm_fp8_e4m3(int M, int N, int K, float alpha, const fp8_e4m3_t* A, int lda,
                   const fp8_e5m2_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_fp8_e4m3(M, N, K, alpha, reinterpret_cast<const uint8_t*>(A), lda,
                         reinterpret_cast<const uint8_t*>(B), ldb, beta, C, ldc);
}

void gemm_fp8_e5m2(int M, int N, int K, float alpha, const fp8_e5m2_t* A, int lda,
                   const fp8_e5m2_t* B, int ldb, float beta, float* C, int ldc) {
    dnnopt_gemm_fp8_e5m2(M, N, K, alpha, reinterpret_cast<const uint8_t*>(A), lda,
                         reinterpret_cast<const uint8_t*>(B), ldb, beta, C, ldc);
}

void gemm_fp8(int M, int N, int K, float alpha, const float* A, int lda, const float* B, int ldb,
              float beta, float* C, int ldc) {
    dnnopt_gemm_fp8(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

bool has_fp8_support() { return dnnopt_has_fp8_support() != 0; }

void gemm_set_num_threads(int n) { dnnopt_gemm_set_num_threads(n); }
int gemm_get_num_threads() { return dnnopt_gemm_get_num_threads(); }

}  // namespace dnnopt

// ---- Conv3D (reference include/dnnopt/conv/conv3d.h) ------------------------
#include "dnnopt/conv/conv3d.h"

namespace dnnopt {

namespace {
dnnopt_conv3d_params to_c(const Conv3DParams& p) {
    dnnopt_conv3d_params c;
    c.N = p.N; c.IC = p.IC; c.ID = p.ID; c.IH = p.IH; c.IW = p.IW;
    c.OC = p.OC; c.KD = p.KD; c.KH = p.KH; c.KW = p.KW;
    c.stride_d = p.stride_d; c.stride_h = p.stride_h; c.stride_w = p.stride_w;
    c.pad_d = p.pad_d; c.pad_h = p.pad_h; c.pad_w = p.pad_w;
    return c;
}
int to_c(Conv3DPostOp op) {
    return op == Conv3DPostOp::kRelu ? DNNOPT_POSTOP_RELU
                                     : (op == Conv3DPostOp::kRelu6 ? DNNOPT_POSTOP_RELU6 : DNNOPT_POSTOP_NONE);
}
}  // namespace

void conv3d_fp32(const Conv3DParams& p, const float* input, const float* filter, const float* bias,
                 float* output, Conv3DPostOp post_op) {
    const dnnopt_conv3d_params c = to_c(p);
    dnnopt_conv3d(DNNOPT_CONV3D_FP32, &c, input, filter, bias, output, to_c(post_op));
}

void conv3d_winograd_3x3x3_s1p1(const Conv3DParams& p, const float* input, const float* filter,
                                float* output) {
    conv3d_fp32(p, input, filter, nullptr, output, Conv3DPostOp::kNone);
}

void conv3d_winograd_dispatch(const Conv3DParams& p, const float* input, const float* filter,
                              const float* bias, float* output, Conv3DPostOp post_op) {
    conv3d_fp32(p, input, filter, bias, output, post_op);
}

void conv3d_bf16(const Conv3DParams& p, const float* input, const float* filter, const float* bias,
                 float* output, Conv3DPostOp post_op) {
    const dnnopt_conv3d_params c = to_c(p);
    dnnopt_conv3d(DNNOPT_CONV3D_BF16, &c, input, filter, bias, output, to_c(post_op));
}

void conv3d_int8(const Conv3DParams& p, const float* input, const float* filter, const float* bias,
                 float* output, Conv3DPostOp post_op) {
    const dnnopt_conv3d_params c = to_c(p);
    dnnopt_conv3d(DNNOPT_CONV3D_INT8, &c, input, filter, bias, output, to_c(post_op));
}

}  // namespace dnnopt
