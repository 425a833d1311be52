#pragma once
// dnnopt:: Conv3D API with the reference's declarations (reference
// include/dnnopt/conv/conv3d.h), implemented by libdnnopt_b200.so on the GPU
// (host or device pointers, synchronous; status via dnnopt_get_last_error()).
//
//   input  [N, ID, IH, IW, IC] (NDHWC), filter [OC, KD, KH, KW, IC],
//   bias   [OC] or nullptr,      output [N, OD, OH, OW, OC] (NDHWC).
#include <cstddef>

namespace dnnopt {

struct Conv3DParams {
    int N;
    int IC;
    int ID, IH, IW;
    int OC;
    int KD, KH, KW;
    int stride_d, stride_h, stride_w;
    int pad_d, pad_h, pad_w;

    int OD() const { return (ID + 2 * pad_d - KD) / stride_d + 1; }
    int OH() const { return (IH + 2 * pad_h - KH) / stride_h + 1; }
    int OW() const { return (IW + 2 * pad_w - KW) / stride_w + 1; }
};

enum class Conv3DPostOp {
    kNone,
    kRelu,
    kRelu6,
};

// FP32 Conv3D: im2col + FP32 GEMM, then bias and the post-op.
void conv3d_fp32(const Conv3DParams& p, const float* input, const float* filter, const float* bias,
                 float* output, Conv3DPostOp post_op = Conv3DPostOp::kNone);

// The reference's Winograd F(2x2, 3x3x3) entry points compute the same
// convolution; on the GPU both run the im2col GEMM of conv3d_fp32.
void conv3d_winograd_3x3x3_s1p1(const Conv3DParams& p, const float* input, const float* filter,
                                float* output);
void conv3d_winograd_dispatch(const Conv3DParams& p, const float* input, const float* filter,
                              const float* bias, float* output, Conv3DPostOp post_op);

// BF16 Conv3D: input and filter rounded to bf16, FP32 accumulation.
void conv3d_bf16(const Conv3DParams& p, const float* input, const float* filter, const float* bias,
                 float* output, Conv3DPostOp post_op = Conv3DPostOp::kNone);

// INT8 Conv3D: per-tensor dynamic quantisation, exact int32 sums, dequantised.
void conv3d_int8(const Conv3DParams& p, const float* input, const float* filter, const float* bias,
                 float* output, Conv3DPostOp post_op = Conv3DPostOp::kNone);

}  // namespace dnnopt
