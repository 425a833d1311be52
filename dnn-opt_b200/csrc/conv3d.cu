// Conv3D as an im2col GEMM on the device: the B200 replacement of the
// reference's conv3d_fp32 / conv3d_bf16 / conv3d_int8 (src/conv/conv3d.cpp),
// the in-tree caller of its FP32, BF16 and INT8 GEMM entries.
//
//   input  [N, ID, IH, IW, IC] (NDHWC), filter [OC, KD, KH, KW, IC],
//   output [N, OD, OH, OW, OC] = im2col(input) [M, K] x filter^T + bias, post-op
//
// with M = N*OD*OH*OW and K = KD*KH*KW*IC.  The column matrix is written once
// in the GEMM's input precision (FP32; BF16 rounded to nearest even as the
// reference's ARM path converts it; INT8 quantised with the per-tensor scale,
// im2col3d_nhwc_int8 :389-457 on the quantised input), the filter is already
// the GEMM's N x K operand, and the library's GEMM entries do the rest (the
// BF16 one on the tcgen05 tall-skinny kernel when OC <= 256).  Bias, the INT8
// dequantisation and relu / relu6 follow in one elementwise pass with the
// reference's rounding order (apply_conv3d_postops :126-148).
#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int kThreads = 256;

// Reference round-half-away quantisation (quantize_fp32_to_int8_3d :366-377).
__device__ __forceinline__ int8_t quant8(float x, float inv) {
    int q = static_cast<int>(roundf(x * inv));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    return static_cast<int8_t>(q);
}

// One CTA per output position (row of the column matrix); threads walk its K
// columns, tap-major then input channel, so reads of a tap are contiguous in
// IC and writes contiguous in K.
template <int MODE>   // 0: FP32, 1: BF16 bits, 2: INT8
__global__ void __launch_bounds__(kThreads) im2col3d_kernel(const Conv3dGeom g, const float* __restrict__ in,
                                                            void* col, const float* scales) {
    __shared__ int s_tap[3 * kConv3dMaxTaps];
    const int taps = g.KD * g.KH * g.KW;
    for (int t = threadIdx.x; t < taps; t += kThreads) {
        const int kw = t % g.KW, r = t / g.KW;
        s_tap[3 * t] = r / g.KH;
        s_tap[3 * t + 1] = r % g.KH;
        s_tap[3 * t + 2] = kw;
    }
    __syncthreads();
    const float inv = MODE == 2 ? scales[2] : 1.0f;
    for (int64_t row = blockIdx.x; row < g.M; row += gridDim.x) {
        const int ow = static_cast<int>(row % g.OW);
        int64_t r = row / g.OW;
        const int oh = static_cast<int>(r % g.OH);
        r /= g.OH;
        const int od = static_cast<int>(r % g.OD);
        const int n = static_cast<int>(r / g.OD);
        for (int k = threadIdx.x; k < g.K; k += kThreads) {
            const int t = k / g.IC, ic = k - t * g.IC;
            const int id = od * g.sd - g.pd + s_tap[3 * t];
            const int ih = oh * g.sh - g.ph + s_tap[3 * t + 1];
            const int iw = ow * g.sw - g.pw + s_tap[3 * t + 2];
            float x = 0.0f;
            if (id >= 0 && id < g.ID && ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW)
                x = in[((((int64_t)n * g.ID + id) * g.IH + ih) * g.IW + iw) * g.IC + ic];
            const int64_t o = row * g.K + k;
            if constexpr (MODE == 0) static_cast<float*>(col)[o] = x;
            else if constexpr (MODE == 1) static_cast<uint16_t*>(col)[o] = f32_to_bf16_bits_ref(x);
            else static_cast<int8_t*>(col)[o] = quant8(x, inv);
        }
    }
}

// Filter [OC, K] in the GEMM precision: BF16 (RNE) or INT8 (scale scales[1]).
template <int MODE>
__global__ void conv3d_filter_kernel(const float* __restrict__ f, void* out, int64_t n, const float* scales) {
    const float inv = MODE == 2 ? scales[3] : 1.0f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if constexpr (MODE == 1) static_cast<uint16_t*>(out)[i] = f32_to_bf16_bits_ref(f[i]);
        else static_cast<int8_t*>(out)[i] = quant8(f[i], inv);
    }
}

// Per-tensor absmax of input and filter as float bit patterns (non-negative
// floats order like unsigned integers); NaN never wins, as in `a > max`.
__global__ void conv3d_absmax_kernel(const float* __restrict__ in, int64_t nin, const float* __restrict__ f,
                                     int64_t nf, uint32_t* bits) {
    uint32_t m0 = 0, m1 = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nin + nf; i += (int64_t)gridDim.x * blockDim.x) {
        const float a = fabsf(i < nin ? in[i] : f[i - nin]);
        const uint32_t u = a == a ? __float_as_uint(a) : 0u;
        if (i < nin) m0 = u > m0 ? u : m0; else m1 = u > m1 ? u : m1;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        m0 = max(m0, __shfl_xor_sync(0xFFFFFFFFu, m0, o));
        m1 = max(m1, __shfl_xor_sync(0xFFFFFFFFu, m1, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(&bits[0], m0);
        atomicMax(&bits[1], m1);
    }
}

// scales[0..3] = s_in, s_f, 1/s_in, 1/s_f with s = max_abs / 127 (1 when all
// inputs are zero), compute_quant_scale_3d :355-364.
__global__ void conv3d_scales_kernel(const uint32_t* bits, float* scales) {
    if (threadIdx.x < 2) {
        const float m = __uint_as_float(bits[threadIdx.x]);
        const float s = m == 0.0f ? 1.0f : __fdiv_rn(m, 127.0f);
        scales[threadIdx.x] = s;
        scales[2 + threadIdx.x] = __fdiv_rn(1.0f, s);
    }
}

// output = post(v + bias[oc]), v = the GEMM result, or float(acc) * (s_in*s_f)
// for INT8 (dequantize_int32_to_fp32_3d :379-386, apply_conv3d_postops).
__global__ void conv3d_post_kernel(float* out, const int32_t* acc, const float* scales, const float* bias,
                                   int64_t M, int OC, int op) {
    const float dq = acc ? __fmul_rn(scales[0], scales[1]) : 1.0f;
    const int64_t n = M * OC;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v = acc ? __fmul_rn(static_cast<float>(acc[i]), dq) : out[i];
        if (bias) v = __fadd_rn(v, bias[i % OC]);
        if (op == 1) v = v > 0.0f ? v : 0.0f;
        else if (op == 2) v = v > 0.0f ? (v < 6.0f ? v : 6.0f) : 0.0f;
        out[i] = v;
    }
}

int grid_for(int64_t n) {
    const int64_t b = (n + kThreads - 1) / kThreads;
    return static_cast<int>(b < 148 * 8 ? (b > 0 ? b : 1) : 148 * 8);
}

}  // namespace

cudaError_t launch_conv3d_im2col(const Conv3dGeom& g, int mode, const float* in, void* col,
                                 const float* scales, cudaStream_t s) {
    if (g.KD * g.KH * g.KW > kConv3dMaxTaps) return cudaErrorInvalidValue;
    const int grid = static_cast<int>(g.M < 148 * 16 ? g.M : 148 * 16);
    switch (mode) {
        case 0: im2col3d_kernel<0><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        case 1: im2col3d_kernel<1><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        case 2: im2col3d_kernel<2><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_conv3d_filter(int mode, const float* f, void* out, int64_t n, const float* scales,
                                 cudaStream_t s) {
    if (mode == 1) conv3d_filter_kernel<1><<<grid_for(n), kThreads, 0, s>>>(f, out, n, scales);
    else if (mode == 2) conv3d_filter_kernel<2><<<grid_for(n), kThreads, 0, s>>>(f, out, n, scales);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_conv3d_scales(const float* in, int64_t nin, const float* f, int64_t nf, uint32_t* bits,
                                 float* scales, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(bits, 0, 2 * sizeof(uint32_t), s);
    if (e != cudaSuccess) return e;
    conv3d_absmax_kernel<<<grid_for(nin + nf), kThreads, 0, s>>>(in, nin, f, nf, bits);
    conv3d_scales_kernel<<<1, 32, 0, s>>>(bits, scales);
    return cudaGetLastError();
}

cudaError_t launch_conv3d_post(float* out, const int32_t* acc, const float* scales, const float* bias,
                               int64_t M, int OC, int op, cudaStream_t s) {
    conv3d_post_kernel<<<grid_for(M * OC), kThreads, 0, s>>>(out, acc, scales, bias, M, OC, op);
    return cudaGetLastError();
}

}  // namespace dnnopt_b200
