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

// Grid-stride over groups of four output positions (rows of the column
// matrix, four loads in flight per thread); each row's
// K columns are walked as chunks of V input channels (V = 4 when IC % 4 == 0
// and the input is 16-byte aligned: one 16-byte load and one 16/8/4-byte store
// per chunk), tap-major then channel, so a tap's reads are contiguous in IC
// and the writes contiguous in K.  A thread's (tap, chunk) position advances
// by a fixed step per iteration, so the inner loop has no division.
template <int MODE, int V>   // MODE 0: FP32, 1: BF16 bits, 2: INT8
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
    const int cpr = g.IC / V;                      // chunks per tap
    const int nchunks = taps * cpr;
    const int t0 = threadIdx.x / cpr, c0 = threadIdx.x - t0 * cpr;
    const int dt = kThreads / cpr, dc = kThreads - dt * cpr;
    const int64_t plane = (int64_t)g.IH * g.IW * g.IC;
    // R rows per pass: a thread keeps R independent loads in flight.
    constexpr int R = 4;
    for (int64_t row0 = (int64_t)blockIdx.x * R; row0 < g.M; row0 += (int64_t)gridDim.x * R) {
        int od[R], oh[R], ow[R];
        const float* src[R];
        bool live[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t row = row0 + q;
            live[q] = row < g.M;
            const int64_t rr = live[q] ? row : row0;
            ow[q] = static_cast<int>(rr % g.OW);
            int64_t r = rr / g.OW;
            oh[q] = static_cast<int>(r % g.OH);
            r /= g.OH;
            od[q] = static_cast<int>(r % g.OD);
            src[q] = in + (r / g.OD) * g.ID * plane;
        }
        int t = t0, c = c0;
        for (int j = threadIdx.x; j < nchunks; j += kThreads) {
            const int kd = s_tap[3 * t], kh = s_tap[3 * t + 1], kw = s_tap[3 * t + 2];
            float x[R][V];
#pragma unroll
            for (int q = 0; q < R; ++q) {
#pragma unroll
                for (int v = 0; v < V; ++v) x[q][v] = 0.0f;
                const int id = od[q] * g.sd - g.pd + kd;
                const int ih = oh[q] * g.sh - g.ph + kh;
                const int iw = ow[q] * g.sw - g.pw + kw;
                if (live[q] && id >= 0 && id < g.ID && ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW) {
                    const float* p = src[q] + id * plane + ((int64_t)ih * g.IW + iw) * g.IC + c * V;
                    if constexpr (V == 4) {
                        const float4 f4 = __ldg(reinterpret_cast<const float4*>(p));
                        x[q][0] = f4.x; x[q][1] = f4.y; x[q][2] = f4.z; x[q][3] = f4.w;
                    } else {
                        x[q][0] = __ldg(p);
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < R; ++q) {
                if (!live[q]) continue;
                const int64_t o = (row0 + q) * g.K + (int64_t)t * g.IC + c * V;
                if constexpr (MODE == 0) {
                    if constexpr (V == 4) *reinterpret_cast<float4*>(static_cast<float*>(col) + o) = make_float4(x[q][0], x[q][1], x[q][2], x[q][3]);
                    else static_cast<float*>(col)[o] = x[q][0];
                } else if constexpr (MODE == 1) {
                    if constexpr (V == 4) {
                        const uint32_t lo = f32_to_bf16_bits_ref(x[q][0]) | (static_cast<uint32_t>(f32_to_bf16_bits_ref(x[q][1])) << 16);
                        const uint32_t hi = f32_to_bf16_bits_ref(x[q][2]) | (static_cast<uint32_t>(f32_to_bf16_bits_ref(x[q][3])) << 16);
                        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(col) + o) = make_uint2(lo, hi);
                    } else {
                        static_cast<uint16_t*>(col)[o] = f32_to_bf16_bits_ref(x[q][0]);
                    }
                } else {
                    if constexpr (V == 4) {
                        uint32_t w = 0;
#pragma unroll
                        for (int v = 0; v < 4; ++v) w |= static_cast<uint32_t>(static_cast<uint8_t>(quant8(x[q][v], inv))) << (8 * v);
                        *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(col) + o) = w;
                    } else {
                        static_cast<int8_t*>(col)[o] = quant8(x[q][0], inv);
                    }
                }
            }
            t += dt;
            c += dc;
            if (c >= cpr) { c -= cpr; ++t; }
        }
    }
}

// im2col of an input already converted to the GEMM precision T (BF16 bits or
// INT8): the same walk as im2col3d_kernel, but every chunk is 16 bytes of one
// tap's channels (IC a multiple of 16 / sizeof(T)) copied as is, so the
// conversion runs once per input element instead of once per tap.  The block
// is sized to a row's chunk count (rounded up to a warp), not a fixed 256, so
// short INT8 rows (K / 16 chunks) leave few threads idle.
template <typename T>
__global__ void __launch_bounds__(kThreads) im2col3d_copy_kernel(const Conv3dGeom g, const T* __restrict__ in,
                                                                 T* __restrict__ col) {
    constexpr int V = 16 / static_cast<int>(sizeof(T));
    __shared__ int s_tap[3 * kConv3dMaxTaps];
    const int taps = g.KD * g.KH * g.KW;
    const int nt = static_cast<int>(blockDim.x);   // a multiple of 32, at most kThreads
    for (int t = threadIdx.x; t < taps; t += nt) {
        const int kw = t % g.KW, r = t / g.KW;
        s_tap[3 * t] = r / g.KH;
        s_tap[3 * t + 1] = r % g.KH;
        s_tap[3 * t + 2] = kw;
    }
    __syncthreads();
    const int cpr = g.IC / V;
    const int nchunks = taps * cpr;
    const int t0 = threadIdx.x / cpr, c0 = threadIdx.x - t0 * cpr;
    const int dt = nt / cpr, dc = nt - dt * cpr;
    const int64_t plane = (int64_t)g.IH * g.IW * g.IC;
    constexpr int R = 4;
    for (int64_t row0 = (int64_t)blockIdx.x * R; row0 < g.M; row0 += (int64_t)gridDim.x * R) {
        int od[R], oh[R], ow[R];
        const T* src[R];
        bool live[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t row = row0 + q;
            live[q] = row < g.M;
            const int64_t rr = live[q] ? row : row0;
            ow[q] = static_cast<int>(rr % g.OW);
            int64_t r = rr / g.OW;
            oh[q] = static_cast<int>(r % g.OH);
            r /= g.OH;
            od[q] = static_cast<int>(r % g.OD);
            src[q] = in + (r / g.OD) * g.ID * plane;
        }
        int t = t0, c = c0;
        for (int j = threadIdx.x; j < nchunks; j += nt) {
            const int kd = s_tap[3 * t], kh = s_tap[3 * t + 1], kw = s_tap[3 * t + 2];
            int4 x[R];
#pragma unroll
            for (int q = 0; q < R; ++q) {
                x[q] = make_int4(0, 0, 0, 0);
                const int id = od[q] * g.sd - g.pd + kd;
                const int ih = oh[q] * g.sh - g.ph + kh;
                const int iw = ow[q] * g.sw - g.pw + kw;
                if (live[q] && id >= 0 && id < g.ID && ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW)
                    x[q] = __ldg(reinterpret_cast<const int4*>(src[q] + id * plane +
                                                               ((int64_t)ih * g.IW + iw) * g.IC + c * V));
            }
#pragma unroll
            for (int q = 0; q < R; ++q)
                if (live[q])
                    *reinterpret_cast<int4*>(col + (row0 + q) * g.K + (int64_t)t * g.IC + c * V) = x[q];
            t += dt;
            c += dc;
            if (c >= cpr) { c -= cpr; ++t; }
        }
    }
}

// Filter [OC, K] or input in the GEMM precision: BF16 (RNE) or INT8 (times
// 1/s = scales[inv_idx]: 3 for the filter, 2 for the input).
template <int MODE>
__global__ void conv3d_filter_kernel(const float* __restrict__ f, void* out, int64_t n, const float* scales,
                                     int inv_idx) {
    const float inv = MODE == 2 ? scales[inv_idx] : 1.0f;
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
    // One atomic per CTA and value (per-warp atomics on the same two words
    // serialise in L2).
    __shared__ uint32_t s_m[2][kThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { s_m[0][warp] = m0; s_m[1][warp] = m1; }
    __syncthreads();
    if (warp == 0) {
        const int nw = static_cast<int>(blockDim.x >> 5);
        m0 = lane < nw ? s_m[0][lane] : 0u;
        m1 = lane < nw ? s_m[1][lane] : 0u;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            m0 = max(m0, __shfl_xor_sync(0xFFFFFFFFu, m0, o));
            m1 = max(m1, __shfl_xor_sync(0xFFFFFFFFu, m1, o));
        }
        if (lane == 0) {
            atomicMax(&bits[0], m0);
            atomicMax(&bits[1], m1);
        }
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

// The scales from the absmax bits (as conv3d_scales_kernel computes them),
// then input and filter quantised in one grid-stride pass; block 0 also stores
// the scales for the GEMM's dequantising epilogue.
__global__ void conv3d_quant_both_kernel(const float* __restrict__ in, int64_t nin, const float* __restrict__ f,
                                         int64_t nf, const uint32_t* bits, float* scales, int8_t* inq,
                                         int8_t* fq) {
    const float m0 = __uint_as_float(bits[0]), m1 = __uint_as_float(bits[1]);
    const float s0 = m0 == 0.0f ? 1.0f : __fdiv_rn(m0, 127.0f);
    const float s1 = m1 == 0.0f ? 1.0f : __fdiv_rn(m1, 127.0f);
    const float inv0 = __fdiv_rn(1.0f, s0), inv1 = __fdiv_rn(1.0f, s1);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        scales[0] = s0;
        scales[1] = s1;
        scales[2] = inv0;
        scales[3] = inv1;
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nin + nf; i += (int64_t)gridDim.x * blockDim.x) {
        if (i < nin) inq[i] = quant8(in[i], inv0);
        else fq[i - nin] = quant8(f[i - nin], inv1);
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
    const int64_t passes = (g.M + 3) / 4;   // four rows per CTA pass
    const int grid = static_cast<int>(passes < 148 * 16 ? passes : 148 * 16);
    const bool v4 = g.IC % 4 == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0;
    switch (mode * 2 + (v4 ? 1 : 0)) {
        case 0: im2col3d_kernel<0, 1><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        case 1: im2col3d_kernel<0, 4><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        case 2: im2col3d_kernel<1, 1><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        case 3: im2col3d_kernel<1, 4><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        case 4: im2col3d_kernel<2, 1><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        case 5: im2col3d_kernel<2, 4><<<grid, kThreads, 0, s>>>(g, in, col, scales); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_conv3d_filter(int mode, const float* f, void* out, int64_t n, const float* scales,
                                 cudaStream_t s, int inv_idx) {
    if (mode == 1) conv3d_filter_kernel<1><<<grid_for(n), kThreads, 0, s>>>(f, out, n, scales, inv_idx);
    else if (mode == 2) conv3d_filter_kernel<2><<<grid_for(n), kThreads, 0, s>>>(f, out, n, scales, inv_idx);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

bool conv3d_copy_im2col_ok(const Conv3dGeom& g, int mode) {
    const int v = mode == 1 ? 8 : (mode == 2 ? 16 : 0);
    return v > 0 && g.IC % v == 0 && g.KD * g.KH * g.KW <= kConv3dMaxTaps;
}

cudaError_t launch_conv3d_im2col_copy(const Conv3dGeom& g, int mode, const void* in_conv, void* col,
                                      cudaStream_t s) {
    if (!conv3d_copy_im2col_ok(g, mode) || reinterpret_cast<uintptr_t>(in_conv) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(col) % 16 != 0)
        return cudaErrorInvalidValue;
    const int64_t nchunks = g.K * (mode == 1 ? 2 : 1) / 16;
    const int threads = static_cast<int>(nchunks >= kThreads ? kThreads : (nchunks + 31) / 32 * 32);
    const int64_t passes = (g.M + 3) / 4;
    const int64_t cap = 148LL * 16 * (kThreads / threads);
    const int grid = static_cast<int>(passes < cap ? passes : cap);
    if (mode == 1)
        im2col3d_copy_kernel<uint16_t><<<grid, threads, 0, s>>>(g, static_cast<const uint16_t*>(in_conv),
                                                                static_cast<uint16_t*>(col));
    else
        im2col3d_copy_kernel<int8_t><<<grid, threads, 0, s>>>(g, static_cast<const int8_t*>(in_conv),
                                                              static_cast<int8_t*>(col));
    return cudaGetLastError();
}

cudaError_t launch_conv3d_scales(const float* in, int64_t nin, const float* f, int64_t nf, uint32_t* bits,
                                 float* scales, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(bits, 0, 2 * sizeof(uint32_t), s);
    if (e != cudaSuccess) return e;
    const int64_t blocks = (nin + nf + 4 * kThreads - 1) / (4 * kThreads);
    const int grid = static_cast<int>(blocks < 148 * 4 ? (blocks > 0 ? blocks : 1) : 148 * 4);
    conv3d_absmax_kernel<<<grid, kThreads, 0, s>>>(in, nin, f, nf, bits);
    conv3d_scales_kernel<<<1, 32, 0, s>>>(bits, scales);
    return cudaGetLastError();
}

cudaError_t launch_conv3d_absmax_quant(const float* in, int64_t nin, const float* f, int64_t nf, uint32_t* bits,
                                       float* scales, int8_t* inq, int8_t* fq, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(bits, 0, 2 * sizeof(uint32_t), s);
    if (e != cudaSuccess) return e;
    const int64_t blocks = (nin + nf + 4 * kThreads - 1) / (4 * kThreads);
    const int grid = static_cast<int>(blocks < 148 * 4 ? (blocks > 0 ? blocks : 1) : 148 * 4);
    conv3d_absmax_kernel<<<grid, kThreads, 0, s>>>(in, nin, f, nf, bits);
    conv3d_quant_both_kernel<<<grid_for(nin + nf), kThreads, 0, s>>>(in, nin, f, nf, bits, scales, inq, fq);
    return cudaGetLastError();
}

cudaError_t launch_conv3d_post(float* out, const int32_t* acc, const float* scales, const float* bias,
                               int64_t M, int OC, int op, cudaStream_t s) {
    conv3d_post_kernel<<<grid_for(M * OC), kThreads, 0, s>>>(out, acc, scales, bias, M, OC, op);
    return cudaGetLastError();
}

}  // namespace dnnopt_b200
