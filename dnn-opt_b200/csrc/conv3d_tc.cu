// Conv3D (stride 1) as an implicit GEMM on the 5th-generation tensor cores:
// the B200 path of the reference's conv3d_bf16 / conv3d_int8
// (src/conv/conv3d.cpp), which materialise im2col columns
// (im2col3d_nhwc_* :389-457) and call the library GEMMs.  Here the column
// matrix is never written: for each filter tap (kd, kh, kw) and chunk of
// input channels, a TMA box of the NDHWC input, shifted by the tap, is the
// A tile of that K-block, and the hardware's out-of-bounds zero fill is the
// convolution padding.
//
//   output [N, OD, OH, OW, OC] = sum_k A[pixel, k] * filter[oc, k],
//   k = ((kd*KH + kh)*KW + kw)*IC + ic (the reference's column order)
//
// INT8: both operands quantised per tensor first (conv3d_int8's
// quantize_fp32_to_int8_3d :366-377, round half away, clamp), int32
// accumulators in TMEM (exact), dequantisation float(acc) * (s_in*s_f), then
// bias and relu / relu6 in the epilogue with the reference's rounding order
// (dequantize_int32_to_fp32_3d :379-386, apply_conv3d_postops :126-148).
// BF16: operands rounded to bf16 (RNE) once, FP32 accumulators.
//
// Tiles: 128 output positions, a box of bw x bh x bd x bn positions (powers
// of two, product 128; positions past the output are computed and dropped),
// by n_mma <= 256 output channels.  A K-block is cb = 32, 64 or 128 bytes of
// channels of one tap, staged with the matching TMA swizzle straight into the
// UMMA K-major layout.  With one channel tile the whole filter stays resident
// in shared memory (loaded with the CTA's first tile), so the ring streams
// only input boxes, which L2 serves (each input position is read once per
// tap).  Roles as in the general tcgen05 GEMM: warp 0 TMA, warp 1 TMEM +
// MMA issue into two accumulators, warps 2-5 epilogue.  Every mbarrier wait
// is bounded; every TMA load targets this CTA's own shared memory.
#include <cuda.h>

#include <mutex>
#include <set>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kMaxN = 256;
constexpr size_t kSmemCap = 232448;   // 227 KB dynamic shared memory per CTA
constexpr size_t kSmemMin = 120 * 1024;   // keeps one CTA per SM (TMEM of up to 512 columns)
constexpr int kBarBytes = 256;
constexpr int kPartMax = 512;          // absmax partials (CTAs of the first INT8 prep kernel)
constexpr int kPrepThreads = 256;

struct ConvTcParams {
    int N, OD, OH, OW, OC;
    int KH, KW;
    int pd, ph, pw;
    int bw, bh, bd, bn;         // output positions per tile along W, H, D, N
    int tw, th, td;             // tiles along W, H, D
    int m_tiles, n_tiles, units;
    int cb, celems, cpt, num_kb;   // K-block bytes / elements, K-blocks per tap, total
    int n_mma, stages, b_res;
    int i8;                     // 1: kind::i8 (int32 accumulators), 0: kind::f16 (bf16, f32)
    int post;                   // 0 none, 1 relu, 2 relu6
    uint32_t a_bytes, b_bytes;  // one K-block of A (128 rows) and of B (n_mma rows)
    uint32_t stage_bytes, ring_off, bar_off;
    const float* scales;        // INT8: {s_in, s_f}
    const float* bias;
    float* out;
    int out_vec;                // 16-byte output stores (OC % 4 == 0, aligned)
    uint32_t* err;
};

__device__ __forceinline__ void tma_load_5d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t c0,
                                            int32_t c1, int32_t c2, int32_t c3, int32_t c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// K-major shared-memory descriptor for rows of cb bytes in the cb-byte
// swizzled layout (8 rows per atom, atoms 8*cb bytes apart): layout code 2
// (128 B), 4 (64 B) or 6 (32 B) at bits 61-63, version 1 at bit 46.
__device__ __forceinline__ uint64_t desc_k_swizzled(uint32_t addr, int cb) {
    const uint64_t layout = cb == 128 ? 2u : (cb == 64 ? 4u : 6u);
    uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>((8u * static_cast<uint32_t>(cb)) >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= layout << 61;
    return d;
}

// Instruction descriptor: D S32 (i8) or F32 (bf16) at bits 4-5, A / B signed
// 8-bit or BF16 (1) at 7-9 / 10-12, both K-major, N >> 3 at 17, M >> 4 at 24.
__device__ __forceinline__ uint32_t conv_idesc(int i8, int n) {
    return ((i8 ? 2u : 1u) << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ float conv_post(float v, const float* bias, int oc, int post) {
    if (bias) v = __fadd_rn(v, __ldg(bias + oc));
    if (post == 1) v = v > 0.0f ? v : 0.0f;
    else if (post == 2) v = v > 0.0f ? (v < 6.0f ? v : 6.0f) : 0.0f;
    return v;
}

__global__ void __launch_bounds__(kThreads, 1)
conv3d_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const ConvTcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* bres = base;                       // resident filter: num_kb x b_bytes (b_res)
    uint8_t* ring = base + p.ring_off;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + p.bar_off);
    uint64_t* empty = full + kMaxStages;
    uint64_t* tfull = empty + kMaxStages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t need = static_cast<uint32_t>(2 * p.n_mma);
    const uint32_t tmem_cols = need <= 32 ? 32u : (need <= 64 ? 64u : (need <= 128 ? 128u : (need <= 256 ? 256u : 512u)));

    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
        *abort_flag = 0u;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();   // the quantised / converted operands come from the previous launch

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t it = 0;
            bool first = true;
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
                const int mt = u % p.m_tiles, nt = u / p.m_tiles;
                int r = mt;
                const int iw = r % p.tw; r /= p.tw;
                const int ih = r % p.th; r /= p.th;
                const int id = r % p.td;
                const int in = r / p.td;
                const int x1 = iw * p.bw - p.pw, x2 = ih * p.bh - p.ph, x3 = id * p.bd - p.pd, x4 = in * p.bn;
                const bool load_b = !p.b_res || first;
                int c = 0, kw = 0, kh = 0, kd = 0;
                bool ok = true;
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    uint8_t* sa = ring + s * p.stage_bytes;
                    mbar_arrive_expect_tx(&full[s], p.a_bytes + (load_b ? p.b_bytes : 0u));
                    tma_load_5d(sa, &tmA, &full[s], c * p.celems, x1 + kw, x2 + kh, x3 + kd, x4);
                    if (load_b)
                        tma_load_2d(p.b_res ? bres + static_cast<uint32_t>(kb) * p.b_bytes : sa + p.a_bytes, &tmB,
                                    &full[s], kb * p.celems, nt * p.n_mma);
                    if (++c == p.cpt) {
                        c = 0;
                        if (++kw == p.KW) {
                            kw = 0;
                            if (++kh == p.KH) { kh = 0; ++kd; }
                        }
                    }
                }
                if (!ok) break;
                first = false;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = conv_idesc(p.i8, p.n_mma);
            const int ksteps = p.cb / 32;   // 32 bytes of K per MMA (K = 32 int8 or 16 bf16)
            uint32_t it = 0, titer = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++titer) {
                const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
                if (!mbar_wait(&tempty[buf], tph ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * static_cast<uint32_t>(p.n_mma);
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
                    if (!mbar_wait(&full[s], ph, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(ring + s * p.stage_bytes);
                    const uint32_t b_addr = p.b_res ? smem_u32(bres) + static_cast<uint32_t>(kb) * p.b_bytes
                                                    : a_addr + p.a_bytes;
                    for (int kk = 0; kk < ksteps; ++kk) {
                        const uint64_t da = desc_k_swizzled(a_addr + kk * 32, p.cb);
                        const uint64_t db = desc_k_swizzled(b_addr + kk * 32, p.cb);
                        if (p.i8) umma_i8(d_tmem, da, db, idesc, (kb | kk) != 0);
                        else umma_f16_ss(d_tmem, da, db, idesc, (kb | kk) != 0);
                    }
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;            // TMEM lanes 32q .. 32q+31
        const int row_in = q * 32 + lane;
        const int ww = row_in % p.bw;
        const int hh = (row_in / p.bw) % p.bh;
        const int dd = (row_in / (p.bw * p.bh)) % p.bd;
        const int nn = row_in / (p.bw * p.bh * p.bd);
        const float dq = p.i8 ? __fmul_rn(p.scales[0], p.scales[1]) : 1.0f;
        uint32_t titer = 0;
        for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x, ++titer) {
            const int mt = u % p.m_tiles, nt = u / p.m_tiles;
            int r = mt;
            const int iw = r % p.tw; r /= p.tw;
            const int ih = r % p.th; r /= p.th;
            const int id = r % p.td;
            const int in = r / p.td;
            const int ow = iw * p.bw + ww, oh = ih * p.bh + hh, od = id * p.bd + dd, on = in * p.bn + nn;
            const bool live = ow < p.OW && oh < p.OH && od < p.OD && on < p.N;
            const int64_t pix = ((static_cast<int64_t>(on) * p.OD + od) * p.OH + oh) * p.OW + ow;
            float* orow = p.out + pix * p.OC;
            const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
            const bool ok = mbar_wait_warp(&tfull[buf], tph, abort_flag, p.err);
            tc_fence_after();
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * static_cast<uint32_t>(p.n_mma);
            const int col0 = nt * p.n_mma;
            for (int c0 = 0; c0 < p.n_mma; c0 += 32) {
                if (col0 + c0 >= p.OC) break;   // uniform across the warp
                uint32_t v[32];
                tmem_ld_32x32b_x16(t_addr + c0, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                tmem_ld_32x32b_x16(t_addr + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                tmem_ld_wait();
                if (!ok || !live) continue;
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float a = p.i8 ? __fmul_rn(static_cast<float>(static_cast<int32_t>(v[j])), dq)
                                         : __uint_as_float(v[j]);
                    f[j] = conv_post(a, p.bias, min(col0 + c0 + j, p.OC - 1), p.post);
                }
                const int cbase = col0 + c0;
                if (p.out_vec && cbase + 32 <= p.OC) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(orow + cbase + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (cbase + j < p.OC) orow[cbase + j] = f[j];
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }

    tc_fence_before();
    __syncthreads();
    pdl_launch_dependents();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, tmem_cols);
    }
}

// ---- operand preparation -------------------------------------------------------
// Reference round-half-away quantisation (quantize_fp32_to_int8_3d :366-377).
__device__ __forceinline__ uint32_t quant8_bits(float x, float inv) {
    int q = static_cast<int>(roundf(x * inv));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q)));
}

__device__ __forceinline__ uint32_t abs_bits(float x) {
    const float a = fabsf(x);
    return a == a ? __float_as_uint(a) : 0u;   // NaN never wins, as in `a > max`
}

// Per-CTA absmax of the input (x) and the filter (y) as float bit patterns
// (non-negative floats order like unsigned integers), one partial per CTA:
// no atomics, nothing to reset between calls.  Vector loads over the
// 16-byte aligned body of each tensor, scalar loads for the rest.
__global__ void __launch_bounds__(kPrepThreads) conv3d_absmax_part_kernel(const float* __restrict__ in, int64_t nin,
                                                                          const float* __restrict__ f, int64_t nf,
                                                                          uint2* part) {
    uint32_t m[2] = {0u, 0u};
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t gs = static_cast<int64_t>(gridDim.x) * blockDim.x;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float* x = t == 0 ? in : f;
        const int64_t n = t == 0 ? nin : nf;
        const int64_t head = (reinterpret_cast<uintptr_t>(x) % 16 == 0) ? 0 : n;   // unaligned: all scalar
        const int64_t nv = (n - head) / 4;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        uint32_t acc = 0u;
        int64_t i = gt;
        for (; i + 3 * gs < nv; i += 4 * gs) {
            float4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __ldg(x4 + i + k * gs);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                acc = max(acc, max(max(abs_bits(v[k].x), abs_bits(v[k].y)), max(abs_bits(v[k].z), abs_bits(v[k].w))));
        }
        for (; i < nv; i += gs) {
            const float4 v = __ldg(x4 + i);
            acc = max(acc, max(max(abs_bits(v.x), abs_bits(v.y)), max(abs_bits(v.z), abs_bits(v.w))));
        }
        for (int64_t j = nv * 4 + gt; j < n; j += gs) acc = max(acc, abs_bits(__ldg(x + j)));
        m[t] = acc;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        m[0] = max(m[0], __shfl_xor_sync(0xFFFFFFFFu, m[0], o));
        m[1] = max(m[1], __shfl_xor_sync(0xFFFFFFFFu, m[1], o));
    }
    __shared__ uint32_t s_m[2][kPrepThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { s_m[0][warp] = m[0]; s_m[1][warp] = m[1]; }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t a = 0u, b = 0u;
        for (int w = 0; w < kPrepThreads / 32; ++w) { a = max(a, s_m[0][w]); b = max(b, s_m[1][w]); }
        part[blockIdx.x] = make_uint2(a, b);
    }
    pdl_launch_dependents();
}

// Scales from the absmax partials (s = max_abs / 127, 1 when all zero,
// compute_quant_scale_3d :355-364; scales[0..3] = s_in, s_f, 1/s_in, 1/s_f),
// then input and filter quantised: four elements per 32-bit store.
__global__ void __launch_bounds__(kPrepThreads) conv3d_quant_kernel(const float* __restrict__ in, int64_t nin,
                                                                    const float* __restrict__ f, int64_t nf,
                                                                    const uint2* part, int nparts, float* scales,
                                                                    int8_t* inq, int8_t* fq) {
    pdl_wait();
    uint32_t m0 = 0u, m1 = 0u;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
        const uint2 v = part[i];
        m0 = max(m0, v.x);
        m1 = max(m1, v.y);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        m0 = max(m0, __shfl_xor_sync(0xFFFFFFFFu, m0, o));
        m1 = max(m1, __shfl_xor_sync(0xFFFFFFFFu, m1, o));
    }
    __shared__ uint32_t s_m[2][kPrepThreads / 32];
    __shared__ float s_inv[2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { s_m[0][warp] = m0; s_m[1][warp] = m1; }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t a = 0u, b = 0u;
        for (int w = 0; w < kPrepThreads / 32; ++w) { a = max(a, s_m[0][w]); b = max(b, s_m[1][w]); }
        const float ma = __uint_as_float(a), mb = __uint_as_float(b);
        const float sa = ma == 0.0f ? 1.0f : __fdiv_rn(ma, 127.0f);
        const float sb = mb == 0.0f ? 1.0f : __fdiv_rn(mb, 127.0f);
        s_inv[0] = __fdiv_rn(1.0f, sa);
        s_inv[1] = __fdiv_rn(1.0f, sb);
        if (blockIdx.x == 0) {
            scales[0] = sa;
            scales[1] = sb;
            scales[2] = s_inv[0];
            scales[3] = s_inv[1];
        }
    }
    __syncthreads();
    pdl_launch_dependents();
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t gs = static_cast<int64_t>(gridDim.x) * blockDim.x;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float* x = t == 0 ? in : f;
        int8_t* y = t == 0 ? inq : fq;
        const int64_t n = t == 0 ? nin : nf;
        const float inv = s_inv[t];
        // y is 256-byte aligned (workspace); vector groups need x aligned too.
        const int64_t nv = reinterpret_cast<uintptr_t>(x) % 16 == 0 ? n / 4 : 0;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        uint32_t* y4 = reinterpret_cast<uint32_t*>(y);
        for (int64_t i = gt; i < nv; i += gs) {
            const float4 v = __ldg(x4 + i);
            y4[i] = quant8_bits(v.x, inv) | (quant8_bits(v.y, inv) << 8) | (quant8_bits(v.z, inv) << 16) |
                    (quant8_bits(v.w, inv) << 24);
        }
        for (int64_t j = nv * 4 + gt; j < n; j += gs)
            y[j] = static_cast<int8_t>(static_cast<uint8_t>(quant8_bits(__ldg(x + j), inv)));
    }
}

// Input and filter to bf16 bits (RNE, the reference's bfloat16_t(float)):
// four elements per 8-byte store.
__global__ void __launch_bounds__(kPrepThreads) conv3d_bf16_prep_kernel(const float* __restrict__ in, int64_t nin,
                                                                        const float* __restrict__ f, int64_t nf,
                                                                        uint16_t* inb, uint16_t* fb) {
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t gs = static_cast<int64_t>(gridDim.x) * blockDim.x;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float* x = t == 0 ? in : f;
        uint16_t* y = t == 0 ? inb : fb;
        const int64_t n = t == 0 ? nin : nf;
        const int64_t nv = reinterpret_cast<uintptr_t>(x) % 16 == 0 ? n / 4 : 0;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        uint2* y4 = reinterpret_cast<uint2*>(y);
        for (int64_t i = gt; i < nv; i += gs) {
            const float4 v = __ldg(x4 + i);
            y4[i] = make_uint2(f32_to_bf16_bits_ref(v.x) | (static_cast<uint32_t>(f32_to_bf16_bits_ref(v.y)) << 16),
                               f32_to_bf16_bits_ref(v.z) | (static_cast<uint32_t>(f32_to_bf16_bits_ref(v.w)) << 16));
        }
        for (int64_t j = nv * 4 + gt; j < n; j += gs) y[j] = f32_to_bf16_bits_ref(__ldg(x + j));
    }
    pdl_launch_dependents();
}

// ---- host helpers ----------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(ptr);
    }();
    return fn;
}

int pow2_at_least(int x, int cap) {
    int p = 1;
    while (p < x && p < cap) p *= 2;
    return p;
}

int chunk_bytes(const Conv3dGeom& g, int mode) {
    const int64_t icb = static_cast<int64_t>(g.IC) * (mode == 1 ? 2 : 1);
    return icb % 128 == 0 ? 128 : (icb % 64 == 0 ? 64 : (icb % 32 == 0 ? 32 : 0));
}

struct ConvTcLayout {
    int bw, bh, bd, bn, tw, th, td, tn, cb, n_mma, n_tiles, num_kb, stages, b_res;
    size_t smem;
    uint32_t a_bytes, b_bytes, stage_bytes, ring_off, bar_off;
};

bool conv_layout(const Conv3dGeom& g, int mode, ConvTcLayout* L) {
    const int cb = chunk_bytes(g, mode);
    if (cb == 0) return false;
    const int eb = mode == 1 ? 2 : 1;
    L->cb = cb;
    L->bw = pow2_at_least(g.OW, BM);
    L->bh = pow2_at_least(g.OH, BM / L->bw);
    L->bd = pow2_at_least(g.OD, BM / (L->bw * L->bh));
    L->bn = BM / (L->bw * L->bh * L->bd);
    L->tw = (g.OW + L->bw - 1) / L->bw;
    L->th = (g.OH + L->bh - 1) / L->bh;
    L->td = (g.OD + L->bd - 1) / L->bd;
    L->tn = (g.N + L->bn - 1) / L->bn;
    int n = g.OC < kMaxN ? g.OC : kMaxN;
    L->n_mma = (n + 31) / 32 * 32;
    L->n_tiles = (g.OC + L->n_mma - 1) / L->n_mma;
    const int64_t cpt = static_cast<int64_t>(g.IC) * eb / cb;
    L->num_kb = static_cast<int>(cpt * g.KD * g.KH * g.KW);
    L->a_bytes = static_cast<uint32_t>(BM * cb);
    L->b_bytes = static_cast<uint32_t>(L->n_mma * cb);
    const size_t fixed = 1024 + kBarBytes;
    const size_t bres = static_cast<size_t>(L->num_kb) * L->b_bytes;
    // The filter stays resident when it leaves room for a ring of at least
    // four input stages.
    L->b_res = L->n_tiles == 1 && fixed + bres + 4 * static_cast<size_t>(L->a_bytes) <= kSmemCap ? 1 : 0;
    L->stage_bytes = L->a_bytes + (L->b_res ? 0u : L->b_bytes);
    const size_t avail = kSmemCap - fixed - (L->b_res ? bres : 0);
    int st = static_cast<int>(avail / L->stage_bytes);
    if (st > kMaxStages) st = kMaxStages;
    if (st < 2) return false;
    L->stages = st;
    L->ring_off = static_cast<uint32_t>(L->b_res ? bres : 0);
    L->bar_off = L->ring_off + static_cast<uint32_t>(st) * L->stage_bytes;
    L->smem = 1024 + L->bar_off + kBarBytes;
    if (L->smem < kSmemMin) L->smem = kSmemMin;
    return L->smem <= kSmemCap;
}

CUtensorMapSwizzle swizzle_for(int cb) {
    return cb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (cb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

int prep_grid(int64_t n4) {
    const int64_t b = (n4 + kPrepThreads - 1) / kPrepThreads;
    return static_cast<int>(b < 1 ? 1 : (b > 148 * 4 ? 148 * 4 : b));
}

}  // namespace

bool conv3d_tc_ok(const Conv3dGeom& g, int mode) {
    if ((mode != 1 && mode != 2) || !encode_fn()) return false;
    if (g.sd != 1 || g.sh != 1 || g.sw != 1) return false;
    if (g.KD * g.KH * g.KW > kConv3dMaxTaps) return false;
    ConvTcLayout L;
    return conv_layout(g, mode, &L);
}

size_t conv3d_tc_part_bytes() { return static_cast<size_t>(kPartMax) * sizeof(uint2); }

cudaError_t launch_conv3d_tc_prep(int mode, const float* in, int64_t nin, const float* f, int64_t nf, void* inq,
                                  void* fq, void* part, float* scales, cudaStream_t s) {
    if (reinterpret_cast<uintptr_t>(inq) % 16 || reinterpret_cast<uintptr_t>(fq) % 16) return cudaErrorInvalidValue;
    if (mode == 1) {
        conv3d_bf16_prep_kernel<<<prep_grid((nin + nf) / 4), kPrepThreads, 0, s>>>(
            in, nin, f, nf, static_cast<uint16_t*>(inq), static_cast<uint16_t*>(fq));
        return cudaGetLastError();
    }
    if (mode != 2 || !part || !scales) return cudaErrorInvalidValue;
    int parts = prep_grid((nin + nf) / 16);   // about four float4 per thread
    if (parts > kPartMax) parts = kPartMax;
    conv3d_absmax_part_kernel<<<parts, kPrepThreads, 0, s>>>(in, nin, f, nf, static_cast<uint2*>(part));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(prep_grid((nin + nf) / 4)));
    cfg.blockDim = dim3(kPrepThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, conv3d_quant_kernel, in, nin, f, nf, static_cast<const uint2*>(part), parts,
                              scales, static_cast<int8_t*>(inq), static_cast<int8_t*>(fq));
}

cudaError_t launch_conv3d_tc(const Conv3dGeom& g, int mode, const void* inq, const void* fq, const float* scales,
                             const float* bias, int op, float* out, uint32_t* err, int num_sms, cudaStream_t s) {
    ConvTcLayout L;
    if (!conv3d_tc_ok(g, mode) || !conv_layout(g, mode, &L)) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(inq) % 16 || reinterpret_cast<uintptr_t>(fq) % 16) return cudaErrorInvalidValue;
    if (mode == 2 && !scales) return cudaErrorInvalidValue;
    const int eb = mode == 1 ? 2 : 1;
    const CUtensorMapDataType dt = mode == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const CUtensorMapSwizzle sw = swizzle_for(L.cb);
    CUtensorMap tmA, tmB;
    {
        const cuuint64_t ic = static_cast<cuuint64_t>(g.IC);
        cuuint64_t dims[5] = {ic, static_cast<cuuint64_t>(g.IW), static_cast<cuuint64_t>(g.IH),
                              static_cast<cuuint64_t>(g.ID), static_cast<cuuint64_t>(g.N)};
        cuuint64_t strides[4] = {ic * eb, ic * eb * g.IW, ic * eb * g.IW * g.IH, ic * eb * g.IW * g.IH * g.ID};
        cuuint32_t box[5] = {static_cast<cuuint32_t>(L.cb / eb), static_cast<cuuint32_t>(L.bw),
                             static_cast<cuuint32_t>(L.bh), static_cast<cuuint32_t>(L.bd), static_cast<cuuint32_t>(L.bn)};
        cuuint32_t estr[5] = {1, 1, 1, 1, 1};
        if (encode_fn()(&tmA, dt, 5, const_cast<void*>(inq), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(g.K), static_cast<cuuint64_t>(g.OC)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(g.K) * eb};
        cuuint32_t box[2] = {static_cast<cuuint32_t>(L.cb / eb), static_cast<cuuint32_t>(L.n_mma)};
        cuuint32_t estr[2] = {1, 1};
        if (encode_fn()(&tmB, dt, 2, const_cast<void*>(fq), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    ConvTcParams p;
    p.N = g.N; p.OD = g.OD; p.OH = g.OH; p.OW = g.OW; p.OC = g.OC;
    p.KH = g.KH; p.KW = g.KW;
    p.pd = g.pd; p.ph = g.ph; p.pw = g.pw;
    p.bw = L.bw; p.bh = L.bh; p.bd = L.bd; p.bn = L.bn;
    p.tw = L.tw; p.th = L.th; p.td = L.td;
    p.m_tiles = L.tw * L.th * L.td * L.tn;
    p.n_tiles = L.n_tiles;
    p.units = p.m_tiles * p.n_tiles;
    p.cb = L.cb;
    p.celems = L.cb / eb;
    p.cpt = static_cast<int>(static_cast<int64_t>(g.IC) * eb / L.cb);
    p.num_kb = L.num_kb;
    p.n_mma = L.n_mma;
    p.stages = L.stages;
    p.b_res = L.b_res;
    p.i8 = mode == 2 ? 1 : 0;
    p.post = op;
    p.a_bytes = L.a_bytes;
    p.b_bytes = L.b_bytes;
    p.stage_bytes = L.stage_bytes;
    p.ring_off = L.ring_off;
    p.bar_off = L.bar_off;
    p.scales = scales;
    p.bias = bias;
    p.out = out;
    p.out_vec = reinterpret_cast<uintptr_t>(out) % 16 == 0 && g.OC % 4 == 0 ? 1 : 0;
    p.err = err;

    static std::mutex mu;
    static std::set<int> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!done.count(dev)) {
            e = cudaFuncSetAttribute(conv3d_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmemCap));
            if (e != cudaSuccess) return e;
            done.insert(dev);
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.units < num_sms ? p.units : num_sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, conv3d_tc_kernel, tmA, tmB, p);
}

}  // namespace dnnopt_b200
