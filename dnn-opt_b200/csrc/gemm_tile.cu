// General-shape int8 SIMT kernel (any M, N, K and leading dimensions) for the
// int8 calls outside the dot-form GEMV class (M > 8, unaligned rows, conv3d's
// column matrices), so that every int8 call the reference accepts has a GPU
// path: dp4a on register tiles (the FP32-accumulate general kernel is
// gemm_simt.cu).
//
// Also here: the FP32-API int8 quantisation (per-tensor absmax / 127,
// lrintf, clamp to [-128, 127]) of reference src/gemm/gemm_smallm_int8.cpp:198-236
// and src/gemm/gemm_driver_generic.cpp:49-67, bit-exact (IEEE division,
// round-to-nearest-even conversion).
#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int BM = 64, BN = 64;
constexpr int BKB = 64;               // K bytes per slice
constexpr int BKW = BKB / 4;          // 32-bit words (four int8 each) per slice
constexpr int kPad = 4;
constexpr int kMaxSplits = 8;

struct S8Params {
    GemmArgs g;
    const float* scales;
    int kchunk;     // K bytes per split (multiple of BKB)
    int vec;        // 1: A and B rows 4-byte aligned (word loads)
    int vec16a;     // 1: A rows 16-byte aligned (16-byte loads)
    int vec16b;     // 1: B rows 16-byte aligned
    // Implicit im2col (CONV kernels only): A[m][k] is the quantised NDHWC
    // input at output position m, tap k / IC, channel k % IC, zero in the padding.
    Conv3dGeom conv;
    const int8_t* conv_in;
    const float* conv_bias;   // CONV epilogue: float(acc) * (s_in * s_f) [+ bias] [relu / relu6]
    int conv_op;
};

// int8 x int8 -> int32 (exact) with A [M, K] and B [N, K] (K contiguous in
// both); optional dequantising epilogue.  64 x 64 CTA tiles, 4 x 4 outputs per
// thread, K in 64-byte slices through two shared-memory buffers (next slice's
// words loaded before the current slice's dp4a), K split over up to 8 CTAs of
// a cluster when the tiles alone leave SMs idle (int32 partials summed
// through distributed shared memory: exact, so the order does not matter).
template <bool DQ, bool CONV = false>
__global__ void __launch_bounds__(kThreads)
gemm_tile_s8_kernel(const S8Params p) {
    // One array carved into the two operands' buffers, so that the split-K
    // partial tile (BM x BN words) can reuse the whole of it.
    __shared__ __align__(16) int32_t smem[2 * BKW * (BM + kPad) + 2 * BKW * (BN + kPad)];
    static_assert(sizeof(smem) >= sizeof(int32_t) * BM * BN, "partial tile must fit");
    auto sA = reinterpret_cast<int32_t (*)[BKW][BM + kPad]>(smem);
    auto sB = reinterpret_cast<int32_t (*)[BKW][BN + kPad]>(smem + 2 * BKW * (BM + kPad));
    pdl_wait();
    pdl_launch_dependents();
    const GemmArgs& g = p.g;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int k_begin = blockIdx.z * p.kchunk;
    const int k_end = min(g.K, k_begin + p.kchunk);
    const int nslices = k_end > k_begin ? (k_end - k_begin + BKB - 1) / BKB : 0;
    const int8_t* A = static_cast<const int8_t*>(g.A);
    const int8_t* B = static_cast<const int8_t*>(g.B);

    // Word w (bytes 4w..4w+3 of the slice) of row r of a [rows, K] int8 matrix.
    auto word = [&](const int8_t* X, int64_t ld, int row, int rows, int k) -> int32_t {
        if (row >= rows || k >= k_end) return 0;
        const int8_t* q = X + (int64_t)row * ld + k;
        if (p.vec && k + 4 <= k_end) return *reinterpret_cast<const int32_t*>(q);
        uint32_t w = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b)
            if (k + b < k_end) w |= static_cast<uint32_t>(static_cast<uint8_t>(q[b])) << (8 * b);
        return static_cast<int32_t>(w);
    };
    constexpr int LW = BM * BKW / kThreads;   // words per thread per operand (4)
    static_assert(BM == BN && LW == 4, "one 16-byte segment per thread and operand");
    // Word w of row r sits at [w][swz(r, w)]: bits 2-4 of the row flipped by
    // w / 4, so the transposing stores of 16-byte row segments (4 threads per
    // 64-byte row, 8 rows per warp) hit 32 distinct banks while the dp4a loop
    // still reads four consecutive rows as one 16-byte load.
    auto swz = [](int r, int w) { return r ^ (4 * ((w >> 2) & 7)); };
    const int vrow = tid >> 2, vq = tid & 3;  // 16-byte path: row, segment
    int32_t ra[LW], rb[LW];
    // Words 4q .. 4q + 3 of row `row` (16-byte aligned rows), zero past the ends.
    auto seg16 = [&](const int8_t* X, int64_t ld, int row, int rows, int k, int32_t (&v)[4]) {
        if (row < rows && k + 16 <= k_end) {
            const int4 x = __ldg(reinterpret_cast<const int4*>(X + (int64_t)row * ld + k));
            v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = word(X, ld, row, rows, k + 4 * j);
        }
    };
    // CONV: this thread's output position (id0, ih0, iw0, batch or -1) and the
    // tap table (kd << 20 | kh << 10 | kw), decoded once.
    __shared__ int s_tap[CONV ? kConv3dMaxTaps : 1];
    int4 crow = make_int4(0, 0, 0, -1);
    if constexpr (CONV) {
        const Conv3dGeom& cg = p.conv;
        const int taps = cg.KD * cg.KH * cg.KW;
        for (int t = tid; t < taps; t += kThreads) {
            const int kw = t % cg.KW, r2 = t / cg.KW;
            s_tap[t] = ((r2 / cg.KH) << 20) | ((r2 % cg.KH) << 10) | kw;
        }
        const int64_t m = static_cast<int64_t>(m0) + vrow;
        if (m < g.M) {
            const int ow = static_cast<int>(m % cg.OW);
            int64_t t = m / cg.OW;
            const int oh = static_cast<int>(t % cg.OH);
            t /= cg.OH;
            const int od = static_cast<int>(t % cg.OD);
            crow = make_int4(od * cg.sd - cg.pd, oh * cg.sh - cg.ph, ow * cg.sw - cg.pw, static_cast<int>(t / cg.OD));
        }
        __syncthreads();
    }
    auto load_slice = [&](int k0) {
        if constexpr (CONV) {
            // 16 channels of one tap (IC % 16 == 0, so K % 16 == 0 and a
            // segment that starts below k_end ends within it).
            const Conv3dGeom& cg = p.conv;
            const int k = k0 + 16 * vq;
            ra[0] = ra[1] = ra[2] = ra[3] = 0;
            if (k < k_end && crow.w >= 0) {
                const int tap = k / cg.IC, c = k - tap * cg.IC;
                const int pk = s_tap[tap];
                const int id = crow.x + (pk >> 20), ih = crow.y + ((pk >> 10) & 1023), iw = crow.z + (pk & 1023);
                if (id >= 0 && id < cg.ID && ih >= 0 && ih < cg.IH && iw >= 0 && iw < cg.IW) {
                    const int4 x = __ldg(reinterpret_cast<const int4*>(
                        p.conv_in + (((static_cast<int64_t>(crow.w) * cg.ID + id) * cg.IH + ih) * cg.IW + iw) * cg.IC + c));
                    ra[0] = x.x; ra[1] = x.y; ra[2] = x.z; ra[3] = x.w;
                }
            }
        } else if (p.vec16a) {
            seg16(A, g.lda, m0 + vrow, g.M, k0 + 16 * vq, ra);
        } else {
#pragma unroll
            for (int i = 0; i < LW; ++i) {
                const int e = tid + i * kThreads;
                ra[i] = word(A, g.lda, m0 + e / BKW, g.M, k0 + 4 * (e % BKW));
            }
        }
        if (p.vec16b) {
            seg16(B, g.ldb, n0 + vrow, g.N, k0 + 16 * vq, rb);
        } else {
#pragma unroll
            for (int i = 0; i < LW; ++i) {
                const int e = tid + i * kThreads;
                rb[i] = word(B, g.ldb, n0 + e / BKW, g.N, k0 + 4 * (e % BKW));
            }
        }
    };
    auto store_slice = [&](int buf) {
#pragma unroll
        for (int i = 0; i < LW; ++i) {
            const int e = tid + i * kThreads;
            const int ra_r = p.vec16a ? vrow : e / BKW, ra_w = p.vec16a ? 4 * vq + i : e % BKW;
            const int rb_r = p.vec16b ? vrow : e / BKW, rb_w = p.vec16b ? 4 * vq + i : e % BKW;
            sA[buf][ra_w][swz(ra_r, ra_w)] = ra[i];
            sB[buf][rb_w][swz(rb_r, rb_w)] = rb[i];
        }
    };

    int32_t acc[4][4] = {};
    if (nslices > 0) {
        load_slice(k_begin);
        store_slice(0);
        __syncthreads();
    }
    for (int t = 0; t < nslices; ++t) {
        const int buf = t & 1;
        if (t + 1 < nslices) load_slice(k_begin + (t + 1) * BKB);
#pragma unroll
        for (int w = 0; w < BKW; ++w) {
            const int4 av = *reinterpret_cast<const int4*>(&sA[buf][w][swz(4 * ty, w)]);
            const int4 bv = *reinterpret_cast<const int4*>(&sB[buf][w][swz(4 * tx, w)]);
            const int a[4] = {av.x, av.y, av.z, av.w};
            const int b[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[r][c] = __dp4a(a[r], b[c], acc[r][c]);
        }
        if (t + 1 < nslices) store_slice(buf ^ 1);
        __syncthreads();
    }

    auto finish = [&](int gi, int gj, int32_t v) {
        if constexpr (DQ) {
            float* cp = static_cast<float*>(g.C) + (int64_t)gi * g.ldc + gj;
            const float scale = __fmul_rn(g.alpha, __fmul_rn(p.scales[0], p.scales[1]));
            const float c0 = (g.beta == 0.0f) ? 0.0f : __fmul_rn(g.beta, *cp);
            *cp = __fadd_rn(c0, __fmul_rn(scale, static_cast<float>(v)));
        } else if constexpr (CONV) {
            float x = __fmul_rn(static_cast<float>(v), __fmul_rn(p.scales[0], p.scales[1]));
            if (p.conv_bias) x = __fadd_rn(x, p.conv_bias[gj]);
            if (p.conv_op == 1) x = x > 0.0f ? x : 0.0f;
            else if (p.conv_op == 2) x = x > 0.0f ? (x < 6.0f ? x : 6.0f) : 0.0f;
            static_cast<float*>(g.C)[(int64_t)gi * g.ldc + gj] = x;
        } else {
            static_cast<int32_t*>(g.C)[(int64_t)gi * g.ldc + gj] = v;
        }
    };
    if (gridDim.z == 1) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int gi = m0 + 4 * ty + r;
            if (gi >= g.M) continue;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int gj = n0 + 4 * tx + c;
                if (gj < g.N) finish(gi, gj, acc[r][c]);
            }
        }
        return;
    }
    // Cluster K split: partial tiles parked in this CTA's (idle) A buffers,
    // CTA q finishes elements q*256 + tid, + S*256, ... over ranks 0..S-1.
    int32_t* part = smem;           // [BM][BN]
#pragma unroll
    for (int r = 0; r < 4; ++r)
        *reinterpret_cast<int4*>(&part[(4 * ty + r) * BN + 4 * tx]) = make_int4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    cluster_sync_all();
    const int S = static_cast<int>(gridDim.z);
    const uint32_t q = cluster_ctarank();
    const uint32_t part_addr = smem_u32(part);
    for (int e = static_cast<int>(q) * kThreads + tid; e < BM * BN; e += S * kThreads) {
        const int mm = e / BN, nn = e - mm * BN;
        int32_t v[kMaxSplits];
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)
            v[r] = r < S ? __float_as_int(ld_dsmem_f32(map_to_cta(part_addr + e * 4u, static_cast<uint32_t>(r)))) : 0;
        int32_t sum = 0;
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r) sum += v[r];
        if (m0 + mm < g.M && n0 + nn < g.N) finish(m0 + mm, n0 + nn, sum);
    }
    cluster_sync_all();   // no CTA leaves while another still reads its tile
}

// Per-tensor absmax of op(A) (M x K) and B (K x N, or N x K when b_trans):
// absmax_bits[0..1] hold the float bit patterns (non-negative floats order
// like unsigned integers).  NaN never wins, as in the reference's `v > max`.
__global__ void absmax2_kernel(const GemmArgs g, uint32_t* absmax_bits) {
    const float* A = static_cast<const float*>(g.A);
    const float* B = static_cast<const float*>(g.B);
    const int64_t na = (int64_t)g.M * g.K, nb = (int64_t)g.K * g.N;
    float ma = 0.0f, mb = 0.0f;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na + nb; i += stride) {
        if (i < na) {
            int64_t m = i / g.K, k = i - m * g.K;
            float v = fabsf(A[g.a_trans ? k * g.lda + m : m * g.lda + k]);
            if (v > ma) ma = v;
        } else {
            int64_t j = i - na;
            int64_t k = j / g.N, n = j - k * g.N;
            float v = fabsf(B[g.b_trans ? n * g.ldb + k : k * g.ldb + n]);
            if (v > mb) mb = v;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ma = fmaxf(ma, __shfl_xor_sync(0xFFFFFFFFu, ma, o));
        mb = fmaxf(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
    }
    if ((threadIdx.x & 31) == 0) {
        if (ma > 0.0f) atomicMax(&absmax_bits[0], __float_as_uint(ma));
        if (mb > 0.0f) atomicMax(&absmax_bits[1], __float_as_uint(mb));
    }
}

__device__ __forceinline__ int8_t quant_s8(float x, float s) {
    int q = __float2int_rn(__fdiv_rn(x, s));
    q = q < -128 ? -128 : (q > 127 ? 127 : q);
    return static_cast<int8_t>(q);
}

// qa: M x K dense; qb: N x K dense (B transposed so the dot-form kernels read
// K-contiguous rows).  scales[0..1] = sA, sB.
__global__ void quantize_s8_kernel(const GemmArgs g, const uint32_t* absmax_bits, float* scales,
                                   int8_t* qa, int8_t* qb) {
    float ma = __uint_as_float(absmax_bits[0]), mb = __uint_as_float(absmax_bits[1]);
    float sa = (ma == 0.0f) ? 1.0f : __fdiv_rn(ma, 127.0f);
    float sb = (mb == 0.0f) ? 1.0f : __fdiv_rn(mb, 127.0f);
    if (blockIdx.x == 0 && threadIdx.x == 0) { scales[0] = sa; scales[1] = sb; }
    const float* A = static_cast<const float*>(g.A);
    const float* B = static_cast<const float*>(g.B);
    const int64_t na = (int64_t)g.M * g.K, nb = (int64_t)g.K * g.N;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na + nb; i += stride) {
        if (i < na) {
            int64_t m = i / g.K, k = i - m * g.K;
            qa[i] = quant_s8(A[g.a_trans ? k * g.lda + m : m * g.lda + k], sa);
        } else {
            // Output-major order for qb (n, k) so writes are coalesced.
            int64_t j = i - na;
            int64_t n = j / g.K, k = j - n * g.K;
            qb[j] = quant_s8(B[g.b_trans ? n * g.ldb + k : k * g.ldb + n], sb);
        }
    }
}

// Reference fp8_e4m3_t(float) / fp8_e5m2_t(float) encoders
// (include/dnnopt/gemm/gemm_types.h:56-85, :131-157), bit for bit.
__device__ __forceinline__ uint8_t enc_re4(float f) {
    uint32_t u = __float_as_uint(f);
    uint32_t sign = (u >> 31) & 1u;
    int32_t ex = static_cast<int32_t>((u >> 23) & 0xFFu) - 127 + 8;
    uint32_t mant = (u >> 20) & 0x7u;
    if (ex > 7) { ex = 7; mant = 7; }
    else if (ex < -6) { ex = 0; mant = 0; }
    if (ex > 0) return static_cast<uint8_t>((sign << 7) | (static_cast<uint32_t>(ex & 0xF) << 3) | mant);
    int shift = -ex;
    if (shift >= 8) return 0;
    mant = (mant >> shift) | (0x8u >> shift);
    return static_cast<uint8_t>((sign << 7) | mant);
}

__device__ __forceinline__ uint8_t enc_re5(float f) {
    uint32_t u = __float_as_uint(f);
    uint32_t sign = (u >> 31) & 1u;
    int32_t ex = static_cast<int32_t>((u >> 23) & 0xFFu) - 127 + 16;
    uint32_t mant = (u >> 21) & 0x3u;
    if (ex > 30) return static_cast<uint8_t>((sign << 7) | (0x1Fu << 2));
    if (ex < -14) return static_cast<uint8_t>(sign << 7);
    if (ex > 0) return static_cast<uint8_t>((sign << 7) | (static_cast<uint32_t>(ex & 0x1F) << 2) | mant);
    int shift = -ex;
    if (shift >= 4) return static_cast<uint8_t>(sign << 7);
    mant = (mant >> shift) | (0x4u >> shift);
    return static_cast<uint8_t>((sign << 7) | mant);
}

// gemm_fp8 (src/gemm/gemm_fp8.cpp:117-146): A -> e4m3 (dense M x K),
// B -> e5m2 (dense K x N).
__global__ void quantize_ref_fp8_kernel(const GemmArgs g, uint8_t* qa, uint8_t* qb) {
    const float* A = static_cast<const float*>(g.A);
    const float* B = static_cast<const float*>(g.B);
    const int64_t na = (int64_t)g.M * g.K, nb = (int64_t)g.K * g.N;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na + nb; i += stride) {
        if (i < na) {
            int64_t m = i / g.K, k = i - m * g.K;
            qa[i] = enc_re4(A[g.a_trans ? k * g.lda + m : m * g.lda + k]);
        } else {
            int64_t j = i - na;
            int64_t k = j / g.N, n = j - k * g.N;
            qb[j] = enc_re5(B[g.b_trans ? n * g.ldb + k : k * g.ldb + n]);
        }
    }
}

}  // namespace

namespace {

cudaError_t launch_s8(const void* fn, S8Params& sp, cudaStream_t s) {
    const GemmArgs& g = sp.g;
    int dev = 0, sms = 148;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    const int64_t tiles = static_cast<int64_t>((g.N + BN - 1) / BN) * ((g.M + BM - 1) / BM);
    int splits = static_cast<int>((2 * static_cast<int64_t>(sms) + tiles - 1) / tiles);
    const int max_by_k = (g.K + 2 * BKB - 1) / (2 * BKB);   // at least two slices per split
    if (splits > max_by_k) splits = max_by_k;
    if (splits > kMaxSplits) splits = kMaxSplits;
    if (splits < 1) splits = 1;
    int kchunk = (g.K + splits - 1) / splits;
    kchunk = (kchunk + BKB - 1) / BKB * BKB;
    if (kchunk < BKB) kchunk = BKB;
    splits = (g.K + kchunk - 1) / kchunk;
    if (splits < 1) splits = 1;
    sp.kchunk = kchunk;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((g.N + BN - 1) / BN), static_cast<unsigned>((g.M + BM - 1) / BM),
                       static_cast<unsigned>(splits));
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int na = 1;
    if (splits > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = static_cast<unsigned>(splits);
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    void* args[] = {&sp};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_gemm_tile_s8(DotKind kind, const GemmArgs& g, const float* scales,
                                cudaStream_t s) {
    if (kind != DotKind::S8S32 && kind != DotKind::S8DQ) return cudaErrorInvalidValue;
    S8Params sp = {};
    sp.g = g;
    sp.scales = scales;
    sp.vec = (reinterpret_cast<uintptr_t>(g.A) % 4 == 0 && reinterpret_cast<uintptr_t>(g.B) % 4 == 0 &&
              g.lda % 4 == 0 && g.ldb % 4 == 0) ? 1 : 0;
    sp.vec16a = (reinterpret_cast<uintptr_t>(g.A) % 16 == 0 && g.lda % 16 == 0) ? 1 : 0;
    sp.vec16b = (reinterpret_cast<uintptr_t>(g.B) % 16 == 0 && g.ldb % 16 == 0) ? 1 : 0;
    const void* fn = kind == DotKind::S8S32 ? reinterpret_cast<const void*>(&gemm_tile_s8_kernel<false>)
                                            : reinterpret_cast<const void*>(&gemm_tile_s8_kernel<true>);
    return launch_s8(fn, sp, s);
}

bool gemm_tile_s8_conv_ok(const Conv3dGeom& cg, const int8_t* in_q, const int8_t* filter_q) {
    return cg.IC % 16 == 0 && cg.M >= 64 && cg.M <= INT32_MAX && cg.K <= INT32_MAX &&
           cg.KD * cg.KH * cg.KW <= kConv3dMaxTaps && cg.KD < 1024 && cg.KH < 1024 && cg.KW < 1024 &&
           reinterpret_cast<uintptr_t>(in_q) % 16 == 0 && reinterpret_cast<uintptr_t>(filter_q) % 16 == 0;
}

cudaError_t launch_gemm_tile_s8_conv(const Conv3dGeom& cg, const int8_t* in_q, const int8_t* filter_q,
                                     const float* scales, const float* bias, int op, float* out,
                                     cudaStream_t s) {
    if (!gemm_tile_s8_conv_ok(cg, in_q, filter_q)) return cudaErrorInvalidValue;
    S8Params sp = {};
    GemmArgs& g = sp.g;
    g.M = static_cast<int>(cg.M);
    g.N = cg.OC;
    g.K = static_cast<int>(cg.K);
    g.alpha = 1.0f;
    g.beta = 0.0f;
    g.A = in_q;               // not read: the CONV kernel gathers from conv_in
    g.lda = cg.K;
    g.a_trans = 0;
    g.B = filter_q;           // [OC, K]
    g.ldb = cg.K;
    g.b_trans = 1;
    g.C = out;                // [M, OC] float, dequantised in the epilogue
    g.ldc = cg.OC;
    sp.scales = scales;       // device: s_in, s_f, 1/s_in, 1/s_f
    sp.conv_bias = bias;
    sp.conv_op = op;
    sp.vec = 1;
    sp.vec16a = 1;            // store mapping of 16-byte row segments
    sp.vec16b = 1;
    sp.conv = cg;
    sp.conv_in = in_q;
    return launch_s8(reinterpret_cast<const void*>(&gemm_tile_s8_kernel<false, true>), sp, s);
}

cudaError_t launch_absmax2(const GemmArgs& g, uint32_t* absmax_bits, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(absmax_bits, 0, 2 * sizeof(uint32_t), s);
    if (e != cudaSuccess) return e;
    int64_t n = (int64_t)g.M * g.K + (int64_t)g.K * g.N;
    int blocks = static_cast<int>(((n + 255) / 256) < 148 * 8 ? (n + 255) / 256 : 148 * 8);
    absmax2_kernel<<<blocks, 256, 0, s>>>(g, absmax_bits);
    return cudaGetLastError();
}

cudaError_t launch_quantize_s8(const GemmArgs& g, const uint32_t* absmax_bits, float* scales,
                               int8_t* qa, int8_t* qb_nk, cudaStream_t s) {
    int64_t n = (int64_t)g.M * g.K + (int64_t)g.K * g.N;
    int blocks = static_cast<int>(((n + 255) / 256) < 148 * 8 ? (n + 255) / 256 : 148 * 8);
    quantize_s8_kernel<<<blocks, 256, 0, s>>>(g, absmax_bits, scales, qa, qb_nk);
    return cudaGetLastError();
}

cudaError_t launch_quantize_ref_fp8(const GemmArgs& g, uint8_t* qa, uint8_t* qb,
                                    cudaStream_t s) {
    int64_t n = (int64_t)g.M * g.K + (int64_t)g.K * g.N;
    int blocks = static_cast<int>(((n + 255) / 256) < 148 * 8 ? (n + 255) / 256 : 148 * 8);
    quantize_ref_fp8_kernel<<<blocks, 256, 0, s>>>(g, qa, qb);
    return cudaGetLastError();
}

// cblas_saxpy (reference src/blas/cblas_saxpy.cpp:13-50): Y[i*incY] += alpha*X[i*incX].
__global__ void saxpy_kernel(int n, float alpha, const float* x, int incx, float* y, int incy) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        y[i * incy] = fmaf(alpha, x[i * incx], y[i * incy]);
}

cudaError_t launch_saxpy(int n, float alpha, const float* x, int incx, float* y, int incy,
                         cudaStream_t s) {
    int blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    saxpy_kernel<<<blocks, 256, 0, s>>>(n, alpha, x, incx, y, incy);
    return cudaGetLastError();
}

// ---- column-major C of the oneDNN entry ------------------------------------
// The entry (integration/onednn/0001-dnnopt-integration.patch:279-365) walks
// the M x N column-major C column by column, j = 0..N-1, so when ldc < M the
// columns overlap in memory and an address can belong to several (i, j)
// pairs.  These kernels give every address of the footprint
// [0, (N-1)*ldc + M) the value that sequential walk leaves: one thread per
// address, pairs (j, i = a - j*ldc) visited in ascending j.  With ldc >= M an
// address has at most one pair.

__device__ __forceinline__ bool colmajor_pairs(int64_t a, int64_t M, int64_t N, int64_t ldc,
                                               int64_t* jlo, int64_t* jhi) {
    int64_t hi = a / ldc;
    if (hi > N - 1) hi = N - 1;
    const int64_t d = a - (M - 1);
    int64_t lo = d <= 0 ? 0 : (d + ldc - 1) / ldc;
    *jlo = lo;
    *jhi = hi;
    return lo <= hi;
}

// K == 0 (:288-303): C = 0 (beta == 0) or C * beta per pair (beta != 1),
// then bias[i] added per pair.
__global__ void colmajor_k0_kernel(float* C, const float* bias, int64_t M, int64_t N, int64_t ldc,
                                   float beta) {
    const int64_t total = (N - 1) * ldc + M;
    for (int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; a < total;
         a += (int64_t)gridDim.x * blockDim.x) {
        int64_t jlo, jhi;
        if (!colmajor_pairs(a, M, N, ldc, &jlo, &jhi)) continue;
        float v = C[a];
        if (beta == 0.0f) {
            v = 0.0f;
        } else if (beta != 1.0f) {
            for (int64_t j = jlo; j <= jhi; ++j) v = __fmul_rn(v, beta);
        }
        if (bias)
            for (int64_t j = jlo; j <= jhi; ++j) v = __fadd_rn(v, bias[a - j * ldc]);
        C[a] = v;
    }
}

// ldc < M (:330-353): C was computed into tmp (rows j of M floats, ld tmp_ld)
// and is copied back row by row, so the last pair's row wins; then the bias
// pass (:355-362) adds bias[i] per pair.
__global__ void colmajor_writeback_kernel(float* C, const float* tmp, int64_t tmp_ld,
                                          const float* bias, int64_t M, int64_t N, int64_t ldc) {
    const int64_t total = (N - 1) * ldc + M;
    for (int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; a < total;
         a += (int64_t)gridDim.x * blockDim.x) {
        int64_t jlo, jhi;
        if (!colmajor_pairs(a, M, N, ldc, &jlo, &jhi)) continue;
        float v = tmp[jhi * tmp_ld + (a - jhi * ldc)];
        if (bias)
            for (int64_t j = jlo; j <= jhi; ++j) v = __fadd_rn(v, bias[a - j * ldc]);
        C[a] = v;
    }
}

// Copy-in of the ldc < M path (:339-343): tmp[j][i] = C[j*ldc + i].
__global__ void colmajor_gather_kernel(float* tmp, const float* C, int64_t M, int64_t N,
                                       int64_t ldc) {
    const int64_t total = N * M;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = e / M, i = e - j * M;
        tmp[e] = C[j * ldc + i];
    }
}

namespace {
int grid_for(int64_t n) {
    int64_t b = (n + 255) / 256;
    return static_cast<int>(b < 148 * 8 ? (b > 0 ? b : 1) : 148 * 8);
}
}  // namespace

cudaError_t launch_colmajor_k0(float* C, const float* bias, int64_t M, int64_t N, int64_t ldc,
                               float beta, cudaStream_t s) {
    colmajor_k0_kernel<<<grid_for((N - 1) * ldc + M), 256, 0, s>>>(C, bias, M, N, ldc, beta);
    return cudaGetLastError();
}

cudaError_t launch_colmajor_writeback(float* C, const float* tmp, int64_t tmp_ld, const float* bias,
                                      int64_t M, int64_t N, int64_t ldc, cudaStream_t s) {
    colmajor_writeback_kernel<<<grid_for((N - 1) * ldc + M), 256, 0, s>>>(C, tmp, tmp_ld, bias, M,
                                                                          N, ldc);
    return cudaGetLastError();
}

cudaError_t launch_colmajor_gather(float* tmp, const float* C, int64_t M, int64_t N, int64_t ldc,
                                   cudaStream_t s) {
    colmajor_gather_kernel<<<grid_for(N * M), 256, 0, s>>>(tmp, C, M, N, ldc);
    return cudaGetLastError();
}

}  // namespace dnnopt_b200
