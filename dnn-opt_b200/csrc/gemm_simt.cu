// General FP32-accumulate GEMM on the CUDA cores for everything the
// specialised kernels do not take: M from 9 up (small-M bands above the GEMV
// kernels' M <= 8), any transposition, any alignment, and the FP32-API
// element encodings (FP32, BF16, FP32 rounded to BF16, the reference's fp8
// codecs).  It replaces the reference's generic paths for these shapes:
// gemm_fp32's adaptive-tile / packed registry range (src/gemm/gemm.cpp:295-347,
// src/gemm/gemm_adaptive_tile_fp32.cpp:664-784) and gemm_driver_generic
// (src/gemm/gemm_driver_generic.cpp:27-248) with C = alpha*A*B + beta*C.
//
// FP32 results must match the reference within 1e-5*K, so the products stay
// FP32 FMAs (no TF32/BF16 tensor-core rounding).  Design:
//   * CTA tile BM x BN (BM = 16, 32 or 64 by M; BN = 128, or 64 when N <= 64 so
//     narrow outputs such as conv3d's OC = 64 waste no columns, with BM = 128
//     when such an output has at least 128 rows per SM), 256 threads,
//     each thread BM*BN/1024 rows x 4 consecutive columns; K in 32-deep slices staged in two
//     shared-memory buffers, the next slice's global loads issued before the
//     current slice's FMAs (register prefetch), one barrier per slice;
//   * both operands are staged k-major in shared memory (a thread's rows and
//     its 4 columns come back as 16-byte loads), with the row index XOR-ed by
//     k / 4 so that the transposing stores of k-contiguous operands (A not
//     transposed, B transposed; 16-byte global loads along k) hit 32 distinct
//     banks;
//   * small tile counts split K over up to 8 CTAs of one thread-block cluster;
//     the partial tiles are summed through distributed shared memory in rank
//     order (deterministic), each CTA finishing 1/S of the tile;
//   * epilogue beta == 0 ? alpha*acc : fma(alpha, acc, beta*C), then + bias[n]
//     when the oneDNN entry passes one.
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "elem.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int BK = 32;
constexpr int kPadA = 4;      // keeps 16-byte alignment of k-major rows
constexpr int kPadB = 4;
constexpr int kMaxSplits = 8;

struct SimtParams {
    GemmArgs g;
    int kchunk;     // K rows per split (multiple of BK)
    int vec_a;      // 1: A's rows start on 4-element boundaries (4-wide loads when not transposed)
    int vec_b;      // 1: B's rows start on 4-element boundaries (4-wide loads in either layout)
    // Implicit im2col (CONV kernels only): A[m][k] is the NDHWC input at
    // output position m, tap k / IC, channel k % IC, zero in the padding.
    Conv3dGeom conv;
    const float* conv_in;
    int conv_op;    // post-op after the bias: 0 none, 1 relu, 2 relu6
};

template <int BM, int BN>
constexpr size_t simt_smem_bytes() {
    return 2 * (static_cast<size_t>(BK) * (BM + kPadA) + static_cast<size_t>(BK) * (BN + kPadB)) *
           sizeof(float);
}

// Four consecutive k of row `row` of a k-contiguous [rows, ld] operand (row
// start and k on 4-element boundaries), zero past the row count and k_end.
template <In I>
__device__ __forceinline__ void load_krow4(const typename Elem<I>::T* X, int64_t ld, int row, int rows, int k,
                                           int k_end, float (&v)[4]) {
    v[0] = v[1] = v[2] = v[3] = 0.0f;
    if (row >= rows || k >= k_end) return;
    const typename Elem<I>::T* q = X + (int64_t)row * ld + k;
    if (k + 4 <= k_end) {
        load4<I>(q, v);
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (k + c < k_end) v[c] = dec<I>(q[c]);
    }
}

template <In IA, In IB, int BM, int BN, bool CONV = false>
__global__ void __launch_bounds__(kThreads, 2)
gemm_simt_kernel(const SimtParams p) {
    using TA = typename Elem<IA>::T;
    using TB = typename Elem<IB>::T;
    constexpr int kColGroups = BN / 4;               // threads across a tile row
    constexpr int kRowGroups = kThreads / kColGroups;
    constexpr int TM = BM / kRowGroups;              // rows per thread
    static_assert(TM >= 1, "tile too small for 256 threads");
    constexpr int LA = BM * BK / kThreads;           // A elements each thread stages per slice
    constexpr int LB = BK * BN / kThreads;           // B elements (16)
    constexpr int SA = BK * (BM + kPadA);            // floats per A buffer
    constexpr int SB = BK * (BN + kPadB);
    extern __shared__ __align__(16) float smem[];
    float* sA = smem;                 // [2][BK][BM + kPadA]
    float* sB = smem + 2 * SA;        // [2][BK][BN + kPadB]

    pdl_wait();
    pdl_launch_dependents();

    const GemmArgs& g = p.g;
    const int tid = threadIdx.x;
    const int tx = tid % kColGroups, ty = tid / kColGroups;   // columns 4*tx.., rows TM*ty..
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int k_begin = blockIdx.z * p.kchunk;
    const int k_end = min(g.K, k_begin + p.kchunk);
    const int nslices = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;
    const TA* A = static_cast<const TA*>(g.A);
    const TB* B = static_cast<const TB*>(g.B);

    // Shared-memory layout: operand element (row, k) of a slice sits at
    // k * (R + 4) + swz(row, k), where swz flips bits 2-4 of the row by k / 4.
    // Groups of four rows stay contiguous (16-byte reads in the FMA loop), and
    // the transposing stores of k-contiguous data (8 threads per 32-k row
    // segment, 4 rows per warp) land in 32 distinct banks.
    constexpr int kSwzA = BM / 4 - 1 < 7 ? BM / 4 - 1 : 7;
    constexpr int kSwzB = BN / 4 - 1 < 7 ? BN / 4 - 1 : 7;
    auto swz = [](int row, int k, int mask) { return row ^ (4 * ((k >> 2) & mask)); };
    // k-contiguous operand (A not transposed, B transposed) with 4-element
    // aligned rows: float4 e4 of a slice is row 4 * (e4 / 32) + lane / 8,
    // k = 4 * (lane % 8), so a warp reads four whole 128-byte row segments.
    auto kvec_coord = [](int e4, int& row, int& k) {
        row = 4 * (e4 >> 5) + ((e4 & 31) >> 3);
        k = 4 * (e4 & 7);
    };
    auto a_coord = [&](int e, int& m, int& k) {
        if (g.a_trans) { m = e % BM; k = e / BM; } else { k = e % BK; m = e / BK; }
    };
    auto b_coord = [&](int e, int& n, int& k) {
        if (g.b_trans) { k = e % BK; n = e / BK; } else { n = e % BN; k = e / BN; }
    };
    const bool vec_a = BM >= 32 && !g.a_trans && p.vec_a;
    const bool vec_bt = g.b_trans && p.vec_b;
    const bool vec_bn = !g.b_trans && p.vec_b;
    // CONV: the tile's output positions (id0, ih0, iw0, batch or -1) and the
    // tap table (kd << 20 | kh << 10 | kw) decoded once, behind the stage buffers.
    const int4* s_rows = nullptr;
    const int* s_tap = nullptr;
    if constexpr (CONV) {
        int4* rows = reinterpret_cast<int4*>(smem + 2 * SA + 2 * SB);
        int* tab = reinterpret_cast<int*>(rows + BM);
        const Conv3dGeom& cg = p.conv;
        for (int r = tid; r < BM; r += kThreads) {
            const int64_t m = static_cast<int64_t>(m0) + r;
            int4 v = make_int4(0, 0, 0, -1);
            if (m < g.M) {
                const int ow = static_cast<int>(m % cg.OW);
                int64_t t = m / cg.OW;
                const int oh = static_cast<int>(t % cg.OH);
                t /= cg.OH;
                const int od = static_cast<int>(t % cg.OD);
                v = make_int4(od * cg.sd - cg.pd, oh * cg.sh - cg.ph, ow * cg.sw - cg.pw, static_cast<int>(t / cg.OD));
            }
            rows[r] = v;
        }
        const int taps = cg.KD * cg.KH * cg.KW;
        for (int t = tid; t < taps; t += kThreads) {
            const int kw = t % cg.KW, r2 = t / cg.KW;
            tab[t] = ((r2 / cg.KH) << 20) | ((r2 % cg.KH) << 10) | kw;
        }
        __syncthreads();
        s_rows = rows;
        s_tap = tab;
    }
    float ra[LA], rb[LB];
    auto load_slice = [&](int k0) {
        if constexpr (CONV) {
            // k (a multiple of 4) is the same for all of a thread's rows; the
            // four channels of a float4 belong to one tap as IC % 4 == 0.
            const Conv3dGeom& cg = p.conv;
            int m, k;
            kvec_coord(tid, m, k);
            const int gk = k0 + k;
            const bool kin = gk < k_end;
            int kd = 0, kh = 0, kw = 0, c = 0;
            if (kin) {
                const int tap = gk / cg.IC;
                c = gk - tap * cg.IC;
                const int pk = s_tap[tap];
                kd = pk >> 20;
                kh = (pk >> 10) & 1023;
                kw = pk & 1023;
            }
#pragma unroll
            for (int i = 0; i < LA / 4; ++i) {
                int mi, ki;
                kvec_coord(tid + i * kThreads, mi, ki);
                const int4 ri = s_rows[mi];
                const int id = ri.x + kd, ih = ri.y + kh, iw = ri.z + kw;
                float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (kin && ri.w >= 0 && id >= 0 && id < cg.ID && ih >= 0 && ih < cg.IH && iw >= 0 && iw < cg.IW)
                    v = __ldg(reinterpret_cast<const float4*>(
                        p.conv_in + (((static_cast<int64_t>(ri.w) * cg.ID + id) * cg.IH + ih) * cg.IW + iw) * cg.IC + c));
                ra[4 * i] = v.x; ra[4 * i + 1] = v.y; ra[4 * i + 2] = v.z; ra[4 * i + 3] = v.w;
            }
        } else if constexpr (BM >= 32) {
            if (vec_a) {
#pragma unroll
                for (int i = 0; i < LA / 4; ++i) {
                    int m, k;
                    kvec_coord(tid + i * kThreads, m, k);
                    float v[4];
                    load_krow4<IA>(A, g.lda, m0 + m, g.M, k0 + k, k_end, v);
#pragma unroll
                    for (int c = 0; c < 4; ++c) ra[4 * i + c] = v[c];
                }
            }
        }
        if (!CONV && !vec_a) {
#pragma unroll
            for (int i = 0; i < LA; ++i) {
                int m, k;
                a_coord(tid + i * kThreads, m, k);
                const int gm = m0 + m, gk = k0 + k;
                ra[i] = (gm < g.M && gk < k_end)
                            ? dec<IA>(A[g.a_trans ? (int64_t)gk * g.lda + gm : (int64_t)gm * g.lda + gk])
                            : 0.0f;
            }
        }
        if (vec_bn) {
#pragma unroll
            for (int i = 0; i < LB / 4; ++i) {
                const int e = tid + i * kThreads;
                const int n4 = e % (BN / 4), k = e / (BN / 4);
                const int gn = n0 + 4 * n4, gk = k0 + k;
                float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (gk < k_end) {
                    const TB* row = B + (int64_t)gk * g.ldb + gn;
                    if (gn + 4 <= g.N) {
                        load4<IB>(row, v);
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            if (gn + c < g.N) v[c] = dec<IB>(row[c]);
                    }
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) rb[4 * i + c] = v[c];
            }
        } else if (vec_bt) {
#pragma unroll
            for (int i = 0; i < LB / 4; ++i) {
                int n, k;
                kvec_coord(tid + i * kThreads, n, k);
                float v[4];
                load_krow4<IB>(B, g.ldb, n0 + n, g.N, k0 + k, k_end, v);
#pragma unroll
                for (int c = 0; c < 4; ++c) rb[4 * i + c] = v[c];
            }
        } else {
#pragma unroll
            for (int i = 0; i < LB; ++i) {
                int n, k;
                b_coord(tid + i * kThreads, n, k);
                const int gn = n0 + n, gk = k0 + k;
                rb[i] = (gn < g.N && gk < k_end)
                            ? dec<IB>(B[g.b_trans ? (int64_t)gn * g.ldb + gk : (int64_t)gk * g.ldb + gn])
                            : 0.0f;
            }
        }
    };
    auto store_slice = [&](int buf) {
        float* a = sA + buf * SA;
        float* b = sB + buf * SB;
        if constexpr (BM >= 32) {
            if (vec_a) {
#pragma unroll
                for (int i = 0; i < LA / 4; ++i) {
                    int m, k;
                    kvec_coord(tid + i * kThreads, m, k);
                    const int col = swz(m, k, kSwzA);     // same for k .. k + 3
#pragma unroll
                    for (int c = 0; c < 4; ++c) a[(k + c) * (BM + kPadA) + col] = ra[4 * i + c];
                }
            }
        }
        if (!vec_a) {
#pragma unroll
            for (int i = 0; i < LA; ++i) {
                int m, k;
                a_coord(tid + i * kThreads, m, k);
                a[k * (BM + kPadA) + swz(m, k, kSwzA)] = ra[i];
            }
        }
        if (vec_bn) {
#pragma unroll
            for (int i = 0; i < LB / 4; ++i) {
                const int e = tid + i * kThreads;
                const int n4 = e % (BN / 4), k = e / (BN / 4);
                *reinterpret_cast<float4*>(&b[k * (BN + kPadB) + swz(4 * n4, k, kSwzB)]) =
                    make_float4(rb[4 * i], rb[4 * i + 1], rb[4 * i + 2], rb[4 * i + 3]);
            }
        } else if (vec_bt) {
#pragma unroll
            for (int i = 0; i < LB / 4; ++i) {
                int n, k;
                kvec_coord(tid + i * kThreads, n, k);
                const int col = swz(n, k, kSwzB);
#pragma unroll
                for (int c = 0; c < 4; ++c) b[(k + c) * (BN + kPadB) + col] = rb[4 * i + c];
            }
        } else {
#pragma unroll
            for (int i = 0; i < LB; ++i) {
                int n, k;
                b_coord(tid + i * kThreads, n, k);
                b[k * (BN + kPadB) + swz(n, k, kSwzB)] = rb[i];
            }
        }
    };

    float acc[TM][4];
#pragma unroll
    for (int r = 0; r < TM; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;

    if (nslices > 0) {
        load_slice(k_begin);
        store_slice(0);
        __syncthreads();
    }
    for (int t = 0; t < nslices; ++t) {
        const int buf = t & 1;
        if (t + 1 < nslices) load_slice(k_begin + (t + 1) * BK);
        const float* a = sA + buf * SA;
        const float* b = sB + buf * SB;
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float av[TM];
            if constexpr (TM >= 4) {
#pragma unroll
                for (int q = 0; q < TM / 4; ++q) {
                    const float4 v = *reinterpret_cast<const float4*>(
                        a + k * (BM + kPadA) + swz(ty * TM + 4 * q, k, kSwzA));
                    av[4 * q] = v.x; av[4 * q + 1] = v.y; av[4 * q + 2] = v.z; av[4 * q + 3] = v.w;
                }
            } else if constexpr (TM == 2) {
                const float2 v = *reinterpret_cast<const float2*>(a + k * (BM + kPadA) + swz(ty * 2, k, kSwzA));
                av[0] = v.x; av[1] = v.y;
            } else {
                av[0] = a[k * (BM + kPadA) + swz(ty, k, kSwzA)];
            }
            const float4 bv = *reinterpret_cast<const float4*>(b + k * (BN + kPadB) + swz(4 * tx, k, kSwzB));
#pragma unroll
            for (int r = 0; r < TM; ++r) {
                acc[r][0] = fmaf(av[r], bv.x, acc[r][0]);
                acc[r][1] = fmaf(av[r], bv.y, acc[r][1]);
                acc[r][2] = fmaf(av[r], bv.z, acc[r][2]);
                acc[r][3] = fmaf(av[r], bv.w, acc[r][3]);
            }
        }
        if (t + 1 < nslices) store_slice(buf ^ 1);
        __syncthreads();
    }

    float* C = static_cast<float*>(g.C);
    auto finish = [&](int gm, int gn, float sum) {
        float* cp = C + (int64_t)gm * g.ldc + gn;
        float v = add_bias((g.beta == 0.0f) ? g.alpha * sum : fmaf(g.alpha, sum, g.beta * *cp), g.bias, gn);
        if constexpr (CONV) {
            if (p.conv_op == 1) v = v > 0.0f ? v : 0.0f;
            else if (p.conv_op == 2) v = v > 0.0f ? (v < 6.0f ? v : 6.0f) : 0.0f;
        }
        *cp = v;
    };
    if (gridDim.z == 1) {
#pragma unroll
        for (int r = 0; r < TM; ++r) {
            const int gm = m0 + ty * TM + r;
            if (gm >= g.M) continue;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int gn = n0 + 4 * tx + c;
                if (gn < g.N) finish(gm, gn, acc[r][c]);
            }
        }
        return;
    }
    // K split over the cluster: every CTA parks its partial tile in its own
    // shared memory (the stage buffers are idle after the last barrier), then
    // CTA q sums elements q, q + S, ... of the tile over ranks 0..S-1.
    float* part = smem;                              // [BM][BN]
#pragma unroll
    for (int r = 0; r < TM; ++r)
        *reinterpret_cast<float4*>(&part[(ty * TM + r) * BN + 4 * tx]) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    cluster_sync_all();
    const uint32_t S = gridDim.z;
    const uint32_t q = cluster_ctarank();
    const uint32_t part_addr = smem_u32(part);
    for (int e = static_cast<int>(q) * kThreads + tid; e < BM * BN; e += static_cast<int>(S) * kThreads) {
        const int m = e / BN, n = e - m * BN;
        const int gm = m0 + m, gn = n0 + n;
        float v[kMaxSplits];
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)
            v[r] = r < static_cast<int>(S) ? ld_dsmem_f32(map_to_cta(part_addr + e * 4u, static_cast<uint32_t>(r)))
                                           : 0.0f;
        float sum = 0.0f;
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)
            if (r < static_cast<int>(S)) sum += v[r];
        if (gm < g.M && gn < g.N) finish(gm, gn, sum);
    }
    cluster_sync_all();   // no CTA leaves while another still reads its tile
}

template <In IA, In IB, int BN>
const void* simt_fn_bn(int bm) {
    switch (bm) {
        case 16: return reinterpret_cast<const void*>(&gemm_simt_kernel<IA, IB, 16, BN>);
        case 32: return reinterpret_cast<const void*>(&gemm_simt_kernel<IA, IB, 32, BN>);
        case 64: return reinterpret_cast<const void*>(&gemm_simt_kernel<IA, IB, 64, BN>);
        case 128:
            if constexpr (BN == 64) return reinterpret_cast<const void*>(&gemm_simt_kernel<IA, IB, 128, 64>);
            return nullptr;
        default: return nullptr;
    }
}

template <In IA, In IB>
const void* simt_fn(int bm, int bn) {
    return bn == 64 ? simt_fn_bn<IA, IB, 64>(bm) : (bn == 128 ? simt_fn_bn<IA, IB, 128>(bm) : nullptr);
}

const void* simt_select(In ia, In ib, int bm, int bn) {
    if (ia == In::F32 && ib == In::F32) return simt_fn<In::F32, In::F32>(bm, bn);
    if (ia == In::BF16 && ib == In::BF16) return simt_fn<In::BF16, In::BF16>(bm, bn);
    if (ia == In::F32R && ib == In::F32R) return simt_fn<In::F32R, In::F32R>(bm, bn);
    if (ia == In::RE4 && ib == In::RE5) return simt_fn<In::RE4, In::RE5>(bm, bn);
    if (ia == In::RE5 && ib == In::RE5) return simt_fn<In::RE5, In::RE5>(bm, bn);
    return nullptr;
}

// Implicit-im2col FP32 kernels (conv3d): the tile shapes the plan picks for M >= 64.
const void* simt_conv_select(int bm, int bn) {
    if (bm == 64 && bn == 64) return reinterpret_cast<const void*>(&gemm_simt_kernel<In::F32, In::F32, 64, 64, true>);
    if (bm == 128 && bn == 64) return reinterpret_cast<const void*>(&gemm_simt_kernel<In::F32, In::F32, 128, 64, true>);
    if (bm == 64 && bn == 128) return reinterpret_cast<const void*>(&gemm_simt_kernel<In::F32, In::F32, 64, 128, true>);
    return nullptr;
}

size_t smem_for(int bm, int bn) {
    if (bn == 64)
        return bm == 16 ? simt_smem_bytes<16, 64>()
                        : (bm == 32 ? simt_smem_bytes<32, 64>()
                                    : (bm == 64 ? simt_smem_bytes<64, 64>() : simt_smem_bytes<128, 64>()));
    return bm == 16 ? simt_smem_bytes<16, 128>() : (bm == 32 ? simt_smem_bytes<32, 128>() : simt_smem_bytes<64, 128>());
}

// Dynamic shared memory above 48 KB needs the attribute once per device and kernel.
cudaError_t prepare(const void* fn, size_t smem) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({dev, fn})) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess) done.insert({dev, fn});
    return e;
}

size_t elem_size(In i) {
    switch (i) {
        case In::F32:
        case In::F32R: return 4;
        case In::BF16: return 2;
        default: return 1;
    }
}

}  // namespace

GemmSimtPlan gemm_simt_plan(const GemmArgs& g, int num_sms) {
    GemmSimtPlan p;
    p.bm = g.M <= 16 ? 16 : (g.M <= 32 ? 32 : 64);
    p.bn = g.N <= 64 ? 64 : 128;
    // Narrow outputs with many rows (conv3d's im2col GEMM: N = OC, M = output
    // positions): 128 x 64 tiles give each thread 8 x 4 outputs, as the 64 x
    // 128 tiles do for wide N, instead of 4 x 4.
    if (p.bn == 64 && g.M >= 128 * static_cast<int64_t>(num_sms > 0 ? num_sms : 148)) p.bm = 128;
    const int64_t tiles = static_cast<int64_t>((g.N + p.bn - 1) / p.bn) * ((g.M + p.bm - 1) / p.bm);
    const int64_t want = 2 * static_cast<int64_t>(num_sms > 0 ? num_sms : 148);
    int s = static_cast<int>((want + tiles - 1) / tiles);
    const int max_by_k = (g.K + 2 * BK - 1) / (2 * BK);      // at least two slices per split
    if (s > max_by_k) s = max_by_k;
    if (s > kMaxSplits) s = kMaxSplits;
    if (s < 1) s = 1;
    int kchunk = (g.K + s - 1) / s;
    kchunk = (kchunk + BK - 1) / BK * BK;
    p.splits = (g.K + kchunk - 1) / kchunk;
    p.kchunk = kchunk;
    return p;
}

namespace {

cudaError_t launch_simt(const void* fn, SimtParams& sp, const GemmSimtPlan& plan, size_t smem, cudaStream_t s) {
    const GemmArgs& g = sp.g;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((g.N + plan.bn - 1) / plan.bn), static_cast<unsigned>((g.M + plan.bm - 1) / plan.bm),
                       static_cast<unsigned>(plan.splits));
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int na = 1;
    if (plan.splits > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = static_cast<unsigned>(plan.splits);
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    void* args[] = {&sp};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_gemm_simt(In ia, In ib, const GemmArgs& g, const GemmSimtPlan& plan,
                             cudaStream_t s) {
    const void* fn = simt_select(ia, ib, plan.bm, plan.bn);
    if (!fn || plan.splits < 1 || plan.splits > kMaxSplits || plan.kchunk < BK) return cudaErrorInvalidValue;
    const size_t smem = smem_for(plan.bm, plan.bn);
    cudaError_t e = prepare(fn, smem);
    if (e != cudaSuccess) return e;
    SimtParams sp = {};
    sp.g = g;
    sp.kchunk = plan.kchunk;
    const size_t eb = elem_size(ib);
    sp.vec_b = (reinterpret_cast<uintptr_t>(g.B) % (4 * eb) == 0 && g.ldb % 4 == 0) ? 1 : 0;
    const size_t ea = elem_size(ia);
    sp.vec_a = (reinterpret_cast<uintptr_t>(g.A) % (4 * ea) == 0 && g.lda % 4 == 0) ? 1 : 0;
    return launch_simt(fn, sp, plan, smem, s);
}

bool gemm_simt_conv_ok(const Conv3dGeom& cg, const float* in, const float* filter) {
    return cg.IC % 4 == 0 && cg.M >= 64 && cg.M <= INT32_MAX && cg.K <= INT32_MAX &&
           cg.KD * cg.KH * cg.KW <= kConv3dMaxTaps && cg.KD < 1024 && cg.KH < 1024 && cg.KW < 1024 &&
           reinterpret_cast<uintptr_t>(in) % 16 == 0 && reinterpret_cast<uintptr_t>(filter) % 16 == 0;
}

cudaError_t launch_gemm_simt_conv(const Conv3dGeom& cg, const float* in, const float* filter, const float* bias,
                                  int op, float* out, int num_sms, cudaStream_t s) {
    if (!gemm_simt_conv_ok(cg, in, filter)) return cudaErrorInvalidValue;
    GemmArgs g;
    g.M = static_cast<int>(cg.M);
    g.N = cg.OC;
    g.K = static_cast<int>(cg.K);
    g.alpha = 1.0f;
    g.beta = 0.0f;
    g.A = in;                 // not read: the CONV kernel gathers from conv_in
    g.lda = cg.K;
    g.a_trans = 0;
    g.B = filter;             // [OC, K]
    g.ldb = cg.K;
    g.b_trans = 1;
    g.C = out;                // [M, OC]
    g.ldc = cg.OC;
    g.bias = bias;            // per output channel, then the post-op, in the epilogue
    const GemmSimtPlan plan = gemm_simt_plan(g, num_sms);
    const void* fn = simt_conv_select(plan.bm, plan.bn);
    if (!fn || plan.splits < 1 || plan.splits > kMaxSplits || plan.kchunk < BK) return cudaErrorInvalidValue;
    const size_t base = smem_for(plan.bm, plan.bn) + static_cast<size_t>(plan.bm) * sizeof(int4);
    cudaError_t e = prepare(fn, base + kConv3dMaxTaps * sizeof(int));
    if (e != cudaSuccess) return e;
    SimtParams sp = {};
    sp.g = g;
    sp.kchunk = plan.kchunk;
    sp.vec_a = 1;
    sp.vec_b = 1;
    sp.conv = cg;
    sp.conv_in = in;
    sp.conv_op = op;
    return launch_simt(fn, sp, plan, base + static_cast<size_t>(cg.KD * cg.KH * cg.KW) * sizeof(int), s);
}

}  // namespace dnnopt_b200
