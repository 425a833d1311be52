// Small-M (M <= 8) dot-form GEMV for a B stored N x K (K contiguous):
//   C[m, n] = epilogue( sum_k A[m, k] * B[n, k] )
//
// Serves:
//   * gemm_int8_int8int8int32 (reference src/gemm/gemm_int8_native.cpp:189-248,
//     whose B is [N, K] with ldb >= K): exact int32 dot products via dp4a.
//   * the FP32-API gemm_int8 after quantisation (reference
//     src/gemm/gemm_smallm_int8.cpp:198-236, :355-390): int8 dot + dequant.
//   * FP32 GEMM with op(B) = B^T (cblas_sgemm with TransB): fp32 FMA.
//   * the config-5 decode-FFN weight GEMM: bf16 activations x OCP-e4m3
//     weights with a per-row FP32 scale, bf16 output (CUDA-core variant).
//
// Each warp owns whole rows of B; lanes stride along K with 16-byte loads, so
// a warp reads 512 contiguous bytes per step and each lane keeps several loads
// in flight.  A (M x K, at most 8 rows) is staged once in shared memory and
// read back with conflict-free 16-byte loads; per-row partial sums are reduced
// with warp shuffles.  Integer accumulation is exact in any order, so the
// int8 path is bit-identical to the reference's scalar loop.
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct NkParams {
    GemmArgs g;
    int rows_per_cta;
    const float* scales;
};

template <DotKind K> struct Tr;

template <> struct Tr<DotKind::F32> {
    using TA = float; using TB = float; using Acc = float;
    static constexpr int EPC = 4;   // B elements per 16-byte chunk
    __device__ static void dot(const uint4& b, const TA* a, Acc& acc) {
        const float4 av = *reinterpret_cast<const float4*>(a);
        acc = fmaf(av.x, __uint_as_float(b.x), acc);
        acc = fmaf(av.y, __uint_as_float(b.y), acc);
        acc = fmaf(av.z, __uint_as_float(b.z), acc);
        acc = fmaf(av.w, __uint_as_float(b.w), acc);
    }
    __device__ static Acc one(TA a, TB b) { return a * b; }
};

template <> struct Tr<DotKind::S8S32> {
    using TA = int8_t; using TB = int8_t; using Acc = int32_t;
    static constexpr int EPC = 16;
    __device__ static void dot(const uint4& b, const TA* a, Acc& acc) {
        const int4 av = *reinterpret_cast<const int4*>(a);
        acc = __dp4a(av.x, static_cast<int>(b.x), acc);
        acc = __dp4a(av.y, static_cast<int>(b.y), acc);
        acc = __dp4a(av.z, static_cast<int>(b.z), acc);
        acc = __dp4a(av.w, static_cast<int>(b.w), acc);
    }
    __device__ static Acc one(TA a, TB b) { return static_cast<int32_t>(a) * static_cast<int32_t>(b); }
};

template <> struct Tr<DotKind::S8DQ> : Tr<DotKind::S8S32> {};

// BF16 appears only in the register-resident rows kernel (A's element type).
template <> struct Tr<DotKind::BF16> {
    using TA = uint16_t; using TB = uint16_t; using Acc = float;
};

template <> struct Tr<DotKind::E4M3> {
    using TA = uint16_t; using TB = uint8_t; using Acc = float;
    static constexpr int EPC = 16;
    __device__ static void dot(const uint4& b, const TA* a, Acc& acc) {
        const uint4 a0 = *reinterpret_cast<const uint4*>(a);
        const uint4 a1 = *reinterpret_cast<const uint4*>(a + 8);
        const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float2 lo = e4m3x2_to_f32x2(static_cast<uint16_t>(bw[q] & 0xFFFFu));
            float2 hi = e4m3x2_to_f32x2(static_cast<uint16_t>(bw[q] >> 16));
            uint32_t x0 = aw[2 * q], x1 = aw[2 * q + 1];
            acc = fmaf(__uint_as_float(x0 << 16), lo.x, acc);
            acc = fmaf(__uint_as_float(x0 & 0xFFFF0000u), lo.y, acc);
            acc = fmaf(__uint_as_float(x1 << 16), hi.x, acc);
            acc = fmaf(__uint_as_float(x1 & 0xFFFF0000u), hi.y, acc);
        }
    }
    __device__ static Acc one(TA a, TB b) {
        float2 v = e4m3x2_to_f32x2(static_cast<uint16_t>(b));
        return bf16_bits_to_f32(a) * v.x;
    }
};

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

template <DotKind KIND, int MT, bool VEC>
__global__ void __launch_bounds__(kThreads)
gemv_nk_kernel(const NkParams p) {
    using T = Tr<KIND>;
    using TA = typename T::TA;
    using TB = typename T::TB;
    using Acc = typename T::Acc;
    constexpr int EPC = T::EPC;
    constexpr int U = 4;   // 16-byte chunks in flight per lane

    extern __shared__ __align__(16) unsigned char smem_raw[];
    TA* sA = reinterpret_cast<TA*>(smem_raw);   // [MT][kpad]

    const GemmArgs& g = p.g;
    const int K = g.K;
    const int kpad = (K + EPC - 1) / EPC * EPC;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const TA* A = static_cast<const TA*>(g.A);
    const TB* B = static_cast<const TB*>(g.B);

    // Stage A (rows >= M and the K tail are zero).
    for (int idx = tid; idx < MT * kpad; idx += kThreads) {
        int m = idx / kpad, k = idx - m * kpad;
        TA v = TA(0);
        if (m < g.M && k < K)
            v = A[g.a_trans ? (int64_t)k * g.lda + m : (int64_t)m * g.lda + k];
        sA[idx] = v;
    }
    __syncthreads();

    const int row_begin = blockIdx.x * p.rows_per_cta;
    const int row_end = min(g.N, row_begin + p.rows_per_cta);
    const int nchunks = VEC ? K / EPC : 0;   // full 16-byte chunks

    for (int n = row_begin + warp; n < row_end; n += kWarps) {
        const TB* brow = B + (int64_t)n * g.ldb;
        Acc acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = Acc(0);

        if constexpr (VEC) {
            const uint4* b4 = reinterpret_cast<const uint4*>(brow);
            for (int q0 = lane; q0 < nchunks; q0 += 32 * U) {
                uint4 bv[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    int q = q0 + 32 * u;
                    bv[u] = (q < nchunks) ? __ldg(b4 + q) : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    int q = q0 + 32 * u;
                    if (q < nchunks) {
#pragma unroll
                        for (int m = 0; m < MT; ++m) T::dot(bv[u], sA + m * kpad + q * EPC, acc[m]);
                    }
                }
            }
        }
        // Scalar remainder (the whole row when rows are not 16-byte aligned).
        for (int k = nchunks * EPC + lane; k < K; k += 32) {
            TB bk = brow[k];
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[m] += T::one(sA[m * kpad + k], bk);
        }

#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = warp_sum(acc[m]);

        if (lane < MT && lane < g.M) {
            Acc s = acc[0];
#pragma unroll
            for (int m = 1; m < MT; ++m) if (lane == m) s = acc[m];
            const int m = lane;
            if constexpr (KIND == DotKind::F32) {
                float* cp = static_cast<float*>(g.C) + (int64_t)m * g.ldc + n;
                *cp = add_bias((g.beta == 0.0f) ? g.alpha * s : fmaf(g.alpha, s, g.beta * *cp), g.bias, n);
            } else if constexpr (KIND == DotKind::S8S32) {
                static_cast<int32_t*>(g.C)[(int64_t)m * g.ldc + n] = s;
            } else if constexpr (KIND == DotKind::S8DQ) {
                // C = (beta == 0 ? 0 : beta*C) + (alpha*(sA*sB)) * float(acc), each op rounded.
                float* cp = static_cast<float*>(g.C) + (int64_t)m * g.ldc + n;
                float scale = __fmul_rn(g.alpha, __fmul_rn(p.scales[0], p.scales[1]));
                float c0 = (g.beta == 0.0f) ? 0.0f : __fmul_rn(g.beta, *cp);
                *cp = __fadd_rn(c0, __fmul_rn(scale, static_cast<float>(s)));
            } else {
                float v = s * p.scales[n];
                static_cast<uint16_t*>(g.C)[(int64_t)m * g.ldc + n] =
                    __bfloat16_as_ushort(__float2bfloat16_rn(v));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Register-resident variant for 16-byte aligned rows and K <= 2 * 256 chunks:
// the CTA's 256 lanes own fixed 16-byte K-chunks (lane L: chunks L and L+256),
// so each lane keeps its slice of A in registers for every row instead of
// re-reading it from shared memory.  A CTA walks its contiguous row range R
// rows at a time (R independent 16-byte loads in flight per chunk and lane),
// accumulates V = MT x R partial dot products, and reduces them with a
// transpose-reduce over lane offsets V/2 .. 1 (lane l keeps value l % V)
// followed by plain butterfly sums over offsets V .. 16, then across the 8
// warps through shared memory in warp order.  V = 32 (MT x R = 4 x 8 or
// 8 x 4) for K up to 512 chunks; V = 8 (MT = 2, R = 4, four chunks per lane)
// carries M <= 2 rows of FP32 up to K = 4096 (inner products y = W x with W
// stored row by row: 16 KB rows, A's 4096 values spread over the CTA's
// registers).
// ---------------------------------------------------------------------------
template <DotKind KIND> struct Chunk;
template <> struct Chunk<DotKind::F32> {
    using Acc = float;
    __device__ static Acc dot(const uint4& b, const uint4& a, Acc acc) {
        acc = fmaf(__uint_as_float(a.x), __uint_as_float(b.x), acc);
        acc = fmaf(__uint_as_float(a.y), __uint_as_float(b.y), acc);
        acc = fmaf(__uint_as_float(a.z), __uint_as_float(b.z), acc);
        acc = fmaf(__uint_as_float(a.w), __uint_as_float(b.w), acc);
        return acc;
    }
    static constexpr int EPC = 4;
};
template <> struct Chunk<DotKind::S8S32> {
    using Acc = int32_t;
    __device__ static Acc dot(const uint4& b, const uint4& a, Acc acc) {
        acc = __dp4a(static_cast<int>(a.x), static_cast<int>(b.x), acc);
        acc = __dp4a(static_cast<int>(a.y), static_cast<int>(b.y), acc);
        acc = __dp4a(static_cast<int>(a.z), static_cast<int>(b.z), acc);
        acc = __dp4a(static_cast<int>(a.w), static_cast<int>(b.w), acc);
        return acc;
    }
    static constexpr int EPC = 16;
};
template <> struct Chunk<DotKind::S8DQ> : Chunk<DotKind::S8S32> {};
template <> struct Chunk<DotKind::BF16> {
    using Acc = float;
    __device__ static float lo(uint32_t w) { return __uint_as_float(w << 16); }
    __device__ static float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
    __device__ static Acc dot(const uint4& b, const uint4& a, Acc acc) {
        acc = fmaf(lo(a.x), lo(b.x), acc); acc = fmaf(hi(a.x), hi(b.x), acc);
        acc = fmaf(lo(a.y), lo(b.y), acc); acc = fmaf(hi(a.y), hi(b.y), acc);
        acc = fmaf(lo(a.z), lo(b.z), acc); acc = fmaf(hi(a.z), hi(b.z), acc);
        acc = fmaf(lo(a.w), lo(b.w), acc); acc = fmaf(hi(a.w), hi(b.w), acc);
        return acc;
    }
    static constexpr int EPC = 8;
};

struct RowsParams {
    GemmArgs g;
    int rows_per_cta;   // multiple of R
    const float* scales;
};

// 16 bytes of A row m starting at element k (zero-filled past K; any alignment).
template <typename TA>
__device__ __forceinline__ uint4 load_a_chunk(const TA* A, int64_t lda, int a_trans, int m, int k,
                                              int K) {
    constexpr int E = 16 / sizeof(TA);
    if (!a_trans && k + E <= K && (reinterpret_cast<uintptr_t>(A + (int64_t)m * lda + k) & 15u) == 0)
        return *reinterpret_cast<const uint4*>(A + (int64_t)m * lda + k);
    TA v[E];
#pragma unroll
    for (int e = 0; e < E; ++e)
        v[e] = (k + e < K) ? A[a_trans ? (int64_t)(k + e) * lda + m : (int64_t)m * lda + k + e] : TA(0);
    uint4 r;
    memcpy(&r, v, 16);
    return r;
}

template <DotKind KIND, int MT, int R, int KCH>
__global__ void __launch_bounds__(kThreads)
gemv_rows_kernel(const RowsParams p) {
    using C = Chunk<KIND>;
    using Acc = typename C::Acc;
    using TA = typename Tr<KIND>::TA;
    constexpr int V = MT * R;
    static_assert(V == 8 || V == 16 || V == 32, "V values per lane, a power of two up to 32");
    __shared__ Acc red[2][kWarps][32];

    pdl_wait();
    pdl_launch_dependents();

    const GemmArgs& g = p.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nchunks = g.K / C::EPC;                 // K % EPC == 0 on this path
    const TA* A = static_cast<const TA*>(g.A);

    uint4 a[KCH][MT];
#pragma unroll
    for (int j = 0; j < KCH; ++j) {
        const int ch = tid + j * kThreads;
#pragma unroll
        for (int m = 0; m < MT; ++m)
            a[j][m] = (m < g.M && ch < nchunks)
                          ? load_a_chunk<TA>(A, g.lda, g.a_trans, m, ch * C::EPC, g.K)
                          : make_uint4(0u, 0u, 0u, 0u);
    }

    const int row_begin = blockIdx.x * p.rows_per_cta;
    const int row_end = min(g.N, row_begin + p.rows_per_cta);
    const uint4* B = static_cast<const uint4*>(g.B);
    const int64_t ldb_chunks = g.ldb / C::EPC;
    auto load_rows = [&](uint4 (&b)[KCH][R], int r0) {
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
            const int ch = tid + j * kThreads;
#pragma unroll
            for (int r = 0; r < R; ++r)
                b[j][r] = (ch < nchunks && r0 + r < row_end) ? __ldg(B + (int64_t)(r0 + r) * ldb_chunks + ch)
                                                            : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    // Software pipeline: the next R rows are requested before the current
    // ones are reduced, so a CTA always has two row groups in flight.
    uint4 bc[KCH][R], bn[KCH][R];
    if (row_begin < row_end) load_rows(bc, row_begin);
    int buf = 0;
    for (int r0 = row_begin; r0 < row_end; r0 += R, buf ^= 1) {
        if (r0 + R < row_end) load_rows(bn, r0 + R);
        Acc v[V];
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                Acc acc = Acc(0);
#pragma unroll
                for (int j = 0; j < KCH; ++j) acc = C::dot(bc[j][r], a[j][m], acc);
                v[m * R + r] = acc;
            }
        // Transpose-reduce: after the step with offset s, a lane keeps the half
        // selected by its bit s; lane l ends with the sum of value l % V over
        // the lanes that differ from it in bits below V, and the butterfly
        // adds the lanes that differ above.
#pragma unroll
        for (int s = V / 2; s >= 1; s >>= 1) {
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int i = 0; i < s; ++i) {
                Acc send = upper ? v[i] : v[i + s];
                Acc keep = upper ? v[i + s] : v[i];
                v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, s);
            }
        }
#pragma unroll
        for (int o = V; o < 32; o <<= 1) v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], o);
        red[buf][warp][lane] = v[0];
        __syncthreads();
        if (warp == 0 && lane < V) {
            Acc t = red[buf][0][lane];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) t += red[buf][w][lane];
            const int m = lane / R, n = r0 + (lane % R);
            if (m < g.M && n < row_end) {
                if constexpr (KIND == DotKind::F32 || KIND == DotKind::BF16) {
                    float* cp = static_cast<float*>(g.C) + (int64_t)m * g.ldc + n;
                    *cp = add_bias((g.beta == 0.0f) ? g.alpha * t : fmaf(g.alpha, t, g.beta * *cp), g.bias, n);
                } else if constexpr (KIND == DotKind::S8S32) {
                    static_cast<int32_t*>(g.C)[(int64_t)m * g.ldc + n] = t;
                } else {
                    float* cp = static_cast<float*>(g.C) + (int64_t)m * g.ldc + n;
                    float scale = __fmul_rn(g.alpha, __fmul_rn(p.scales[0], p.scales[1]));
                    float c0 = (g.beta == 0.0f) ? 0.0f : __fmul_rn(g.beta, *cp);
                    *cp = __fadd_rn(c0, __fmul_rn(scale, static_cast<float>(t)));
                }
            }
        }
        // red[buf] is rewritten two iterations later, after the next barrier.
#pragma unroll
        for (int j = 0; j < KCH; ++j)
#pragma unroll
            for (int r = 0; r < R; ++r) bc[j][r] = bn[j][r];
    }
}

// ---------------------------------------------------------------------------
// Bulk-copy variant of the register-resident dot form (gemv_rows_bulk): the
// same lane -> 16-byte K-chunk ownership (A in registers) and the same
// transpose-reduce, but B's rows reach the CTA through a ring of shared-memory
// stages of R rows, filled by a ninth (producer) warp with cp.async.bulk: one
// copy per stage when the rows are dense in memory (ldb == K), else one per
// row.  The bytes in flight then cost no registers (two CTAs per SM keep up
// to six stages, 192 KB, in flight per SM), and the consumer warps release a
// stage on an mbarrier as soon as their reads of it are done, before the
// reduction.  Every wait is bounded (kMbarTimeoutNs); a timeout records an
// error word and the remaining waits give up.
// ---------------------------------------------------------------------------
constexpr int kBulkThreads = kThreads + 32;   // 8 consumer warps + 1 producer warp
constexpr int kBulkMaxStages = 6;

struct RowsBulkParams {
    GemmArgs g;
    int rows_per_cta;      // multiple of R
    int stages;            // ring depth (2..kBulkMaxStages)
    uint32_t row_bytes;    // K * element size (a multiple of 16)
    const float* scales;
    uint32_t* err;
};

template <DotKind KIND, int MT, int R, int KCH>
__global__ void __launch_bounds__(kBulkThreads, 1)
gemv_rows_bulk_kernel(const RowsBulkParams p) {
    using C = Chunk<KIND>;
    using Acc = typename C::Acc;
    using TA = typename Tr<KIND>::TA;
    constexpr int V = MT * R;
    static_assert(V == 8 || V == 16 || V == 32, "V values per lane, a power of two up to 32");
    extern __shared__ __align__(128) unsigned char stage_mem[];
    __shared__ __align__(8) uint64_t full[kBulkMaxStages];
    __shared__ __align__(8) uint64_t empty[kBulkMaxStages];
    __shared__ Acc red[2][kWarps][32];
    __shared__ uint32_t abort_flag;

    const GemmArgs& g = p.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row_begin = blockIdx.x * p.rows_per_cta;
    const int row_end = min(g.N, row_begin + p.rows_per_cta);
    const int ngroups = row_begin < row_end ? (row_end - row_begin + R - 1) / R : 0;
    const uint32_t stage_bytes = static_cast<uint32_t>(R) * p.row_bytes;

    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        abort_flag = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();
    pdl_launch_dependents();

    if (warp == kWarps) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const unsigned char* Bb = static_cast<const unsigned char*>(g.B);
            const int64_t ldb_bytes = g.ldb * static_cast<int64_t>(sizeof(typename Tr<KIND>::TB));
            const bool dense = ldb_bytes == static_cast<int64_t>(p.row_bytes);
            for (int j = 0; j < ngroups; ++j) {
                const int s = j % p.stages;
                if (j >= p.stages &&
                    !mbar_wait(&empty[s], static_cast<uint32_t>(j / p.stages - 1) & 1u, &abort_flag, p.err))
                    break;
                const int r0 = row_begin + j * R;
                const int nr = min(R, row_end - r0);
                mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nr) * p.row_bytes);
                unsigned char* dst = stage_mem + static_cast<size_t>(s) * stage_bytes;
                if (dense) {
                    bulk_load_1d(dst, Bb + r0 * ldb_bytes, static_cast<uint32_t>(nr) * p.row_bytes, &full[s]);
                } else {
                    for (int r = 0; r < nr; ++r)
                        bulk_load_1d(dst + static_cast<size_t>(r) * p.row_bytes, Bb + (r0 + r) * ldb_bytes,
                                     p.row_bytes, &full[s]);
                }
            }
        }
        return;
    }

    // ---------------- consumers (warps 0..7) ----------------
    const int nchunks = g.K / C::EPC;
    const TA* A = static_cast<const TA*>(g.A);
    uint4 a[KCH][MT];
#pragma unroll
    for (int j = 0; j < KCH; ++j) {
        const int ch = tid + j * kThreads;
#pragma unroll
        for (int m = 0; m < MT; ++m)
            a[j][m] = (m < g.M && ch < nchunks)
                          ? load_a_chunk<TA>(A, g.lda, g.a_trans, m, ch * C::EPC, g.K)
                          : make_uint4(0u, 0u, 0u, 0u);
    }
    int buf = 0;
    for (int j = 0; j < ngroups; ++j, buf ^= 1) {
        const int s = j % p.stages;
        const bool ok = mbar_wait(&full[s], static_cast<uint32_t>(j / p.stages) & 1u, &abort_flag, p.err);
        const int r0 = row_begin + j * R;
        Acc v[V];
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = Acc(0);
        if (ok) {
            const unsigned char* st = stage_mem + static_cast<size_t>(s) * stage_bytes;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                uint4 b[KCH];
#pragma unroll
                for (int kc = 0; kc < KCH; ++kc) {
                    const int ch = tid + kc * kThreads;
                    b[kc] = ch < nchunks ? *reinterpret_cast<const uint4*>(st + r * p.row_bytes + ch * 16)
                                         : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    Acc acc = Acc(0);
#pragma unroll
                    for (int kc = 0; kc < KCH; ++kc) acc = C::dot(b[kc], a[kc][m], acc);
                    v[m * R + r] = acc;
                }
            }
        }
        // This warp is done with the stage.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
        for (int sh = V / 2; sh >= 1; sh >>= 1) {
            const bool upper = (lane & sh) != 0;
#pragma unroll
            for (int i = 0; i < sh; ++i) {
                Acc send = upper ? v[i] : v[i + sh];
                Acc keep = upper ? v[i + sh] : v[i];
                v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, sh);
            }
        }
#pragma unroll
        for (int o = V; o < 32; o <<= 1) v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], o);
        red[buf][warp][lane] = v[0];
        named_barrier_sync(1, kThreads);
        if (warp == 0 && lane < V && ok) {
            Acc t = red[buf][0][lane];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) t += red[buf][w][lane];
            const int m = lane / R, n = r0 + (lane % R);
            if (m < g.M && n < row_end) {
                if constexpr (KIND == DotKind::F32 || KIND == DotKind::BF16) {
                    float* cp = static_cast<float*>(g.C) + (int64_t)m * g.ldc + n;
                    *cp = add_bias((g.beta == 0.0f) ? g.alpha * t : fmaf(g.alpha, t, g.beta * *cp), g.bias, n);
                } else if constexpr (KIND == DotKind::S8S32) {
                    static_cast<int32_t*>(g.C)[(int64_t)m * g.ldc + n] = t;
                } else {
                    float* cp = static_cast<float*>(g.C) + (int64_t)m * g.ldc + n;
                    float scale = __fmul_rn(g.alpha, __fmul_rn(p.scales[0], p.scales[1]));
                    float c0 = (g.beta == 0.0f) ? 0.0f : __fmul_rn(g.beta, *cp);
                    *cp = __fadd_rn(c0, __fmul_rn(scale, static_cast<float>(t)));
                }
            }
        }
        // red[buf] is rewritten two groups later, after the next barrier.
    }
}

template <DotKind KIND, int KCH>
const void* rows_bulk_select_mt(int mt) {
    switch (mt) {
        case 1:
        case 2:
        case 4: return reinterpret_cast<const void*>(&gemv_rows_bulk_kernel<KIND, 4, 8, KCH>);
        case 8: return reinterpret_cast<const void*>(&gemv_rows_bulk_kernel<KIND, 8, 4, KCH>);
        default: return nullptr;
    }
}

template <DotKind KIND, int KCH>
const void* rows_select_mt(int mt) {
    switch (mt) {
        case 1:
        case 2:   // rows >= M of A are zero: the MT=4 kernel, R=8 keeps registers down
        case 4: return reinterpret_cast<const void*>(&gemv_rows_kernel<KIND, 4, 8, KCH>);
        case 8: return reinterpret_cast<const void*>(&gemv_rows_kernel<KIND, 8, 4, KCH>);
        default: return nullptr;
    }
}

// Kernel and rows per step for `kch` 16-byte chunks per lane (1, 2, or 3-4
// for the deep FP32 variant, M <= 2 only).
struct RowsCfg {
    const void* fn;
    int R;
};
RowsCfg rows_cfg(DotKind kind, int mt, int kch) {
    if (kch > 2) {
        if (mt > 2 || kch > 4) return {nullptr, 0};
        if (kind == DotKind::F32) return {reinterpret_cast<const void*>(&gemv_rows_kernel<DotKind::F32, 2, 4, 4>), 4};
        if (kind == DotKind::BF16) return {reinterpret_cast<const void*>(&gemv_rows_kernel<DotKind::BF16, 2, 4, 4>), 4};
        return {nullptr, 0};
    }
    const int R = mt <= 4 ? 8 : 4;
    switch (kind) {
        case DotKind::F32: return {kch == 1 ? rows_select_mt<DotKind::F32, 1>(mt) : rows_select_mt<DotKind::F32, 2>(mt), R};
        case DotKind::BF16: return {kch == 1 ? rows_select_mt<DotKind::BF16, 1>(mt) : rows_select_mt<DotKind::BF16, 2>(mt), R};
        case DotKind::S8S32: return {kch == 1 ? rows_select_mt<DotKind::S8S32, 1>(mt) : rows_select_mt<DotKind::S8S32, 2>(mt), R};
        case DotKind::S8DQ: return {kch == 1 ? rows_select_mt<DotKind::S8DQ, 1>(mt) : rows_select_mt<DotKind::S8DQ, 2>(mt), R};
        default: return {nullptr, 0};
    }
}

template <DotKind KIND, int MT, bool VEC>
const void* nk_fn() {
    return reinterpret_cast<const void*>(&gemv_nk_kernel<KIND, MT, VEC>);
}

template <DotKind KIND>
const void* nk_select_mt(int mt, int vec) {
    switch (mt) {
        case 1: return vec ? nk_fn<KIND, 1, true>() : nk_fn<KIND, 1, false>();
        case 2: return vec ? nk_fn<KIND, 2, true>() : nk_fn<KIND, 2, false>();
        case 4: return vec ? nk_fn<KIND, 4, true>() : nk_fn<KIND, 4, false>();
        case 8: return vec ? nk_fn<KIND, 8, true>() : nk_fn<KIND, 8, false>();
        default: return nullptr;
    }
}

const void* nk_select(DotKind kind, int mt, int vec) {
    switch (kind) {
        case DotKind::F32: return nk_select_mt<DotKind::F32>(mt, vec);
        case DotKind::S8S32: return nk_select_mt<DotKind::S8S32>(mt, vec);
        case DotKind::S8DQ: return nk_select_mt<DotKind::S8DQ>(mt, vec);
        case DotKind::E4M3: return nk_select_mt<DotKind::E4M3>(mt, vec);
        default: break;   // BF16: rows kernel only
    }
    return nullptr;
}

size_t elem_a_bytes(DotKind kind) {
    switch (kind) {
        case DotKind::F32: return 4;
        case DotKind::E4M3:
        case DotKind::BF16: return 2;
        default: return 1;
    }
}

int epc(DotKind kind) { return kind == DotKind::F32 ? 4 : (kind == DotKind::BF16 ? 8 : 16); }

}  // namespace

size_t gemv_nk_smem_bytes(DotKind kind, int mt, int K) {
    int e = epc(kind);
    size_t kpad = (static_cast<size_t>(K) + e - 1) / e * e;
    return static_cast<size_t>(mt) * kpad * elem_a_bytes(kind);
}

// Raises the kernel's dynamic shared-memory limit once per (device, kernel)
// to the library maximum, so later launches (including under stream capture)
// make no attribute calls.
static cudaError_t prepare_nk(const void* fn, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({dev, fn})) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kGemvNkMaxSmem));
    if (e == cudaSuccess) done.insert({dev, fn});
    return e;
}

cudaError_t gemv_nk_occupancy(DotKind kind, int mt, int vec, int K, int* blocks_per_sm) {
    const void* fn = nk_select(kind, mt, vec);
    if (!fn) return cudaErrorInvalidValue;
    size_t smem = gemv_nk_smem_bytes(kind, mt, K);
    cudaError_t e = prepare_nk(fn, smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, kThreads, smem);
}

cudaError_t launch_gemv_nk(DotKind kind, const GemmArgs& g, const GemvNkPlan& p,
                           const float* scales, cudaStream_t s) {
    const void* fn = nk_select(kind, p.mt, p.vec);
    if (!fn || g.M > p.mt || p.grid < 1) return cudaErrorInvalidValue;
    size_t smem = gemv_nk_smem_bytes(kind, p.mt, g.K);
    if (smem > kGemvNkMaxSmem) return cudaErrorInvalidValue;
    cudaError_t e = prepare_nk(fn, smem);
    if (e != cudaSuccess) return e;
    NkParams kp;
    kp.g = g;
    kp.rows_per_cta = (g.N + p.grid - 1) / p.grid;
    kp.scales = scales;
    int grid = (g.N + kp.rows_per_cta - 1) / kp.rows_per_cta;
    void* args[] = {&kp};
    return cudaLaunchKernel(fn, dim3(grid), dim3(kThreads), args, smem, s);
}

bool gemv_rows_supported(DotKind kind, const GemmArgs& g) {
    if (kind == DotKind::E4M3 || g.M < 1 || g.M > 8) return false;
    const int epc_ = epc(kind);
    const size_t eb = kind == DotKind::F32 ? 4 : (kind == DotKind::BF16 ? 2 : 1);
    const bool deep = (kind == DotKind::F32 || kind == DotKind::BF16) && g.M <= 2;
    const int max_chunks = deep ? 4 * kThreads : 2 * kThreads;
    if (g.K % epc_ != 0 || g.K / epc_ > max_chunks) return false;
    return reinterpret_cast<uintptr_t>(g.B) % 16 == 0 && (static_cast<size_t>(g.ldb) * eb) % 16 == 0;
}

cudaError_t gemv_rows_occupancy(DotKind kind, int mt, int K, int* blocks_per_sm) {
    const int kch = (K / epc(kind) + kThreads - 1) / kThreads;
    const void* fn = rows_cfg(kind, mt, kch <= 1 ? 1 : kch).fn;
    if (!fn) return cudaErrorInvalidValue;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, kThreads, 0);
}

cudaError_t launch_gemv_rows(DotKind kind, const GemmArgs& g, int mt, int grid, const float* scales,
                             cudaStream_t s) {
    if (!gemv_rows_supported(kind, g) || g.M > mt) return cudaErrorInvalidValue;
    const int kch = (g.K / epc(kind) + kThreads - 1) / kThreads;
    const RowsCfg rc = rows_cfg(kind, mt, kch <= 1 ? 1 : kch);
    const void* fn = rc.fn;
    if (!fn) return cudaErrorInvalidValue;
    const int R = rc.R;
    const int groups = (g.N + R - 1) / R;
    if (grid < 1) grid = 1;
    if (grid > groups) grid = groups;
    const int per = (groups + grid - 1) / grid;
    RowsParams rp;
    rp.g = g;
    rp.rows_per_cta = per * R;
    rp.scales = scales;
    const int blocks = (g.N + rp.rows_per_cta - 1) / rp.rows_per_cta;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&rp};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// ---- bulk-copy rows kernel -------------------------------------------------
namespace {

struct RowsBulkCfg {
    const void* fn;
    int R;
    int stages;
    uint32_t row_bytes;
    size_t smem;
};

// K of at most 2 x 256 chunks; stage depth for two CTAs per SM (96 KB each)
// when a stage is at most 48 KB, else one CTA per SM (200 KB).  Measured on
// config 3: three stages at two CTAs per SM 10.5 us, two stages at three CTAs
// per SM 11.3 us.
RowsBulkCfg rows_bulk_cfg(DotKind kind, int mt, int K) {
    RowsBulkCfg c{nullptr, 0, 0, 0, 0};
    const int kch = (K / epc(kind) + kThreads - 1) / kThreads;
    if (kch < 1 || kch > 2) return c;
    switch (kind) {
        case DotKind::F32: c.fn = kch == 1 ? rows_bulk_select_mt<DotKind::F32, 1>(mt) : rows_bulk_select_mt<DotKind::F32, 2>(mt); break;
        case DotKind::BF16: c.fn = kch == 1 ? rows_bulk_select_mt<DotKind::BF16, 1>(mt) : rows_bulk_select_mt<DotKind::BF16, 2>(mt); break;
        case DotKind::S8S32: c.fn = kch == 1 ? rows_bulk_select_mt<DotKind::S8S32, 1>(mt) : rows_bulk_select_mt<DotKind::S8S32, 2>(mt); break;
        case DotKind::S8DQ: c.fn = kch == 1 ? rows_bulk_select_mt<DotKind::S8DQ, 1>(mt) : rows_bulk_select_mt<DotKind::S8DQ, 2>(mt); break;
        default: return c;
    }
    if (!c.fn) return c;
    c.R = mt <= 4 ? 8 : 4;
    const size_t eb = kind == DotKind::F32 ? 4 : (kind == DotKind::BF16 ? 2 : 1);
    c.row_bytes = static_cast<uint32_t>(static_cast<size_t>(K) * eb);
    const size_t stage = static_cast<size_t>(c.R) * c.row_bytes;
    const size_t budget = stage <= 48 * 1024 ? 96 * 1024 : 200 * 1024;
    int st = static_cast<int>(budget / stage);
    st = st > kBulkMaxStages ? kBulkMaxStages : st;
    if (st < 2) { c.fn = nullptr; return c; }
    c.stages = st;
    c.smem = static_cast<size_t>(st) * stage;
    return c;
}

cudaError_t prepare_rows_bulk(const void* fn) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({dev, fn})) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess) done.insert({dev, fn});
    return e;
}

}  // namespace

bool gemv_rows_bulk_supported(DotKind kind, const GemmArgs& g) {
    return gemv_rows_supported(kind, g) && rows_bulk_cfg(kind, 8, g.K).fn != nullptr &&
           rows_bulk_cfg(kind, 4, g.K).fn != nullptr;
}

cudaError_t gemv_rows_bulk_occupancy(DotKind kind, int mt, int K, int* blocks_per_sm) {
    const RowsBulkCfg c = rows_bulk_cfg(kind, mt, K);
    if (!c.fn) return cudaErrorInvalidValue;
    cudaError_t e = prepare_rows_bulk(c.fn);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, c.fn, kBulkThreads, c.smem);
}

cudaError_t launch_gemv_rows_bulk(DotKind kind, const GemmArgs& g, int mt, int grid, const float* scales,
                                  uint32_t* err, cudaStream_t s) {
    if (!gemv_rows_bulk_supported(kind, g) || g.M > mt) return cudaErrorInvalidValue;
    const RowsBulkCfg c = rows_bulk_cfg(kind, mt, g.K);
    if (!c.fn) return cudaErrorInvalidValue;
    cudaError_t e = prepare_rows_bulk(c.fn);
    if (e != cudaSuccess) return e;
    const int groups = (g.N + c.R - 1) / c.R;
    if (grid < 1) grid = 1;
    if (grid > groups) grid = groups;
    const int per = (groups + grid - 1) / grid;
    RowsBulkParams rp;
    rp.g = g;
    rp.rows_per_cta = per * c.R;
    rp.stages = c.stages;
    rp.row_bytes = c.row_bytes;
    rp.scales = scales;
    rp.err = err;
    const int blocks = (g.N + rp.rows_per_cta - 1) / rp.rows_per_cta;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks, 1, 1);
    cfg.blockDim = dim3(kBulkThreads, 1, 1);
    cfg.dynamicSmemBytes = c.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&rp};
    return cudaLaunchKernelExC(&cfg, c.fn, args);
}

}  // namespace dnnopt_b200
