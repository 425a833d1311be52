// Small-M (M <= 8) GEMV-class kernel for a K x N row-major B (N contiguous):
//   C[M,N] = alpha * op(A)[M,K] * B[K,N] + beta * C
//
// Replaces the reference's small-M FP32 drivers (gemm_1xn_fp32,
// src/gemm/gemm_tiny_fp32.cpp:167-218; gemm_smallm_wide_driver_fp32,
// src/gemm/gemm_smallm_wide_fp32.cpp:412-490) and serves the same shapes for
// the bf16 / FP32-API bf16 / reference-fp8 entry points.
//
// B200 design: the op is HBM-bound (about 0.5*M flop per byte of B), so the
// kernel is shaped for bytes in flight, not arithmetic.
//   * A CTA owns a 128-column strip of B and one K-split; each warp streams
//     rows of the strip with coalesced 16-byte loads (4-byte loads when the
//     rows are not 16-byte aligned, e.g. prime N), U rows unrolled so every
//     thread keeps U independent loads in flight.
//   * The A panel for the split is staged transposed in shared memory so a
//     row's M coefficients arrive with one broadcast vector load.
//   * Warps reduce through shared memory in a fixed order; K-splits reduce
//     through a global workspace by the last CTA of each strip (atomic
//     ticket), again in split order, so results are deterministic.
//   * The grid is sized by the host to one wave of resident CTAs over the
//     148 SMs (splits = resident CTAs / strips).
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "dnnopt_b200.h"
#include "elem.cuh"
#include "kernels.h"
#include "plan.h"

namespace dnnopt_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTileN = 128;

struct KnParams {
    GemmArgs g;
    int splits, kchunk, n_pad;
    float* ws;
    uint32_t* counters;
};

// Four B elements of one row as loaded: a 16-, 8- or 4-byte word for 4-, 2-
// and 1-byte encodings (kept packed until the FMAs so that narrow types keep
// as many rows in flight per register as FP32).
template <size_t EB> struct RawWord;
template <> struct RawWord<4> { using T = uint4; };
template <> struct RawWord<2> { using T = uint2; };
template <> struct RawWord<1> { using T = uint32_t; };

template <In I>
__device__ __forceinline__ void unpack4(const typename RawWord<sizeof(typename Elem<I>::T)>::T& w,
                                        float (&o)[4]) {
    using T = typename Elem<I>::T;
    if constexpr (sizeof(T) == 4) {
        o[0] = dec<I>(__uint_as_float(w.x)); o[1] = dec<I>(__uint_as_float(w.y));
        o[2] = dec<I>(__uint_as_float(w.z)); o[3] = dec<I>(__uint_as_float(w.w));
    } else if constexpr (sizeof(T) == 2) {
        o[0] = dec<I>(static_cast<uint16_t>(w.x & 0xFFFFu)); o[1] = dec<I>(static_cast<uint16_t>(w.x >> 16));
        o[2] = dec<I>(static_cast<uint16_t>(w.y & 0xFFFFu)); o[3] = dec<I>(static_cast<uint16_t>(w.y >> 16));
    } else {
        o[0] = dec<I>(static_cast<uint8_t>(w & 0xFFu)); o[1] = dec<I>(static_cast<uint8_t>((w >> 8) & 0xFFu));
        o[2] = dec<I>(static_cast<uint8_t>((w >> 16) & 0xFFu)); o[3] = dec<I>(static_cast<uint8_t>(w >> 24));
    }
}

// Element c of a packed word (scalar-load path).
template <typename T, typename W>
__device__ __forceinline__ void set_elem(W& w, int c, T v) {
    if constexpr (sizeof(T) == 4) {
        const uint32_t u = __float_as_uint(v);
        if (c == 0) w.x = u; else if (c == 1) w.y = u; else if (c == 2) w.z = u; else w.w = u;
    } else if constexpr (sizeof(T) == 2) {
        const uint32_t u = static_cast<uint32_t>(v);
        if (c == 0) w.x = (w.x & 0xFFFF0000u) | u;
        else if (c == 1) w.x = (w.x & 0xFFFFu) | (u << 16);
        else if (c == 2) w.y = (w.y & 0xFFFF0000u) | u;
        else w.y = (w.y & 0xFFFFu) | (u << 16);
    } else {
        const uint32_t u = static_cast<uint32_t>(v);
        w = (w & ~(0xFFu << (8 * c))) | (u << (8 * c));
    }
}

// Column (within the 128-wide strip) held in accumulator slot c of `lane`.
template <bool VEC4>
__device__ __forceinline__ int slot_col(int lane, int c) {
    return VEC4 ? 4 * lane + c : lane + 32 * c;
}

// One kernel, two ways to reduce the K-splits of a strip:
//   CLUSTER == false: partial strips go to the workspace; the last CTA of the
//     strip (atomic ticket) sums them in split order;
//   CLUSTER == true: the splits form one thread-block cluster and sum the
//     partial strips through distributed shared memory.
// Per CTA the critical path is kept to as few memory round trips as possible:
//   1. the first batch of B rows is requested before anything else; A for the
//      pass is staged in shared memory while those loads are in flight;
//   2. the remaining rows stream with register double-buffering (two batches
//      of U rows in flight per thread);
//   3. the 8 warps reduce in shared memory in warp order, then the splits:
//      the last CTA of a strip loads every split's partial (8-16 splits
//      per round of independent loads, vector width matched to MT so that all
//      256 threads take part) and the C values it needs, and sums the splits
//      in order.
constexpr int kPassRows = 1024;   // K rows of A staged per pass

// Register caps (measured on B200): MT = 1 at four CTAs per SM, MT = 2 at
// three (2 x 4096 x 4096: 19.9 -> 17.6 us); MT = 4, 8 uncapped (three CTAs
// per SM made 8 x 4096 x 4096 slower: more splits to reduce).
template <In IA, In IB, int MT, bool VEC4, bool CLUSTER>
__global__ void __launch_bounds__(kThreads, MT == 1 ? 4 : (MT == 2 ? 3 : 1))
gemv_kn_kernel(const KnParams p) {
    using TA = typename Elem<IA>::T;
    using TB = typename Elem<IB>::T;
    using Raw = typename RawWord<sizeof(TB)>::T;
    // Rows per warp per batch (x2 in flight): 4 for FP32, 8 for 2-byte and 16
    // for 1-byte encodings, i.e. the same 16 bytes per lane and row group.
    constexpr int U = 16 / static_cast<int>(sizeof(TB));
    constexpr int kRowsPerBatch = kWarps * U;

    extern __shared__ __align__(16) float dsm[];
    const int pass_rows = p.kchunk < kPassRows ? p.kchunk : kPassRows;
    const int stage_floats = pass_rows * MT;
    const int red_floats = stage_floats > kWarps * MT * kTileN ? stage_floats : kWarps * MT * kTileN;
    float* sA = dsm;
    float* red = dsm;
    float* part = dsm + red_floats;            // [MT][128] this CTA's partial strip
    __shared__ int s_last;

    pdl_wait();
    pdl_launch_dependents();

    const GemmArgs& g = p.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kTileN;
    const int split = blockIdx.y;
    const int k_begin = split * p.kchunk;
    const int k_end = min(g.K, k_begin + p.kchunk);
    const bool full_tile = (n0 + kTileN) <= g.N;
    const TA* A = static_cast<const TA*>(g.A);
    const TB* B = static_cast<const TB*>(g.B);
    float* C = static_cast<float*>(g.C);

    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0.0f;

    for (int kp = k_begin; kp < k_end; kp += kPassRows) {
        const int kn = min(kPassRows, k_end - kp);
        const int nb = (kn + kRowsPerBatch - 1) / kRowsPerBatch;

        auto load_batch = [&](Raw (&b)[U], int it) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int r = it * kRowsPerBatch + u * kWarps + warp;
                b[u] = Raw{};
                if (r < kn) {
                    const TB* row = B + (int64_t)(kp + r) * g.ldb + n0;
                    if (VEC4 && full_tile) {
                        b[u] = __ldg(reinterpret_cast<const Raw*>(row + 4 * lane));
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            int col = slot_col<VEC4>(lane, c);
                            if (n0 + col < g.N) set_elem<TB>(b[u], c, row[col]);
                        }
                    }
                }
            }
        };
        auto compute_batch = [&](const Raw (&braw)[U], int it) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int r = it * kRowsPerBatch + u * kWarps + warp;
                if (r < kn) {
                    float bu[4];
                    unpack4<IB>(braw[u], bu);
                    float a[MT];
                    if constexpr (MT % 4 == 0) {
#pragma unroll
                        for (int q = 0; q < MT / 4; ++q) {
                            float4 v = *reinterpret_cast<const float4*>(&sA[r * MT + 4 * q]);
                            a[4 * q] = v.x; a[4 * q + 1] = v.y; a[4 * q + 2] = v.z; a[4 * q + 3] = v.w;
                        }
                    } else {
#pragma unroll
                        for (int m = 0; m < MT; ++m) a[m] = sA[r * MT + m];
                    }
#pragma unroll
                    for (int m = 0; m < MT; ++m)
#pragma unroll
                        for (int c = 0; c < 4; ++c) acc[m][c] = fmaf(a[m], bu[c], acc[m][c]);
                }
            }
        };

        Raw b0[U], b1[U];
        if (nb > 0) load_batch(b0, 0);
        if (kp > k_begin) __syncthreads();   // the previous pass is done with sA
        for (int idx = tid; idx < kn * MT; idx += kThreads) {
            const int r = idx / MT, m = idx - r * MT;
            float v = 0.0f;
            if (m < g.M) {
                const int64_t off = g.a_trans ? (int64_t)(kp + r) * g.lda + m : (int64_t)m * g.lda + (kp + r);
                v = dec<IA>(A[off]);
            }
            sA[idx] = v;
        }
        __syncthreads();
        for (int it = 0; it < nb; it += 2) {
            if (it + 1 < nb) load_batch(b1, it + 1);
            compute_batch(b0, it);
            if (it + 1 < nb) {
                if (it + 2 < nb) load_batch(b0, it + 2);
                compute_batch(b1, it + 1);
            }
        }
    }
    __syncthreads();   // sA is reused for the warp partials below

#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[(warp * MT + m) * kTileN + slot_col<VEC4>(lane, c)] = acc[m][c];
    __syncthreads();
    for (int idx = tid; idx < MT * kTileN; idx += kThreads) {
        int m = idx / kTileN, j = idx - m * kTileN;
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += red[(w * MT + m) * kTileN + j];
        part[idx] = sum;
    }

    // C = beta == 0 ? alpha*sum : fma(alpha, sum, beta*C), the reference's
    // epilogue; C is read only where it is written.
    auto store = [&](int m, int j, float sum) {
        if (m < g.M && n0 + j < g.N) {
            float* cp = C + (int64_t)m * g.ldc + n0 + j;
            *cp = add_bias((g.beta == 0.0f) ? g.alpha * sum : fmaf(g.alpha, sum, g.beta * *cp), g.bias, n0 + j);
        }
    };

    if (p.splits == 1) {
        // Each thread stores what it reduced itself: no barrier needed.
        for (int idx = tid; idx < MT * kTileN; idx += kThreads) store(idx / kTileN, idx % kTileN, part[idx]);
        return;
    }
    if constexpr (CLUSTER) {
        cluster_sync_all();
        const uint32_t rank = cluster_ctarank();
        const uint32_t part_addr = smem_u32(part);
        const int S = p.splits;
        const int ncol = (kTileN - static_cast<int>(rank) + S - 1) / S;
        for (int idx = tid; idx < MT * ncol; idx += kThreads) {
            int m = idx / ncol, jj = idx - m * ncol;
            int j = static_cast<int>(rank) + jj * S;
            float sum = 0.0f;
            for (int q = 0; q < S; ++q)
                sum += ld_dsmem_f32(map_to_cta(part_addr + static_cast<uint32_t>((m * kTileN + j) * 4),
                                               static_cast<uint32_t>(q)));
            store(m, j, sum);
        }
        cluster_sync_all();
    } else {
        // Publish this split's strip (16-byte stores; the workspace rows are
        // n_pad floats, a multiple of 128); the last CTA of the strip (ticket
        // splits-1) sums the splits in order and writes C.
        float4* ws4 = reinterpret_cast<float4*>(p.ws);
        const int q_per_split = MT * kTileN / 4;           // float4 groups of one strip
        const int row4 = p.n_pad / 4;
        __syncthreads();   // part[] was written by other threads
        for (int q = tid; q < q_per_split; q += kThreads) {
            const int m = q / (kTileN / 4), j4 = q - m * (kTileN / 4);
            __stcg(&ws4[((int64_t)split * MT + m) * row4 + n0 / 4 + j4],
                   *reinterpret_cast<const float4*>(&part[m * kTileN + 4 * j4]));
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            uint32_t ticket = atomicAdd(&p.counters[blockIdx.x], 1u);
            s_last = (ticket == static_cast<uint32_t>(p.splits - 1));
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        // Each thread owns VW consecutive columns of one row m (every thread
        // of the CTA when MT >= 2) and issues all its split loads in rounds of
        // kSumRound before adding them in split order.
        constexpr int VW = MT >= 8 ? 4 : (MT >= 4 ? 2 : 1);
        constexpr int kGroupsPerRow = kTileN / VW;
        constexpr int kSumRound = VW == 4 ? 8 : 16;
        const float* wsf = p.ws;
        for (int q = tid; q < MT * kGroupsPerRow; q += kThreads) {
            const int m = q / kGroupsPerRow, j0 = (q - m * kGroupsPerRow) * VW;
            if (m >= g.M || n0 + j0 >= g.N) continue;
            float* crow = C + (int64_t)m * g.ldc + n0 + j0;
            float cv[VW];
#pragma unroll
            for (int u = 0; u < VW; ++u)
                cv[u] = (g.beta != 0.0f && n0 + j0 + u < g.N) ? crow[u] : 0.0f;
            float sum[VW];
#pragma unroll
            for (int u = 0; u < VW; ++u) sum[u] = 0.0f;
            const float* src = wsf + (int64_t)m * p.n_pad + n0 + j0;
            const int64_t sstride = (int64_t)MT * p.n_pad;
            for (int sp0 = 0; sp0 < p.splits; sp0 += kSumRound) {
                float v[kSumRound][VW];
#pragma unroll
                for (int r = 0; r < kSumRound; ++r) {
                    if (sp0 + r < p.splits) {
                        const float* ps = src + (sp0 + r) * sstride;
                        if constexpr (VW == 4) {
                            const float4 t = __ldcg(reinterpret_cast<const float4*>(ps));
                            v[r][0] = t.x; v[r][1] = t.y; v[r][2] = t.z; v[r][3] = t.w;
                        } else if constexpr (VW == 2) {
                            const float2 t = __ldcg(reinterpret_cast<const float2*>(ps));
                            v[r][0] = t.x; v[r][1] = t.y;
                        } else {
                            v[r][0] = __ldcg(ps);
                        }
                    }
                }
#pragma unroll
                for (int r = 0; r < kSumRound; ++r)
                    if (sp0 + r < p.splits) {
#pragma unroll
                        for (int u = 0; u < VW; ++u) sum[u] += v[r][u];
                    }
            }
#pragma unroll
            for (int u = 0; u < VW; ++u)
                if (n0 + j0 + u < g.N)
                    crow[u] = add_bias((g.beta == 0.0f) ? g.alpha * sum[u] : fmaf(g.alpha, sum[u], g.beta * cv[u]),
                                       g.bias, n0 + j0 + u);
        }
        if (tid == 0) p.counters[blockIdx.x] = 0u;   // ready for the next launch on this stream
    }
}

size_t kn_smem_bytes(int mt, int kchunk) {
    size_t rows = kchunk < kPassRows ? kchunk : kPassRows;
    size_t stage = rows * mt;
    size_t red = static_cast<size_t>(kWarps) * mt * kTileN;
    return ((stage > red ? stage : red) + static_cast<size_t>(mt) * kTileN) * sizeof(float);
}

template <In IA, In IB, int MT, bool VEC4, bool CL>
const void* kn_fn() {
    return reinterpret_cast<const void*>(&gemv_kn_kernel<IA, IB, MT, VEC4, CL>);
}

template <In IA, In IB, bool CL>
const void* kn_select_mt(int mt, int vec4) {
    switch (mt) {
        case 1: return vec4 ? kn_fn<IA, IB, 1, true, CL>() : kn_fn<IA, IB, 1, false, CL>();
        case 2: return vec4 ? kn_fn<IA, IB, 2, true, CL>() : kn_fn<IA, IB, 2, false, CL>();
        case 4: return vec4 ? kn_fn<IA, IB, 4, true, CL>() : kn_fn<IA, IB, 4, false, CL>();
        case 8: return vec4 ? kn_fn<IA, IB, 8, true, CL>() : kn_fn<IA, IB, 8, false, CL>();
        default: return nullptr;
    }
}

template <bool CL>
const void* kn_select_t(In ia, In ib, int mt, int vec4) {
    if (ia == In::F32 && ib == In::F32) return kn_select_mt<In::F32, In::F32, CL>(mt, vec4);
    if (ia == In::BF16 && ib == In::BF16) return kn_select_mt<In::BF16, In::BF16, CL>(mt, vec4);
    if (ia == In::F32R && ib == In::F32R) return kn_select_mt<In::F32R, In::F32R, CL>(mt, vec4);
    if (ia == In::RE4 && ib == In::RE5) return kn_select_mt<In::RE4, In::RE5, CL>(mt, vec4);
    if (ia == In::RE5 && ib == In::RE5) return kn_select_mt<In::RE5, In::RE5, CL>(mt, vec4);
    return nullptr;
}

const void* kn_select(In ia, In ib, int mt, int vec4) { return kn_select_t<false>(ia, ib, mt, vec4); }
const void* kn_cluster_select(In ia, In ib, int mt, int vec4) {
    return kn_select_t<true>(ia, ib, mt, vec4);
}

}  // namespace

int gemv_kn_tiles(int N) { return (N + kTileN - 1) / kTileN; }

size_t gemv_kn_ws_floats(const GemvKnPlan& p, int N) {
    if (p.splits <= 1) return 0;
    return static_cast<size_t>(p.splits) * p.mt * gemv_kn_tiles(N) * kTileN;
}

cudaError_t gemv_kn_occupancy(In ia, In ib, int mt, int vec4, int* blocks_per_sm) {
    const void* fn = kn_select(ia, ib, mt, vec4);
    if (!fn) return cudaErrorInvalidValue;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, kThreads,
                                                         kn_smem_bytes(mt, 256));
}

int gemv_kn_cluster_max_chunk() { return kPassRows; }

cudaError_t gemv_kn_cluster_occupancy(In ia, In ib, int mt, int vec4, int kchunk, int* blocks_per_sm) {
    const void* fn = kn_cluster_select(ia, ib, mt, vec4);
    if (!fn) return cudaErrorInvalidValue;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, kThreads,
                                                         kn_smem_bytes(mt, kchunk));
}

cudaError_t launch_gemv_kn_cluster(In ia, In ib, const GemmArgs& g, const GemvKnPlan& p,
                                   cudaStream_t s) {
    const void* fn = kn_cluster_select(ia, ib, p.mt, p.vec4);
    if (!fn || g.M > p.mt || p.splits < 1 || p.splits > 16 || p.kchunk < 1 ||
        p.kchunk > kPassRows)
        return cudaErrorInvalidValue;
    if (p.splits > 8) {
        static std::mutex mu;
        static std::set<std::pair<int, const void*>> done;
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        std::lock_guard<std::mutex> lk(mu);
        if (!done.count({dev, fn})) {
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return e;
            done.insert({dev, fn});
        }
    }
    KnParams kp;
    kp.g = g;
    kp.splits = p.splits;
    kp.kchunk = p.kchunk;
    kp.n_pad = gemv_kn_tiles(g.N) * kTileN;
    kp.ws = nullptr;
    kp.counters = nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(gemv_kn_tiles(g.N), p.splits, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kn_smem_bytes(p.mt, p.kchunk);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(p.splits);
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    void* args[] = {&kp};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_gemv_kn(In ia, In ib, const GemmArgs& g, const GemvKnPlan& p, float* ws,
                           uint32_t* counters, cudaStream_t s) {
    const void* fn = kn_select(ia, ib, p.mt, p.vec4);
    if (!fn || g.M > p.mt || p.splits < 1 || p.kchunk < 1) return cudaErrorInvalidValue;
    if (p.splits > 1 && (!ws || !counters)) return cudaErrorInvalidValue;
    KnParams kp;
    kp.g = g;
    kp.splits = p.splits;
    kp.kchunk = p.kchunk;
    kp.n_pad = gemv_kn_tiles(g.N) * kTileN;
    kp.ws = ws;
    kp.counters = counters;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(gemv_kn_tiles(g.N), p.splits, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kn_smem_bytes(p.mt, p.kchunk);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&kp};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace dnnopt_b200

// ---------------------------------------------------------------------------
// Allocation-free entry point: dnnopt_cuda_gemm_f32_noalloc.
//
// Some callers cannot call cudaMalloc: code whose device memory is owned by a
// framework's caching allocator (allocating behind its back breaks the pool's
// accounting and out-of-memory handling), serving loops that forbid any
// allocation after warm-up because cudaMalloc can synchronise the device, and
// runtimes that fix their memory budget at start-up.  For them this entry
// point runs the small-M split-K GEMV kernel with the planner's split rule
// (dnnopt_cuda_gemm_f32 may pick the slab or cluster kernel for the same
// shape; results then agree within FP32 rounding, not bitwise) and takes its
// scratch (split-K partial strips and the per-strip tickets) from the
// file-scope device array below instead of the per-stream workspace.
//
// * Capacity: kNoAllocTicketWords strips of 128 columns (N <= 131072) and
//   kNoAllocPartialFloats partial floats (4 MiB); larger requests are
//   rejected with DNNOPT_STATUS_EXCEEDS_SCRATCH.  The array (4 MiB + 4 KiB)
//   is held by every GPU that loads the library until the process exits.
// * The first call on a device looks up the array's device address with
//   cudaGetSymbolAddress (host code cannot use the symbol itself: on the host
//   it names a stand-in, not device memory) and loads the eight FP32 kernel
//   instantiations; make that first call before any stream capture.  The
//   address is cached for the life of the process: after cudaDeviceReset the
//   entry point must not be called again.
// * Every call shares the array and it keeps the last call's contents: the
//   tickets are cleared on the call's stream before each launch, the partials
//   are fully rewritten before they are read.  Calls that overlap on the GPU
//   (different streams, or several host threads) race on the array and must
//   be serialised by the caller.
// * No cudaMalloc, cudaFree or allocating library routine is called.
// ---------------------------------------------------------------------------
namespace dnnopt_b200 {
namespace {

constexpr size_t kNoAllocTicketWords = 1024;
constexpr size_t kNoAllocPartialFloats = static_cast<size_t>(1) << 20;
constexpr size_t kNoAllocScratchBytes = kNoAllocTicketWords * 4 + kNoAllocPartialFloats * 4;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
// Per-device set-up, done once under g_noalloc_mu by the first call on that
// device: the scratch array's device address, the SM count and the resident
// CTAs per SM of each of the eight FP32 instantiations (M class 1/2/4/8 x
// vector width), which also loads every one of them, so that later calls make
// no driver query and load no code.
struct NoAllocDevice {
    void* scratch = nullptr;
    int sms = 0;
    int occ[4][2] = {};
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];

int noalloc_mt(int M) { return M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8)); }
int noalloc_mt_index(int mt) { return mt == 1 ? 0 : (mt == 2 ? 1 : (mt == 4 ? 2 : 3)); }

int noalloc_setup(int dev, NoAllocDevice* out) {
    NoAllocDevice d;
    if (cudaGetSymbolAddress(&d.scratch, g_noalloc_scratch) != cudaSuccess || !d.scratch) {
        cudaGetLastError();
        return DNNOPT_STATUS_CUDA_ERROR;
    }
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return DNNOPT_STATUS_CUDA_ERROR;
    }
    const int mts[4] = {1, 2, 4, 8};
    for (int i = 0; i < 4; ++i) {
        for (int v = 0; v < 2; ++v) {
            const void* fn = kn_select(In::F32, In::F32, mts[i], v);
            cudaFuncAttributes fa;
            int occ = 0;
            if (!fn || cudaFuncGetAttributes(&fa, fn) != cudaSuccess ||
                gemv_kn_occupancy(In::F32, In::F32, mts[i], v, &occ) != cudaSuccess) {
                cudaGetLastError();
                return DNNOPT_STATUS_CUDA_ERROR;
            }
            d.occ[i][v] = occ < 1 ? 1 : occ;
        }
    }
    *out = d;
    return DNNOPT_STATUS_SUCCESS;
}

}  // namespace
}  // namespace dnnopt_b200

extern "C" __attribute__((visibility("default"))) int dnnopt_cuda_gemm_f32_noalloc(
    const dnnopt_gemm_desc* d, const float* A, const float* B, float* C, void* stream) {
    using namespace dnnopt_b200;
    if (!d || d->M < 0 || d->N < 0 || d->K < 0) return DNNOPT_STATUS_INVALID_VALUE;
    if (d->M == 0 || d->N == 0 || d->K == 0) return DNNOPT_STATUS_SUCCESS;
    if (!A || !B || !C) return DNNOPT_STATUS_INVALID_VALUE;
    if (d->lda < (d->trans_a ? d->M : d->K) || d->ldc < d->N) return DNNOPT_STATUS_INVALID_VALUE;
    if (d->trans_b || d->M > 8) return DNNOPT_STATUS_NOT_SUPPORTED;   // small-M, B K x N only
    if (d->ldb < d->N) return DNNOPT_STATUS_INVALID_VALUE;
    const int tiles = gemv_kn_tiles(d->N);
    if (static_cast<size_t>(tiles) > kNoAllocTicketWords) return DNNOPT_STATUS_EXCEEDS_SCRATCH;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return DNNOPT_STATUS_NO_DEVICE;
    }
    if (dev < 0 || dev >= kNoAllocMaxDevices) return DNNOPT_STATUS_NOT_SUPPORTED;
    NoAllocDevice nd;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_dev[dev].scratch) {
            const int st = noalloc_setup(dev, &g_noalloc_dev[dev]);
            if (st != DNNOPT_STATUS_SUCCESS) return st;
        }
        nd = g_noalloc_dev[dev];
    }
    void* scratch = nd.scratch;

    GemmArgs g;
    g.M = d->M; g.N = d->N; g.K = d->K;
    g.alpha = d->alpha; g.beta = d->beta;
    g.A = A; g.lda = d->lda; g.a_trans = d->trans_a ? 1 : 0;
    g.B = B; g.ldb = d->ldb; g.b_trans = 0;
    g.C = C; g.ldc = d->ldc;

    // The planner's split-K rule for this kernel (kn_plan_rule, the one
    // dnnopt_cuda_gemm_f32 uses when it picks the split-K kernel), then fewer
    // splits if the partial strips would not fit the fixed array.  The rule
    // keeps splits x strips within one wave of resident CTAs, at most 8 x 128
    // x 3 x 148 floats, so the clamp is a guard that B200 shapes do not reach.
    const int mt = noalloc_mt(g.M);
    const int vec4 = (reinterpret_cast<uintptr_t>(B) % 16 == 0 && g.ldb % 4 == 0) ? 1 : 0;
    GemvKnPlan p = kn_plan_rule(g, mt, vec4, nd.occ[noalloc_mt_index(mt)][vec4], nd.sms, 0, false);
    const size_t per_split = static_cast<size_t>(p.mt) * tiles * 128;
    if (p.splits > 1 && static_cast<size_t>(p.splits) * per_split > kNoAllocPartialFloats) {
        int splits = p.splits;
        while (splits > 1 && static_cast<size_t>(splits) * per_split > kNoAllocPartialFloats) --splits;
        p = kn_plan_rule(g, mt, vec4, 1, nd.sms, splits, false);
    }
    if (p.splits > 1 && static_cast<size_t>(p.splits) * per_split > kNoAllocPartialFloats)
        return DNNOPT_STATUS_EXCEEDS_SCRATCH;

    uint32_t* tickets = static_cast<uint32_t*>(scratch);
    float* partials = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) +
                                               kNoAllocTicketWords * 4);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (p.splits > 1 &&
        cudaMemsetAsync(tickets, 0, static_cast<size_t>(tiles) * sizeof(uint32_t), s) != cudaSuccess) {
        cudaGetLastError();
        return DNNOPT_STATUS_CUDA_ERROR;
    }
    if (launch_gemv_kn(In::F32, In::F32, g, p, partials, tickets, s) != cudaSuccess) {
        cudaGetLastError();
        return DNNOPT_STATUS_CUDA_ERROR;
    }
    return DNNOPT_STATUS_SUCCESS;
}
