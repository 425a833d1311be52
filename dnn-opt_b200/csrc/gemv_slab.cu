// Small-M (M <= 8) GEMV for a K x N row-major B with a few thousand columns:
// the column-slab form.  C[M,N] = alpha * op(A)[M,K] * B[K,N] + beta * C.
//
// Serves the same reference entry points as the split-K kernel (gemm_1xn_fp32,
// src/gemm/gemm_tiny_fp32.cpp:167-218; gemm_smallm_wide_driver_fp32,
// src/gemm/gemm_smallm_wide_fp32.cpp:412-490) on the shapes where a split-K
// reduction through global memory costs more than the B stream itself: N of a
// few thousand columns and K of a few thousand rows, e.g. the irregular-N
// sweep M in {2,3,5,7} x N in {1009, 2039, 4093} x K = 1024, whose B matrices
// (4-17 MB) stream in under 3 us at HBM speed.
//
// B200 design, for latency:
//   * a CTA owns a slab of W = 8 (or 16) consecutive columns and the whole K
//     extent, so each output is finished inside the CTA: no workspace, no
//     atomic ticket, no second pass over memory; the host picks W = 16 when
//     8-column slabs would need more than one wave of resident CTAs, or for
//     M <= 4 from 1536 columns on;
//   * no bias epilogue: it costs the no-bias form registers (63 -> 68 at
//     M <= 2) and sweep time; calls with a bias vector take the split-K
//     kernel instead;
//   * lane l reads column l % W of rows l / W + (32 / W) * warp + 256 / W * i:
//     a warp load covers 32 / W row segments of 4W bytes (rows need no
//     alignment, so prime N works), and every thread issues its first 2 x 16
//     row loads before it stages A, so one DRAM round trip covers most of a
//     1024-row slab;
//   * the A panel is staged in shared memory k-major, MT floats per row
//     (thread t loads column t of A from every row m and writes its MT values
//     as 16-byte stores), so a row's MT coefficients come back with MT/4
//     vector loads;
//   * lanes of a column reduce with two shuffles, warps through shared memory
//     in warp order: the result is deterministic.
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "elem.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kBatch = 16;                    // rows per register batch (2 batches in flight)
constexpr int kPassRows = 1024;               // K rows of A staged per pass

struct SlabParams {
    GemmArgs g;
};

// One slab (columns [slab*W, slab*W + W) of one GEMM) computed by the whole
// CTA.  sA: dynamic shared memory of at least MT * min(K, kPassRows) floats.
template <In IA, In IB, int MT, int W>
__device__ __forceinline__ void slab_body(const GemmArgs& g, int slab, float* sA,
                                          float (&red)[kWarps][MT][W]) {
    using TA = typename Elem<IA>::T;
    using TB = typename Elem<IB>::T;
    constexpr int kSlabW = W;                       // columns per CTA (8 or 16)
    constexpr int kRowsPerLoad = 32 / kSlabW;       // rows one warp load covers
    constexpr int kRowStep = kWarps * kRowsPerLoad; // rows one CTA-wide load covers

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int col = lane % kSlabW, rsub = lane / kSlabW;
    const int n0 = slab * kSlabW;
    const bool col_ok = n0 + col < g.N;
    const TA* A = static_cast<const TA*>(g.A);
    const TB* B = static_cast<const TB*>(g.B) + n0 + col;
    float* C = static_cast<float*>(g.C);

    // The threads that write C (tid < MT * W: m = tid / W, column tid % W)
    // fetch their C element now, in the shadow of the B stream.
    const int wm = tid / kSlabW, wc = tid % kSlabW;
    const bool writer = tid < MT * kSlabW && wm < g.M && n0 + wc < g.N;
    float c_old = 0.0f;
    if (writer && g.beta != 0.0f) c_old = C[(int64_t)wm * g.ldc + n0 + wc];

    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;

    const int r0 = warp * kRowsPerLoad + rsub;   // this thread's first row of a pass
    for (int kp = 0; kp < g.K; kp += kPassRows) {
        const int kn = min(kPassRows, g.K - kp);
        const int nrows = kn > r0 ? (kn - r0 + kRowStep - 1) / kRowStep : 0;   // rows of this thread
        const int nb = (nrows + kBatch - 1) / kBatch;
        const TB* Bp = B + (int64_t)(kp + r0) * g.ldb;
        const int64_t bstep = (int64_t)kRowStep * g.ldb;

        auto load_batch = [&](float (&b)[kBatch], int j) {
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                const int i = j * kBatch + u;
                b[u] = (col_ok && i < nrows) ? dec<IB>(__ldg(Bp + i * bstep)) : 0.0f;
            }
        };
        auto compute_batch = [&](const float (&b)[kBatch], int j) {
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                const int i = j * kBatch + u;
                if (i < nrows) {
                    const int r = r0 + i * kRowStep;
                    float a[MT];
                    if constexpr (MT >= 4) {
#pragma unroll
                        for (int q = 0; q < MT / 4; ++q) {
                            const float4 v = *reinterpret_cast<const float4*>(&sA[r * MT + 4 * q]);
                            a[4 * q] = v.x; a[4 * q + 1] = v.y; a[4 * q + 2] = v.z; a[4 * q + 3] = v.w;
                        }
                    } else if constexpr (MT == 2) {
                        const float2 v = *reinterpret_cast<const float2*>(&sA[r * 2]);
                        a[0] = v.x; a[1] = v.y;
                    } else {
                        a[0] = sA[r];
                    }
#pragma unroll
                    for (int m = 0; m < MT; ++m) acc[m] = fmaf(a[m], b[u], acc[m]);
                }
            }
        };

        float b0[kBatch], b1[kBatch];
        if (nb > 0) load_batch(b0, 0);
        if (nb > 1) load_batch(b1, 1);
        if (kp > 0) __syncthreads();   // the previous pass is done with sA
        // Stage A rows kp .. kp+kn as sA[r][m]; m >= M is zero.  Thread t
        // takes rows t, t+256, ...: all its loads are issued before any store.
        constexpr int kRowsPerThread = kPassRows / kThreads;   // 4
        float v[kRowsPerThread][MT];
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j) {
            const int r = tid + j * kThreads;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                v[j][m] = 0.0f;
                if (r < kn && m < g.M) {
                    const int64_t off = g.a_trans ? (int64_t)(kp + r) * g.lda + m : (int64_t)m * g.lda + (kp + r);
                    v[j][m] = dec<IA>(A[off]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j) {
            const int r = tid + j * kThreads;
            if (r < kn) {
                if constexpr (MT >= 4) {
#pragma unroll
                    for (int q = 0; q < MT / 4; ++q)
                        *reinterpret_cast<float4*>(&sA[r * MT + 4 * q]) =
                            make_float4(v[j][4 * q], v[j][4 * q + 1], v[j][4 * q + 2], v[j][4 * q + 3]);
                } else if constexpr (MT == 2) {
                    *reinterpret_cast<float2*>(&sA[r * 2]) = make_float2(v[j][0], v[j][1]);
                } else {
                    sA[r] = v[j][0];
                }
            }
        }
        __syncthreads();
        for (int j = 0; j < nb; j += 2) {
            compute_batch(b0, j);
            if (j + 2 < nb) load_batch(b0, j + 2);
            if (j + 1 < nb) {
                compute_batch(b1, j + 1);
                if (j + 3 < nb) load_batch(b1, j + 3);
            }
        }
    }

    // Lanes l, l + W, ... hold the same column: fixed shuffle tree.
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int o = kSlabW; o < 32; o <<= 1) acc[m] += __shfl_xor_sync(0xFFFFFFFFu, acc[m], o);
    }
    if (rsub == 0) {
#pragma unroll
        for (int m = 0; m < MT; ++m) red[warp][m][col] = acc[m];
    }
    __syncthreads();
    if (writer) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += red[w][wm][wc];
        C[(int64_t)wm * g.ldc + n0 + wc] = (g.beta == 0.0f) ? g.alpha * sum : fmaf(g.alpha, sum, g.beta * c_old);
    }
}

template <In IA, In IB, int MT, int W>
__global__ void __launch_bounds__(kThreads)
gemv_slab_kernel(const SlabParams p) {
    extern __shared__ __align__(16) float sA[];          // [pass rows][MT]
    __shared__ float red[kWarps][MT][W];
    pdl_wait();
    pdl_launch_dependents();
    slab_body<IA, IB, MT, W>(p.g, blockIdx.x, sA, red);
}

template <In IA, In IB, int MT>
const void* slab_fn(int w) {
    return w == 16 ? reinterpret_cast<const void*>(&gemv_slab_kernel<IA, IB, MT, 16>)
                   : reinterpret_cast<const void*>(&gemv_slab_kernel<IA, IB, MT, 8>);
}

template <In IA, In IB>
const void* slab_select_mt(int mt, int w) {
    switch (mt) {
        case 1: return slab_fn<IA, IB, 1>(w);
        case 2: return slab_fn<IA, IB, 2>(w);
        case 4: return slab_fn<IA, IB, 4>(w);
        case 8: return slab_fn<IA, IB, 8>(w);
        default: return nullptr;
    }
}

const void* slab_select(In ia, In ib, int mt, int w) {
    if (w != 8 && w != 16) return nullptr;
    if (ia == In::F32 && ib == In::F32) return slab_select_mt<In::F32, In::F32>(mt, w);
    if (ia == In::BF16 && ib == In::BF16) return slab_select_mt<In::BF16, In::BF16>(mt, w);
    if (ia == In::F32R && ib == In::F32R) return slab_select_mt<In::F32R, In::F32R>(mt, w);
    if (ia == In::RE4 && ib == In::RE5) return slab_select_mt<In::RE4, In::RE5>(mt, w);
    if (ia == In::RE5 && ib == In::RE5) return slab_select_mt<In::RE5, In::RE5>(mt, w);
    return nullptr;
}

size_t slab_smem_bytes(int mt, int K) {
    const int rows = K < kPassRows ? K : kPassRows;
    return static_cast<size_t>(mt) * rows * sizeof(float);
}

}  // namespace

int gemv_slab_ctas(int N, int w) { return (N + w - 1) / w; }

cudaError_t gemv_slab_occupancy(In ia, In ib, int mt, int w, int K, int* blocks_per_sm) {
    const void* fn = slab_select(ia, ib, mt, w);
    if (!fn) return cudaErrorInvalidValue;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, kThreads,
                                                         slab_smem_bytes(mt, K));
}

// Shared-memory carveout: just enough for the register-limited number of
// CTAs per SM at the kernel's largest footprint (K >= kPassRows), the rest
// stays L1.  Measured on B200: the default split can hold fewer CTAs than the
// registers allow (start times spread over a second wave), while the largest
// split leaves so little L1 that far fewer loads stay in flight (2-3x
// slower).  Set once per device and kernel.
cudaError_t set_carveout(const void* fn, int mt) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({dev, fn})) return cudaSuccess;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, fn);
    if (e != cudaSuccess) return e;
    int occ = 0;
    const size_t dyn = slab_smem_bytes(mt, kPassRows);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kThreads, dyn);
    if (e != cudaSuccess) return e;
    int smem_per_sm = 0;
    e = cudaDeviceGetAttribute(&smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (e != cudaSuccess) return e;
    const size_t need = static_cast<size_t>(occ > 0 ? occ : 1) * (dyn + fa.sharedSizeBytes + 1024);
    int pct = static_cast<int>((need * 100 + smem_per_sm - 1) / static_cast<size_t>(smem_per_sm)) + 2;
    if (pct > 100) pct = 100;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, pct);
    if (e == cudaSuccess) done.insert({dev, fn});
    return e;
}

cudaError_t launch_gemv_slab(In ia, In ib, const GemmArgs& g, int mt, int w, cudaStream_t s) {
    const void* fn = slab_select(ia, ib, mt, w);
    if (!fn || g.M > mt || g.M < 1 || g.N < 1 || g.K < 1) return cudaErrorInvalidValue;
    cudaError_t pe = set_carveout(fn, mt);
    if (pe != cudaSuccess) return pe;
    SlabParams sp;
    sp.g = g;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(gemv_slab_ctas(g.N, w)), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = slab_smem_bytes(mt, g.K);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&sp};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace dnnopt_b200
