// Small-M (M <= 8) FP32 GEMV for a K x N row-major B: the row-panel form.
// C[M,N] = alpha * op(A)[M,K] * B[K,N] + beta * C.
//
// Serves the reference's small-M FP32 entry points (gemm_1xn_fp32,
// src/gemm/gemm_tiny_fp32.cpp:167-218; gemm_smallm_wide_driver_fp32,
// src/gemm/gemm_smallm_wide_fp32.cpp:412-490, whose 48-column panels with a
// 256-row K block are the CPU analogue) on shapes such as the irregular-N
// sweep M in {2,3,5,7} x N in {1009, 2039, 4093} x K = 1024, where B (4-17 MB)
// is the whole HBM stream and N is prime, so B's rows have no alignment.
//
// B200 design, for aggregate HBM throughput when several such GEMMs overlap:
//   * a CTA owns a panel of 128 consecutive columns and one of S K-ranges;
//     warp w reads rows w, w + 8, ... of the range, lane l columns l + 32 q
//     (q < 4), so every warp load is one 128-byte piece of a 512-byte row
//     segment and a warp covers the whole segment (coalesced 4-byte loads:
//     prime N rules out wider ones).  Measured on B200 with the sweep's twelve
//     B reads in one graph on six streams: 512-byte row segments by 8 CTAs
//     per panel stream at 4.9 TB/s, the column-slab pattern (32-64-byte
//     strips, whole K per CTA) at 1.8-2.5 TB/s, one bulk copy per row segment
//     (cp.async.bulk) is issue-bound at about one 0.5 KB copy per 20-40 ns
//     per SM, 16-byte cp.async stages at a few GB/s per CTA;
//   * U rows per warp are loaded one batch ahead into registers (two
//     batches in flight), the A panel sits in shared memory k-major (MT floats
//     per row, broadcast reads), each lane accumulates MT x 4 outputs;
//   * the eight warps' partial panels are summed through shared memory in
//     warp order; with S > 1 each CTA publishes its partial panel to an
//     L2-resident workspace and the last CTA of the panel (atomic ticket)
//     sums the S partials in split order and applies alpha / beta (and the
//     oneDNN entry's bias), so results are bit-deterministic.  Measured on
//     B200 against reducing the K-ranges of a panel inside a thread-block
//     cluster through distributed shared memory: the cluster form costs
//     17 us more per sweep (50 against 33 us without any cross-CTA step), as
//     every CTA of a cluster waits for the slowest and holds its slot until
//     the peers have read its partial; the ticket form lets CTAs retire
//     independently.
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxRows = 512;        // K rows per CTA (bounds the staged A panel)

struct PanelParams {
    GemmArgs g;
    int rows;          // K rows per CTA (multiple of 8); the last CTA may get fewer
    int n_pad;         // workspace row length (panels * 128)
    float* ws;         // [S][MT][n_pad] partial panels (S > 1)
    uint32_t* counters;  // one ticket per panel, zero on entry, left zero
};

template <int MT, int U, int kPanel>
__global__ void __launch_bounds__(kThreads, (kPanel == 64 && U <= 8) ? 3 : 2)
gemv_panel_kernel(const PanelParams p) {
    constexpr int kQ = kPanel / 32;                        // columns per lane
    constexpr int kMaxOut = (MT * kPanel + kThreads - 1) / kThreads;
    constexpr int VW = (MT * kPanel) / kThreads >= 4 ? 4 : ((MT * kPanel) / kThreads >= 2 ? 2 : 1);
    constexpr int kGroups = MT * kPanel / VW;             // <= kThreads
    static_assert(kGroups <= kThreads, "one column group per thread");
    extern __shared__ __align__(16) float smem[];
    __shared__ int s_last;

    const GemmArgs& g = p.g;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kPanel;
    const int split = blockIdx.y;
    const int S = gridDim.y;
    const int k0 = split * p.rows;
    const int R = max(0, min(p.rows, g.K - k0));
    const int vc = min(kPanel, g.N - n0);         // valid columns of this panel

    float* sA = smem;                             // [p.rows][MT]
    float* red = smem + p.rows * MT;              // [kWarps][MT][kPanel]; [0] ends as the CTA's partial

    pdl_wait();

    // Rows of this warp: warp + 8 * i, i < nrows; batch j holds i in [j*U, j*U + U).
    const int nrows = R > warp ? (R - warp + kWarps - 1) / kWarps : 0;
    const int nb = (nrows + U - 1) / U;
    const float* Bp = static_cast<const float*>(g.B) + (static_cast<int64_t>(k0) + warp) * g.ldb + n0 + lane;
    const int64_t rstep = static_cast<int64_t>(kWarps) * g.ldb;
    bool colok[kQ];
#pragma unroll
    for (int q = 0; q < kQ; ++q) colok[q] = lane + 32 * q < vc;

    auto load_batch = [&](float (&b)[U][kQ], int j) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = j * U + u;
#pragma unroll
            for (int q = 0; q < kQ; ++q)
                b[u][q] = (i < nrows && colok[q]) ? __ldg(Bp + i * rstep + 32 * q) : 0.0f;
        }
    };
    float b0[U][kQ], b1[U][kQ];
    if (nb > 0) load_batch(b0, 0);
    if (nb > 1) load_batch(b1, 1);

    // Stage A rows k0 .. k0+R as sA[r][m] (m >= M zero): thread t loads row t
    // of every m (coalesced along k) and writes its MT values as vector stores.
    const float* A = static_cast<const float*>(g.A);
    for (int r = tid; r < R; r += kThreads) {
        float v[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            v[m] = 0.0f;
            if (m < g.M) {
                const int64_t off = g.a_trans ? static_cast<int64_t>(k0 + r) * g.lda + m
                                              : static_cast<int64_t>(m) * g.lda + (k0 + r);
                v[m] = __ldg(A + off);
            }
        }
        if constexpr (MT >= 4) {
#pragma unroll
            for (int q = 0; q < MT / 4; ++q)
                *reinterpret_cast<float4*>(&sA[r * MT + 4 * q]) =
                    make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else if constexpr (MT == 2) {
            *reinterpret_cast<float2*>(&sA[r * 2]) = make_float2(v[0], v[1]);
        } else {
            sA[r] = v[0];
        }
    }

    // Thread t finishes VW consecutive columns of row m (t < kGroups) in the
    // last CTA of the panel; every CTA reads those C values now, in the shadow
    // of the B stream, as it cannot know yet whether it will be the last.
    const int gm = tid / (kPanel / VW), gc = (tid % (kPanel / VW)) * VW;
    const bool gown = tid < kGroups && gm < g.M;
    float* C = static_cast<float*>(g.C);
    float c_old[VW];
#pragma unroll
    for (int u = 0; u < VW; ++u)
        c_old[u] = (gown && g.beta != 0.0f && n0 + gc + u < g.N) ? C[static_cast<int64_t>(gm) * g.ldc + n0 + gc + u]
                                                                  : 0.0f;
    __syncthreads();   // sA complete

    float acc[MT][kQ];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int q = 0; q < kQ; ++q) acc[m][q] = 0.0f;
    auto compute_batch = [&](const float (&b)[U][kQ], int j) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = j * U + u;
            if (i < nrows) {
                const int r = warp + kWarps * i;
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
                for (int m = 0; m < MT; ++m)
#pragma unroll
                    for (int q = 0; q < kQ; ++q) acc[m][q] = fmaf(a[m], b[u][q], acc[m][q]);
            }
        }
    };
    for (int j = 0; j < nb; j += 2) {
        compute_batch(b0, j);
        if (j + 2 < nb) load_batch(b0, j + 2);
        if (j + 1 < nb) {
            compute_batch(b1, j + 1);
            if (j + 3 < nb) load_batch(b1, j + 3);
        }
    }

    // The B stream of this CTA is done: let the next kernel on the stream
    // start launching.  Triggered here rather than at entry, so that a
    // dependent grid's CTAs do not sit resident (holding registers and SM
    // slots) at their griddepcontrol.wait for this kernel's whole run.
    pdl_launch_dependents();

    // Warp partials -> red[warp][m][c], then the CTA's partial panel
    // red[0][m][c] = sum over warps 0..7 in order.
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int q = 0; q < kQ; ++q) red[(warp * MT + m) * kPanel + lane + 32 * q] = acc[m][q];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxOut; ++i) {
        const int o = tid + i * kThreads;     // o = m * kPanel + c
        if (o < MT * kPanel) {
            float s = red[o];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) s += red[w * MT * kPanel + o];
            red[o] = s;
        }
    }
    __syncthreads();

    float sum[VW];
    if (S == 1) {
#pragma unroll
        for (int u = 0; u < VW; ++u) sum[u] = gown ? red[gm * kPanel + gc + u] : 0.0f;
    } else {
        // Publish this split's partial panel, then the last CTA of the panel
        // (ticket S - 1) sums the S partials in split order.
        if (tid < kGroups) {
            float* dst = p.ws + (static_cast<int64_t>(split) * MT + gm) * p.n_pad + n0 + gc;
            if constexpr (VW == 4) __stcg(reinterpret_cast<float4*>(dst), *reinterpret_cast<const float4*>(&red[gm * kPanel + gc]));
            else if constexpr (VW == 2) __stcg(reinterpret_cast<float2*>(dst), *reinterpret_cast<const float2*>(&red[gm * kPanel + gc]));
            else __stcg(dst, red[gm * kPanel + gc]);
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t ticket = atomicAdd(&p.counters[blockIdx.x], 1u);
            s_last = ticket == static_cast<uint32_t>(S - 1);
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        float v[8][VW];
        const float* src = p.ws + static_cast<int64_t>(gm) * p.n_pad + n0 + gc;
        const int64_t sstride = static_cast<int64_t>(MT) * p.n_pad;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (q < S && tid < kGroups) {
                const float* ps = src + q * sstride;
                if constexpr (VW == 4) {
                    const float4 t = __ldcg(reinterpret_cast<const float4*>(ps));
                    v[q][0] = t.x; v[q][1] = t.y; v[q][2] = t.z; v[q][3] = t.w;
                } else if constexpr (VW == 2) {
                    const float2 t = __ldcg(reinterpret_cast<const float2*>(ps));
                    v[q][0] = t.x; v[q][1] = t.y;
                } else {
                    v[q][0] = __ldcg(ps);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < VW; ++u) sum[u] = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
            if (q < S) {
#pragma unroll
                for (int u = 0; u < VW; ++u) sum[u] += v[q][u];
            }
        if (tid == 0) p.counters[blockIdx.x] = 0u;   // ready for the next launch on this stream
    }
    if (gown) {
#pragma unroll
        for (int u = 0; u < VW; ++u) {
            const int n = n0 + gc + u;
            if (n < g.N) {
                const float val = (g.beta == 0.0f) ? g.alpha * sum[u] : fmaf(g.alpha, sum[u], g.beta * c_old[u]);
                C[static_cast<int64_t>(gm) * g.ldc + n] = add_bias(val, g.bias, n);
            }
        }
    }
}

// Rows per warp batch (two batches in flight): 4 for 128-column panels, 8
// for 64-column ones (16 KB of loads in flight per CTA either way), 16 for
// 64-column panels over the whole K (one CTA streams a 64-column panel alone,
// so it keeps 32 KB in flight).
template <int MT>
const void* panel_fn(int w, int splits) {
    if (w == 64) return splits == 1 ? reinterpret_cast<const void*>(&gemv_panel_kernel<MT, 16, 64>)
                                    : reinterpret_cast<const void*>(&gemv_panel_kernel<MT, 8, 64>);
    return reinterpret_cast<const void*>(&gemv_panel_kernel<MT, 4, 128>);
}

const void* panel_select(int mt, int w, int splits) {
    if (w != 64 && w != 128) return nullptr;
    switch (mt) {
        case 1: return panel_fn<1>(w, splits);
        case 2: return panel_fn<2>(w, splits);
        case 4: return panel_fn<4>(w, splits);
        case 8: return panel_fn<8>(w, splits);
        default: return nullptr;
    }
}

size_t panel_smem_bytes(int mt, int w, int rows) {
    return static_cast<size_t>(rows) * mt * 4 + static_cast<size_t>(kWarps) * mt * w * 4;
}

cudaError_t panel_prepare(const void* fn) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({dev, fn})) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(panel_smem_bytes(8, 128, kMaxRows)));
    if (e == cudaSuccess) done.insert({dev, fn});
    return e;
}

}  // namespace

int gemv_panel_rows(int K, int splits) {
    if (splits < 1) return 0;
    const int rows = (K + splits - 1) / splits;
    return (rows + 7) / 8 * 8;
}

bool gemv_panel_supported(const GemmArgs& g, int mt, int w, int splits) {
    if (!panel_select(mt, w, splits) || g.M < 1 || g.M > mt || g.N < 1 || g.K < 1 || g.b_trans) return false;
    if (splits != 1 && splits != 2 && splits != 4 && splits != 8) return false;
    const int rows = gemv_panel_rows(g.K, splits);
    // Every split holds at least one row and at most kMaxRows.
    return rows <= kMaxRows && static_cast<int64_t>(rows) * (splits - 1) < g.K;
}

int gemv_panel_ctas(int N, int w, int splits) { return (N + w - 1) / w * splits; }

cudaError_t gemv_panel_occupancy(int mt, int w, int splits, int rows, int* blocks_per_sm) {
    const void* fn = panel_select(mt, w, splits);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = panel_prepare(fn);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, kThreads,
                                                         panel_smem_bytes(mt, w, rows));
}

size_t gemv_panel_ws_floats(int N, int mt, int w, int splits) {
    if (splits <= 1) return 0;
    return static_cast<size_t>(splits) * mt * ((N + w - 1) / w) * w;
}

int gemv_panel_tickets(int N, int w) { return (N + w - 1) / w; }

cudaError_t launch_gemv_panel(const GemmArgs& g, int mt, int w, int splits, float* ws, uint32_t* counters,
                              cudaStream_t s) {
    if (!gemv_panel_supported(g, mt, w, splits)) return cudaErrorInvalidValue;
    if (splits > 1 && (!ws || !counters)) return cudaErrorInvalidValue;
    const void* fn = panel_select(mt, w, splits);
    cudaError_t e = panel_prepare(fn);
    if (e != cudaSuccess) return e;
    PanelParams pp;
    pp.g = g;
    pp.rows = gemv_panel_rows(g.K, splits);
    pp.n_pad = gemv_panel_tickets(g.N, w) * w;
    pp.ws = ws;
    pp.counters = counters;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(gemv_panel_tickets(g.N, w)), static_cast<unsigned>(splits), 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = panel_smem_bytes(mt, w, pp.rows);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&pp};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace dnnopt_b200
