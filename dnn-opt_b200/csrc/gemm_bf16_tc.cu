// BF16 x BF16 -> FP32 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM)
// for the tall-skinny class: large M, N <= 256, B small enough to stay resident
// in shared memory.  This is the B200 replacement of the reference's BLIS
// BFMMLA driver gemm_bf16_bf16bf16f32 (src/gemm/gemm_driver_bf16.cpp:134-218,
// micro-kernel src/gemm/gemm_ukernel_bf16_neon.cpp:30-160) on its headline
// shape (M=65536, N=64, K=256).
//
// Shape physics: at N=64, K=256 the GEMM does 43 flop per HBM byte, far below
// the BF16 ridge (~250 flop/B), so the kernel streams A and C at HBM speed and
// keeps the tensor cores a few percent busy.  Design:
//   * persistent CTAs walk 128-row tiles of A;
//   * warp 0 issues TMA loads of A in 128 x 64 K-blocks (128-byte swizzle)
//     into an N-stage shared-memory ring (mbarrier full/empty pairs);
//   * the first ring of A loads is issued before B (K x N) is gathered once
//     per CTA into the same K-major swizzled layout (16-byte row loads);
//   * warp 1 issues tcgen05.mma (M=128, N=n_pad, K=16) into one of two TMEM
//     accumulators, so the epilogue of tile t overlaps the MMAs of tile t+1;
//   * warps 2-5 drain TMEM with tcgen05.ld, apply alpha/beta (the reference
//     epilogue: beta == 0 ? alpha*acc : fma(alpha, acc, beta*C)) and store
//     each thread's row with 16-byte stores;
//   * two CTAs per SM when B leaves room (a shallow 4-stage ring each).
// No cluster multicast is used anywhere.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int BM = 128;                // rows per tile (UMMA M)
constexpr int kKBlock = 64;            // bf16 elements per 128-byte swizzle row
constexpr int kStageBytes = BM * 128;  // one A K-block
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr size_t kSmemLimit = 227 * 1024;

struct TcParams {
    int M, N, K;
    int n_pad, num_kb, num_tiles, stages;
    float alpha, beta;
    const uint16_t* B;
    int64_t ldb;
    int b_trans;
    int b_vec;         // B is K x N with 16-byte aligned rows (vector gather)
    float* C;
    int64_t ldc;
    uint32_t tmem_cols;
    uint32_t* err;
};

__global__ void __launch_bounds__(kThreads, 2)
gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int sb_bytes = p.num_kb * p.n_pad * 128;
    uint8_t* sB = base;
    uint8_t* sA = sB + sb_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sA + p.stages * kStageBytes);
    uint64_t* empty = full + p.stages;
    uint64_t* tfull = empty + p.stages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // Tiles of this CTA: blockIdx.x, +gridDim.x, ...; producer iteration i
    // loads K-block (i % num_kb) of the (i / num_kb)-th of them.
    const int my_tiles = (p.num_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x);
    const uint32_t total_iters = static_cast<uint32_t>(my_tiles > 0 ? my_tiles : 0) * p.num_kb;
    auto issue_load = [&](uint32_t i) {
        const uint32_t s = i % p.stages;
        const int tile = static_cast<int>(blockIdx.x) + static_cast<int>(i / p.num_kb) * static_cast<int>(gridDim.x);
        const int kb = static_cast<int>(i % p.num_kb);
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(sA + s * kStageBytes, &tmA, &full[s], kb * kKBlock, tile * BM);
    };
    const uint32_t pre = total_iters < static_cast<uint32_t>(p.stages) ? total_iters
                                                                       : static_cast<uint32_t>(p.stages);

    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
        *abort_flag = 0u;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        // The first ring of A loads goes out before B is gathered: every stage
        // starts empty, so these need no wait.
        for (uint32_t i = 0; i < pre; ++i) issue_load(i);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, p.tmem_cols);
        tmem_relinquish();
    }

    // Gather B into K-major 128B-swizzled rows (the UMMA B operand):
    // byte offset of (n, k) = kb*n_pad*128 + n*128 + ((c ^ (n&7))*16) + (k%8)*2,
    // kb = k/64, c = (k%64)/8.
    if (p.b_vec) {
        // B is K x N with 16-byte aligned rows: one 16-byte load brings 8
        // consecutive n of row k; consecutive threads take consecutive k so
        // the 2-byte shared stores of a warp fall in distinct banks.  Loads
        // are issued in groups of kGather before any store so that a thread
        // has kGather requests in flight instead of one.
        constexpr int kGather = 8;
        const int kpad = p.num_kb * kKBlock;
        const int n8s = p.n_pad / 8;
        const int total = kpad * n8s;
        for (int base_idx = tid; base_idx < total; base_idx += kThreads * kGather) {
            uint4 v[kGather];
#pragma unroll
            for (int j = 0; j < kGather; ++j) {
                const int idx = base_idx + j * kThreads;
                const int k = idx % kpad, n8 = idx / kpad;
                v[j] = make_uint4(0u, 0u, 0u, 0u);
                if (idx < total && k < p.K) {
                    if (n8 * 8 + 8 <= p.N) {
                        v[j] = __ldg(reinterpret_cast<const uint4*>(p.B + (int64_t)k * p.ldb + n8 * 8));
                    } else {
                        uint32_t w[4] = {0u, 0u, 0u, 0u};
                        for (int e = 0; e < 8 && n8 * 8 + e < p.N; ++e)
                            w[e >> 1] |= static_cast<uint32_t>(p.B[(int64_t)k * p.ldb + n8 * 8 + e]) << ((e & 1) * 16);
                        v[j] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kGather; ++j) {
                const int idx = base_idx + j * kThreads;
                if (idx >= total) break;
                const int k = idx % kpad, n8 = idx / kpad;
                const uint32_t w4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
                const int kb = k >> 6, c = (k & 63) >> 3;
                uint8_t* base_kb = sB + kb * p.n_pad * 128 + (k & 7) * 2;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int n = n8 * 8 + e;
                    const uint16_t val = static_cast<uint16_t>(w4[e >> 1] >> ((e & 1) * 16));
                    *reinterpret_cast<uint16_t*>(base_kb + n * 128 + ((c ^ (n & 7)) * 16)) = val;
                }
            }
        }
    } else {
        const int total = p.num_kb * 8 * p.n_pad;
        for (int idx = tid; idx < total; idx += kThreads) {
            const int n = idx % p.n_pad, rest = idx / p.n_pad;
            const int c = rest & 7, kb = rest >> 3;
            const int k0 = kb * kKBlock + c * 8;
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                uint32_t lo = 0, hi = 0;
                if (n < p.N) {
                    int ka = k0 + e, kb2 = k0 + e + 1;
                    if (ka < p.K) lo = p.B[p.b_trans ? (int64_t)n * p.ldb + ka : (int64_t)ka * p.ldb + n];
                    if (kb2 < p.K) hi = p.B[p.b_trans ? (int64_t)n * p.ldb + kb2 : (int64_t)kb2 * p.ldb + n];
                }
                w[e >> 1] = lo | (hi << 16);
            }
            uint8_t* dst = sB + kb * p.n_pad * 128 + n * 128 + ((c ^ (n & 7)) * 16);
            *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            for (uint32_t i = pre; i < total_iters && !*abort_flag; ++i) {
                const uint32_t s = i % p.stages, ph = (i / p.stages) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err)) break;
                issue_load(i);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16_f32(BM, p.n_pad);
            uint32_t it = 0, titer = 0;
            for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++titer) {
                const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
                if (!mbar_wait(&tempty[buf], tph ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * p.n_pad;
                bool ok = true;
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
                    if (!mbar_wait(&full[s], ph, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * kStageBytes);
                    const uint32_t b_addr = smem_u32(sB + kb * p.n_pad * 128);
#pragma unroll
                    for (int kk = 0; kk < kKBlock / 16; ++kk) {
                        umma_f16_ss(d_tmem, umma_desc_k_sw128(a_addr + kk * 32),
                                    umma_desc_k_sw128(b_addr + kk * 32), idesc,
                                    (kb | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);   // stage is free once these MMAs retire
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);     // accumulator ready for the epilogue
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        // Each thread owns one output row: 16-column groups come out of TMEM
        // and go straight to global memory as 16-byte stores (a thread's
        // consecutive stores complete each 32-byte sector of its row).
        const int q = warp & 3;                      // TMEM lane quadrant of this warp
        uint32_t titer = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++titer) {
            const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
            if (!mbar_wait(&tfull[buf], tph, abort_flag, p.err)) break;
            tc_fence_after();
            const int row = tile * BM + q * 32 + lane;
            const bool row_ok = row < p.M;
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * p.n_pad;
            float* crow = p.C + (int64_t)row * p.ldc;
            for (int cg = 0; cg < p.n_pad / 16; ++cg) {
                uint32_t r[16];
                tmem_ld_32x32b_x16(t_addr + cg * 16, r);
                tmem_ld_wait();
                if (!row_ok) continue;
                const int c0 = cg * 16;
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const int col = c0 + j4 * 4;
                    float v[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[j] = p.alpha * __uint_as_float(r[j4 * 4 + j]);
                    if (col + 4 <= p.N) {
                        float4* dst = reinterpret_cast<float4*>(crow + col);
                        if (p.beta != 0.0f) {
                            const float4 old = *dst;
                            v[0] = fmaf(p.alpha, __uint_as_float(r[j4 * 4 + 0]), p.beta * old.x);
                            v[1] = fmaf(p.alpha, __uint_as_float(r[j4 * 4 + 1]), p.beta * old.y);
                            v[2] = fmaf(p.alpha, __uint_as_float(r[j4 * 4 + 2]), p.beta * old.z);
                            v[3] = fmaf(p.alpha, __uint_as_float(r[j4 * 4 + 3]), p.beta * old.w);
                        }
                        *dst = make_float4(v[0], v[1], v[2], v[3]);
                    } else {
                        for (int j = 0; j < 4 && col + j < p.N; ++j) {
                            float o = v[j];
                            if (p.beta != 0.0f) o = fmaf(p.alpha, __uint_as_float(r[j4 * 4 + j]), p.beta * crow[col + j]);
                            crow[col + j] = o;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);  // TMEM buffer may be overwritten
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

// ---- host helpers ----------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                             cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(ptr);
    }();
    return fn;
}

struct Layout {
    int n_pad, num_kb, stages, ctas_per_sm;
    size_t smem;
};

// Measured on B200: two CTAs per SM with a 4-stage ring stream A faster than
// one CTA with a deep ring.  Fall back to one CTA per SM (up to 8 stages)
// when B does not leave room for two.
Layout plan_layout(const GemmArgs& g) {
    Layout L;
    L.n_pad = (g.N + 15) / 16 * 16;
    L.num_kb = (g.K + kKBlock - 1) / kKBlock;
    const size_t fixed = 1024 + static_cast<size_t>(L.num_kb) * L.n_pad * 128 + 256;
    const size_t half = kSmemLimit / 2 - 1024;
    int st2 = fixed < half ? static_cast<int>((half - fixed) / kStageBytes) : 0;
    if (st2 >= 3) {
        L.stages = st2 > 4 ? 4 : st2;
        L.ctas_per_sm = 2;
    } else {
        int st = fixed < kSmemLimit ? static_cast<int>((kSmemLimit - fixed) / kStageBytes) : 0;
        L.stages = st > kMaxStages ? kMaxStages : st;
        L.ctas_per_sm = 1;
    }
    L.smem = fixed + static_cast<size_t>(L.stages) * kStageBytes;
    return L;
}

}  // namespace

bool gemm_bf16_tc_supported(const GemmArgs& g) {
    if (g.M < 1 || g.N < 1 || g.K < 1 || g.N > 256 || g.a_trans) return false;
    if (reinterpret_cast<uintptr_t>(g.A) % 16 || g.lda % 8 || g.lda < g.K) return false;
    if (reinterpret_cast<uintptr_t>(g.C) % 16 || g.ldc % 4 || g.ldc < g.N) return false;
    if (get_encode_fn() == nullptr) return false;
    return plan_layout(g).stages >= 2;
}

cudaError_t launch_gemm_bf16_tc(const GemmArgs& g, int num_sms, uint32_t* err, cudaStream_t s) {
    if (!gemm_bf16_tc_supported(g)) return cudaErrorInvalidValue;
    const Layout L = plan_layout(g);
    EncodeTiledFn encode = get_encode_fn();

    CUtensorMap tmA;
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(g.K), static_cast<cuuint64_t>(g.M)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(g.lda) * 2};
        cuuint32_t box[2] = {kKBlock, BM};
        cuuint32_t estr[2] = {1, 1};
        if (encode(&tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(g.A), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }

    TcParams p;
    p.M = g.M; p.N = g.N; p.K = g.K;
    p.n_pad = L.n_pad; p.num_kb = L.num_kb; p.stages = L.stages;
    p.num_tiles = (g.M + BM - 1) / BM;
    p.alpha = g.alpha; p.beta = g.beta;
    p.B = static_cast<const uint16_t*>(g.B); p.ldb = g.ldb; p.b_trans = g.b_trans;
    p.b_vec = (!g.b_trans && reinterpret_cast<uintptr_t>(g.B) % 16 == 0 && g.ldb % 8 == 0) ? 1 : 0;
    p.C = static_cast<float*>(g.C); p.ldc = g.ldc;
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(2 * L.n_pad)) cols <<= 1;
    p.tmem_cols = cols;
    p.err = err;

    // The attribute is per device; set it once to the largest size requested
    // so that launches under stream capture make no further attribute calls.
    static thread_local int smem_set_dev = -1;
    static thread_local size_t smem_set = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != smem_set_dev || L.smem > smem_set) {
        e = cudaFuncSetAttribute(gemm_bf16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemLimit));
        if (e != cudaSuccess) return e;
        smem_set_dev = dev;
        smem_set = kSmemLimit;
    }
    const int slots = num_sms * L.ctas_per_sm;
    int grid = p.num_tiles < slots ? p.num_tiles : slots;
    gemm_bf16_tc_kernel<<<grid, kThreads, L.smem, s>>>(tmA, p);
    return cudaGetLastError();
}

}  // namespace dnnopt_b200
