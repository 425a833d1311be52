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
//   * persistent CTAs walk 128-row tiles of A: one CTA per SM with four
//     K-blocks per ring stage when K spans four or more K-blocks, else two
//     CTAs per SM when shared memory and TMEM allow;
//   * one thread issues every TMA load: B once per CTA, straight into the UMMA
//     operand layout (MN-major 128-byte swizzle when B is K x N, K-major when B
//     is N x K; an element gather only when B's rows are not 16-byte aligned),
//     then A in 128 x 64 K-blocks into the shared-memory ring (mbarrier
//     full/empty pairs);
//   * warp 1 issues tcgen05.mma (M=128, N=n_mma, K=16) into one of two TMEM
//     accumulators, so the epilogue of tile t overlaps the MMAs of tile t+1;
//   * warps 2-5 drain TMEM with tcgen05.ld, apply alpha/beta (the reference
//     epilogue: beta == 0 ? alpha*acc : fma(alpha, acc, beta*C)), stage 32 x 32
//     float blocks in 128-byte-swizzled shared memory and write them with TMA
//     stores (rows >= M and columns >= N are clipped by the tensor map);
//   * programmatic dependent launch: the prologue (barrier init, TMEM
//     allocation, descriptor prefetch) overlaps the previous kernel's tail and
//     every global access waits for it (griddepcontrol.wait).
// Every TMA load targets this CTA's own shared memory.
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
constexpr int kStageCBytes = 32 * 128;           // one 32 x 32 FP32 store block
constexpr int kCStagingBytes = 4 * 2 * kStageCBytes;  // 4 warps x 2 buffers
constexpr size_t kSmemLimit = 227 * 1024;
constexpr size_t kSmemPerSm = 228 * 1024;        // per SM, 1 KB of it reserved per CTA

enum BMode : int {
    kBGather = 0,    // element gather into the K-major swizzled layout
    kBTmaMN = 1,     // B is K x N: TMA boxes of 64 n x 64 k, MN-major operand
    kBTmaK = 2,      // B is N x K: TMA boxes of 64 k x n_mma rows, K-major operand
};

struct TcParams {
    int M, N, K;
    int n_mma, num_kb, kpad, n_chunks, num_tiles, stages, b_mode;
    int kbs, groups;   // A K-blocks per ring stage, stages per tile
    uint32_t sb_bytes;
    float alpha, beta;
    const uint16_t* B;
    int64_t ldb;
    int b_trans;
    const float* C;     // read for beta != 0
    int64_t ldc;
    uint32_t tmem_cols;
    uint32_t* err;
};

// Shared-memory descriptor of an MN-major operand in the canonical 128-byte
// swizzled layout: 64 elements along N per 128-byte row, eight K rows per
// 1024-byte atom, atoms of one 64-column chunk stacked densely along K (SBO =
// 1024 B) and chunks `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// MN: B in the MN-major layout (kBTmaMN), else K-major.  A compile-time
// choice: a run-time branch between MMA forms in the issue loop measured twice
// the issue time per MMA on B200.
template <bool MN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sB = base;
    uint8_t* sA = sB + p.sb_bytes;
    const uint32_t stage_bytes = static_cast<uint32_t>(p.kbs) * kStageBytes;
    uint8_t* sC = sA + p.stages * stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sC + kCStagingBytes);
    uint64_t* empty = full + p.stages;
    uint64_t* tfull = empty + p.stages;
    uint64_t* tempty = tfull + 2;
    uint64_t* bfull = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bfull + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // Tiles of this CTA: blockIdx.x, +gridDim.x, ...; producer iteration i
    // loads K-block group (i % groups) of the (i / groups)-th of them: kbs
    // K-blocks per stage (a stage costs a roughly fixed mbarrier round trip,
    // so larger stages stream faster).
    const int my_tiles = (p.num_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x);
    const uint32_t total_iters = static_cast<uint32_t>(my_tiles > 0 ? my_tiles : 0) * p.groups;
    auto issue_load = [&](uint32_t i) {
        const uint32_t s = i % p.stages;
        const int tile = static_cast<int>(blockIdx.x) + static_cast<int>(i / p.groups) * static_cast<int>(gridDim.x);
        const int kb0 = static_cast<int>(i % p.groups) * p.kbs;
        const int nsub = min(p.kbs, p.num_kb - kb0);
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nsub) * kStageBytes);
        for (int sub = 0; sub < nsub; ++sub)
            tma_load_2d(sA + s * stage_bytes + sub * kStageBytes, &tmA, &full[s], (kb0 + sub) * kKBlock, tile * BM);
    };
    const uint32_t pre = total_iters < static_cast<uint32_t>(p.stages) ? total_iters
                                                                       : static_cast<uint32_t>(p.stages);

    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
        mbar_init(bfull, 1);
        *abort_flag = 0u;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmC);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, p.tmem_cols);
        tmem_relinquish();
    }
    pdl_wait();   // inputs and C may be written by the preceding kernel
    if (tid == 0) {
        // B first (the first MMA needs all of it), then the first ring of A:
        // every stage starts empty, so these loads need no wait.
        if (p.b_mode == kBTmaMN) {
            mbar_arrive_expect_tx(bfull, p.sb_bytes);
            for (int j = 0; j < p.n_chunks; ++j)
                for (int kb = 0; kb < p.num_kb; ++kb)
                    tma_load_2d(sB + (j * p.kpad + kb * kKBlock) * 128, &tmB, bfull, j * 64, kb * kKBlock);
        } else if (p.b_mode == kBTmaK) {
            mbar_arrive_expect_tx(bfull, p.sb_bytes);
            for (int kb = 0; kb < p.num_kb; ++kb)
                tma_load_2d(sB + kb * p.n_mma * 128, &tmB, bfull, kb * kKBlock, 0);
        }
        for (uint32_t i = 0; i < pre; ++i) issue_load(i);
    }

    if (p.b_mode == kBGather) {
        // B rows are not 16-byte aligned: gather element pairs into the
        // K-major 128B-swizzled layout, byte offset of (n, k) =
        // kb*n_mma*128 + n*128 + ((c ^ (n&7))*16) + (k%8)*2, kb = k/64, c = (k%64)/8.
        const int total = p.num_kb * 8 * p.n_mma;
        for (int idx = tid; idx < total; idx += kThreads) {
            const int n = idx % p.n_mma, rest = idx / p.n_mma;
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
            uint8_t* dst = sB + kb * p.n_mma * 128 + n * 128 + ((c ^ (n & 7)) * 16);
            *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Dependent kernels may start once every CTA holds its TMEM: one that
    // allocated first could otherwise leave this grid waiting on it.
    pdl_launch_dependents();

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
            uint32_t idesc = umma_idesc_bf16_f32(BM, p.n_mma);
            if constexpr (MN) idesc |= 1u << 16;                 // B operand MN-major
            const uint32_t sb_addr = smem_u32(sB);
            const uint32_t lbo = static_cast<uint32_t>(p.kpad) * 128u;
            bool ok = p.b_mode == kBGather || mbar_wait(bfull, 0, abort_flag, p.err);
            uint32_t it = 0, titer = 0;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++titer) {
                const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
                if (!mbar_wait(&tempty[buf], tph ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * p.n_mma;
                for (int grp = 0; grp < p.groups; ++grp, ++it) {
                    const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
                    if (!mbar_wait(&full[s], ph, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const int kb0 = grp * p.kbs;
                    const int nsub = min(p.kbs, p.num_kb - kb0);
                    for (int sub = 0; sub < nsub; ++sub) {
                        const int kb = kb0 + sub;
                        const uint32_t a_addr = smem_u32(sA + s * stage_bytes + sub * kStageBytes);
                        // K step of 16: 32 bytes along a K-major row, or two
                        // 1024-byte 8-row atoms down an MN-major chunk (the B
                        // layout branch taken once per K-block).
                        if constexpr (MN) {
#pragma unroll
                            for (int kk = 0; kk < kKBlock / 16; ++kk)
                                umma_f16_ss(d_tmem, umma_desc_k_sw128(a_addr + kk * 32),
                                            umma_desc_mn_sw128(sb_addr + (kb * 8 + kk * 2) * 1024, lbo), idesc,
                                            (kb | kk) != 0 ? 1u : 0u);
                        } else {
#pragma unroll
                            for (int kk = 0; kk < kKBlock / 16; ++kk)
                                umma_f16_ss(d_tmem, umma_desc_k_sw128(a_addr + kk * 32),
                                            umma_desc_k_sw128(sb_addr + kb * p.n_mma * 128 + kk * 32), idesc,
                                            (kb | kk) != 0 ? 1u : 0u);
                        }
                    }
                    umma_commit(&empty[s]);   // stage is free once these MMAs retire
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);     // accumulator ready for the epilogue
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        // Warp q owns TMEM lanes / tile rows [32q, 32q+32).  Columns go out in
        // 32-wide groups through two 4 KB staging buffers per warp: lane l
        // writes row l as eight 16-byte chunks at ((c ^ (l&7))*16), the
        // 128-byte swizzle the C tensor map uses, so a warp's shared stores
        // are conflict-free; lane 0 then issues one TMA store per group.
        const int q = warp & 3;
        uint8_t* stg = sC + q * 2 * kStageCBytes;
        const int n_groups = (p.N + 31) / 32;
        uint32_t titer = 0, gcount = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++titer) {
            const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
            if (!mbar_wait_warp(&tfull[buf], tph, abort_flag, p.err)) break;
            tc_fence_after();
            const int row = tile * BM + q * 32 + lane;
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * p.n_mma;
            for (int g0 = 0; g0 < n_groups; g0 += 2) {
                uint32_t r[2][32];
                const int ng = n_groups - g0 < 2 ? n_groups - g0 : 2;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (h < ng) {
                        tmem_ld_32x32b_x16(t_addr + (g0 + h) * 32, *reinterpret_cast<uint32_t(*)[16]>(&r[h][0]));
                        tmem_ld_32x32b_x16(t_addr + (g0 + h) * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[h][16]));
                    }
                }
                tmem_ld_wait();
                if (g0 + 2 >= n_groups) {
                    // Every column of this tile is in registers: release the
                    // accumulator so the next tile's MMAs can start.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[buf]);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (h >= ng) break;
                    const int col0 = (g0 + h) * 32;
                    uint8_t* sbuf = stg + (gcount & 1u) * kStageCBytes;
                    if (lane == 0) tma_store_wait_read<1>();   // this buffer's previous store has read it
                    __syncwarp();
                    const float* crow = p.C + (int64_t)row * p.ldc;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        float v[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) v[j] = p.alpha * __uint_as_float(r[h][c * 4 + j]);
                        if (p.beta != 0.0f && row < p.M) {
                            const int col = col0 + c * 4;
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                if (col + j < p.N)
                                    v[j] = fmaf(p.alpha, __uint_as_float(r[h][c * 4 + j]), p.beta * crow[col + j]);
                        }
                        *reinterpret_cast<float4*>(sbuf + lane * 128 + ((c ^ (lane & 7)) * 16)) =
                            make_float4(v[0], v[1], v[2], v[3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, sbuf, col0, tile * BM + q * 32);
                        tma_store_commit();
                    }
                    ++gcount;
                }
            }
        }
        if (lane == 0) tma_store_wait_all<0>();   // staging must outlive the stores' reads
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
    int b_mode, n_mma, num_kb, kpad, n_chunks, stages, ctas_per_sm, kbs;
    uint32_t sb_bytes, tmem_cols;
    size_t smem;
};

// B operand mode, shared-memory plan and CTAs per SM.  Measured on B200: one
// CTA per SM with four K-blocks per stage streams A fastest when K has four
// or more K-blocks; for shallower K two CTAs per SM with a 2-4 stage ring beat
// one CTA with a deep ring of single K-blocks; one CTA per SM (up to 8 stages)
// when B or TMEM leaves no room for two.
Layout plan_layout(const GemmArgs& g) {
    Layout L;
    const bool b_aligned = reinterpret_cast<uintptr_t>(g.B) % 16 == 0 && g.ldb % 8 == 0;
    L.num_kb = (g.K + kKBlock - 1) / kKBlock;
    L.kpad = L.num_kb * kKBlock;
    if (b_aligned && !g.b_trans && L.kpad * 128 < (1 << 18)) {
        L.b_mode = kBTmaMN;
        L.n_mma = (g.N + 63) / 64 * 64;
        L.n_chunks = L.n_mma / 64;
        L.sb_bytes = static_cast<uint32_t>(L.n_chunks * L.kpad * 128);
    } else {
        L.b_mode = b_aligned && g.b_trans ? kBTmaK : kBGather;
        L.n_mma = (g.N + 15) / 16 * 16;
        L.n_chunks = 0;
        L.sb_bytes = static_cast<uint32_t>(L.num_kb * L.n_mma * 128);
    }
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(2 * L.n_mma)) cols <<= 1;
    L.tmem_cols = cols;
    const size_t fixed = 1024 + static_cast<size_t>(L.sb_bytes) + kCStagingBytes + 256;
    const size_t per_cta2 = kSmemPerSm / 2 - 1024;
    const int st2 = fixed < per_cta2 ? static_cast<int>((per_cta2 - fixed) / kStageBytes) : 0;
    L.kbs = 1;
    // Four or more K-blocks per tile: one CTA per SM with four K-blocks per
    // ring stage (a stage costs a roughly fixed mbarrier round trip; measured
    // on 65536 x 64 x 256: 11.9 us against 12.8 us for two CTAs per SM with
    // one K-block per stage).  Shallower K: two CTAs per SM.
    const int st4 = fixed < kSmemLimit ? static_cast<int>((kSmemLimit - fixed) / (4 * kStageBytes)) : 0;
    if (L.num_kb >= 4 && st4 >= 2) {
        L.kbs = 4;
        L.stages = st4 > kMaxStages ? kMaxStages : st4;
        L.ctas_per_sm = 1;
    } else if (st2 >= 2 && 2 * L.tmem_cols <= 512) {
        L.stages = st2 > 4 ? 4 : st2;
        L.ctas_per_sm = 2;
    } else {
        const int st = fixed < kSmemLimit ? static_cast<int>((kSmemLimit - fixed) / kStageBytes) : 0;
        L.stages = st > kMaxStages ? kMaxStages : st;
        L.ctas_per_sm = 1;
    }
    L.smem = fixed + static_cast<size_t>(L.stages) * L.kbs * kStageBytes;
    return L;
}

bool encode_2d(CUtensorMap* m, CUtensorMapDataType t, const void* ptr, uint64_t d0, uint64_t d1,
               uint64_t row_bytes, uint32_t b0, uint32_t b1) {
    cuuint64_t dims[2] = {d0, d1};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {b0, b1};
    cuuint32_t estr[2] = {1, 1};
    return get_encode_fn()(m, t, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace {
bool shape_ok(const GemmArgs& g) {
    if (g.M < 1 || g.N < 1 || g.K < 1 || g.N > 256 || g.a_trans) return false;
    if (reinterpret_cast<uintptr_t>(g.A) % 16 || g.lda % 8 || g.lda < g.K) return false;
    if (reinterpret_cast<uintptr_t>(g.C) % 16 || g.ldc % 4 || g.ldc < g.N) return false;
    return get_encode_fn() != nullptr;
}
}  // namespace

bool gemm_bf16_tc_supported(const GemmArgs& g) {
    return shape_ok(g) && plan_layout(g).stages >= 2;
}

// B stays resident in shared memory, so a deep K (conv3d's im2col GEMMs:
// K = 27*IC) may not fit: the caller then runs K in chunks of this many rows
// (a multiple of the 64-row K-block), accumulating into C with beta = 1.
int gemm_bf16_tc_kchunk(const GemmArgs& g) {
    if (!shape_ok(g)) return 0;
    if (plan_layout(g).stages >= 2) return g.K;
    GemmArgs t = g;
    for (int kc = (g.K - 1) / kKBlock * kKBlock; kc >= kKBlock; kc -= kKBlock) {
        t.K = kc;
        if (plan_layout(t).stages >= 2) return kc;
    }
    return 0;
}

cudaError_t launch_gemm_bf16_tc(const GemmArgs& g, int num_sms, uint32_t* err, cudaStream_t s) {
    if (!gemm_bf16_tc_supported(g)) return cudaErrorInvalidValue;
    const Layout L = plan_layout(g);

    // Inner dimension first; every row stride is a multiple of 16 bytes and
    // every box's inner extent is 128 bytes (the swizzle span).
    CUtensorMap tmA, tmB, tmC;
    if (!encode_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.A, g.K, g.M,
                   static_cast<uint64_t>(g.lda) * 2, kKBlock, BM))
        return cudaErrorInvalidValue;
    if (!encode_2d(&tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.C, g.N, g.M,
                   static_cast<uint64_t>(g.ldc) * 4, 32, 32))
        return cudaErrorInvalidValue;
    if (L.b_mode == kBTmaMN) {
        if (!encode_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.B, g.N, g.K,
                       static_cast<uint64_t>(g.ldb) * 2, 64, kKBlock))
            return cudaErrorInvalidValue;
    } else if (L.b_mode == kBTmaK) {
        if (!encode_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.B, g.K, g.N,
                       static_cast<uint64_t>(g.ldb) * 2, kKBlock, static_cast<uint32_t>(L.n_mma)))
            return cudaErrorInvalidValue;
    } else {
        tmB = tmA;   // unused
    }

    TcParams p;
    p.M = g.M; p.N = g.N; p.K = g.K;
    p.n_mma = L.n_mma; p.num_kb = L.num_kb; p.kpad = L.kpad; p.n_chunks = L.n_chunks;
    p.num_tiles = (g.M + BM - 1) / BM;
    p.stages = L.stages; p.b_mode = L.b_mode; p.sb_bytes = L.sb_bytes;
    p.kbs = L.kbs; p.groups = (L.num_kb + L.kbs - 1) / L.kbs;
    p.alpha = g.alpha; p.beta = g.beta;
    p.B = static_cast<const uint16_t*>(g.B); p.ldb = g.ldb; p.b_trans = g.b_trans;
    p.C = static_cast<const float*>(g.C); p.ldc = g.ldc;
    p.tmem_cols = L.tmem_cols;
    p.err = err;

    // The attribute is per device; set it once so that launches under stream
    // capture make no further attribute calls.
    static thread_local int smem_set_dev = -1;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != smem_set_dev) {
        e = cudaFuncSetAttribute(gemm_bf16_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemLimit));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_bf16_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmemLimit));
        if (e != cudaSuccess) return e;
        smem_set_dev = dev;
    }
    const int slots = num_sms * L.ctas_per_sm;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.num_tiles < slots ? p.num_tiles : slots));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return L.b_mode == kBTmaMN ? cudaLaunchKernelEx(&cfg, gemm_bf16_tc_kernel<true>, tmA, tmB, tmC, p)
                               : cudaLaunchKernelEx(&cfg, gemm_bf16_tc_kernel<false>, tmA, tmB, tmC, p);
}

}  // namespace dnnopt_b200
