// General GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), both
// operands streamed by TMA, for the shapes the GEMV kernels and the
// tall-skinny BF16 kernel do not take:
//   * INT8 x INT8 -> INT32 (gemm_int8_int8int8int32, reference
//     src/gemm/gemm_int8_native.cpp:37-181, the 8x8 SMMLA tile) and the
//     FP32-API gemm_int8 after quantisation (dequantising epilogue,
//     src/gemm/gemm_driver_generic.cpp:49-67) for M > 8: tcgen05.mma.kind::i8,
//     int32 accumulators (exact, so bit-identical to the reference's sums);
//   * BF16 x BF16 -> FP32 (gemm_bf16_bf16bf16f32, reference
//     src/gemm/gemm_driver_bf16.cpp:134-218) for M > 8 and N > 256:
//     tcgen05.mma.kind::f16, FP32 accumulators, the reference epilogue
//     beta == 0 ? alpha*acc : fma(alpha, acc, beta*C).
//
// Layout: A [M, K] K-major (lda); B either [N, K] K-major (INT8 always, BF16
// with trans_b) or [K, N] MN-major (BF16 without trans_b).  Every K-block is
// 128 bytes of K (64 bf16 or 128 int8), staged by TMA with the 128-byte
// swizzle straight into the UMMA operand layout; four MMAs of 32 bytes of K
// consume it (K = 16 bf16 or K = 32 int8 per instruction).
//
// Work units are (split, m-tile, n-tile) with 128-row m-tiles and n-tiles of
// n_mma <= 256 columns; persistent CTAs (one per SM, a 192 KB ring of stages
// of up to 64 KB: one K-block at n_mma = 256, several for narrower tiles or
// small M, whose A blocks hold only M rows) walk the units.  Roles: warp 0 issues TMA loads, warp 1 owns TMEM and
// issues the MMAs into one of two accumulators (so the epilogue of a unit
// overlaps the MMAs of the next), warps 2-5 drain TMEM with tcgen05.ld (warp
// q owns TMEM lanes / tile rows 32(q%4) ...) and write C directly.  With a
// K split (units of one tile in different CTAs) the epilogue writes its
// partial tile to the workspace; the last CTA of the tile (atomic ticket)
// sums the splits in split order and writes C.
//
// Every TMA load targets this CTA's own shared memory.  Every mbarrier wait is
// bounded (kMbarTimeoutNs); a timeout records an error word and makes the
// other roles give up.
#include <cuda.h>

#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int BM = 128;
constexpr int kKBytes = 128;                       // bytes of K per K-block
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kRingBytes = 4 * (128 * 128 + 256 * 128);   // 192 KB of stages
constexpr int kMaxN = 256;
constexpr int kMaxSplits = 4;                      // K splits reduced through the global workspace
constexpr int kMaxClusterSplits = 8;               // K splits reduced inside a cluster (portable size)
constexpr int kRedItems = 4;                       // column quads per thread per reduction round
constexpr int kCStageBytes = 32 * 128;                // one 32 x 32 4-byte store block
constexpr int kCStaging = 4 * 2 * kCStageBytes;       // 4 epilogue warps x 2 buffers
constexpr size_t kSmem = 1024 + static_cast<size_t>(kRingBytes) + kCStaging + 256;

enum TcOp : int {
    kOpBf16K = 0,    // bf16, B [N, K] K-major
    kOpBf16MN = 1,   // bf16, B [K, N] MN-major
    kOpI8 = 2,       // int8, B [N, K] K-major
};
enum TcEpi : int {
    kEpiF32 = 0,     // C fp32 = beta == 0 ? alpha*acc : fma(alpha, acc, beta*C)
    kEpiS32 = 1,     // C int32 = acc
    kEpiS8DQ = 2,    // C fp32 = (beta*C) + (alpha*sA*sB) * float(acc)
};

struct TcGemmParams {
    int M, N, K;
    int n_mma, num_kb, kb_per_split, splits;
    int kbs;               // 128-byte K-blocks per ring stage (stages of up to 64 KB)
    int stages;            // ring depth: kRingBytes / stage bytes, at most kMaxStages
    int a_rows;            // A rows loaded per K-block: 128, or M rounded up to 8 when M < 128
    uint32_t a_bytes, sub_bytes;   // a_rows * 128; one K-block of A and B
    int m_tiles, n_tiles, units;
    int op, epi;
    float alpha, beta;
    void* C;
    int64_t ldc;
    const float* scales;   // {sA, sB} for kEpiS8DQ
    int c_vec;             // 1: C 16-byte aligned with ldc % 4 == 0 (vector epilogue)
    int c_tma;             // 1: unsplit tiles with beta == 0 go out by TMA stores (tmC)
    int cluster;           // 1: the splits of a tile are one thread-block cluster (one unit per CTA)
    void* ws;              // [tiles][splits][BM][n_mma] partials (splits > 1, not cluster)
    uint32_t* tickets;     // one per tile, zero on entry, left zero
    uint32_t* err;
};

__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor (tcgen05 .kind::f16 / .kind::i8): D format bits
// 4-5 (1 = F32, 2 = S32), A / B format bits 7-9 / 10-12 (BF16 = 1, signed
// 8-bit = 1), B major bit 16 (1 = MN-major), N >> 3 at 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t tc_idesc(int op, int m, int n) {
    const uint32_t dfmt = op == kOpI8 ? 2u : 1u;
    return (dfmt << 4) | (1u << 7) | (1u << 10) | ((op == kOpBf16MN ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// MN-major operand in the 128-byte swizzled layout: 64 bf16 along N per
// 128-byte row, 8 K rows per 1024-byte atom, 64-column chunks `lbo` bytes apart.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

__device__ __forceinline__ void st_dsmem_v4(uint32_t cluster_addr, uint4 v) {
    asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// Epilogue of four consecutive outputs (row, col .. col+3) from raw
// accumulator words: int32 as is, FP32 with alpha / beta, or the int8
// dequantisation float(acc) * (alpha * sA * sB) (+ beta * C) with the
// reference's rounding order.  16-byte accesses when C allows and the four
// columns are inside N.
__device__ __forceinline__ void store4(const TcGemmParams& p, int row, int col, const uint32_t* w) {
    const int64_t off = static_cast<int64_t>(row) * p.ldc + col;
    const bool vec = p.c_vec && col + 3 < p.N;
    if (p.epi == kEpiS32) {
        int32_t* cp = static_cast<int32_t*>(p.C) + off;
        if (vec) {
            *reinterpret_cast<int4*>(cp) = make_int4(static_cast<int>(w[0]), static_cast<int>(w[1]),
                                                     static_cast<int>(w[2]), static_cast<int>(w[3]));
        } else {
            for (int j = 0; j < 4 && col + j < p.N; ++j) cp[j] = static_cast<int32_t>(w[j]);
        }
        return;
    }
    float* cp = static_cast<float*>(p.C) + off;
    float old[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (p.beta != 0.0f) {
        if (vec) {
            const float4 t = *reinterpret_cast<const float4*>(cp);
            old[0] = t.x; old[1] = t.y; old[2] = t.z; old[3] = t.w;
        } else {
            for (int j = 0; j < 4 && col + j < p.N; ++j) old[j] = cp[j];
        }
    }
    float v[4];
    if (p.epi == kEpiF32) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float acc = __uint_as_float(w[j]);
            v[j] = (p.beta == 0.0f) ? p.alpha * acc : fmaf(p.alpha, acc, p.beta * old[j]);
        }
    } else {
        const float scale = __fmul_rn(p.alpha, __fmul_rn(p.scales[0], p.scales[1]));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float c_0 = (p.beta == 0.0f) ? 0.0f : __fmul_rn(p.beta, old[j]);
            v[j] = __fadd_rn(c_0, __fmul_rn(scale, static_cast<float>(static_cast<int32_t>(w[j]))));
        }
    }
    if (vec) {
        *reinterpret_cast<float4*>(cp) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        for (int j = 0; j < 4 && col + j < p.N; ++j) cp[j] = v[j];
    }
}

// OP is a template parameter: a run-time branch between MMA forms in the
// issue loop measured twice the issue time per MMA on B200.
template <int OP>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const TcGemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* stages = base;
    const int kStages = p.stages;
    // Stage = kbs x [A K-block (a_rows rows)][B K-block].  With a_rows < 128
    // the MMA's M = 128 rows read past the loaded A rows into neighbouring
    // shared memory: those accumulator rows are >= M and never stored.
    const uint32_t kSubBytes = p.sub_bytes;
    const uint32_t kStageBytes = static_cast<uint32_t>(p.kbs) * kSubBytes;
    uint8_t* sC = base + kRingBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kRingBytes + kCStaging);
    uint64_t* empty = full + kMaxStages;
    uint64_t* tfull = empty + kMaxStages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    volatile uint32_t* last_flag = tmem_slot + 2;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tmem_cols = static_cast<uint32_t>(2 * p.n_mma) <= 32 ? 32u
                             : (static_cast<uint32_t>(2 * p.n_mma) <= 64 ? 64u
                             : (static_cast<uint32_t>(2 * p.n_mma) <= 128 ? 128u
                             : (static_cast<uint32_t>(2 * p.n_mma) <= 256 ? 256u : 512u)));

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
        *abort_flag = 0u;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (p.c_tma) prefetch_tmap(&tmC);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();

    // Unit u -> (split, m-tile, n-tile); the splits of a tile are adjacent
    // unit indices so that they run at the same time.
    auto unit_coords = [&](int u, int& split, int& mt, int& nt) {
        split = u % p.splits;
        const int t = u / p.splits;
        mt = t % p.m_tiles;
        nt = t / p.m_tiles;
    };
    auto unit_kbs = [&](int split, int& kb0, int& nkb) {
        kb0 = split * p.kb_per_split;
        nkb = min(p.kb_per_split, p.num_kb - kb0);
    };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t it = 0;
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
                int split, mt, nt, kb0, nkb;
                unit_coords(u, split, mt, nt);
                unit_kbs(split, kb0, nkb);
                for (int kb = kb0; kb < kb0 + nkb; kb += p.kbs, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err)) break;
                    const int nsub = min(p.kbs, kb0 + nkb - kb);
                    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nsub) * kSubBytes);
                    for (int sub = 0; sub < nsub; ++sub) {
                        uint8_t* sa = stages + s * kStageBytes + sub * kSubBytes;
                        uint8_t* sb = sa + p.a_bytes;
                        const int kx = OP == kOpI8 ? (kb + sub) * kKBytes : (kb + sub) * (kKBytes / 2);   // elements
                        tma_load_2d(sa, &tmA, &full[s], kx, mt * BM);
                        if constexpr (OP == kOpBf16MN) {
                            // 64-column chunks of 64 K rows: chunk j at j * 8 KB.
                            for (int j = 0; j < p.n_mma / 64; ++j)
                                tma_load_2d(sb + j * 8192, &tmB, &full[s], nt * p.n_mma + j * 64, kx);
                        } else {
                            tma_load_2d(sb, &tmB, &full[s], kx, nt * p.n_mma);
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // One instruction form per operand kind, hoisted out of the K loop:
        // 32 bytes of K per MMA, +32 B along a K-major 128-byte row, or two
        // 1024-B atoms (16 K rows) down an MN-major chunk.
        if (lane == 0) {
            const uint32_t idesc = tc_idesc(OP, BM, p.n_mma);
            uint32_t it = 0, titer = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++titer) {
                int split, mt, nt, kb0, nkb;
                unit_coords(u, split, mt, nt);
                unit_kbs(split, kb0, nkb);
                const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
                if (!mbar_wait(&tempty[buf], tph ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * static_cast<uint32_t>(p.n_mma);
                for (int kb = 0; kb < nkb; kb += p.kbs, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!mbar_wait(&full[s], ph, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const int nsub = min(p.kbs, nkb - kb);
                    for (int sub = 0; sub < nsub; ++sub) {
                        const uint32_t a_addr = smem_u32(stages + s * kStageBytes + sub * kSubBytes);
                        const uint32_t b_addr = a_addr + p.a_bytes;
                        const int kl = kb + sub;
                        if constexpr (OP == kOpI8) {
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                umma_i8_ss(d_tmem, umma_desc_k_sw128(a_addr + kk * 32),
                                           umma_desc_k_sw128(b_addr + kk * 32), idesc, (kl | kk) != 0);
                        } else if constexpr (OP == kOpBf16MN) {
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                umma_f16_ss(d_tmem, umma_desc_k_sw128(a_addr + kk * 32),
                                            desc_mn_sw128(b_addr + kk * 2048, 8192), idesc, (kl | kk) != 0);
                        } else {
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                umma_f16_ss(d_tmem, umma_desc_k_sw128(a_addr + kk * 32),
                                            umma_desc_k_sw128(b_addr + kk * 32), idesc, (kl | kk) != 0);
                        }
                    }
                    umma_commit(&empty[s]);   // stage free once these MMAs retire
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);     // accumulator ready for the epilogue
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;           // TMEM lanes 32q .. 32q+31 (warp id mod 4)
        const int ep_tid = tid - 64;      // 0..127
        uint32_t titer = 0, cgrp = 0;
        if (p.cluster) {
            // Cluster split-K: this CTA's one unit is done once its
            // accumulator is complete; the rows leave TMEM after the cluster
            // barrier below.
            if (!mbar_wait_warp(&tfull[0], 0u, abort_flag, p.err) && lane == 0) *abort_flag = 1u;
        }
        for (int u = blockIdx.x; !p.cluster && u < p.units && !*abort_flag; u += gridDim.x, ++titer) {
            int split, mt, nt;
            unit_coords(u, split, mt, nt);
            const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
            const bool ok = mbar_wait_warp(&tfull[buf], tph, abort_flag, p.err);
            tc_fence_after();
            const int row_in = q * 32 + lane;
            const int row = mt * BM + row_in;
            const int col0 = nt * p.n_mma;
            const int tile = mt + nt * p.m_tiles;
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * static_cast<uint32_t>(p.n_mma);
            const bool partial = p.splits > 1;
            // Drain the accumulator 32 columns at a time: to C, or (split-K) to
            // this split's partial tile in the workspace.
            uint32_t* wrow = partial ? static_cast<uint32_t*>(p.ws) +
                                           ((static_cast<int64_t>(tile) * p.splits + split) * BM + row_in) * p.n_mma
                                     : nullptr;
            for (int c0 = 0; c0 < p.n_mma; c0 += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x16(t_addr + c0, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
                tmem_ld_32x32b_x16(t_addr + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
                tmem_ld_wait();
                if (!ok) continue;
                if (partial) {
                    if (row >= p.M) continue;   // rows past M are never summed
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        __stcg(reinterpret_cast<uint4*>(wrow + c0 + j), make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]));
                } else if (p.c_tma) {
                    // beta == 0: the 32 x 32 block (rows 32q.., columns c0..)
                    // through 128-byte-swizzled shared memory and one TMA store
                    // (rows >= M, columns >= N clipped by the tensor map).
                    if (col0 + c0 >= p.N) continue;
                    uint8_t* sbuf = sC + (q * 2 + (cgrp & 1u)) * kCStageBytes;
                    if (lane == 0) tma_store_wait_read<1>();   // this buffer's previous store has read it
                    __syncwarp();
                    const float dq = p.epi == kEpiS8DQ ? __fmul_rn(p.alpha, __fmul_rn(p.scales[0], p.scales[1])) : 0.0f;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        uint32_t w[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint32_t raw = r[c * 4 + j];
                            w[j] = p.epi == kEpiS32 ? raw
                                 : (p.epi == kEpiF32 ? __float_as_uint(p.alpha * __uint_as_float(raw))
                                                     : __float_as_uint(__fadd_rn(0.0f, __fmul_rn(dq, static_cast<float>(static_cast<int32_t>(raw))))));
                        }
                        *reinterpret_cast<uint4*>(sbuf + lane * 128 + ((c ^ (lane & 7)) * 16)) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, sbuf, col0 + c0, mt * BM + q * 32);
                        tma_store_commit();
                    }
                    ++cgrp;
                } else if (row < p.M) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const int col = col0 + c0 + j;
                        if (col >= p.N) break;
                        store4(p, row, col, &r[j]);
                    }
                }
            }
            // Accumulator drained: the next unit's MMAs may reuse it.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            if (!partial || !ok) continue;
            // Split-K: publish, then the last split of the tile sums all splits
            // in split order (int32: exact; FP32: a fixed order).
            __threadfence();
            named_barrier_sync(1, 128);
            if (ep_tid == 0) {
                const uint32_t t = atomicAdd(&p.tickets[tile], 1u);
                *last_flag = t == static_cast<uint32_t>(p.splits - 1) ? 1u : 0u;
            }
            named_barrier_sync(1, 128);
            const bool last = *last_flag != 0u;
            named_barrier_sync(1, 128);   // everyone has read last_flag before the next unit rewrites it
            if (!last) continue;
            __threadfence();
            {
                // The tile's valid rows x n_mma/4 column quads, row-major over
                // the 128 epilogue threads (coalesced 16-byte loads),
                // kRedItems quads per thread per round with every split's load
                // in flight.
                const uint32_t* tbase = static_cast<const uint32_t*>(p.ws) +
                                        static_cast<int64_t>(tile) * p.splits * BM * p.n_mma;
                const int64_t sstride = static_cast<int64_t>(BM) * p.n_mma;
                const int mrows = min(BM, p.M - mt * BM);
                const int quads = p.n_mma / 4;
                const int items = mrows * quads;
                for (int i0 = ep_tid; i0 < items; i0 += kRedItems * 128) {
                    uint4 v[kRedItems][kMaxSplits];
#pragma unroll
                    for (int h = 0; h < kRedItems; ++h) {
                        const int item = i0 + h * 128;
#pragma unroll
                        for (int sp = 0; sp < kMaxSplits; ++sp)
                            if (item < items && sp < p.splits)
                                v[h][sp] = __ldcg(reinterpret_cast<const uint4*>(
                                    tbase + sp * sstride + (item / quads) * p.n_mma + (item % quads) * 4));
                    }
#pragma unroll
                    for (int h = 0; h < kRedItems; ++h) {
                        const int item = i0 + h * 128;
                        if (item >= items) break;
                        const int r_in = item / quads, c4 = (item % quads) * 4;
                        if (col0 + c4 >= p.N) continue;
                        int32_t si[4] = {0, 0, 0, 0};
                        float sf[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                        for (int sp = 0; sp < kMaxSplits; ++sp) {
                            if (sp >= p.splits) break;
                            const uint32_t w4[4] = {v[h][sp].x, v[h][sp].y, v[h][sp].z, v[h][sp].w};
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                si[j] += static_cast<int32_t>(w4[j]);
                                sf[j] += __uint_as_float(w4[j]);
                            }
                        }
                        uint32_t w[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            w[j] = p.epi == kEpiF32 ? __float_as_uint(sf[j]) : static_cast<uint32_t>(si[j]);
                        store4(p, mt * BM + r_in, col0 + c4, w);
                    }
                }
            }
            if (ep_tid == 0) p.tickets[tile] = 0u;   // ready for the next launch on this stream
        }
        if (p.c_tma && lane == 0) tma_store_wait_all<0>();   // staging must outlive the stores' reads
    }

    tc_fence_before();
    __syncthreads();
    if (p.cluster) {
        // Barrier A: every CTA of the cluster has its accumulator complete, so
        // every ring is idle.  Each split then pushes its partial rows from
        // TMEM into the owning CTA's ring with remote (fire-and-forget)
        // stores: CTA `rank` owns tile rows [rank*per, (rank+1)*per), laid
        // out [split][row][n_mma + 4] (16-byte chunks of consecutive rows in
        // different banks).  Barrier B makes them visible; the owner sums its
        // rows over the splits in split order (int32: exact; FP32: a fixed
        // order) from its own shared memory and applies the epilogue.
        cluster_sync_all();
        int split, mt, nt;
        unit_coords(static_cast<int>(blockIdx.x), split, mt, nt);
        const int mrows = min(BM, p.M - mt * BM);
        const int per = (mrows + p.splits - 1) / p.splits;
        const int pstride = p.n_mma + 4;
        const uint32_t part0 = smem_u32(stages);
        if (warp >= 2) {
            tc_fence_after();
            const int q = warp & 3;
            const int row_in = q * 32 + lane;
            const int owner = row_in < mrows ? row_in / per : 0;
            const uint32_t dst = map_to_cta(
                part0 + static_cast<uint32_t>(((split * per) + (row_in - owner * per)) * pstride) * 4u,
                static_cast<uint32_t>(owner));
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
            for (int c0 = 0; c0 < p.n_mma; c0 += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x16(t_addr + c0, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
                tmem_ld_32x32b_x16(t_addr + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
                tmem_ld_wait();
                if (row_in >= mrows) continue;
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    st_dsmem_v4(dst + static_cast<uint32_t>(c0 + j) * 4u, make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]));
            }
        }
        cluster_sync_all();
        const uint32_t rank = cluster_ctarank();
        const int r0 = static_cast<int>(rank) * per;
        const int r1 = min(mrows, r0 + per);
        const int quads = p.n_mma / 4;
        const int col0 = nt * p.n_mma;
        const int items = r0 < r1 ? (r1 - r0) * quads : 0;
        const uint32_t* part = reinterpret_cast<const uint32_t*>(stages);
        for (int item = tid; item < items; item += kThreads) {
            const int lr = item / quads, c4 = (item % quads) * 4;
            if (col0 + c4 >= p.N) continue;
            int32_t si[4] = {0, 0, 0, 0};
            float sf[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int k = 0; k < p.splits; ++k) {
                const uint4 v = *reinterpret_cast<const uint4*>(part + ((k * per) + lr) * pstride + c4);
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    si[j] += static_cast<int32_t>(w4[j]);
                    sf[j] += __uint_as_float(w4[j]);
                }
            }
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                w[j] = p.epi == kEpiF32 ? __float_as_uint(sf[j]) : static_cast<uint32_t>(si[j]);
            if (!*abort_flag) store4(p, mt * BM + r0 + lr, col0 + c4, w);
        }
    }
    pdl_launch_dependents();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, tmem_cols);
    }
}

// ---- host helpers ----------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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

bool encode(CUtensorMap* m, CUtensorMapDataType t, const void* ptr, uint64_t d0, uint64_t d1, uint64_t row_bytes,
            uint32_t b0, uint32_t b1) {
    cuuint64_t dims[2] = {d0, d1};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {b0, b1};
    cuuint32_t estr[2] = {1, 1};
    return encode_fn()(m, t, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

bool gemm_tc_supported(TcKind kind, const GemmArgs& g) {
    if (g.M < 1 || g.N < 1 || g.K < 1 || g.a_trans || !encode_fn()) return false;
    const size_t eb = kind == TcKind::BF16 ? 2 : 1;
    if (!aligned16(g.A) || (static_cast<size_t>(g.lda) * eb) % 16 != 0) return false;
    if (!aligned16(g.B) || (static_cast<size_t>(g.ldb) * eb) % 16 != 0) return false;
    if (kind != TcKind::BF16 && !g.b_trans) return false;   // int8 B is always [N, K]
    if (kind == TcKind::BF16 && !g.b_trans && g.N < 64) return false;
    return !g.bias;
}

// Tile width, K split and grid for a shape: n_mma up to 256 (a multiple of 64
// for MN-major B, else of 32: the epilogue drains 32 columns at a time); the K extent split so that units ~ SMs when the
// output tiles alone leave most SMs idle, at least 4 K-blocks per split.
TcPlan gemm_tc_plan(TcKind kind, const GemmArgs& g, int num_sms) {
    TcPlan pl{};
    const bool mn = kind == TcKind::BF16 && !g.b_trans;
    int n = g.N < kMaxN ? g.N : kMaxN;
    n = mn ? (n + 63) / 64 * 64 : (n + 31) / 32 * 32;
    const int m_tiles = (g.M + BM - 1) / BM;
    // Narrower tiles before a K split: a split tile's last CTA sums every
    // split's partial tile alone, so more tiles (B columns read by more CTAs,
    // A re-read from L2) cost less than deep splits.
    // Narrow no further than 128 columns: every MMA instruction and every ring
    // stage has a roughly fixed cost (measured on B200), so a K split keeps
    // more work per MMA than a narrower tile does.
    while (n > 128 && m_tiles * ((g.N + n - 1) / n) * 2 <= num_sms) n /= 2;
    pl.n_mma = n;
    const int n_tiles = (g.N + n - 1) / n;
    const int elems = kind == TcKind::BF16 ? kKBytes / 2 : kKBytes;
    const int num_kb = (g.K + elems - 1) / elems;
    const int tiles = m_tiles * n_tiles;
    // Splits double while every unit still gets its own CTA, so a split tile
    // is reduced inside its thread-block cluster (up to 8 CTAs).
    int splits = 1;
    while (tiles * splits * 2 <= num_sms && num_kb / (splits * 2) >= 4 && splits < kMaxClusterSplits) splits *= 2;
    pl.kb_per_split = (num_kb + splits - 1) / splits;
    pl.splits = (num_kb + pl.kb_per_split - 1) / pl.kb_per_split;
    return pl;
}

size_t gemm_tc_ws_bytes(const GemmArgs& g, const TcPlan& pl) {
    if (pl.splits <= 1) return 0;
    const int m_tiles = (g.M + BM - 1) / BM, n_tiles = (g.N + pl.n_mma - 1) / pl.n_mma;
    return static_cast<size_t>(m_tiles) * n_tiles * pl.splits * BM * pl.n_mma * 4;
}

int gemm_tc_tickets(const GemmArgs& g, const TcPlan& pl) {
    return ((g.M + BM - 1) / BM) * ((g.N + pl.n_mma - 1) / pl.n_mma);
}

cudaError_t launch_gemm_tc(TcKind kind, DotKind epi, const GemmArgs& g, const TcPlan& pl, const float* scales,
                           void* ws, uint32_t* tickets, uint32_t* err, int num_sms, cudaStream_t s) {
    if (!gemm_tc_supported(kind, g) || pl.n_mma < 16 || pl.n_mma > kMaxN) return cudaErrorInvalidValue;
    const int units = ((g.M + BM - 1) / BM) * ((g.N + pl.n_mma - 1) / pl.n_mma) * pl.splits;
    // Split tiles are reduced inside a cluster when every unit has its own CTA,
    // else through the workspace by a ticketed last CTA.
    const bool cluster = pl.splits > 1 && units <= num_sms && pl.splits <= kMaxClusterSplits;
    if (!cluster && (pl.splits > kMaxSplits || (pl.splits > 1 && (!ws || !tickets)))) return cudaErrorInvalidValue;
    const bool mn = kind == TcKind::BF16 && !g.b_trans;
    const int op = kind == TcKind::BF16 ? (mn ? kOpBf16MN : kOpBf16K) : kOpI8;
    CUtensorMap tmA, tmB;
    // A rows per K-block: the whole 128-row tile, or only M (rounded up to 8)
    // when M < 128, so a small-M GEMM loads no zero rows.
    const int a_rows = g.M >= BM ? BM : (g.M + 7) / 8 * 8;
    if (kind == TcKind::BF16) {
        if (!encode(&tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.A, g.K, g.M, static_cast<uint64_t>(g.lda) * 2, 64,
                    static_cast<uint32_t>(a_rows)))
            return cudaErrorInvalidValue;
        if (mn) {
            if (!encode(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.B, g.N, g.K, static_cast<uint64_t>(g.ldb) * 2, 64, 64))
                return cudaErrorInvalidValue;
        } else if (!encode(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.B, g.K, g.N, static_cast<uint64_t>(g.ldb) * 2, 64,
                           static_cast<uint32_t>(pl.n_mma))) {
            return cudaErrorInvalidValue;
        }
    } else {
        if (!encode(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.A, g.K, g.M, static_cast<uint64_t>(g.lda), 128,
                    static_cast<uint32_t>(a_rows)) ||
            !encode(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.B, g.K, g.N, static_cast<uint64_t>(g.ldb), 128,
                    static_cast<uint32_t>(pl.n_mma)))
            return cudaErrorInvalidValue;
    }
    // Unsplit tiles with beta == 0 store C by TMA when C's rows are 16-byte
    // strided and aligned.
    CUtensorMap tmC = tmA;
    const bool c_tma = pl.splits == 1 && g.beta == 0.0f && aligned16(g.C) && (g.ldc * 4) % 16 == 0 &&
                       encode(&tmC, epi == DotKind::S8S32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                              g.C, g.N, g.M, static_cast<uint64_t>(g.ldc) * 4, 32, 32);
    if (!c_tma) tmC = tmA;   // unused
    TcGemmParams p;
    p.c_tma = c_tma ? 1 : 0;
    p.M = g.M; p.N = g.N; p.K = g.K;
    p.n_mma = pl.n_mma;
    const int elems = kind == TcKind::BF16 ? kKBytes / 2 : kKBytes;
    p.num_kb = (g.K + elems - 1) / elems;
    p.kb_per_split = pl.kb_per_split;
    p.splits = pl.splits;
    p.m_tiles = (g.M + BM - 1) / BM;
    p.n_tiles = (g.N + pl.n_mma - 1) / pl.n_mma;
    p.units = p.m_tiles * p.n_tiles * p.splits;
    p.op = op;
    p.epi = epi == DotKind::S8S32 ? kEpiS32 : (epi == DotKind::S8DQ ? kEpiS8DQ : kEpiF32);
    p.alpha = g.alpha; p.beta = g.beta;
    p.C = g.C; p.ldc = g.ldc;
    // Up to 64 KB per ring stage: a stage's cost (barrier round trips, commit)
    // is roughly fixed, so small K-blocks travel several to a stage.
    p.a_rows = a_rows;
    p.a_bytes = static_cast<uint32_t>(a_rows) * kKBytes;
    p.sub_bytes = p.a_bytes + static_cast<uint32_t>(pl.n_mma) * kKBytes;
    p.kbs = 4 * p.sub_bytes <= 65536u ? 4 : (2 * p.sub_bytes <= 65536u ? 2 : 1);
    p.stages = kRingBytes / (p.kbs * static_cast<int>(p.sub_bytes));
    if (p.stages > kMaxStages) p.stages = kMaxStages;
    p.scales = scales;
    p.c_vec = aligned16(g.C) && g.ldc % 4 == 0 ? 1 : 0;
    p.cluster = cluster ? 1 : 0;
    p.ws = ws;
    p.tickets = tickets;
    p.err = err;

    static std::mutex mu;
    static std::set<int> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!done.count(dev)) {
            e = cudaFuncSetAttribute(gemm_tc_kernel<kOpBf16K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmem));
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(gemm_tc_kernel<kOpBf16MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmem));
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(gemm_tc_kernel<kOpI8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmem));
            if (e != cudaSuccess) return e;
            done.insert(dev);
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.units < num_sms ? p.units : num_sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cluster) {
        cfg.gridDim = dim3(static_cast<unsigned>(p.units));
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = static_cast<unsigned>(pl.splits);
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    if (op == kOpI8) return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<kOpI8>, tmA, tmB, tmC, p);
    if (op == kOpBf16MN) return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<kOpBf16MN>, tmA, tmB, tmC, p);
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<kOpBf16K>, tmA, tmB, tmC, p);
}

}  // namespace dnnopt_b200
