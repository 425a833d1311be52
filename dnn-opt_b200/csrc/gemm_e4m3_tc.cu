// Decode-FFN weight GEMM on the tensor cores:
//   C[m, n] = bf16_rne( scale[n] * sum_k A[m, k] * W[n, k] ),   M <= 8,
// A bf16 [M, K], W OCP-E4M3FN [N, K] (K contiguous), scale FP32 [N], C bf16.
// The reference has no implementation (its FP8 path, src/gemm/gemm_fp8.cpp:51-83,
// dequantises to FP32 and calls the scalar GEMM); this is the B200 design.
//
// The weights are the HBM stream (235 MB at the config's shape), so they go
// TMA -> shared memory -> tcgen05.mma.kind::f8f6f4 untouched: 128 weight rows
// are the UMMA M dimension, the activations the N dimension.  A small prep
// kernel first splits the bf16 activations into two e4m3 operands,
// hi = e4m3(a*s) and lo = e4m3(a*s - hi), with s a power of two per row
// (max |a*s| in [128, 256)).  a*s carries bf16's 8 significant bits, hi the
// top 4 and lo the rest, so hi + lo reproduces a*s exactly while the
// residual's last bit is at least e4m3's subnormal step 2^-9, i.e. for
// |a*s| >= 2^-2, values down to 2^9-2^10 below the row maximum; smaller values
// are off by at most 2^-10, about 2^-17-2^-18 of the row maximum, well inside
// the bf16 output rounding.  UMMA N = 16 holds the 8 hi rows and 8 lo rows (one
// 2 KB TMA box per K-block, loaded with the weight box), so
// D[:, m] + D[:, 8+m] is the full-precision product sum, undone by 1/s.
//
// K is split into S ranges (S chosen for an even wave count over the SMs);
// S > 1 partial [8 x 128] strips reduce through the workspace by the last CTA
// of each tile (atomic ticket), in split order, so the result is deterministic.
// Roles: warp 0 TMA producer, warp 1 MMA issuer + TMEM owner, warps 2-5 drain
// TMEM (tcgen05.ld) and write C.
//
// Fused all-gather (N-sharded over ranks, one process per GPU): the epilogue
// stores each finished column into every rank's output buffer (peer memory
// mapped through CUDA IPC, plain stores over NVLink), and the last tile of
// the grid raises this rank's flag on every rank (release, system scope); a
// one-CTA wait kernel then blocks the stream until every rank's flag has
// arrived (bounded wait) and advances the device-side call counter.  The
// transfer of a tile overlaps the MMAs of the tiles still running.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int BM = 128;                 // weight rows per tile (UMMA M)
constexpr int KB = 128;                 // e4m3 elements per K-block (128-byte swizzle row)
constexpr int kWStage = BM * KB;        // 16 KB of weights per K-block
constexpr int kActBlock = 16 * KB;      // 16 activation rows x 128 B per K-block
constexpr int kStage = kWStage + kActBlock;
constexpr int kThreads = 192;
constexpr int kMaxKc = 4096;            // K elements per CTA (activation operand 64 KB)
constexpr size_t kSmemLimit = 227 * 1024;
constexpr int kMaxPeers = kAllGatherMaxRanks;

struct E4Params {
    int M, N, K;
    int kc, splits, stages;
    const float* inv_sigma;   // [8] from the prep kernel
    const float* scale;
    int64_t ldc;
    float* ws;
    uint32_t* tickets;
    uint32_t* err;
    // Outputs: nout copies of C (nout == 1: local C; nout == world: every
    // rank's output buffer, this rank's column block already applied).
    int nout;
    uint16_t* out[kMaxPeers];
    // All-gather (done != nullptr): the call number is *seq + 1; output copy
    // o goes to out[o] + (call & 1) * out_stride; `done` counts finished tiles
    // on this GPU and the last tile raises flag[q][rank] = call on every rank q.
    int64_t out_stride;
    const uint32_t* seq;
    uint32_t* done;
    uint32_t* flag[kMaxPeers];
    int rank;
};

// Instruction descriptor, kind::f8f6f4: A = B = E4M3 (format 0), D = F32,
// both K-major, M = 128, N = 16.
constexpr uint32_t kIdescE4M3 = (1u << 4) | (0u << 7) | (0u << 10) | ((16u >> 3) << 17) |
                                ((128u >> 4) << 24);

__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Two floats -> two OCP e4m3 bytes (RNE, saturate): x0 in the low byte.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float x0, float x1) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    return r;
}

__device__ __forceinline__ float e4m3_byte_to_f32(uint32_t b) {
    return e4m3x2_to_f32x2(static_cast<uint16_t>(b & 0xFFu)).x;
}

// Activation operand: one CTA per activation row m (8 rows; rows >= M are
// zero).  act is [16][kpad] e4m3 (row m = hi, row 8+m = lo), K-tail zero.
// Each thread owns 16-byte chunks (8 bf16) c = tid + 256 i of its row: with
// 16-byte aligned rows and K <= 16384 every chunk is loaded once, all loads
// in flight together, and kept in registers for both the row maximum and the
// split (one memory round trip); otherwise elements are read one at a time,
// twice.  Either way the scale and the conversions are the same.
constexpr int kPrepChunks = 8;   // chunks per thread held in registers (K <= 256 * 8 * 8)

__device__ __forceinline__ void act_split8(const float (&x)[8], float sigma, uint2& hi, uint2& lo) {
    float v[8], r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = x[j] * sigma;
    hi.x = f32x2_to_e4m3x2(v[0], v[1]) | (f32x2_to_e4m3x2(v[2], v[3]) << 16);
    hi.y = f32x2_to_e4m3x2(v[4], v[5]) | (f32x2_to_e4m3x2(v[6], v[7]) << 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        r[j] = v[j] - e4m3_byte_to_f32(hi.x >> (8 * j));
        r[4 + j] = v[4 + j] - e4m3_byte_to_f32(hi.y >> (8 * j));
    }
    lo.x = f32x2_to_e4m3x2(r[0], r[1]) | (f32x2_to_e4m3x2(r[2], r[3]) << 16);
    lo.y = f32x2_to_e4m3x2(r[4], r[5]) | (f32x2_to_e4m3x2(r[6], r[7]) << 16);
}

__global__ void __launch_bounds__(256)
e4m3_act_prep_kernel(const uint16_t* __restrict__ A, int64_t lda, int M, int K, int kpad,
                     uint8_t* __restrict__ act, float* __restrict__ inv_sigma) {
    __shared__ float wmax[8];
    pdl_wait();
    pdl_launch_dependents();
    const int m = blockIdx.x, tid = threadIdx.x;
    const bool live = m < M;
    const uint16_t* arow = A + (int64_t)m * lda;
    const int nch = kpad / 8;   // kpad is a multiple of 128
    const bool vec = (reinterpret_cast<uintptr_t>(arow) & 15u) == 0 && nch <= 256 * kPrepChunks;
    float x[kPrepChunks][8];
    float amax = 0.0f;
    if (vec) {
#pragma unroll
        for (int i = 0; i < kPrepChunks; ++i) {
            const int c = tid + 256 * i;
            uint4 w = make_uint4(0u, 0u, 0u, 0u);
            if (live && c < nch && c * 8 + 8 <= K) w = __ldg(reinterpret_cast<const uint4*>(arow) + c);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                x[i][2 * j] = __uint_as_float(ww[j] << 16);
                x[i][2 * j + 1] = __uint_as_float(ww[j] & 0xFFFF0000u);
            }
            if (live && c < nch && c * 8 < K && c * 8 + 8 > K) {   // the K tail chunk
#pragma unroll
                for (int j = 0; j < 8; ++j) x[i][j] = c * 8 + j < K ? bf16_bits_to_f32(arow[c * 8 + j]) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[i][j]));
        }
    } else if (live) {
        for (int k = tid; k < K; k += 256) amax = fmaxf(amax, fabsf(bf16_bits_to_f32(arow[k])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    if ((tid & 31) == 0) wmax[tid >> 5] = amax;
    __syncthreads();
    amax = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) amax = fmaxf(amax, wmax[w]);
    // s = 2^(8 - E) with amax < 2^E: max |a*s| in [128, 256).
    int e = 0;
    if (amax > 0.0f) frexpf(amax, &e);
    e = max(-100, min(100, 8 - e));
    const float sigma = ldexpf(1.0f, e);
    if (tid == 0) inv_sigma[m] = ldexpf(1.0f, -e);
    if (vec) {
#pragma unroll
        for (int i = 0; i < kPrepChunks; ++i) {
            const int c = tid + 256 * i;
            if (c >= nch) break;
            uint2 hi, lo;
            act_split8(x[i], sigma, hi, lo);
            *reinterpret_cast<uint2*>(act + (int64_t)m * kpad + c * 8) = hi;
            *reinterpret_cast<uint2*>(act + (int64_t)(8 + m) * kpad + c * 8) = lo;
        }
        return;
    }
    for (int c = tid; c < nch; c += 256) {
        float xx[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) xx[j] = (live && c * 8 + j < K) ? bf16_bits_to_f32(arow[c * 8 + j]) : 0.0f;
        uint2 hi, lo;
        act_split8(xx, sigma, hi, lo);
        *reinterpret_cast<uint2*>(act + (int64_t)m * kpad + c * 8) = hi;
        *reinterpret_cast<uint2*>(act + (int64_t)(8 + m) * kpad + c * 8) = lo;
    }
}

__global__ void __launch_bounds__(kThreads, 4)
gemm_e4m3_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmAct,
                    const E4Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tile = blockIdx.x, split = blockIdx.y;
    const int n0 = tile * BM;
    const int k0 = split * p.kc;
    const int klen = min(p.kc, p.K - k0);
    const int nkb = (klen + KB - 1) / KB;

    uint8_t* sStage = base;                      // stages x (16 KB weights + 2 KB activations)
    uint64_t* full = reinterpret_cast<uint64_t*>(sStage + p.stages * kStage);
    uint64_t* empty = full + p.stages;
    uint64_t* mma_done = empty + p.stages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    volatile int* s_last = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    auto issue = [&](int kb, int s) {
        mbar_arrive_expect_tx(&full[s], kStage);
        tma_load_2d(sStage + s * kStage, &tmW, &full[s], k0 + kb * KB, n0);
        tma_load_2d(sStage + s * kStage + kWStage, &tmAct, &full[s], k0 + kb * KB, 0);
    };
    const int pre = nkb < p.stages ? nkb : p.stages;
    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(mma_done, 1);
        *abort_flag = 0u;
        fence_mbar_init();
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmAct);
        // The first ring of weights goes out before griddepcontrol.wait: the
        // prep kernel does not write them, and every kernel before the prep
        // kernel has completed when this grid starts (the prep kernel
        // releases it only after its own wait).  The weight stream thus
        // overlaps the prep kernel.
        for (int kb = 0; kb < pre; ++kb) {
            mbar_arrive_expect_tx(&full[kb], kStage);
            tma_load_2d(sStage + kb * kStage, &tmW, &full[kb], k0 + kb * KB, n0);
        }
    }
    pdl_wait();          // the activation operand and 1/s come from the prep kernel
    if (tid == 0)
        for (int kb = 0; kb < pre; ++kb)
            tma_load_2d(sStage + kb * kStage + kWStage, &tmAct, &full[kb], k0 + kb * KB, 0);
    if (warp == 1) {
        tmem_alloc(tmem_slot, 32);
        tmem_relinquish();
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
            for (int kb = pre; kb < nkb && !*abort_flag; ++kb) {
                const int s = kb % p.stages;
                const uint32_t ph = static_cast<uint32_t>(kb / p.stages) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err)) break;
                issue(kb, s);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % p.stages;
                const uint32_t ph = static_cast<uint32_t>(kb / p.stages) & 1u;
                if (!mbar_wait(&full[s], ph, abort_flag, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sStage + s * kStage);
                const uint32_t b_addr = a_addr + kWStage;
#pragma unroll
                for (int kk = 0; kk < KB / 32; ++kk)
                    umma_f8_ss(tmem_base, umma_desc_k_sw128(a_addr + kk * 32),
                               umma_desc_k_sw128(b_addr + kk * 32), kIdescE4M3,
                               (kb | kk) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            if (ok) umma_commit(mma_done);
        }
    } else {
        // ---------------- epilogue ----------------
        const int q = warp & 3;
        const int nl = q * 32 + lane;          // tile row = output column n0 + nl
        const int n = n0 + nl;
        float v[8];
        bool ok = mbar_wait(mma_done, 0u, abort_flag, p.err);
        if (ok) {
            tc_fence_after();
            uint32_t r[16];
            tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(q * 32) << 16), r);
            tmem_ld_wait();
#pragma unroll
            for (int m = 0; m < 8; ++m)
                v[m] = (__uint_as_float(r[m]) + __uint_as_float(r[8 + m])) * p.inv_sigma[m];
        }
        const float sc = (n < p.N) ? p.scale[n] : 0.0f;
        const uint32_t call = p.seq ? *p.seq + 1u : 0u;
        const int64_t obase = p.seq ? static_cast<int64_t>(call & 1u) * p.out_stride : 0;
        // Writes one finished column n (rows 0..M-1) into every output copy;
        // the stores of a warp cover 64 contiguous bytes per row and copy.
        auto write_col = [&](const float (&c)[8]) {
            uint16_t bits[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) bits[m] = __bfloat16_as_ushort(__float2bfloat16_rn(c[m] * sc));
            for (int o = 0; o < p.nout; ++o)
                for (int m = 0; m < p.M; ++m) p.out[o][obase + (int64_t)m * p.ldc + n] = bits[m];
        };
        bool wrote = false;    // this CTA finished its tile (the epilogue group agrees)
        if (p.splits == 1) {
            if (ok && n < p.N) write_col(v);
            wrote = true;
        } else {
            // Every epilogue thread takes both barriers, whatever `ok` says.
            if (ok) {
                float* wsp = p.ws + ((int64_t)tile * p.splits + split) * (8 * BM);
#pragma unroll
                for (int m = 0; m < 8; ++m) __stcg(&wsp[m * BM + nl], v[m]);
            }
            __threadfence();
            named_barrier_sync(1, 128);
            if (tid == 64) {
                uint32_t t = atomicAdd(&p.tickets[tile], 1u);
                *s_last = (t == static_cast<uint32_t>(p.splits - 1)) ? 1 : 0;
            }
            named_barrier_sync(1, 128);
            if (*s_last) {
                __threadfence();
                const float* wt = p.ws + (int64_t)tile * p.splits * (8 * BM);
                if (ok && n < p.N) {
                    float sum[8];
#pragma unroll
                    for (int m = 0; m < 8; ++m) {
                        sum[m] = 0.0f;
                        if (m < p.M)
                            for (int sp = 0; sp < p.splits; ++sp) sum[m] += __ldcg(&wt[sp * 8 * BM + m * BM + nl]);
                    }
                    write_col(sum);
                }
                if (tid == 64) p.tickets[tile] = 0u;
                wrote = true;
            }
        }
        if (p.done && wrote) {
            // All-gather completion.  After the epilogue barrier one thread
            // counts the tile with an acq_rel atomic at GPU scope: its release
            // covers the group's stores (ordered before it by the barrier),
            // and the last tile's acquire gathers every tile's.  That thread
            // then fences once at system scope and raises this rank's flag on
            // every rank with relaxed system-scope stores (fence + relaxed
            // store = release), which the peers read with system-scope acquire
            // loads.  Measured: a system-scope fence per tile costs 6 us per
            // call, a release store per flag ~2 us per rank.
            named_barrier_sync(1, 128);
            if (tid == 64) {
                const uint32_t ntiles = gridDim.x;
                const uint32_t t = atom_add_acq_rel_gpu_u32(p.done, 1u);
                if (t == ntiles - 1) {
                    fence_acq_rel_sys();
                    for (int q = 0; q < p.nout; ++q) st_relaxed_sys_u32(&p.flag[q][p.rank], call);
                    *p.done = 0u;   // ready for the next call on this stream
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 32);
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

size_t smem_bytes(int stages, int /*kc*/) {
    return 1024 + static_cast<size_t>(stages) * kStage + 256;
}

}  // namespace

bool gemm_e4m3_tc_supported(const GemmArgs& g) {
    if (g.M < 1 || g.M > 8 || g.N < 1 || g.K < 16 || g.a_trans) return false;
    if (g.K % 16 || g.ldb % 16 || reinterpret_cast<uintptr_t>(g.B) % 16) return false;
    return encode_fn() != nullptr;
}

E4m3TcPlan gemm_e4m3_tc_plan_splits(const GemmArgs& g, int splits, int stages) {
    E4m3TcPlan p{1, 0, 0};
    if (splits < 1) splits = 1;
    int kc = ((g.K + splits - 1) / splits + KB - 1) / KB * KB;
    if (kc > kMaxKc) kc = kMaxKc;
    p.kc = kc;
    p.splits = (g.K + kc - 1) / kc;
    int st = stages < 2 ? 2 : stages;
    while (st > 2 && smem_bytes(st, kc) > kSmemLimit) --st;
    p.stages = smem_bytes(st, kc) <= kSmemLimit ? st : 0;
    return p;
}

E4m3TcPlan gemm_e4m3_tc_plan(const GemmArgs& g, int num_sms) {
    // Measured on B200 (M = 8, K = 8192, N = 3584 .. 28672): several CTAs per
    // SM with a shallow ring stream the weights faster than one CTA with a
    // deep ring, and the best split count puts about three CTAs on every SM
    // (tiles x splits ~ 3 x SMs); past 4 splits a 2-stage ring is as fast.
    const int tiles = (g.N + BM - 1) / BM;
    int s = (3 * num_sms + tiles / 2) / tiles;
    const int max_s = g.K / KB > 1 ? g.K / KB : 1;
    if (s > 16) s = 16;
    if (s > max_s) s = max_s;
    if (s < 1) s = 1;
    return gemm_e4m3_tc_plan_splits(g, s, s > 4 ? 2 : 3);
}

size_t gemm_e4m3_tc_ws_floats(const GemmArgs& g, const E4m3TcPlan& p) {
    if (p.splits <= 1) return 0;
    return static_cast<size_t>((g.N + BM - 1) / BM) * p.splits * 8 * BM;
}

size_t gemm_e4m3_tc_act_bytes(const GemmArgs& g) {
    const size_t kpad = (static_cast<size_t>(g.K) + KB - 1) / KB * KB;
    return 16 * kpad + 64;
}

cudaError_t launch_gemm_e4m3_tc(const GemmArgs& g, const E4m3TcPlan& plan, const float* scale,
                                float* ws, uint32_t* tickets, void* act_buf, uint32_t* err,
                                cudaStream_t s, const AllGatherArgs* ag) {
    if (!gemm_e4m3_tc_supported(g) || plan.kc <= 0 || plan.stages < 2 || !act_buf)
        return cudaErrorInvalidValue;
    if (plan.splits > 1 && (!ws || !tickets)) return cudaErrorInvalidValue;
    if (ag && (ag->world < 1 || ag->world > kMaxPeers || ag->rank < 0 || ag->rank >= ag->world ||
               !ag->done))
        return cudaErrorInvalidValue;
    const int kpad = (g.K + KB - 1) / KB * KB;
    uint8_t* act = static_cast<uint8_t*>(act_buf);
    float* inv_sigma = reinterpret_cast<float*>(act + 16 * static_cast<size_t>(kpad));
    if (reinterpret_cast<uintptr_t>(act) % 16) return cudaErrorInvalidValue;
    CUtensorMap tmW, tmAct;
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(g.K), static_cast<cuuint64_t>(g.N)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(g.ldb)};
        cuuint32_t box[2] = {KB, BM};
        cuuint32_t estr[2] = {1, 1};
        if (encode_fn()(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(g.B), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(kpad), 16};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(kpad)};
        cuuint32_t box[2] = {KB, 16};
        cuuint32_t estr[2] = {1, 1};
        if (encode_fn()(&tmAct, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, act, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    static thread_local int attr_dev = -1;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (attr_dev != dev) {
        e = cudaFuncSetAttribute(gemm_e4m3_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemLimit));
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(8, 1, 1);
        cfg.blockDim = dim3(256, 1, 1);
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, e4m3_act_prep_kernel, static_cast<const uint16_t*>(g.A),
                               static_cast<int64_t>(g.lda), g.M, g.K, kpad, act, inv_sigma);
        if (e != cudaSuccess) return e;
    }
    E4Params p;
    p.M = g.M; p.N = g.N; p.K = g.K;
    p.kc = plan.kc; p.splits = plan.splits; p.stages = plan.stages;
    p.inv_sigma = inv_sigma;
    p.scale = scale;
    p.ldc = g.ldc;
    p.ws = ws; p.tickets = tickets; p.err = err;
    for (int q = 0; q < kMaxPeers; ++q) { p.out[q] = nullptr; p.flag[q] = nullptr; }
    if (ag) {
        p.nout = ag->world;
        for (int q = 0; q < ag->world; ++q) {
            if (!ag->out[q] || !ag->flag[q]) return cudaErrorInvalidValue;
            p.out[q] = static_cast<uint16_t*>(ag->out[q]) + static_cast<int64_t>(ag->rank) * g.N;
            p.flag[q] = ag->flag[q];
        }
        p.done = ag->done;
        p.rank = ag->rank;
        p.seq = ag->seq;
        p.out_stride = ag->out_stride_elems;
        if (!ag->seq) return cudaErrorInvalidValue;
    } else {
        p.nout = 1;
        p.out[0] = static_cast<uint16_t*>(g.C);
        p.done = nullptr;
        p.rank = 0;
        p.seq = nullptr;
        p.out_stride = 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((g.N + BM - 1) / BM, plan.splits, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes(plan.stages, plan.kc);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_e4m3_tc_kernel, tmW, tmAct, p);
}

}  // namespace dnnopt_b200
