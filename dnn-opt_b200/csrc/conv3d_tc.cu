// Conv3D (stride 1) as an implicit GEMM on the 5th-generation tensor cores:
// the B200 path of the reference's conv3d_bf16 / conv3d_int8
// (src/conv/conv3d.cpp), which materialise im2col columns
// (im2col3d_nhwc_* :389-457) and call the library GEMMs.  Here the column
// matrix is never written.  The operands are prepared once: the input
// converted (BF16, RNE) or quantised (INT8, per-tensor scale, round half
// away, quantize_fp32_to_int8_3d :366-377) into a zero-padded NDHWC copy
// [N, ID+2pd, IH+2ph, IW+2pw, IC], the filter likewise.  In the padded copy,
// viewed as rows of IC channels, output position (n, od, oh, ow) is row
//   P = ((n*Dp + od)*Hp + oh)*Wp + ow
// and its filter tap (kd, kh, kw) reads row P + (kd*Hp + kh)*Wp + kw, so the
// A tiles of all KH x KW taps of one depth slice kd and one chunk of channels,
// for 128 consecutive rows P, are 128-row windows at offsets kh*Wp + kw of
// ONE 2-D TMA box of 128 + (KH-1)*Wp + KW - 1 rows (one box per filter row,
// 128 + KW - 1 rows, when that exceeds the 256-row box limit): each tap's
// UMMA descriptor starts that many rows into the box, which the swizzled
// layout allows (the swizzle follows the absolute shared-memory address;
// checked on B200).  Rows P that are not output positions (the padding
// columns / planes) are computed and dropped.
//
//   output [N, OD, OH, OW, OC] = sum_k A[P, k] * filter[oc, k],
//   k = ((kd*KH + kh)*KW + kw)*IC + ic (the reference's column order)
//
// INT8: int32 accumulators in TMEM (exact), dequantisation float(acc) *
// (s_in*s_f), then bias and relu / relu6 in the epilogue with the reference's
// rounding order (dequantize_int32_to_fp32_3d :379-386, apply_conv3d_postops
// :126-148).  BF16: FP32 accumulators, then bias and post-op.
//
// A K-block is cb = 32, 64 or 128 bytes of channels of one tap, staged with
// the matching TMA swizzle straight into the UMMA K-major layout; each ring
// stage carries one or more window boxes (up to 64 KB: on B200 a stage costs
// a roughly fixed mbarrier round trip of about 0.3 us and a 128-row box about
// 0.12 us more, so one window box instead of a box per tap cuts the TMA rows
// several-fold).  With one channel tile (OC <= 256) the whole filter stays
// resident
// in shared memory, loaded with the CTA's first tile.  Roles: warp 0 TMA,
// warp 1 TMEM + MMA issue into two accumulators, warps 2-5 epilogue (32 x 32
// blocks transposed through swizzled shared memory into whole 128-byte row
// stores).  Every mbarrier wait and the prep kernel's grid barrier are
// bounded; every TMA load targets this CTA's own shared memory.
#include <cuda.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

namespace {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kMaxN = 256;
constexpr size_t kSmemCap = 232448;       // 227 KB dynamic shared memory per CTA
constexpr size_t kSmemMin = 120 * 1024;   // keeps one CTA per SM (TMEM of up to 512 columns)
constexpr int kBarBytes = 256;
constexpr int kStaging = 4 * 4096;        // one 32 x 32 fp32 block per epilogue warp
constexpr int kPrepThreads = 256;         // BF16 conversion
constexpr int kQuantThreads = 1024;       // INT8 prep: one CTA per SM (cooperative)

struct ConvTcParams {
    int N, OD, OH, OW, OC;
    int Dp, Hp, Wp;             // padded input extents
    int KH, KW;
    int m_tiles, n_tiles, units;
    int p_last;                 // padded row of the last output position
    int cb, celems, cpt, num_kb;   // K-block bytes / elements, K-blocks per tap, total
    int n_mma, stages, b_res;
    // Windows: one A box of rows_win rows (128 + (hwin-1)*Wp + KW - 1,
    // rounded up to 8) per (kd, group of hwin filter rows, channel chunk)
    // serves hwin*KW taps, whose A operands start kh*Wp + kw rows into it
    // (the UMMA descriptor may start at any row of a swizzled tile: the
    // swizzle follows the absolute address).
    int num_win, kws;           // windows per tile (KD*(KH/hwin)*cpt), windows per ring stage
    int hwin;                   // filter rows per window: KH when 128 + (KH-1)*Wp + KW - 1 <= 256 rows, else 1
    uint32_t a_slot, win_bytes; // A box slot (1024-byte multiple); A slot + KW B blocks unless resident
    int post;                   // 0 none, 1 relu, 2 relu6
    uint32_t a_bytes, b_bytes;  // one A window box (rows_win rows) and one B K-block (n_mma rows)
    uint32_t stage_bytes;       // kws windows
    uint32_t ring_off, stg_off, bar_off;
    const float* scales;        // INT8: {s_in, s_f}
    const float* bias;
    float* out;
    int out_vec;                // 16-byte output stores (OC % 4 == 0, aligned)
    uint32_t* err;
};

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// K-major shared-memory descriptor for rows of cb bytes in the cb-byte
// swizzled layout (8 rows per atom, atoms 8*cb bytes apart): layout code 2
// (128 B), 4 (64 B) or 6 (32 B) at bits 61-63, version 1 at bit 46.
__device__ __forceinline__ uint64_t desc_k_swizzled(uint32_t addr, int cb) {
    const uint64_t layout = cb == 128 ? 2u : (cb == 64 ? 4u : 6u);
    uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>((8u * static_cast<uint32_t>(cb)) >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= layout << 61;
    return d;
}

// Instruction descriptor: D S32 (i8) or F32 (bf16) at bits 4-5, A / B signed
// 8-bit or BF16 (1) at 7-9 / 10-12, both K-major, N >> 3 at 17, M >> 4 at 24.
__device__ __forceinline__ uint32_t conv_idesc(int i8, int n) {
    return ((i8 ? 2u : 1u) << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ float conv_post(float v, const float* bias, int oc, int post) {
    if (bias) v = __fadd_rn(v, __ldg(bias + oc));
    if (post == 1) v = v > 0.0f ? v : 0.0f;
    else if (post == 2) v = v > 0.0f ? (v < 6.0f ? v : 6.0f) : 0.0f;
    return v;
}

// I8: kind::i8 with int32 accumulators (INT8), else kind::f16 (BF16, FP32
// accumulators).  KS: MMAs per tap and channel chunk (cb / 32).  Both
// compile-time: on B200 one thread issuing tcgen05.mma at N = 64 is bound by
// its own instruction stream (a straight-line sequence measured ~54 cycles
// per MMA, the math ~32), and every run-time branch in the loop adds to it — a
// branch between the two MMA forms doubled the cost, nested tap / K-step
// loops made the conv kernel ~20 % (INT8) and ~27 % (BF16) slower than this
// flat loop.
template <bool I8, int KS>
__global__ void __launch_bounds__(kThreads, 1)
conv3d_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const ConvTcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* bres = base;                       // resident filter: num_kb x b_bytes (b_res)
    uint8_t* ring = base + p.ring_off;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + p.bar_off);
    uint64_t* empty = full + kMaxStages;
    uint64_t* tfull = empty + kMaxStages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t need = static_cast<uint32_t>(2 * p.n_mma);
    const uint32_t tmem_cols = need <= 32 ? 32u : (need <= 64 ? 64u : (need <= 128 ? 128u : (need <= 256 ? 256u : 512u)));

    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
        *abort_flag = 0u;
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();   // the prepared operands come from the previous launch

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t it = 0;
            bool first = true;
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
                const int mt = u % p.m_tiles, nt = u / p.m_tiles;
                const int p0 = mt * BM;
                const bool load_b = !p.b_res || first;
                // Window walk: off = (kd*Hp + kh0)*Wp, tap0 = (kd*KH + kh0)*KW
                // with kh0 the window's first filter row, channel chunk c
                // fastest.
                int c = 0, kh = 0, off = 0, tap0 = 0;
                bool ok = true;
                const int wtaps = p.hwin * p.KW;   // taps per window
                const uint32_t b_load = load_b ? static_cast<uint32_t>(wtaps) * p.b_bytes : 0u;
                for (int w = 0; w < p.num_win; w += p.kws, ++it) {
                    const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    uint8_t* sa = ring + s * p.stage_bytes;
                    const int nsub = min(p.kws, p.num_win - w);
                    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nsub) * (p.a_bytes + b_load));
                    for (int sub = 0; sub < nsub; ++sub) {
                        uint8_t* wb = sa + sub * p.win_bytes;
                        tma_load_2d(wb, &tmA, &full[s], c * p.celems, p0 + off);
                        if (load_b)
                            for (int t = 0; t < wtaps; ++t) {
                                const int kb = (tap0 + t) * p.cpt + c;
                                tma_load_2d(p.b_res ? bres + static_cast<uint32_t>(kb) * p.b_bytes
                                                    : wb + p.a_slot + t * p.b_bytes,
                                            &tmB, &full[s], kb * p.celems, nt * p.n_mma);
                            }
                        if (++c == p.cpt) {
                            c = 0;
                            off += p.hwin * p.Wp;
                            tap0 += wtaps;
                            kh += p.hwin;
                            if (kh == p.KH) {
                                kh = 0;
                                off += (p.Hp - p.KH) * p.Wp;
                            }
                        }
                    }
                }
                if (!ok) break;
                first = false;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = conv_idesc(I8 ? 1 : 0, p.n_mma);
            uint32_t it = 0, titer = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++titer) {
                const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
                if (!mbar_wait(&tempty[buf], tph ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * static_cast<uint32_t>(p.n_mma);
                int c = 0, tap0 = 0;
                const int wtaps = p.hwin * p.KW;
                uint32_t acc = 0u;   // 0 until the tile's first MMA
                const uint32_t bres_addr = smem_u32(bres);
                // B block of tap kw: resident copy (cpt blocks per tap) or the
                // window's own KW blocks; chosen once per window so that the
                // issue loop is branch-free.
                const uint32_t b_step16 = (p.b_res ? static_cast<uint32_t>(p.cpt) * p.b_bytes : p.b_bytes) >> 4;
                constexpr uint32_t cb16 = 2u * KS;   // one row of the chunk, in 16-byte units
                // From tap (kh, KW-1) to tap (kh+1, 0): Wp - KW + 1 rows down.
                const uint32_t a_wrap = static_cast<uint32_t>(p.Wp - p.KW + 1) * cb16;
                for (int w = 0; w < p.num_win; w += p.kws, ++it) {
                    const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
                    if (!mbar_wait(&full[s], ph, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t st_addr = smem_u32(ring + s * p.stage_bytes);
                    const int nsub = min(p.kws, p.num_win - w);
                    for (int sub = 0; sub < nsub; ++sub) {
                        const uint32_t win = st_addr + sub * p.win_bytes;
                        const uint32_t b0 = p.b_res ? bres_addr + static_cast<uint32_t>(tap0 * p.cpt + c) * p.b_bytes
                                                    : win + p.a_slot;
                        // Descriptors of the window's first tap; tap (kh_i, kw)
                        // starts kh_i*Wp + kw rows into the A box and K step kk
                        // 32 bytes further.  The start address field holds
                        // address >> 4 in bits 0-13 and shared-memory addresses
                        // stay below 2^18, so these offsets (in 16-byte units)
                        // are added to the descriptor without a carry.
                        const uint64_t da0 = desc_k_swizzled(win, KS * 32);
                        const uint64_t db0 = desc_k_swizzled(b0, KS * 32);
                        // Taps in (kh_i, kw) order as one flat loop; the step to
                        // the next tap's A rows is a select, not a nested loop.
                        uint32_t a_off = 0u, b_off = 0u;
                        int kw = 0;
                        for (int t = 0; t < wtaps; ++t) {
#pragma unroll
                            for (int kk = 0; kk < KS; ++kk) {
                                const uint64_t da = da0 + (a_off + 2u * kk);
                                const uint64_t db = db0 + (b_off + 2u * kk);
                                if constexpr (I8) umma_i8(d_tmem, da, db, idesc, acc);
                                else umma_f16_ss(d_tmem, da, db, idesc, acc);
                                acc = 1u;
                            }
                            const bool wrap = ++kw == p.KW;
                            kw = wrap ? 0 : kw;
                            a_off += wrap ? a_wrap : cb16;
                            b_off += b_step16;
                        }
                        if (++c == p.cpt) {
                            c = 0;
                            tap0 += wtaps;
                        }
                    }
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;            // TMEM lanes 32q .. 32q+31 = tile rows
        uint8_t* stg = base + p.stg_off + q * 4096;
        const float dq = I8 ? __fmul_rn(p.scales[0], p.scales[1]) : 1.0f;
        const int plane = p.Hp * p.Wp, vol = p.Dp * plane;
        uint32_t titer = 0;
        for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x, ++titer) {
            const int mt = u % p.m_tiles, nt = u / p.m_tiles;
            // This lane's row: padded position P -> output position (or none).
            const int P = mt * BM + q * 32 + lane;
            const int n = P / vol;
            int r = P - n * vol;
            const int d = r / plane;
            r -= d * plane;
            const int h = r / p.Wp, w = r - h * p.Wp;
            const int live = P <= p.p_last && d < p.OD && h < p.OH && w < p.OW;
            const int64_t pix = ((static_cast<int64_t>(n) * p.OD + d) * p.OH + h) * p.OW + w;
            const uint32_t buf = titer & 1u, tph = (titer >> 1) & 1u;
            const bool ok = mbar_wait_warp(&tfull[buf], tph, abort_flag, p.err);
            tc_fence_after();
            const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * static_cast<uint32_t>(p.n_mma);
            const int col0 = nt * p.n_mma;
            for (int c0 = 0; c0 < p.n_mma; c0 += 32) {
                const int cbase = col0 + c0;
                if (cbase >= p.OC) break;   // uniform across the warp
                uint32_t v[32];
                tmem_ld_32x32b_x16(t_addr + c0, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                tmem_ld_32x32b_x16(t_addr + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                tmem_ld_wait();
                // Row `lane` into the staging block: 16-byte chunk j of the
                // row at chunk position j ^ (lane % 8) (conflict-free both ways).
                __syncwarp();   // the previous block's reads are done
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float f[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int col = cbase + 4 * j + e;
                        const float a = I8 ? __fmul_rn(static_cast<float>(static_cast<int32_t>(v[4 * j + e])), dq)
                                           : __uint_as_float(v[4 * j + e]);
                        f[e] = conv_post(a, p.bias, min(col, p.OC - 1), p.post);
                    }
                    *reinterpret_cast<float4*>(stg + lane * 128 + ((j ^ (lane & 7)) * 16)) =
                        make_float4(f[0], f[1], f[2], f[3]);
                }
                __syncwarp();
                // Whole rows out: eight lanes per 128-byte row, four rows per step.
#pragma unroll
                for (int rd = 0; rd < 8; ++rd) {
                    const int row = rd * 4 + (lane >> 3), ch = lane & 7;
                    const int64_t prow = __shfl_sync(0xFFFFFFFFu, pix, row);
                    const int lrow = __shfl_sync(0xFFFFFFFFu, live, row);
                    const float4 val = *reinterpret_cast<const float4*>(stg + row * 128 + ((ch ^ (row & 7)) * 16));
                    const int col = cbase + ch * 4;
                    if (!ok || !lrow || col >= p.OC) continue;
                    float* dst = p.out + prow * p.OC + col;
                    if (p.out_vec) {
                        *reinterpret_cast<float4*>(dst) = val;
                    } else {
                        const float vv[4] = {val.x, val.y, val.z, val.w};
                        for (int e = 0; e < 4 && col + e < p.OC; ++e) dst[e] = vv[e];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }

    tc_fence_before();
    __syncthreads();
    pdl_launch_dependents();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, tmem_cols);
    }
}

// ---- operand preparation -------------------------------------------------------
struct PrepGeom {
    int N, ID, IH, IW, IC;
    int pd, ph, pw, Dp, Hp, Wp;
    int cpp;          // 16-byte chunks per padded pixel
    int64_t nin, nf;  // input / filter elements
    int64_t nchunks;  // 16-byte chunks of the padded input
    int in_vec;       // input 16-byte aligned
    int f_vec;        // filter 16-byte aligned
};

// Reference round-half-away quantisation (quantize_fp32_to_int8_3d :366-377).
__device__ __forceinline__ uint32_t quant8_bits(float x, float inv) {
    int q = static_cast<int>(roundf(x * inv));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q)));
}

__device__ __forceinline__ uint32_t quant8x4(float4 v, float inv) {
    return quant8_bits(v.x, inv) | (quant8_bits(v.y, inv) << 8) | (quant8_bits(v.z, inv) << 16) |
           (quant8_bits(v.w, inv) << 24);
}

__device__ __forceinline__ uint32_t abs_bits(float x) {
    const float a = fabsf(x);
    return a == a ? __float_as_uint(a) : 0u;   // NaN never wins, as in `a > max`
}

__device__ __forceinline__ uint32_t abs_bits4(float4 v) {
    return max(max(abs_bits(v.x), abs_bits(v.y)), max(abs_bits(v.z), abs_bits(v.w)));
}

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Source of padded chunk `ch` (16 bytes of the padded copy, `per` input
// elements), or nullptr for a padding chunk.
// 32-bit index arithmetic: the padded copy has fewer than 2^31 rows.
__device__ __forceinline__ const float* pad_source(const PrepGeom& g, const float* in, int64_t ch, int per) {
    const uint32_t c32 = static_cast<uint32_t>(ch);
    const uint32_t pixel = c32 / static_cast<uint32_t>(g.cpp);
    const int cc = static_cast<int>(c32 - pixel * static_cast<uint32_t>(g.cpp));
    uint32_t t = pixel;
    const int wp = static_cast<int>(t % static_cast<uint32_t>(g.Wp)); t /= static_cast<uint32_t>(g.Wp);
    const int hp = static_cast<int>(t % static_cast<uint32_t>(g.Hp)); t /= static_cast<uint32_t>(g.Hp);
    const int dp = static_cast<int>(t % static_cast<uint32_t>(g.Dp));
    const int64_t n = t / static_cast<uint32_t>(g.Dp);
    const int d = dp - g.pd, h = hp - g.ph, w = wp - g.pw;
    if (d < 0 || d >= g.ID || h < 0 || h >= g.IH || w < 0 || w >= g.IW) return nullptr;
    return in + (((n * g.ID + d) * g.IH + h) * static_cast<int64_t>(g.IW) + w) * g.IC + static_cast<int64_t>(cc) * per;
}

// Grid barrier for a cooperative launch: arrive, the last CTA clears the two
// words `clear2` (the other call parity's absmax slot), resets the count and
// advances the generation; the others wait (bounded, about 2 s of SM clocks)
// for the generation to move.  false: timed out (error recorded).
__device__ bool grid_barrier(uint32_t* count, uint32_t* gen, uint32_t* clear2, uint32_t* err) {
    __shared__ uint32_t s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t ok = 1u;
        const uint32_t g0 = ld_acquire_gpu_u32(gen);
        __threadfence();
        const uint32_t t = atomicAdd(count, 1u);
        if (t == gridDim.x - 1) {
            clear2[0] = 0u;
            clear2[1] = 0u;
            atomicExch(count, 0u);
            __threadfence();
            atomicAdd(gen, 1u);
        } else {
            long long t0;
            asm volatile("mov.u64 %0, %%clock64;" : "=l"(t0));
            for (;;) {
                if (ld_acquire_gpu_u32(gen) != g0) break;
                long long t1;
                asm volatile("mov.u64 %0, %%clock64;" : "=l"(t1));
                if (t1 - t0 > (4LL << 30)) {
                    record_kernel_error(err, kKerrMbarTimeout);
                    ok = 0u;
                    break;
                }
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0u;
}

// INT8 operands in one cooperative launch of one CTA per SM: absmax of input
// and filter (float bit patterns: non-negative floats order like unsigned
// integers), folded per CTA into this call's slot of `maxslots` (two slots
// alternating with the barrier generation's parity, so the slot is clean
// without a reset launch), grid barrier, the scales (s = max_abs / 127, 1
// when all zero, compute_quant_scale_3d :355-364; scales[0..3] = s_in, s_f,
// 1/s_in, 1/s_f), then the padded input (zero padding written too) and the
// filter quantised; the second read of the input is served by L2.
__global__ void __launch_bounds__(kQuantThreads) conv3d_quant_pad_kernel(const float* __restrict__ in,
                                                                         const float* __restrict__ f, const PrepGeom g,
                                                                         uint32_t* sync, uint32_t* maxslots,
                                                                         float* scales, int8_t* inq, int8_t* fq,
                                                                         uint32_t* err) {
    __shared__ uint32_t s_m[2][kQuantThreads / 32];
    __shared__ float s_inv[2];
    __shared__ uint32_t s_slot;
    // This call's slot: the generation cannot move before every CTA arrived.
    if (threadIdx.x == 0) s_slot = ld_acquire_gpu_u32(sync + 1) & 1u;
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t gs = static_cast<int64_t>(gridDim.x) * blockDim.x;
    uint32_t m[2] = {0u, 0u};
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float* x = t == 0 ? in : f;
        const int64_t n = t == 0 ? g.nin : g.nf;
        const int64_t nv = (t == 0 ? g.in_vec : g.f_vec) ? n / 4 : 0;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        uint32_t acc = 0u;
        for (int64_t i0 = gt; i0 < nv; i0 += 4 * gs) {
            float4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = i0 + k * gs < nv ? __ldg(x4 + i0 + k * gs) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 4; ++k) acc = max(acc, abs_bits4(v[k]));
        }
        for (int64_t j = nv * 4 + gt; j < n; j += gs) acc = max(acc, abs_bits(__ldg(x + j)));
        m[t] = acc;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        m[0] = max(m[0], __shfl_xor_sync(0xFFFFFFFFu, m[0], o));
        m[1] = max(m[1], __shfl_xor_sync(0xFFFFFFFFu, m[1], o));
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { s_m[0][warp] = m[0]; s_m[1][warp] = m[1]; }
    __syncthreads();
    const uint32_t slot = s_slot;
    if (threadIdx.x == 0) {
        uint32_t a = 0u, b = 0u;
        for (int w = 0; w < kQuantThreads / 32; ++w) { a = max(a, s_m[0][w]); b = max(b, s_m[1][w]); }
        atomicMax(maxslots + 2 * slot, a);
        atomicMax(maxslots + 2 * slot + 1, b);
    }
    grid_barrier(sync, sync + 1, maxslots + 2 * (slot ^ 1u), err);
    if (threadIdx.x == 0) {
        const float ma = __uint_as_float(__ldcg(maxslots + 2 * slot));
        const float mb = __uint_as_float(__ldcg(maxslots + 2 * slot + 1));
        const float sa = ma == 0.0f ? 1.0f : __fdiv_rn(ma, 127.0f);
        const float sb = mb == 0.0f ? 1.0f : __fdiv_rn(mb, 127.0f);
        s_inv[0] = __fdiv_rn(1.0f, sa);
        s_inv[1] = __fdiv_rn(1.0f, sb);
        if (blockIdx.x == 0) {
            scales[0] = sa;
            scales[1] = sb;
            scales[2] = s_inv[0];
            scales[3] = s_inv[1];
        }
    }
    __syncthreads();
    pdl_launch_dependents();
    const float inv0 = s_inv[0], inv1 = s_inv[1];
    // Padded input: 16 int8 per chunk.
    uint4* out4 = reinterpret_cast<uint4*>(inq);
    for (int64_t ch = gt; ch < g.nchunks; ch += gs) {
        const float* src = pad_source(g, in, ch, 16);
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (src) {
            if (g.in_vec) {
                const float4* s4 = reinterpret_cast<const float4*>(src);
                o.x = quant8x4(__ldg(s4), inv0);
                o.y = quant8x4(__ldg(s4 + 1), inv0);
                o.z = quant8x4(__ldg(s4 + 2), inv0);
                o.w = quant8x4(__ldg(s4 + 3), inv0);
            } else {
                uint32_t wv[4];
                for (int k = 0; k < 4; ++k)
                    wv[k] = quant8x4(make_float4(__ldg(src + 4 * k), __ldg(src + 4 * k + 1), __ldg(src + 4 * k + 2),
                                                 __ldg(src + 4 * k + 3)), inv0);
                o = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
        }
        out4[ch] = o;
    }
    // Filter [OC, K]: four elements per 32-bit store (fq is 16-byte aligned).
    const int64_t nfv = g.f_vec ? g.nf / 4 : 0;
    for (int64_t i = gt; i < nfv; i += gs)
        reinterpret_cast<uint32_t*>(fq)[i] = quant8x4(__ldg(reinterpret_cast<const float4*>(f) + i), inv1);
    for (int64_t j = nfv * 4 + gt; j < g.nf; j += gs)
        fq[j] = static_cast<int8_t>(static_cast<uint8_t>(quant8_bits(__ldg(f + j), inv1)));
}

__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
    return f32_to_bf16_bits_ref(a) | (static_cast<uint32_t>(f32_to_bf16_bits_ref(b)) << 16);
}

// BF16 operands: the padded input (8 bf16 per 16-byte chunk, zero padding
// written too) and the filter, RNE as the reference's bfloat16_t(float).
__global__ void __launch_bounds__(kPrepThreads) conv3d_bf16_pad_kernel(const float* __restrict__ in,
                                                                       const float* __restrict__ f, const PrepGeom g,
                                                                       uint16_t* inb, uint16_t* fb) {
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t gs = static_cast<int64_t>(gridDim.x) * blockDim.x;
    uint4* out4 = reinterpret_cast<uint4*>(inb);
    for (int64_t ch = gt; ch < g.nchunks; ch += gs) {
        const float* src = pad_source(g, in, ch, 8);
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (src) {
            float x[8];
            if (g.in_vec) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(src));
                const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
                x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
            } else {
                for (int k = 0; k < 8; ++k) x[k] = __ldg(src + k);
            }
            o = make_uint4(bf16x2(x[0], x[1]), bf16x2(x[2], x[3]), bf16x2(x[4], x[5]), bf16x2(x[6], x[7]));
        }
        out4[ch] = o;
    }
    const int64_t nfv = g.f_vec ? g.nf / 4 : 0;
    for (int64_t i = gt; i < nfv; i += gs) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(f) + i);
        reinterpret_cast<uint2*>(fb)[i] = make_uint2(bf16x2(v.x, v.y), bf16x2(v.z, v.w));
    }
    for (int64_t j = nfv * 4 + gt; j < g.nf; j += gs) fb[j] = f32_to_bf16_bits_ref(__ldg(f + j));
    pdl_launch_dependents();
}

// ---- host helpers ----------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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

int chunk_bytes(const Conv3dGeom& g, int mode) {
    const int64_t icb = static_cast<int64_t>(g.IC) * (mode == 1 ? 2 : 1);
    return icb % 128 == 0 ? 128 : (icb % 64 == 0 ? 64 : (icb % 32 == 0 ? 32 : 0));
}

struct ConvTcLayout {
    int Dp, Hp, Wp, cb, n_mma, n_tiles, num_kb, stages, b_res, m_tiles;
    int rows_win, num_win, kws, hwin;
    uint32_t a_slot, win_bytes;
    int64_t rows, p_last;
    size_t smem;
    uint32_t a_bytes, b_bytes, stage_bytes, ring_off, stg_off, bar_off;
};

bool conv_layout(const Conv3dGeom& g, int mode, ConvTcLayout* L) {
    const int cb = chunk_bytes(g, mode);
    if (cb == 0) return false;
    const int eb = mode == 1 ? 2 : 1;
    L->cb = cb;
    L->Dp = g.ID + 2 * g.pd;
    L->Hp = g.IH + 2 * g.ph;
    L->Wp = g.IW + 2 * g.pw;
    L->rows = static_cast<int64_t>(g.N) * L->Dp * L->Hp * L->Wp;
    L->p_last = ((static_cast<int64_t>(g.N - 1) * L->Dp + g.OD - 1) * L->Hp + g.OH - 1) * L->Wp + g.OW - 1;
    // Row indices (tile rows plus the largest tap offset) stay in int32.
    const int64_t max_off = (static_cast<int64_t>(g.KD - 1) * L->Hp + g.KH - 1) * L->Wp + g.KW - 1;
    if (L->rows + max_off + BM >= (int64_t(1) << 31)) return false;
    L->m_tiles = static_cast<int>((L->p_last + BM) / BM);
    const int n = g.OC < kMaxN ? g.OC : kMaxN;
    L->n_mma = (n + 31) / 32 * 32;
    L->n_tiles = (g.OC + L->n_mma - 1) / L->n_mma;
    const int64_t cpt = static_cast<int64_t>(g.IC) * eb / cb;
    L->num_kb = static_cast<int>(cpt * g.KD * g.KH * g.KW);
    // One A window per (kd, chunk) covering all KH x KW taps when
    // 128 + (KH-1)*Wp + KW - 1 rows fit a TMA box (256 rows), else one per
    // (kd, kh, chunk) of 128 + KW - 1 rows; rounded up to 8 rows.
    const int64_t full_rows = BM + static_cast<int64_t>(g.KH - 1) * L->Wp + g.KW - 1;
    L->hwin = full_rows <= 256 ? g.KH : 1;
    L->rows_win = static_cast<int>(((L->hwin == g.KH ? full_rows : BM + g.KW - 1) + 7) / 8 * 8);
    if (L->rows_win > 256) return false;   // TMA box limit
    L->num_win = static_cast<int>(cpt * g.KD * (g.KH / L->hwin));
    L->a_bytes = static_cast<uint32_t>(L->rows_win * cb);
    L->a_slot = (L->a_bytes + 1023u) / 1024u * 1024u;
    L->b_bytes = static_cast<uint32_t>(L->n_mma * cb);
    const size_t fixed = 1024 + kBarBytes + kStaging;
    const size_t bres = static_cast<size_t>(L->num_kb) * L->b_bytes;
    // The filter stays resident when it leaves room for a ring of at least
    // three input windows.
    L->b_res = L->n_tiles == 1 && fixed + bres + 3 * static_cast<size_t>(L->a_slot) <= kSmemCap ? 1 : 0;
    L->win_bytes = L->a_slot + (L->b_res ? 0u : static_cast<uint32_t>(L->hwin * g.KW) * L->b_bytes);
    // Several windows per ring stage (up to 64 KB), preferably three stages.
    const size_t avail = kSmemCap - fixed - (L->b_res ? bres : 0);
    L->kws = 1;
    for (int k = 8; k > 1; --k)
        if (k * L->win_bytes <= 65536u && avail / (k * L->win_bytes) >= 3) { L->kws = k; break; }
    if (L->kws > L->num_win) L->kws = L->num_win;
    L->stage_bytes = static_cast<uint32_t>(L->kws) * L->win_bytes;
    int st = static_cast<int>(avail / L->stage_bytes);
    if (st > kMaxStages) st = kMaxStages;
    if (st < 2) return false;
    L->stages = st;
    L->ring_off = static_cast<uint32_t>(L->b_res ? bres : 0);
    L->stg_off = L->ring_off + static_cast<uint32_t>(st) * L->stage_bytes;
    L->bar_off = L->stg_off + kStaging;
    L->smem = 1024 + L->bar_off + kBarBytes;
    if (L->smem < kSmemMin) L->smem = kSmemMin;
    return L->smem <= kSmemCap;
}

CUtensorMapSwizzle swizzle_for(int cb) {
    return cb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (cb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

PrepGeom prep_geom(const Conv3dGeom& g, int mode, const float* in, const float* f) {
    PrepGeom pg;
    pg.N = g.N; pg.ID = g.ID; pg.IH = g.IH; pg.IW = g.IW; pg.IC = g.IC;
    pg.pd = g.pd; pg.ph = g.ph; pg.pw = g.pw;
    pg.Dp = g.ID + 2 * g.pd; pg.Hp = g.IH + 2 * g.ph; pg.Wp = g.IW + 2 * g.pw;
    pg.cpp = g.IC * (mode == 1 ? 2 : 1) / 16;
    pg.nin = static_cast<int64_t>(g.N) * g.ID * g.IH * g.IW * g.IC;
    pg.nf = static_cast<int64_t>(g.OC) * g.K;
    pg.nchunks = static_cast<int64_t>(g.N) * pg.Dp * pg.Hp * pg.Wp * pg.cpp;
    pg.in_vec = reinterpret_cast<uintptr_t>(in) % 16 == 0 ? 1 : 0;
    pg.f_vec = reinterpret_cast<uintptr_t>(f) % 16 == 0 ? 1 : 0;
    return pg;
}

// CTAs of the INT8 prep kernel: one per SM when one 1024-thread CTA fits
// (cooperative launch), else 0.
int coop_grid(int num_sms) {
    static std::mutex mu;
    static std::unordered_map<int, int> per_sm;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(mu);
    auto it = per_sm.find(dev);
    if (it == per_sm.end()) {
        int nb = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, conv3d_quant_pad_kernel, kQuantThreads, 0) != cudaSuccess)
            nb = 0;
        it = per_sm.emplace(dev, nb).first;
    }
    return it->second >= 1 ? num_sms : 0;
}

}  // namespace

bool conv3d_tc_ok(const Conv3dGeom& g, int mode) {
    if ((mode != 1 && mode != 2) || !encode_fn()) return false;
    if (g.sd != 1 || g.sh != 1 || g.sw != 1) return false;
    if (g.KD * g.KH * g.KW > kConv3dMaxTaps) return false;
    ConvTcLayout L;
    return conv_layout(g, mode, &L);
}

size_t conv3d_tc_input_bytes(const Conv3dGeom& g, int mode) {
    return static_cast<size_t>(g.N) * (g.ID + 2 * g.pd) * (g.IH + 2 * g.ph) * (g.IW + 2 * g.pw) * g.IC *
           (mode == 1 ? 2 : 1);
}

cudaError_t launch_conv3d_tc_prep(const Conv3dGeom& g, int mode, const float* in, const float* f, void* inq, void* fq,
                                  uint32_t* sync, uint32_t* maxslots, float* scales, uint32_t* err, int num_sms,
                                  cudaStream_t s) {
    if (!conv3d_tc_ok(g, mode)) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(inq) % 16 || reinterpret_cast<uintptr_t>(fq) % 16) return cudaErrorInvalidValue;
    const PrepGeom pg = prep_geom(g, mode, in, f);
    if (mode == 1) {
        const int64_t work = pg.nchunks > pg.nf / 4 ? pg.nchunks : pg.nf / 4;
        int64_t grid = (work + kPrepThreads - 1) / kPrepThreads;
        if (grid > 4LL * num_sms) grid = 4LL * num_sms;
        if (grid < 1) grid = 1;
        conv3d_bf16_pad_kernel<<<static_cast<unsigned>(grid), kPrepThreads, 0, s>>>(
            in, f, pg, static_cast<uint16_t*>(inq), static_cast<uint16_t*>(fq));
        return cudaGetLastError();
    }
    if (!sync || !maxslots || !scales) return cudaErrorInvalidValue;
    int grid = coop_grid(num_sms);
    if (grid < 1) return cudaErrorNotSupported;
    // Fewer CTAs for small tensors: four float4 per thread for the absmax,
    // one 16-byte chunk per thread for the quantisation.
    const int64_t w1 = (pg.nin / 4 + 4 * kQuantThreads - 1) / (4 * kQuantThreads);
    const int64_t w2 = (pg.nchunks + kQuantThreads - 1) / kQuantThreads;
    const int64_t need = w1 > w2 ? w1 : w2;
    if (need < grid) grid = static_cast<int>(need > 0 ? need : 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kQuantThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, conv3d_quant_pad_kernel, in, f, pg, sync, maxslots, scales,
                              static_cast<int8_t*>(inq), static_cast<int8_t*>(fq), err);
}

cudaError_t launch_conv3d_tc(const Conv3dGeom& g, int mode, const void* inq, const void* fq, const float* scales,
                             const float* bias, int op, float* out, uint32_t* err, int num_sms, cudaStream_t s) {
    ConvTcLayout L;
    if (!conv3d_tc_ok(g, mode) || !conv_layout(g, mode, &L)) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(inq) % 16 || reinterpret_cast<uintptr_t>(fq) % 16) return cudaErrorInvalidValue;
    if (mode == 2 && !scales) return cudaErrorInvalidValue;
    const int eb = mode == 1 ? 2 : 1;
    const CUtensorMapDataType dt = mode == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const CUtensorMapSwizzle sw = swizzle_for(L.cb);
    CUtensorMap tmA, tmB;
    {
        // Padded input as rows of IC channels; box: one chunk x rows_win rows.
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(g.IC), static_cast<cuuint64_t>(L.rows)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(g.IC) * eb};
        cuuint32_t box[2] = {static_cast<cuuint32_t>(L.cb / eb), static_cast<cuuint32_t>(L.rows_win)};
        cuuint32_t estr[2] = {1, 1};
        if (encode_fn()(&tmA, dt, 2, const_cast<void*>(inq), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(g.K), static_cast<cuuint64_t>(g.OC)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(g.K) * eb};
        cuuint32_t box[2] = {static_cast<cuuint32_t>(L.cb / eb), static_cast<cuuint32_t>(L.n_mma)};
        cuuint32_t estr[2] = {1, 1};
        if (encode_fn()(&tmB, dt, 2, const_cast<void*>(fq), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    ConvTcParams p;
    p.N = g.N; p.OD = g.OD; p.OH = g.OH; p.OW = g.OW; p.OC = g.OC;
    p.Dp = L.Dp; p.Hp = L.Hp; p.Wp = L.Wp;
    p.KH = g.KH; p.KW = g.KW;
    p.m_tiles = L.m_tiles;
    p.n_tiles = L.n_tiles;
    p.units = p.m_tiles * p.n_tiles;
    p.p_last = static_cast<int>(L.p_last);
    p.cb = L.cb;
    p.celems = L.cb / eb;
    p.cpt = static_cast<int>(static_cast<int64_t>(g.IC) * eb / L.cb);
    p.num_kb = L.num_kb;
    p.n_mma = L.n_mma;
    p.stages = L.stages;
    p.b_res = L.b_res;
    p.num_win = L.num_win;
    p.hwin = L.hwin;
    p.kws = L.kws;
    p.a_slot = L.a_slot;
    p.win_bytes = L.win_bytes;
    p.post = op;
    p.a_bytes = L.a_bytes;
    p.b_bytes = L.b_bytes;
    p.stage_bytes = L.stage_bytes;
    p.ring_off = L.ring_off;
    p.stg_off = L.stg_off;
    p.bar_off = L.bar_off;
    p.scales = scales;
    p.bias = bias;
    p.out = out;
    p.out_vec = reinterpret_cast<uintptr_t>(out) % 16 == 0 && g.OC % 4 == 0 ? 1 : 0;
    p.err = err;

    static std::mutex mu;
    static std::unordered_map<int, bool> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!done.count(dev)) {
            const void* fns[6] = {reinterpret_cast<const void*>(conv3d_tc_kernel<true, 1>),
                                  reinterpret_cast<const void*>(conv3d_tc_kernel<true, 2>),
                                  reinterpret_cast<const void*>(conv3d_tc_kernel<true, 4>),
                                  reinterpret_cast<const void*>(conv3d_tc_kernel<false, 1>),
                                  reinterpret_cast<const void*>(conv3d_tc_kernel<false, 2>),
                                  reinterpret_cast<const void*>(conv3d_tc_kernel<false, 4>)};
            for (const void* fn : fns) {
                e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemCap));
                if (e != cudaSuccess) return e;
            }
            done[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.units < num_sms ? p.units : num_sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // MMAs per tap and chunk: cb / 32 (cb is 32, 64 or 128).
    if (mode == 2)
        return L.cb == 128 ? cudaLaunchKernelEx(&cfg, conv3d_tc_kernel<true, 4>, tmA, tmB, p)
             : L.cb == 64  ? cudaLaunchKernelEx(&cfg, conv3d_tc_kernel<true, 2>, tmA, tmB, p)
                           : cudaLaunchKernelEx(&cfg, conv3d_tc_kernel<true, 1>, tmA, tmB, p);
    return L.cb == 128 ? cudaLaunchKernelEx(&cfg, conv3d_tc_kernel<false, 4>, tmA, tmB, p)
         : L.cb == 64  ? cudaLaunchKernelEx(&cfg, conv3d_tc_kernel<false, 2>, tmA, tmB, p)
                       : cudaLaunchKernelEx(&cfg, conv3d_tc_kernel<false, 1>, tmA, tmB, p);
}

}  // namespace dnnopt_b200
