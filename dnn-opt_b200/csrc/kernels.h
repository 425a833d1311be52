// Host-side launch interface of the sm_100a kernels (internal to the library).
// The public boundary is include/dnnopt_b200.h; these entry points take plain
// device pointers and a stream and return cudaError_t.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace dnnopt_b200 {

// Element encodings an FP32-accumulating kernel can read.
enum class In : int {
    F32 = 0,    // float
    BF16 = 1,   // bfloat16 bits (uint16_t)
    F32R = 2,   // float, rounded to bf16 (RNE) on load: the FP32-API gemm_bf16
    RE4 = 3,    // reference fp8_e4m3_t byte (bias-8 codec, gemm_types.h:51-121)
    RE5 = 4,    // reference fp8_e5m2_t byte (bias-16 codec, gemm_types.h:127-197)
};

// op(A)[M,K] * op(B)[K,N]: row-major views with optional transposition.
// a_trans: A is stored K x M (element (m,k) at A[k*lda + m]).
// b_trans: B is stored N x K (element (k,n) at B[n*ldb + k]).
struct GemmArgs {
    int M, N, K;
    float alpha, beta;
    const void* A;
    int64_t lda;
    int a_trans;
    const void* B;
    int64_t ldb;
    int b_trans;
    void* C;
    int64_t ldc;
    // FP32-output paths only: bias[n] added to C[m][n] after the alpha/beta
    // epilogue (the oneDNN entry's bias pass); nullptr for none.
    const float* bias = nullptr;
};

// ---- small-M FP32-output GEMV, B is K x N (N contiguous) -------------------
// Split-K over gridDim.y with a deterministic last-CTA reduction through
// `ws` (splits * MT * n_pad floats) and `counters` (one per 128-column tile,
// zero on entry, left zero on exit).
struct GemvKnPlan {
    int mt;        // 1, 2, 4 or 8 (M <= mt)
    int vec4;      // 1: 4-wide vector loads of B rows (aligned rows)
    int splits;    // K splits (gridDim.y)
    int kchunk;    // rows of K per split
    int cluster;   // 1: splits form a cluster (DSMEM reduction, no workspace)
};
int gemv_kn_tiles(int N);
size_t gemv_kn_ws_floats(const GemvKnPlan& p, int N);
cudaError_t gemv_kn_occupancy(In ia, In ib, int mt, int vec4, int* blocks_per_sm);
cudaError_t launch_gemv_kn(In ia, In ib, const GemmArgs& g, const GemvKnPlan& p, float* ws,
                           uint32_t* counters, cudaStream_t s);
// Cluster variant: splits <= 16 form one thread-block cluster per strip and
// reduce through distributed shared memory (no workspace); kchunk must not
// exceed gemv_kn_cluster_max_chunk().  Launched with programmatic dependent
// launch so its prologue overlaps the previous kernel on the stream.
int gemv_kn_cluster_max_chunk();
cudaError_t gemv_kn_cluster_occupancy(In ia, In ib, int mt, int vec4, int kchunk, int* blocks_per_sm);
cudaError_t launch_gemv_kn_cluster(In ia, In ib, const GemmArgs& g, const GemvKnPlan& p,
                                   cudaStream_t s);

// ---- small-M column-slab GEMV, B is K x N -----------------------------------
// One CTA per 8 or 16 consecutive columns over the whole K extent (reduced
// inside the CTA: no workspace).  Launched with programmatic dependent launch.
// `w` = columns per CTA (8 or 16).
int gemv_slab_ctas(int N, int w);
cudaError_t gemv_slab_occupancy(In ia, In ib, int mt, int w, int K, int* blocks_per_sm);
cudaError_t launch_gemv_slab(In ia, In ib, const GemmArgs& g, int mt, int w, cudaStream_t s);

// ---- small-M row-panel GEMV, FP32, B is K x N ------------------------------
// A CTA owns a panel of `w` (64 or 128) columns and one of `splits` (1, 2,
// 4, 8) K-ranges of gemv_panel_rows(K, splits) rows, read as whole row
// segments (4w bytes) per warp.  splits > 1: partial panels go to `ws`
// (gemv_panel_ws_floats) and the last CTA of each panel (ticket in
// `counters`, gemv_panel_tickets of them, zero on entry and left zero) sums
// them in split order.  Launched with programmatic dependent launch.
int gemv_panel_rows(int K, int splits);
bool gemv_panel_supported(const GemmArgs& g, int mt, int w, int splits);
int gemv_panel_ctas(int N, int w, int splits);
size_t gemv_panel_ws_floats(int N, int mt, int w, int splits);
int gemv_panel_tickets(int N, int w);
cudaError_t gemv_panel_occupancy(int mt, int w, int splits, int rows, int* blocks_per_sm);
cudaError_t launch_gemv_panel(const GemmArgs& g, int mt, int w, int splits, float* ws, uint32_t* counters,
                              cudaStream_t s);

// ---- small-M dot-form GEMV, B is N x K (K contiguous) ----------------------
enum class DotKind : int {
    F32 = 0,     // fp32 x fp32 -> fp32, alpha/beta epilogue
    S8S32 = 1,   // int8 x int8 -> int32 (exact), C overwritten
    E4M3 = 2,    // bf16 x OCP e4m3 * scale[n] -> bf16
    S8DQ = 3,    // int8 x int8 -> fp32 dequant: C = (alpha*sA*sB)*acc + beta*C
    BF16 = 4,    // bf16 x bf16 -> fp32, alpha/beta epilogue (register-resident rows kernel)
};
struct GemvNkPlan {
    int mt;       // 1, 2, 4 or 8
    int vec;      // 1: 16-byte vector loads of B rows
    int grid;     // CTAs (rows are split evenly across them)
};
// The whole A panel (mt x K) is staged in shared memory, so K is bounded by
// kGemvNkMaxSmem / (mt * sizeof(A element)).
constexpr size_t kGemvNkMaxSmem = 200 * 1024;
size_t gemv_nk_smem_bytes(DotKind kind, int mt, int K);
cudaError_t launch_gemv_nk(DotKind kind, const GemmArgs& g, const GemvNkPlan& p,
                           const float* scales, cudaStream_t s);
cudaError_t gemv_nk_occupancy(DotKind kind, int mt, int vec, int K, int* blocks_per_sm);

// Register-resident dot form (F32 / S8S32 / S8DQ): B rows 16-byte aligned,
// K a multiple of the 16-byte chunk and at most 512 chunks.  `grid` CTAs split
// the rows evenly in groups of R (32 / mt) rows.
bool gemv_rows_supported(DotKind kind, const GemmArgs& g);
cudaError_t gemv_rows_occupancy(DotKind kind, int mt, int K, int* blocks_per_sm);
cudaError_t launch_gemv_rows(DotKind kind, const GemmArgs& g, int mt, int grid, const float* scales,
                             cudaStream_t s);

// Bulk-copy variant of the register-resident dot form (F32 / BF16 / S8S32 /
// S8DQ, same preconditions, K of at most 2 x 256 chunks): B rows reach the
// CTA through a ring of shared-memory stages filled with cp.async.bulk by a
// producer warp.  `err` receives a KernelErrorCode when a bounded wait gives
// up (may be null).
bool gemv_rows_bulk_supported(DotKind kind, const GemmArgs& g);
cudaError_t gemv_rows_bulk_occupancy(DotKind kind, int mt, int K, int* blocks_per_sm);
cudaError_t launch_gemv_rows_bulk(DotKind kind, const GemmArgs& g, int mt, int grid, const float* scales,
                                  uint32_t* err, cudaStream_t s);

// ---- general tiled SIMT kernels (any M, N, K, strides, transposes) ----------
// General FP32-accumulate GEMM on the CUDA cores (gemm_simt.cu): BM x BN
// tiles (BM = 16, 32, 64 by M; BN = 64 for N <= 64, else 128), K split over up to 8 CTAs of a cluster when
// the tiles alone would leave SMs idle.
struct GemmSimtPlan {
    int bm = 64;
    int bn = 128;
    int splits = 1;
    int kchunk = 0;
};
GemmSimtPlan gemm_simt_plan(const GemmArgs& g, int num_sms);
cudaError_t launch_gemm_simt(In ia, In ib, const GemmArgs& g, const GemmSimtPlan& plan,
                             cudaStream_t s);
// int8: A is M x K (lda), B is N x K (ldb); kind S8S32 or S8DQ (scales = {sA, sB} on device).
cudaError_t launch_gemm_tile_s8(DotKind kind, const GemmArgs& g, const float* scales,
                                cudaStream_t s);

// ---- FP32-API int8 quantisation (per-tensor absmax / 127, lrintf, clamp) ----
// scales[0..1] receive sA, sB; absmax[0..1] is scratch (zeroed by this call).
cudaError_t launch_absmax2(const GemmArgs& g, uint32_t* absmax_bits, cudaStream_t s);
cudaError_t launch_quantize_s8(const GemmArgs& g, const uint32_t* absmax_bits, float* scales,
                               int8_t* qa, int8_t* qb_nk, cudaStream_t s);

// gemm_fp8 FP32 API: encode A with the reference e4m3 codec (dense M x K) and
// B with the reference e5m2 codec (dense K x N).
cudaError_t launch_quantize_ref_fp8(const GemmArgs& g, uint8_t* qa, uint8_t* qb, cudaStream_t s);

// ---- Conv3D as an im2col GEMM (conv3d.cu) ------------------------------------
constexpr int kConv3dMaxTaps = 1024;   // KD * KH * KW
struct Conv3dGeom {
    int N, IC, ID, IH, IW, OC, KD, KH, KW, sd, sh, sw, pd, ph, pw, OD, OH, OW;
    int64_t M, K;   // column matrix: M = N*OD*OH*OW rows of K = KD*KH*KW*IC
};
// mode 0: FP32 columns, 1: BF16 (RNE), 2: INT8 quantised with 1/scales[2].
cudaError_t launch_conv3d_im2col(const Conv3dGeom& g, int mode, const float* in, void* col,
                                 const float* scales, cudaStream_t s);
// Filter (or input) to BF16 (mode 1) or INT8 with 1/scales[inv_idx] (mode 2;
// 3 for the filter, 2 for the input).
cudaError_t launch_conv3d_filter(int mode, const float* f, void* out, int64_t n, const float* scales,
                                 cudaStream_t s, int inv_idx = 3);
// im2col of an input already in the GEMM precision (mode 1: BF16 bits, 2:
// INT8), 16-byte channel chunks copied as is; needs IC % (16 / element size)
// == 0 (conv3d_copy_im2col_ok) and 16-byte aligned buffers.
bool conv3d_copy_im2col_ok(const Conv3dGeom& g, int mode);
cudaError_t launch_conv3d_im2col_copy(const Conv3dGeom& g, int mode, const void* in_conv, void* col,
                                      cudaStream_t s);
// Absmax, then scales[0..3] and the INT8 input and filter in one pass (two launches).
cudaError_t launch_conv3d_absmax_quant(const float* in, int64_t nin, const float* f, int64_t nf, uint32_t* bits,
                                       float* scales, int8_t* inq, int8_t* fq, cudaStream_t s);
// scales[0..3] = s_in, s_f, 1/s_in, 1/s_f from the per-tensor absmax (bits: 2 words).
cudaError_t launch_conv3d_scales(const float* in, int64_t nin, const float* f, int64_t nf, uint32_t* bits,
                                 float* scales, cudaStream_t s);
// FP32 conv3d as one implicit-GEMM launch of the SIMT kernel (gemm_simt.cu):
// out[M, OC] = im2col(in) x filter^T with the column matrix gathered tile by
// tile from the NDHWC input (never materialised), bias and post-op (0 none,
// 1 relu, 2 relu6) in the epilogue.  Needs IC % 4 == 0, M >= 64, 16-byte
// aligned input and filter, at most kConv3dMaxTaps taps.
bool gemm_simt_conv_ok(const Conv3dGeom& g, const float* in, const float* filter);
cudaError_t launch_gemm_simt_conv(const Conv3dGeom& g, const float* in, const float* filter, const float* bias,
                                  int op, float* out, int num_sms, cudaStream_t s);
// INT8 conv3d as one implicit-GEMM launch of the dp4a tile kernel
// (gemm_tile.cu): out[M, OC] = post(float(im2col(in_q) x filter_q^T) *
// (scales[0] * scales[1]) + bias) with exact int32 sums and 16-byte channel
// segments gathered from the quantised NDHWC input.  Needs IC % 16 == 0,
// M >= 64, 16-byte aligned operands, at most kConv3dMaxTaps taps.
bool gemm_tile_s8_conv_ok(const Conv3dGeom& g, const int8_t* in_q, const int8_t* filter_q);
cudaError_t launch_gemm_tile_s8_conv(const Conv3dGeom& g, const int8_t* in_q, const int8_t* filter_q,
                                     const float* scales, const float* bias, int op, float* out,
                                     cudaStream_t s);
// BF16 / INT8 conv3d with stride 1 as an implicit GEMM on tcgen05
// (conv3d_tc.cu): the input prepared once into a zero-padded NDHWC copy, in
// which every filter tap of 128 consecutive output rows is one 2-D TMA box
// (no column matrix); the filter resident in shared memory when it fits;
// bias / dequantisation / post-op in the epilogue.  Needs IC * element size a
// multiple of 32 bytes.  mode 1: BF16, 2: INT8.
bool conv3d_tc_ok(const Conv3dGeom& g, int mode);
// Bytes of the padded input copy.
size_t conv3d_tc_input_bytes(const Conv3dGeom& g, int mode);
// Operands for launch_conv3d_tc: BF16 bits of the padded input and the
// filter, or INT8 in one cooperative launch (absmax into this call's slot of
// the four zero-initialised words `maxslots`, grid barrier on the two
// zero-initialised words `sync`, scales[0..3], quantised padded input and
// filter).  inq / fq 16-byte aligned.
cudaError_t launch_conv3d_tc_prep(const Conv3dGeom& g, int mode, const float* in, const float* f, void* inq, void* fq,
                                  uint32_t* sync, uint32_t* maxslots, float* scales, uint32_t* err, int num_sms,
                                  cudaStream_t s);
cudaError_t launch_conv3d_tc(const Conv3dGeom& g, int mode, const void* inq, const void* fq, const float* scales,
                             const float* bias, int op, float* out, uint32_t* err, int num_sms, cudaStream_t s);
// out = post_op(v + bias[oc]); v = out, or float(acc) * (scales[0] * scales[1]) when acc.
cudaError_t launch_conv3d_post(float* out, const int32_t* acc, const float* scales, const float* bias,
                               int64_t M, int OC, int op, cudaStream_t s);

// Column-major C fix-ups of the oneDNN entry (footprint [0, (N-1)*ldc + M),
// overlapping columns handled in the entry's sequential order).
cudaError_t launch_colmajor_k0(float* C, const float* bias, int64_t M, int64_t N, int64_t ldc,
                               float beta, cudaStream_t s);
cudaError_t launch_colmajor_writeback(float* C, const float* tmp, int64_t tmp_ld, const float* bias,
                                      int64_t M, int64_t N, int64_t ldc, cudaStream_t s);
cudaError_t launch_colmajor_gather(float* tmp, const float* C, int64_t M, int64_t N, int64_t ldc,
                                   cudaStream_t s);

cudaError_t launch_saxpy(int n, float alpha, const float* x, int incx, float* y, int incy,
                         cudaStream_t s);

// ---- general tcgen05 GEMM, both operands by TMA (gemm_tc.cu) ----------------
// INT8 (A [M,K], B [N,K], int32 accumulators: S8S32 or the S8DQ dequantising
// epilogue with scales = {sA, sB}) or BF16 (A [M,K], B [K,N] or [N,K] with
// b_trans, FP32 accumulators, alpha / beta).  Operands 16-byte aligned with
// 16-byte row strides, A not transposed, no bias.  Units = 128-row x n_mma
// tiles x K splits; splits > 1 reduce through `ws` (gemm_tc_ws_bytes) with one
// ticket per tile in `tickets` (zero on entry, left zero).  `err` receives a
// KernelErrorCode when a bounded wait gives up.
enum class TcKind : int { I8 = 0, BF16 = 1 };
struct TcPlan {
    int n_mma;          // columns per tile (<= 256)
    int kb_per_split;   // 128-byte K-blocks per split
    int splits;
};
bool gemm_tc_supported(TcKind kind, const GemmArgs& g);
TcPlan gemm_tc_plan(TcKind kind, const GemmArgs& g, int num_sms);
size_t gemm_tc_ws_bytes(const GemmArgs& g, const TcPlan& pl);
int gemm_tc_tickets(const GemmArgs& g, const TcPlan& pl);
cudaError_t launch_gemm_tc(TcKind kind, DotKind epi, const GemmArgs& g, const TcPlan& pl, const float* scales,
                           void* ws, uint32_t* tickets, uint32_t* err, int num_sms, cudaStream_t s);

// ---- BF16 tall-skinny tcgen05 GEMM (A row-major K-contiguous, TMA) ----------
bool gemm_bf16_tc_supported(const GemmArgs& g);
// Rows of K one launch can take (g.K when B fits whole, 0 when the shape has no tcgen05 path).
int gemm_bf16_tc_kchunk(const GemmArgs& g);
// ---- config-5 e4m3 weight GEMM on tcgen05 (kind::f8f6f4), M <= 8 ------------
struct E4m3TcPlan {
    int splits;   // K ranges (gridDim.y); > 1 reduces through ws + tickets
    int kc;       // K elements per range (multiple of 128)
    int stages;   // weight ring depth (0: shape not supported)
};
bool gemm_e4m3_tc_supported(const GemmArgs& g);
E4m3TcPlan gemm_e4m3_tc_plan(const GemmArgs& g, int num_sms);
E4m3TcPlan gemm_e4m3_tc_plan_splits(const GemmArgs& g, int splits, int stages);
size_t gemm_e4m3_tc_ws_floats(const GemmArgs& g, const E4m3TcPlan& p);
// Scratch for the activation operand (hi/lo e4m3 rows + per-row scales).
size_t gemm_e4m3_tc_act_bytes(const GemmArgs& g);
// Two launches (activation prep, then the GEMM), both with programmatic
// dependent launch.
// Fused all-gather of an N-sharded e4m3 GEMM: out[q] is rank q's first
// output buffer [M x ldc] (mapped in this process; the second starts
// out_stride_elems later), flag[q] rank q's flag array; `seq` is this rank's
// device-side call counter (call number = *seq + 1, advanced by the wait
// kernel); `done` is a zeroed local counter.
constexpr int kAllGatherMaxRanks = 8;
struct AllGatherArgs {
    int world, rank;
    void* out[kAllGatherMaxRanks];
    uint32_t* flag[kAllGatherMaxRanks];
    const uint32_t* seq;
    int64_t out_stride_elems;
    uint32_t* done;
};
cudaError_t launch_gemm_e4m3_tc(const GemmArgs& g, const E4m3TcPlan& plan, const float* scale,
                                float* ws, uint32_t* tickets, void* act_buf, uint32_t* err,
                                cudaStream_t s, const AllGatherArgs* ag = nullptr);
// One CTA: waits (bounded by timeout_ns of %globaltimer) until flag[q] has
// reached the call number for every q < world; on timeout records
// kKerrPeerTimeout in *err and returns.  The call number is *seq + 1 when
// `seq` is given (then *seq is advanced to it after the wait), else `epoch`.
cudaError_t launch_peer_wait(const uint32_t* flag, int world, uint32_t epoch, uint32_t* seq,
                             uint64_t timeout_ns, uint32_t* err, cudaStream_t s);

// err: device word that receives a KernelErrorCode when a bounded wait gives up.
cudaError_t launch_gemm_bf16_tc(const GemmArgs& g, int num_sms, uint32_t* err, cudaStream_t s);


}  // namespace dnnopt_b200
