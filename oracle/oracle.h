/* TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's (xuefenghao5121/DNN-Opt) arithmetic for
 * the small-M / irregular-N / tall-skinny GEMM path.  This library is the
 * parity checker for the CUDA product path: only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg load it.  The product library
 * (dnn-opt_b200/lib/libdnnopt_b200.so) never links or calls it.
 *
 * Every function names the reference file:line whose arithmetic it restates.
 * All matrices are row-major with explicit leading dimensions, as in the
 * reference's include/dnnopt/gemm/gemm.h:10-102.
 */
#ifndef DNNOPT_ORACLE_H
#define DNNOPT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar codecs ---------------------------------------------------- */
uint16_t oracle_bf16_from_f32(float f);   /* gemm_types.h:18-24 (RNE by +0x7FFF+lsb) */
float oracle_bf16_to_f32(uint16_t b);     /* gemm_types.h:27-31 */
float oracle_e4m3fn_to_f32(uint8_t b);    /* OCP 8-bit FP spec, E4M3FN (bias 7, 0x7F/0xFF NaN) */
uint8_t oracle_e4m3fn_from_f32(float f);  /* OCP E4M3FN, round-to-nearest-even, saturate to 448 */
float oracle_refe4m3_to_f32(uint8_t b);   /* reference fp8_e4m3_t decode, gemm_types.h:88-115 */
uint8_t oracle_refe4m3_from_f32(float f); /* reference fp8_e4m3_t encode, gemm_types.h:56-85 */
float oracle_refe5m2_to_f32(uint8_t b);   /* reference fp8_e5m2_t decode, gemm_types.h:160-191 */
uint8_t oracle_refe5m2_from_f32(float f); /* reference fp8_e5m2_t encode, gemm_types.h:131-157 */

/* ---- GEMMs ------------------------------------------------------------ */
/* gemm_naive_fp32, src/gemm/gemm.cpp:88-100: sequential-k FP32 accumulation,
 * C = alpha*acc + beta*C (C is read even when beta == 0). */
void oracle_gemm_f32_naive(int M, int N, int K, float alpha, const float* A, int lda,
                           const float* B, int ldb, float beta, float* C, int ldc);

/* Same contraction accumulated in FP64 (the "ideal" used for tolerance
 * analysis); C64 is M x N dense (ld = N); beta*C uses the incoming C. */
void oracle_gemm_f32_f64(int M, int N, int K, float alpha, const float* A, int lda,
                         const float* B, int ldb, float beta, const float* C, int ldc,
                         double* C64, int threads);

/* gemm_int8_int8int8int32, src/gemm/gemm_int8_native.cpp:238-247.
 * B is [N, K] (K contiguous, ldb >= K); C is overwritten (no alpha/beta). */
void oracle_gemm_s8s32(int M, int N, int K, const int8_t* A, int lda, const int8_t* B,
                       int ldb, int32_t* C, int ldc, int threads);

/* gemm_bf16_bf16bf16f32, src/gemm/gemm_driver_bf16.cpp:134-218 with the
 * epilogue of gemm_ukernel_bf16_8x8 (gemm_ukernel_bf16_neon.cpp:141-153):
 * FP32 accumulation of exact bf16 products, then beta == 0 ? alpha*acc
 * : fma(alpha, acc, beta*C).  If C64 != NULL the FP64 ideal is also written. */
void oracle_gemm_bf16f32(int M, int N, int K, float alpha, const uint16_t* A, int lda,
                         const uint16_t* B, int ldb, float beta, float* C, int ldc,
                         double* C64, int threads);

/* FP32-API gemm_int8 on its I8MM path, src/gemm/gemm_smallm_int8.cpp:130-176 (M=1)
 * and :198-236, :355-390 (M=2..8), src/gemm/gemm_driver_generic.cpp:49-67 (M>8):
 * per-tensor absmax scales, q = clamp(lrintf(x/scale), -128, 127), exact int32
 * dot products, C = (alpha*sA*sB)*float(acc) + (beta == 0 ? 0 : beta*C). */
void oracle_gemm_int8_f32api(int M, int N, int K, float alpha, const float* A, int lda,
                             const float* B, int ldb, float beta, float* C, int ldc);

/* BASELINE config 5 (no reference implementation exists; the reference FP8 path
 * is a stub, src/gemm/gemm_fp8.cpp:51-83):
 * C[m,n] = bf16_rne( sum_k bf16(A[m,k]) * e4m3fn(W[n,k]) * scale[n] ).
 * W is [N, K] K-contiguous.  The sum is accumulated in FP64; C64 (M x N dense)
 * receives the FP64 value before bf16 rounding when non-NULL. */
void oracle_gemm_e4m3bf16(int M, int N, int K, const uint16_t* A, int lda, const uint8_t* W,
                          int ldw, const float* scale, uint16_t* C, int ldc, double* C64,
                          int threads);

/* Per-output-channel quantisation used to build config-5 weights:
 * scale[n] = absmax_k |W[n,k]| / 448 (1 when the row is all zero),
 * q[n,k] = e4m3fn_rne(W[n,k] / scale[n]). */
void oracle_quantize_e4m3_rows(int N, int K, const float* W, int ldw, uint8_t* q, float* scale,
                               int threads);

/* dnnopt::gemm_fp8_e4m3 / gemm_fp8_e5m2 (src/gemm/gemm_fp8.cpp:51-113): decode
 * with the reference's own (non-OCP) codecs, then the naive FP32 GEMM. */
void oracle_gemm_refe4m3_refe5m2(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                                 const uint8_t* B, int ldb, float beta, float* C, int ldc);
void oracle_gemm_refe5m2_refe5m2(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                                 const uint8_t* B, int ldb, float beta, float* C, int ldc);

/* The oneDNN integration's dnnopt_sgemm (integration/onednn/
 * 0001-dnnopt-integration.patch:279-365, with dnnopt_gemm_row_major
 * :243-267): column-major arguments, C(M x N, ldc) = alpha*op(A)*op(B) +
 * beta*C through RowMajor(op B, op A, N, M, K, B, ldb, A, lda, C, ldc) on
 * dense transposed copies and the naive FP32 GEMM, the ldc < M temporary
 * buffer and its copy-back, then C[i + j*ldc] += bias[i] (column by column).
 * Returns 0, or -1 for packed ('P') operands. */
int oracle_sgemm_colmajor(char transa, char transb, int64_t M, int64_t N, int64_t K, float alpha,
                          const float* A, int64_t lda, const float* B, int64_t ldb, float beta,
                          float* C, int64_t ldc, const float* bias);

/* Conv3D (reference src/conv/conv3d.cpp): NDHWC input, filter [OC, KD, KH,
 * KW, IC], output [N, OD, OH, OW, OC]; p = N, IC, ID, IH, IW, OC, KD, KH, KW,
 * stride d/h/w, pad d/h/w.  The GEMM view is im2col3d (:57-124, columns in
 * (kd, kh, kw, ic) order, zeros for padding) times the filter, then
 * apply_conv3d_postops (:126-148: + bias[oc], then relu / relu6).
 *   precision 0: FP32, accumulated in column order exactly as im2col + the
 *                naive GEMM does (bit-exact with the reference on x86);
 *   precision 1: the ARM BF16 path (:290-340): input and filter rounded to
 *                bf16 (RNE), products accumulated; out64 gets the float64 sum;
 *   precision 2: the ARM INT8 path (:355-518): per-tensor scale absmax/127
 *                (1 when all zero), q = clamp(round(x * (1/scale))), exact
 *                int32 sums, float(acc) * (s_in * s_f), then bias / post-op.
 * post_op: 0 none, 1 relu, 2 relu6.  out64 may be NULL. */
void oracle_conv3d(int precision, const int* p, const float* input, const float* filter,
                   const float* bias, float* output, int post_op, double* out64);

#ifdef __cplusplus
}
#endif
#endif
