/*
 * dnnopt_b200.h -- C ABI of the B200-native small-M / irregular-N /
 * tall-skinny GEMM library (libdnnopt_b200.so).
 *
 * Drop-in boundary for the GEMM hot path of xuefenghao5121/DNN-Opt.  Plain C
 * types only (no CUDA, torch or C++ types), so cgo / JNI / ctypes / N-API can
 * bind it directly.  Two families of entry points:
 *
 *   dnnopt_gemm_*       Same arguments as the reference's public C++ API
 *                       (include/dnnopt/gemm/gemm.h:10-102): row-major,
 *                       C = alpha*A*B + beta*C, pointers may be host memory
 *                       (pageable or pinned) or device memory.  Synchronous:
 *                       results are in C when the call returns.  They run on
 *                       the stream set with dnnopt_set_stream (default: a
 *                       library-owned stream of the current device).
 *
 *   dnnopt_cuda_gemm_*  Device pointers only, asynchronous on `stream` (a
 *                       cudaStream_t passed as void*; NULL is the legacy
 *                       default stream).  Nothing is copied or synchronised.
 *
 * Error behaviour: the reference's functions return void and silently return
 * on M, N or K <= 0 (src/gemm/gemm.cpp:180).  Here every function returns a
 * dnnopt_status; M, N or K == 0 is a successful no-op exactly as in the
 * reference, while negative sizes, too-small leading dimensions and NULL
 * operands are DNNOPT_STATUS_INVALID_VALUE.  The C++ mirror (libdnnopt_b200.so
 * also exports dnnopt::gemm_fp32 etc. with the reference's void signatures)
 * records the status for dnnopt_get_last_error().
 *
 * Matrix conventions: A is M x K, B is K x N, C is M x N, all row-major with
 * leading dimensions lda, ldb, ldc (elements), except where an entry point
 * says otherwise (the int8 entry points read B as N x K, K contiguous, exactly
 * as the reference implementation does: src/gemm/gemm_int8_native.cpp:217).
 */
#ifndef DNNOPT_B200_H
#define DNNOPT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DNNOPT_B200_ABI_VERSION 1

typedef enum dnnopt_status {
    DNNOPT_STATUS_SUCCESS = 0,
    DNNOPT_STATUS_INVALID_VALUE = 1,   /* negative size, ld too small, NULL operand */
    DNNOPT_STATUS_NOT_SUPPORTED = 2,   /* no GPU path for this combination */
    DNNOPT_STATUS_CUDA_ERROR = 3,      /* a CUDA runtime call failed */
    DNNOPT_STATUS_ALLOC_FAILED = 4,    /* device or pinned allocation failed */
    DNNOPT_STATUS_NO_DEVICE = 5,       /* no CUDA device visible */
    DNNOPT_STATUS_KERNEL_TIMEOUT = 6,  /* a bounded in-kernel wait gave up */
    DNNOPT_STATUS_INJECTED_FAULT = 7,  /* host-side fault injection (tests) */
    DNNOPT_STATUS_EXCEEDS_SCRATCH = 8  /* request larger than a fixed scratch area */
} dnnopt_status;

/* Shape and epilogue of one GEMM call for the dnnopt_cuda_* entry points.
 * trans_a: A is stored K x M (op(A) = A^T).  trans_b: B is stored N x K
 * (op(B) = B^T).  Leading dimensions refer to the stored matrices. */
typedef struct dnnopt_gemm_desc {
    int M, N, K;
    int lda, ldb, ldc;
    float alpha, beta;
    int trans_a, trans_b;
} dnnopt_gemm_desc;

/* ------------------------------------------------------------------------
 * Reference-signature entry points (host or device pointers, synchronous)
 * ---------------------------------------------------------------------- */

/* Replaces dnnopt::gemm_fp32 (include/dnnopt/gemm/gemm.h:14-17,
 * src/gemm/gemm.cpp:168-377).  FP32 FMA accumulation (never TF32). */
int dnnopt_gemm_fp32(int M, int N, int K, float alpha, const float* A, int lda,
                     const float* B, int ldb, float beta, float* C, int ldc);

/* Replaces dnnopt::gemm_bf16 (gemm.h:28-31, src/gemm/gemm.cpp:379-416): FP32
 * in/out, operands rounded to bf16 (round-to-nearest-even, gemm_types.h:18-24),
 * FP32 accumulation. */
int dnnopt_gemm_bf16(int M, int N, int K, float alpha, const float* A, int lda,
                     const float* B, int ldb, float beta, float* C, int ldc);

/* Replaces dnnopt::gemm_bf16_bf16bf16f32 (gemm.h:36-39,
 * src/gemm/gemm_driver_bf16.cpp:134-218).  A, B are bf16 bit patterns. */
int dnnopt_gemm_bf16_bf16bf16f32(int M, int N, int K, float alpha, const uint16_t* A, int lda,
                                 const uint16_t* B, int ldb, float beta, float* C, int ldc);

/* Replaces dnnopt::gemm_int8 (gemm.h:44-47, src/gemm/gemm.cpp:418-455) on its
 * I8MM path: per-tensor absmax/127 scales, lrintf quantisation clamped to
 * [-128, 127], exact int32 accumulation, C = (alpha*sA*sB)*acc + beta*C
 * (src/gemm/gemm_smallm_int8.cpp:198-236, :355-390). */
int dnnopt_gemm_int8(int M, int N, int K, float alpha, const float* A, int lda,
                     const float* B, int ldb, float beta, float* C, int ldc);

/* Replaces dnnopt::gemm_int8_int8int8int32 (gemm.h:55-58,
 * src/gemm/gemm_int8_native.cpp:189-248).  B is N x K (K contiguous,
 * ldb >= K), C is overwritten with exact int32 dot products. */
int dnnopt_gemm_int8_int8int8int32(int M, int N, int K, const int8_t* A, int lda,
                                   const int8_t* B, int ldb, int32_t* C, int ldc);

/* Replace dnnopt::gemm_fp8_e4m3 / gemm_fp8_e5m2 / gemm_fp8 / has_fp8_support
 * (gemm.h:70-93, src/gemm/gemm_fp8.cpp:32-146).  Operands use the reference's
 * own fp8_e4m3_t / fp8_e5m2_t codecs (include/dnnopt/gemm/gemm_types.h:51-200),
 * decoded exactly; FP32 accumulation.  dnnopt_gemm_fp8 quantises FP32 inputs
 * with those codecs first (the reference's FP8-hardware branch). */
int dnnopt_gemm_fp8_e4m3(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                         const uint8_t* B, int ldb, float beta, float* C, int ldc);
int dnnopt_gemm_fp8_e5m2(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                         const uint8_t* B, int ldb, float beta, float* C, int ldc);
int dnnopt_gemm_fp8(int M, int N, int K, float alpha, const float* A, int lda, const float* B,
                    int ldb, float beta, float* C, int ldc);
int dnnopt_has_fp8_support(void);

/* Decode-FFN weight GEMM (the reference has only the
 * FP32 stub above): C[m,n] = bf16_rne(scale[n] * sum_k A[m,k] * W[n,k]),
 * A bf16 M x K, W OCP-E4M3FN N x K (K contiguous, ldw >= K), scale FP32[N],
 * FP32 accumulation, C bf16 M x N. */
int dnnopt_gemm_e4m3_bf16(int M, int N, int K, const uint16_t* A, int lda, const uint8_t* W,
                          int ldw, const float* scale, uint16_t* C, int ldc);

/* FP32 GEMM with transposition flags (host or device pointers, synchronous):
 * the row-major core that cblas_sgemm / sgemm_ reduce to (reference
 * src/blas/cblas_sgemm.cpp:67-99), without materialising transposes. */
int dnnopt_gemm_f32_desc(const dnnopt_gemm_desc* d, const float* A, const float* B, float* C);

/* Replaces the oneDNN integration's dnnopt_sgemm (reference
 * integration/onednn/0001-dnnopt-integration.patch:279-365), the hook the
 * patched extended_sgemm calls: column-major (Fortran) arguments by pointer,
 * C(M x N, ldc) = alpha * op(A) * op(B) + beta * C, then C[i + j*ldc] +=
 * bias[i] when bias is non-null.  transa / transb: 'T'/'t' transposed,
 * 'P'/'p' (packed) -> DNNOPT_STATUS_NOT_SUPPORTED (dnnl_unimplemented),
 * anything else not transposed.  M == 0 or N == 0: no-op; K == 0: C is
 * scaled by beta (zeroed for beta == 0) and the bias added.  ldc < M (the
 * reference's temporary-buffer path, :330-353) gives what its column-by-column
 * copy-back leaves.  Host or device pointers, synchronous; transposes are
 * kernel flags (no transposed copies) and the bias is fused into the GEMM
 * epilogue. */
int dnnopt_sgemm_colmajor(const char* transa, const char* transb, const int64_t* M,
                          const int64_t* N, const int64_t* K, const float* alpha, const float* A,
                          const int64_t* lda, const float* B, const int64_t* ldb,
                          const float* beta, float* C, const int64_t* ldc, const float* bias);

/* ------------------------------------------------------------------------
 * Conv3D (replaces dnnopt::conv3d_fp32 / conv3d_bf16 / conv3d_int8, reference
 * include/dnnopt/conv/conv3d.h:52-127, src/conv/conv3d.cpp:151-525).
 *   input  [N, ID, IH, IW, IC] (NDHWC), filter [OC, KD, KH, KW, IC],
 *   bias [OC] or NULL, output [N, OD, OH, OW, OC], O* = (I* + 2*pad - K*) / stride + 1.
 * precision: DNNOPT_CONV3D_FP32, _BF16 (input and filter rounded to bf16,
 * FP32 accumulation: the reference's ARM BFMMLA path) or _INT8 (per-tensor
 * absmax/127 quantisation, exact int32 sums, dequantised: its SMMLA path).
 * post_op: DNNOPT_POSTOP_NONE, _RELU, _RELU6, applied after the bias.
 * N, IC or OC <= 0, or an empty output: no-op (the reference's early return).
 * KD*KH*KW is limited to 1024.  The column matrix (M x K in the compute
 * precision, M = N*OD*OH*OW, K = KD*KH*KW*IC) is library scratch.
 * ---------------------------------------------------------------------- */
enum { DNNOPT_CONV3D_FP32 = 0, DNNOPT_CONV3D_BF16 = 1, DNNOPT_CONV3D_INT8 = 2 };
enum { DNNOPT_POSTOP_NONE = 0, DNNOPT_POSTOP_RELU = 1, DNNOPT_POSTOP_RELU6 = 2 };
typedef struct dnnopt_conv3d_params {
    int N, IC, ID, IH, IW, OC, KD, KH, KW;
    int stride_d, stride_h, stride_w;
    int pad_d, pad_h, pad_w;
} dnnopt_conv3d_params;
/* Host or device pointers, synchronous. */
int dnnopt_conv3d(int precision, const dnnopt_conv3d_params* p, const float* input,
                  const float* filter, const float* bias, float* output, int post_op);

/* Replaces cblas_saxpy (reference src/blas/cblas_saxpy.cpp:13-50):
 * Y[i*incY] += alpha * X[i*incX] for i < N; N <= 0 or alpha == 0 is a no-op;
 * negative increments are rejected. */
int dnnopt_saxpy(int N, float alpha, const float* X, int incX, float* Y, int incY);

/* Replaces dnnopt::gemm_set_num_threads / gemm_get_num_threads
 * (gemm.h:97-100).  The value is stored and reported; GPU parallelism is
 * chosen by the plan selector. */
void dnnopt_gemm_set_num_threads(int n);
int dnnopt_gemm_get_num_threads(void);

/* ------------------------------------------------------------------------
 * Device-pointer entry points (asynchronous on `stream`)
 * ---------------------------------------------------------------------- */
int dnnopt_cuda_gemm_f32(const dnnopt_gemm_desc* d, const float* A, const float* B, float* C,
                         void* stream);
/* dnnopt_sgemm_colmajor on device pointers, stream-ordered. */
int dnnopt_cuda_sgemm_colmajor(const char* transa, const char* transb, const int64_t* M,
                               const int64_t* N, const int64_t* K, const float* alpha,
                               const float* A, const int64_t* lda, const float* B,
                               const int64_t* ldb, const float* beta, float* C, const int64_t* ldc,
                               const float* bias, void* stream);
/* dnnopt_conv3d on device pointers, stream-ordered. */
int dnnopt_cuda_conv3d(int precision, const dnnopt_conv3d_params* p, const float* input,
                       const float* filter, const float* bias, float* output, int post_op,
                       void* stream);
int dnnopt_cuda_gemm_bf16f32(const dnnopt_gemm_desc* d, const uint16_t* A, const uint16_t* B,
                             float* C, void* stream);
/* FP32 operands rounded to bf16 on load (dnnopt_gemm_bf16 semantics). */
int dnnopt_cuda_gemm_f32_bf16round(const dnnopt_gemm_desc* d, const float* A, const float* B,
                                   float* C, void* stream);
/* FP32-API int8 (dnnopt_gemm_int8 semantics). */
int dnnopt_cuda_gemm_f32_s8quant(const dnnopt_gemm_desc* d, const float* A, const float* B,
                                 float* C, void* stream);
/* B is N x K (d->trans_b is ignored); alpha/beta are ignored. */
int dnnopt_cuda_gemm_s8s32(const dnnopt_gemm_desc* d, const int8_t* A, const int8_t* B,
                           int32_t* C, void* stream);
/* W is N x K with leading dimension d->ldb; scale has N entries. */
int dnnopt_cuda_gemm_e4m3bf16(const dnnopt_gemm_desc* d, const uint16_t* A, const uint8_t* W,
                              const float* scale, uint16_t* C, void* stream);
/* Reference fp8 codecs: A e4m3 (or e5m2) bytes, B e5m2 bytes. */
int dnnopt_cuda_gemm_refe4m3_e5m2(const dnnopt_gemm_desc* d, const uint8_t* A, const uint8_t* B,
                                  float* C, void* stream);
int dnnopt_cuda_gemm_refe5m2_e5m2(const dnnopt_gemm_desc* d, const uint8_t* A, const uint8_t* B,
                                  float* C, void* stream);

/* Allocation-free FP32 small-M GEMM (no counterpart in the reference).  For
 * callers that cannot call cudaMalloc -- code whose device memory belongs to
 * a framework's caching allocator, serving loops that allow no allocation
 * after warm-up, runtimes with a memory budget fixed at start-up.  M <= 8
 * with B stored K x N (otherwise DNNOPT_STATUS_NOT_SUPPORTED), on the split-K
 * GEMV kernel with the planner's split rule.  dnnopt_cuda_gemm_f32 may pick
 * the column-slab or cluster kernel for the same shape, which sum in another
 * order: results agree within FP32 rounding, not bit for bit.  The split-K
 * scratch is a fixed 4 MiB device array inside the library (N <= 131072,
 * larger requests return DNNOPT_STATUS_EXCEEDS_SCRATCH).  The first call on a
 * device looks up that array and loads the kernel; make it before any stream
 * capture.  The looked-up address belongs to the device's primary context:
 * after cudaDeviceReset the entry point must not be called again in this
 * process.  All calls share the array: calls that overlap on the GPU race and
 * must be serialised by the caller. */
int dnnopt_cuda_gemm_f32_noalloc(const dnnopt_gemm_desc* d, const float* A, const float* B,
                                 float* C, void* stream);

/* ------------------------------------------------------------------------
 * Multi-GPU (one process per GPU).  No reference counterpart: the reference
 * is single-process CPU code.  Config 5's weight GEMM is N-sharded over the
 * ranks and its output all-gathered inside the GEMM kernel over peer memory.
 * ---------------------------------------------------------------------- */
#define DNNOPT_MAX_RANKS 8

/* Device buffers another process can map: zero-filled cudaMalloc memory on
 * the current device, its 64-byte CUDA IPC handle, and the mapping of a
 * peer's handle into this process (peer access over NVLink). */
int dnnopt_peer_alloc(size_t bytes, void** ptr);
int dnnopt_peer_free(void* ptr);
int dnnopt_ipc_handle(const void* ptr, unsigned char handle[64]);
int dnnopt_ipc_open(const unsigned char handle[64], void** ptr);
int dnnopt_ipc_close(void* ptr);

typedef struct {
    int world;                                /* 1 .. DNNOPT_MAX_RANKS */
    int rank;                                 /* this process's rank */
    void* out[DNNOPT_MAX_RANKS];              /* rank q's first output buffer [M x ldc] bf16, mapped here */
    unsigned int* flags[DNNOPT_MAX_RANKS];    /* rank q's flag array (world words), mapped here */
    unsigned int* seq;                        /* this rank's call counter (device word, starts at 0) */
    size_t out_stride;                        /* bytes from each rank's first output buffer to its
                                                 second; 0 = one buffer */
} dnnopt_allgather_desc;

/* Fused N-sharded e4m3 decode-FFN GEMM + all-gather.  d->N is this rank's
 * shard width n and d->ldc the full output row length (>= world * n); W and
 * scale hold this rank's n weight rows.  The call numbers itself on the
 * device: call c = *seq + 1 writes the rank's columns [rank*n, rank*n + n) of
 * bf16(scale * A W^T) into buffer (c & 1) of every rank (out[q] + (c & 1) *
 * out_stride), raises flags[q][rank] = c on every rank q once all of them are
 * written, and the stream then waits (bounded, 2 s) until every rank's flag
 * has reached c in this rank's array and sets *seq = c: work queued after the
 * call on `stream` sees the full [M x world*n] result.  Nothing in the
 * arguments changes from call to call, so the call can be captured in a CUDA
 * graph and replayed.  With two buffers a rank one call ahead never
 * overwrites a buffer its peers may still read.  M <= 8.  A flag that does
 * not arrive in time makes dnnopt_stream_status() return
 * DNNOPT_STATUS_KERNEL_TIMEOUT. */
int dnnopt_cuda_gemm_e4m3bf16_allgather(const dnnopt_gemm_desc* d, const uint16_t* A,
                                        const uint8_t* W, const float* scale,
                                        const dnnopt_allgather_desc* ag, void* stream);
/* The bounded wait alone: blocks `stream` until flags[q] has reached epoch
 * for every q < world, or until timeout_us has passed (then the stream's
 * status becomes DNNOPT_STATUS_KERNEL_TIMEOUT). */
int dnnopt_cuda_peer_wait(const unsigned int* flags, int world, unsigned int epoch,
                          unsigned int timeout_us, void* stream);
/* Synchronises `stream` and reports (then clears) a bounded wait that gave up
 * in a kernel this library queued on it. */
int dnnopt_stream_status(void* stream);

/* ------------------------------------------------------------------------
 * Runtime control
 * ---------------------------------------------------------------------- */
/* Stream used by the dnnopt_gemm_* (host-signature) entry points on the
 * current device; NULL restores the library-owned stream. */
int dnnopt_set_stream(void* stream);
/* Status of the last call made by this thread (for the void C++ mirror). */
int dnnopt_get_last_error(void);
const char* dnnopt_status_string(int status);
/* Number of library kernel launches issued by this process so far. */
uint64_t dnnopt_launch_count(void);
/* Name of the kernel the plan selector picks for a call (diagnostics):
 * kind 0 = f32, 1 = bf16f32, 2 = f32_bf16round, 3 = f32_s8quant, 4 = s8s32,
 * 5 = e4m3bf16, 6 = refe4m3_e5m2, 7 = refe5m2_e5m2.  Writes a NUL-terminated
 * string into buf (at most len bytes); needs no device for the name. */
int dnnopt_plan_describe(int kind, const dnnopt_gemm_desc* d, char* buf, int len);

/* Plan autotuning (replaces src/gemm/gemm_autotune.cpp's CPU blocking
 * autotune; enabled like the reference with DNNOPT_AUTOTUNE=1 or this call):
 * candidate split-K / grid choices are timed with CUDA events on first use of
 * a shape and cached; the cache persists in a "DNNAUTO" v4 file. */
int dnnopt_autotune_enable(int on);
int dnnopt_autotune_save(const char* path);
int dnnopt_autotune_load(const char* path);
int dnnopt_autotune_entries(void);

/* Host-side fault injection for failure-path tests: the next `count` calls
 * that reach `site` fail with DNNOPT_STATUS_INJECTED_FAULT before touching the
 * GPU.  site 1 = workspace allocation, 2 = kernel launch, 3 = host staging
 * copy.  count 0 clears.  Also settable with DNNOPT_FAULT_INJECT=site:count. */
int dnnopt_debug_inject_fault(int site, int count);

#ifdef __cplusplus
}
#endif
#endif /* DNNOPT_B200_H */
