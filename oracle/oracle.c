/* TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference arithmetic.
 * See oracle.h for the contract; each function cites the reference lines it
 * restates.  Built with -ffp-contract=off so that every float operation is
 * rounded exactly where the reference source rounds it on a non-FMA host. */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* Minimal static-partition parallel-for over [0, n) on `threads` pthreads
 * (the image has no OpenMP runtime).  fn(ctx, begin, end). */
typedef void (*range_fn)(void* ctx, int begin, int end);
typedef struct { range_fn fn; void* ctx; int b, e; } range_job;
static void* range_tramp(void* p) { range_job* j = (range_job*)p; j->fn(j->ctx, j->b, j->e); return NULL; }
static void parallel_for(int n, int threads, range_fn fn, void* ctx) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads == 1 || n < 2) { fn(ctx, 0, n); return; }
    pthread_t tid[256];
    range_job job[256];
    int chunk = (n + threads - 1) / threads, used = 0;
    for (int t = 0; t < threads; ++t) {
        int b = t * chunk, e = b + chunk < n ? b + chunk : n;
        if (b >= e) break;
        job[t].fn = fn; job[t].ctx = ctx; job[t].b = b; job[t].e = e;
        if (pthread_create(&tid[t], NULL, range_tramp, &job[t]) != 0) { fn(ctx, b, e); continue; }
        used = t + 1;
    }
    for (int t = 0; t < used; ++t) pthread_join(tid[t], NULL);
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---------------- bf16 (gemm_types.h:18-31) ---------------- */
uint16_t oracle_bf16_from_f32(float f) {
    uint32_t u = f2u(f);
    uint32_t round = 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)((u + round) >> 16);
}
float oracle_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* ---------------- OCP E4M3FN ---------------- */
float oracle_e4m3fn_to_f32(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
    float v;
    if (e == 0xF && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);              /* subnormal: m * 2^-9 */
    else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);    /* normal */
    return s ? -v : v;
}

uint8_t oracle_e4m3fn_from_f32(float f) {
    if (isnan(f)) return 0x7F;
    uint8_t s = signbit(f) ? 0x80 : 0x00;
    double a = fabs((double)f);
    if (a == 0.0) return s;
    if (a >= 448.0) return s | 0x7E;                   /* saturate to max finite */
    int E;
    frexp(a, &E);
    E -= 1;                                            /* a in [2^E, 2^(E+1)) */
    if (E < -6) {                                      /* subnormal quantum 2^-9 */
        double q = nearbyint(ldexp(a, 9));
        return s | (uint8_t)q;                         /* q == 8 is min normal 0x08 */
    }
    double q = nearbyint(ldexp(a, 3 - E));             /* q in [8, 16] */
    if (q >= 16.0) { q = 8.0; E += 1; }
    if (E > 8) return s | 0x7E;
    uint8_t bits = (uint8_t)(((E + 7) << 3) | ((int)q - 8));
    if (bits == 0x7F) bits = 0x7E;
    return s | bits;
}

/* ---------------- reference fp8_e4m3_t (gemm_types.h:56-115) ----------- */
uint8_t oracle_refe4m3_from_f32(float f) {
    uint32_t u = f2u(f);
    uint32_t sign = (u >> 31) & 1u;
    int32_t ex = (int32_t)((u >> 23) & 0xFFu) - 127 + 8;
    uint32_t mant = (u >> 20) & 0x7u;
    if (ex > 7) { ex = 7; mant = 7; }
    else if (ex < -6) { ex = 0; mant = 0; }
    if (ex > 0) return (uint8_t)((sign << 7) | ((uint32_t)(ex & 0xF) << 3) | mant);
    int shift = -ex;
    if (shift >= 8) return 0;
    mant = (mant >> shift) | (0x8u >> shift);
    return (uint8_t)((sign << 7) | mant);
}

float oracle_refe4m3_to_f32(uint8_t b) {
    uint32_t sign = (b >> 7) & 1u, e = (b >> 3) & 0xFu, m = b & 7u;
    if (e == 0) {
        if (m == 0) return u2f(sign << 31);
        int ae = -6;
        while (!(m & 0x8u)) { m <<= 1; ae--; }
        m &= 7u;
        return u2f((sign << 31) | ((uint32_t)(ae + 127) << 23) | (m << 20));
    }
    if (e == 0xF && m == 7) return sign ? -448.0f : 448.0f;
    return u2f((sign << 31) | ((uint32_t)((int)e - 8 + 127) << 23) | (m << 20));
}

/* ---------------- reference fp8_e5m2_t (gemm_types.h:131-191) ----------- */
uint8_t oracle_refe5m2_from_f32(float f) {
    uint32_t u = f2u(f);
    uint32_t sign = (u >> 31) & 1u;
    int32_t ex = (int32_t)((u >> 23) & 0xFFu) - 127 + 16;
    uint32_t mant = (u >> 21) & 0x3u;
    if (ex > 30) return (uint8_t)((sign << 7) | (0x1Fu << 2));
    if (ex < -14) return (uint8_t)(sign << 7);
    if (ex > 0) return (uint8_t)((sign << 7) | ((uint32_t)(ex & 0x1F) << 2) | mant);
    int shift = -ex;
    if (shift >= 4) return (uint8_t)(sign << 7);
    mant = (mant >> shift) | (0x4u >> shift);
    return (uint8_t)((sign << 7) | mant);
}

float oracle_refe5m2_to_f32(uint8_t b) {
    uint32_t sign = (b >> 7) & 1u, e = (b >> 2) & 0x1Fu, m = b & 3u;
    if (e == 0) {
        if (m == 0) return u2f(sign << 31);
        int ae = -14;
        while (!(m & 0x4u)) { m <<= 1; ae--; }
        m &= 3u;
        return u2f((sign << 31) | ((uint32_t)(ae + 127) << 23) | (m << 21));
    }
    if (e == 0x1F) return u2f((sign << 31) | (0xFFu << 23) | (m << 21));
    return u2f((sign << 31) | ((uint32_t)((int)e - 16 + 127) << 23) | (m << 21));
}

/* ---------------- oneDNN entry (0001-dnnopt-integration.patch:243-365) --------- */
int oracle_sgemm_colmajor(char transa, char transb, int64_t M, int64_t N, int64_t K, float alpha,
                          const float* A, int64_t lda, const float* B, int64_t ldb, float beta,
                          float* C, int64_t ldc, const float* bias) {
    if (transa == 'P' || transa == 'p' || transb == 'P' || transb == 'p') return -1;   /* :284-286 */
    if (M == 0 || N == 0) return 0;                                                  /* :289 */
    if (K == 0) {                                                                    /* :290-304 */
        if (beta == 0.0f) {
            for (int64_t j = 0; j < N; ++j) memset(C + j * ldc, 0, (size_t)M * sizeof(float));
        } else if (beta != 1.0f) {
            for (int64_t j = 0; j < N; ++j)
                for (int64_t i = 0; i < M; ++i) C[j * ldc + i] *= beta;
        }
        if (bias)
            for (int64_t j = 0; j < N; ++j)
                for (int64_t i = 0; i < M; ++i) C[j * ldc + i] += bias[i];
        return 0;
    }
    const int tA = transa == 'T' || transa == 't', tB = transb == 'T' || transb == 't';
    /* Row-major view (:306-322): rm = op(B)^T-side first.  X (rm_M x K) is
     * op(B) read row-major, Y (K x rm_N) is op(A) read row-major. */
    const int rm_M = (int)N, rm_N = (int)M, rm_K = (int)K;
    const float* X = B;
    int ldx = (int)ldb;
    float* xt = NULL;
    if (tB) {            /* dnnopt_gemm_row_major transA: stored K x rm_M -> dense rm_M x K (:249-253) */
        xt = (float*)malloc((size_t)rm_M * rm_K * sizeof(float));
        for (int r = 0; r < rm_M; ++r)
            for (int k = 0; k < rm_K; ++k) xt[(size_t)r * rm_K + k] = B[(size_t)k * ldb + r];
        X = xt; ldx = rm_K;
    }
    const float* Y = A;
    int ldy = (int)lda;
    float* yt = NULL;
    if (tA) {            /* transB: stored rm_N x K -> dense K x rm_N (:254-258) */
        yt = (float*)malloc((size_t)rm_K * rm_N * sizeof(float));
        for (int k = 0; k < rm_K; ++k)
            for (int c = 0; c < rm_N; ++c) yt[(size_t)k * rm_N + c] = A[(size_t)c * lda + k];
        Y = yt; ldy = rm_N;
    }
    if (ldc >= rm_N) {
        oracle_gemm_f32_naive(rm_M, rm_N, rm_K, alpha, X, ldx, Y, ldy, beta, C, (int)ldc);
    } else {             /* :330-353 */
        float* tmp = (float*)calloc((size_t)rm_M * rm_N, sizeof(float));
        if (beta != 0.0f)
            for (int r = 0; r < rm_M; ++r)
                for (int c = 0; c < rm_N; ++c) tmp[(size_t)r * rm_N + c] = C[(size_t)r * ldc + c];
        oracle_gemm_f32_naive(rm_M, rm_N, rm_K, alpha, X, ldx, Y, ldy, beta, tmp, rm_N);
        for (int r = 0; r < rm_M; ++r)
            for (int c = 0; c < rm_N; ++c) C[(size_t)r * ldc + c] = tmp[(size_t)r * rm_N + c];
        free(tmp);
    }
    free(xt);
    free(yt);
    if (bias)            /* :355-362, column by column */
        for (int64_t j = 0; j < N; ++j)
            for (int64_t i = 0; i < M; ++i) C[j * ldc + i] += bias[i];
    return 0;
}

/* ---------------- Conv3D (src/conv/conv3d.cpp) ---------------- */
static float conv_post(float v, const float* bias, int oc, int op) {   /* :126-148 */
    if (bias) v += bias[oc];
    if (op == 1) v = v > 0 ? v : 0;
    else if (op == 2) v = v > 0 ? (v < 6 ? v : 6) : 0;
    return v;
}
static float absmax_scale(const float* x, size_t n) {                  /* :355-364 */
    float m = 0.0f;
    for (size_t i = 0; i < n; ++i) { float a = fabsf(x[i]); if (a > m) m = a; }
    return m == 0.0f ? 1.0f : m / 127.0f;
}
static int8_t quant8(float x, float inv) {                             /* :366-377 */
    int q = (int)roundf(x * inv);
    if (q > 127) q = 127; else if (q < -128) q = -128;
    return (int8_t)q;
}
void oracle_conv3d(int precision, const int* p, const float* input, const float* filter,
                   const float* bias, float* output, int post_op, double* out64) {
    const int N = p[0], IC = p[1], ID = p[2], IH = p[3], IW = p[4], OC = p[5];
    const int KD = p[6], KH = p[7], KW = p[8], sd = p[9], sh = p[10], sw = p[11];
    const int pd = p[12], ph = p[13], pw = p[14];
    const int OD = (ID + 2 * pd - KD) / sd + 1, OH = (IH + 2 * ph - KH) / sh + 1;
    const int OW = (IW + 2 * pw - KW) / sw + 1;
    if (N <= 0 || OC <= 0 || IC <= 0) return;
    const size_t nin = (size_t)N * ID * IH * IW * IC, nflt = (size_t)OC * KD * KH * KW * IC;
    float s_in = 1.0f, s_f = 1.0f, inv_in = 1.0f, inv_f = 1.0f;
    if (precision == 2) {
        s_in = absmax_scale(input, nin); s_f = absmax_scale(filter, nflt);
        inv_in = 1.0f / s_in; inv_f = 1.0f / s_f;
    }
    for (int n = 0; n < N; ++n)
    for (int od = 0; od < OD; ++od)
    for (int oh = 0; oh < OH; ++oh)
    for (int ow = 0; ow < OW; ++ow) {
        const size_t row = (((size_t)n * OD + od) * OH + oh) * OW + ow;
        for (int oc = 0; oc < OC; ++oc) {
            float acc = 0.0f;
            double acc64 = 0.0;
            int32_t acc8 = 0;
            for (int kd = 0; kd < KD; ++kd)
            for (int kh = 0; kh < KH; ++kh)
            for (int kw = 0; kw < KW; ++kw)
            for (int ic = 0; ic < IC; ++ic) {
                const int id = od * sd - pd + kd, ih = oh * sh - ph + kh, iw = ow * sw - pw + kw;
                const int inside = id >= 0 && id < ID && ih >= 0 && ih < IH && iw >= 0 && iw < IW;
                const float x = inside ? input[((((size_t)n * ID + id) * IH + ih) * IW + iw) * IC + ic] : 0.0f;
                const float w = filter[((((size_t)oc * KD + kd) * KH + kh) * KW + kw) * IC + ic];
                if (precision == 0) {
                    acc += x * w;                   /* im2col zeros included, column order */
                } else if (precision == 1) {
                    const float xb = oracle_bf16_to_f32(oracle_bf16_from_f32(x));
                    const float wb = oracle_bf16_to_f32(oracle_bf16_from_f32(w));
                    acc += xb * wb;
                    acc64 += (double)xb * (double)wb;
                } else {
                    acc8 += (int32_t)quant8(x, inv_in) * (int32_t)quant8(w, inv_f);
                }
            }
            float v = precision == 2 ? (float)acc8 * (s_in * s_f) : acc;
            output[row * OC + oc] = conv_post(v, bias, oc, post_op);
            if (out64) {
                double d = precision == 1 ? acc64 : (double)v;
                if (bias) d += bias[oc];
                if (post_op == 1) d = d > 0 ? d : 0;
                else if (post_op == 2) d = d > 0 ? (d < 6 ? d : 6) : 0;
                out64[row * OC + oc] = d;
            }
        }
    }
}

/* ---------------- FP32 (gemm.cpp:88-100) ---------------- */
void oracle_gemm_f32_naive(int M, int N, int K, float alpha, const float* A, int lda,
                           const float* B, int ldb, float beta, float* C, int ldc) {
    if (M <= 0 || N <= 0 || K <= 0) return;           /* gemm.cpp:180 */
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += A[(size_t)i * lda + k] * B[(size_t)k * ldb + j];
            C[(size_t)i * ldc + j] = alpha * acc + beta * C[(size_t)i * ldc + j];
        }
}

typedef struct {
    int M, N, K, lda, ldb, ldc;
    float alpha, beta;
    const float* A; const float* B; const float* C; double* C64;
} f64_ctx;
static void f64_range(void* p, int b, int e) {
    const f64_ctx* c = (const f64_ctx*)p;
    for (int blk = b; blk < e; ++blk) {
        int j0 = blk * 64, j1 = j0 + 64 < c->N ? j0 + 64 : c->N;
        for (int i = 0; i < c->M; ++i) {
            double acc[64];
            for (int j = j0; j < j1; ++j) acc[j - j0] = 0.0;
            for (int k = 0; k < c->K; ++k) {
                double a = c->A[(size_t)i * c->lda + k];
                const float* bb = c->B + (size_t)k * c->ldb;
                for (int j = j0; j < j1; ++j) acc[j - j0] += a * (double)bb[j];
            }
            for (int j = j0; j < j1; ++j) {
                double cc = (c->beta == 0.0f) ? 0.0 : (double)c->beta * c->C[(size_t)i * c->ldc + j];
                c->C64[(size_t)i * c->N + j] = (double)c->alpha * acc[j - j0] + cc;
            }
        }
    }
}
void oracle_gemm_f32_f64(int M, int N, int K, float alpha, const float* A, int lda,
                         const float* B, int ldb, float beta, const float* C, int ldc,
                         double* C64, int threads) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    f64_ctx c = {M, N, K, lda, ldb, ldc, alpha, beta, A, B, C, C64};
    parallel_for((N + 63) / 64, threads, f64_range, &c);
}

/* ---------------- INT8 -> INT32 (gemm_int8_native.cpp:238-247) ---------- */
typedef struct {
    int M, K, lda, ldb, ldc;
    const int8_t* A; const int8_t* B; int32_t* C;
} s8_ctx;
static void s8_range(void* p, int b, int e) {
    const s8_ctx* c = (const s8_ctx*)p;
    for (int j = b; j < e; ++j) {
        const int8_t* bb = c->B + (size_t)j * c->ldb;
        for (int i = 0; i < c->M; ++i) {
            const int8_t* a = c->A + (size_t)i * c->lda;
            int32_t sum = 0;
            for (int k = 0; k < c->K; ++k) sum += (int32_t)a[k] * (int32_t)bb[k];
            c->C[(size_t)i * c->ldc + j] = sum;
        }
    }
}
void oracle_gemm_s8s32(int M, int N, int K, const int8_t* A, int lda, const int8_t* B,
                       int ldb, int32_t* C, int ldc, int threads) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    s8_ctx c = {M, K, lda, ldb, ldc, A, B, C};
    parallel_for(N, threads, s8_range, &c);
}

/* ---------------- BF16 -> FP32 (gemm_driver_bf16.cpp:134-218) ------------ */
typedef struct {
    int N, K, lda, ldb, ldc;
    float alpha, beta;
    const uint16_t* A; const uint16_t* B; float* C; double* C64;
} bf_ctx;
static void bf_range(void* p, int b, int e) {
    const bf_ctx* c = (const bf_ctx*)p;
    float accf[256];
    double accd[256];
    for (int i = b; i < e; ++i) {
        for (int j0 = 0; j0 < c->N; j0 += 256) {
            int j1 = j0 + 256 < c->N ? j0 + 256 : c->N;
            for (int j = j0; j < j1; ++j) { accf[j - j0] = 0.0f; accd[j - j0] = 0.0; }
            for (int k = 0; k < c->K; ++k) {
                float a = oracle_bf16_to_f32(c->A[(size_t)i * c->lda + k]);
                const uint16_t* bb = c->B + (size_t)k * c->ldb;
                for (int j = j0; j < j1; ++j) {
                    float pr = a * oracle_bf16_to_f32(bb[j]);  /* exact: 8x8-bit significands */
                    accf[j - j0] += pr;
                    accd[j - j0] += (double)pr;
                }
            }
            for (int j = j0; j < j1; ++j) {
                size_t o = (size_t)i * c->ldc + j;
                double cd = (c->beta == 0.0f) ? 0.0 : (double)c->beta * (double)c->C[o];
                if (c->C64) c->C64[(size_t)i * c->N + j] = (double)c->alpha * accd[j - j0] + cd;
                if (c->beta == 0.0f) c->C[o] = c->alpha * accf[j - j0];
                else c->C[o] = fmaf(c->alpha, accf[j - j0], c->beta * c->C[o]);
            }
        }
    }
}
void oracle_gemm_bf16f32(int M, int N, int K, float alpha, const uint16_t* A, int lda,
                         const uint16_t* B, int ldb, float beta, float* C, int ldc,
                         double* C64, int threads) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    bf_ctx c = {N, K, lda, ldb, ldc, alpha, beta, A, B, C, C64};
    parallel_for(M, threads, bf_range, &c);
}

/* ---------------- FP32-API INT8 (gemm_smallm_int8.cpp) ------------------ */
void oracle_gemm_int8_f32api(int M, int N, int K, float alpha, const float* A, int lda,
                             const float* B, int ldb, float beta, float* C, int ldc) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    float max_a = 0.0f, max_b = 0.0f;
    for (int i = 0; i < M; ++i)
        for (int k = 0; k < K; ++k) {
            float v = fabsf(A[(size_t)i * lda + k]);
            if (v > max_a) max_a = v;
        }
    for (int k = 0; k < K; ++k)
        for (int j = 0; j < N; ++j) {
            float v = fabsf(B[(size_t)k * ldb + j]);
            if (v > max_b) max_b = v;
        }
    float sa = (max_a == 0.0f) ? 1.0f : max_a / 127.0f;
    float sb = (max_b == 0.0f) ? 1.0f : max_b / 127.0f;
    float scale = alpha * (sa * sb);
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            int32_t acc = 0;
            for (int k = 0; k < K; ++k) {
                long qa = lrintf(A[(size_t)i * lda + k] / sa);
                long qb = lrintf(B[(size_t)k * ldb + j] / sb);
                qa = qa < -128 ? -128 : (qa > 127 ? 127 : qa);
                qb = qb < -128 ? -128 : (qb > 127 ? 127 : qb);
                acc += (int32_t)(qa * qb);
            }
            size_t o = (size_t)i * ldc + j;
            float c0 = (beta == 0.0f) ? 0.0f : beta * C[o];
            C[o] = c0 + scale * (float)acc;
        }
}

/* ---------------- config 5: bf16 x e4m3 (per-channel scale) -> bf16 ------ */
typedef struct {
    int M, N, K, lda, ldw, ldc;
    const uint16_t* A; const uint8_t* W; const float* scale; uint16_t* C; double* C64;
    const float* lut;
} e4_ctx;
static void e4_range(void* p, int b, int e) {
    const e4_ctx* c = (const e4_ctx*)p;
    for (int n = b; n < e; ++n) {
        const uint8_t* w = c->W + (size_t)n * c->ldw;
        for (int m = 0; m < c->M; ++m) {
            const uint16_t* a = c->A + (size_t)m * c->lda;
            double acc = 0.0;
            for (int k = 0; k < c->K; ++k)
                acc += (double)oracle_bf16_to_f32(a[k]) * (double)c->lut[w[k]];
            acc *= (double)c->scale[n];
            if (c->C64) c->C64[(size_t)m * c->N + n] = acc;
            c->C[(size_t)m * c->ldc + n] = oracle_bf16_from_f32((float)acc);
        }
    }
}
void oracle_gemm_e4m3bf16(int M, int N, int K, const uint16_t* A, int lda, const uint8_t* W,
                          int ldw, const float* scale, uint16_t* C, int ldc, double* C64,
                          int threads) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    float lut[256];
    for (int b = 0; b < 256; ++b) lut[b] = oracle_e4m3fn_to_f32((uint8_t)b);
    e4_ctx c = {M, N, K, lda, ldw, ldc, A, W, scale, C, C64, lut};
    parallel_for(N, threads, e4_range, &c);
}

typedef struct { int K, ldw; const float* W; uint8_t* q; float* scale; } q_ctx;
static void q_range(void* p, int b, int e) {
    const q_ctx* c = (const q_ctx*)p;
    for (int n = b; n < e; ++n) {
        const float* w = c->W + (size_t)n * c->ldw;
        float amax = 0.0f;
        for (int k = 0; k < c->K; ++k) { float v = fabsf(w[k]); if (v > amax) amax = v; }
        float s = (amax == 0.0f) ? 1.0f : amax / 448.0f;
        c->scale[n] = s;
        for (int k = 0; k < c->K; ++k) c->q[(size_t)n * c->K + k] = oracle_e4m3fn_from_f32(w[k] / s);
    }
}
void oracle_quantize_e4m3_rows(int N, int K, const float* W, int ldw, uint8_t* q, float* scale,
                               int threads) {
    q_ctx c = {K, ldw, W, q, scale};
    parallel_for(N, threads, q_range, &c);
}

/* ---------------- FP8 API stubs (gemm_fp8.cpp:51-113) ------------------ */
static void fp8_gemm_common(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                            const uint8_t* B, int ldb, float beta, float* C, int ldc,
                            float (*deca)(uint8_t), float (*decb)(uint8_t), float* abuf,
                            float* bbuf) {
    for (int i = 0; i < M; ++i)
        for (int k = 0; k < K; ++k) abuf[(size_t)i * K + k] = deca(A[(size_t)i * lda + k]);
    for (int k = 0; k < K; ++k)
        for (int j = 0; j < N; ++j) bbuf[(size_t)k * N + j] = decb(B[(size_t)k * ldb + j]);
    oracle_gemm_f32_naive(M, N, K, alpha, abuf, K, bbuf, N, beta, C, ldc);
}

void oracle_gemm_refe4m3_refe5m2(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                                 const uint8_t* B, int ldb, float beta, float* C, int ldc) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    float* a = (float*)malloc(sizeof(float) * (size_t)M * K);
    float* b = (float*)malloc(sizeof(float) * (size_t)K * N);
    fp8_gemm_common(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, oracle_refe4m3_to_f32,
                    oracle_refe5m2_to_f32, a, b);
    free(a);
    free(b);
}

void oracle_gemm_refe5m2_refe5m2(int M, int N, int K, float alpha, const uint8_t* A, int lda,
                                 const uint8_t* B, int ldb, float beta, float* C, int ldc) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    float* a = (float*)malloc(sizeof(float) * (size_t)M * K);
    float* b = (float*)malloc(sizeof(float) * (size_t)K * N);
    fp8_gemm_common(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, oracle_refe5m2_to_f32,
                    oracle_refe5m2_to_f32, a, b);
    free(a);
    free(b);
}
