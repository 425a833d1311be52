"""GPU parity: the CUDA path through the C ABI against the reference's golden
outputs and the CPU oracle.

Tolerances (written here):
  * FP32:   max|gpu - ref| <= 1e-5 * K          (reference test uses K*2e-5)
  * BF16:   |gpu - fp64| <= 1e-2 * max(1, |ref|) (and a much tighter FP32 check)
  * INT8 -> INT32 and the FP32-API int8 path: bit-exact
  * FP8 (config 5): |gpu - fp64| <= 2^-7 |ref| + 1e-4 max|ref| (one bf16 ulp)
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle.oracle import bf16_bits, bf16_to_f32, int8_uniform, ref_uniform
from tests.conftest import plan_file_bytes, plan_key

pytestmark = pytest.mark.gpu

GEMM_SHAPES = [(1, 1, 1), (4, 4, 4), (8, 8, 8), (16, 16, 16), (32, 32, 32), (64, 64, 64),
               (1, 128, 64), (7, 13, 5), (3, 3, 1000), (128, 1, 768), (1, 1000, 2048),
               (5, 7, 11), (13, 17, 19), (127, 127, 127)]
CBLAS_SIZES = [(4, 4, 4), (16, 16, 16), (32, 64, 48), (7, 13, 11), (1, 64, 32)]
C2_SHAPES = [(m, n, 1024) for m in (2, 3, 5, 7) for n in (1009, 2039, 4093)]
INT8_SHAPES = [(1, 1, 1), (4, 37, 67), (3, 129, 1000), (8, 64, 4096), (5, 7, 11), (13, 17, 19)]


def fp32_tol(K):
    return 1e-5 * K


@pytest.fixture(scope="module")
def gpu(torch_cuda, dn):
    return torch_cuda


# ------------------------------------------------------------------ FP32 ----
@pytest.mark.parametrize("shape", GEMM_SHAPES)
def test_fp32_reference_shapes(gpu, dn, golden, shape):
    M, N, K = shape
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 42)
    C = np.zeros(M * N, np.float32)
    dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.0, C, N))
    assert np.max(np.abs(C - golden[f"fp32_{M}x{N}x{K}"])) <= fp32_tol(K)


def test_fp32_alpha_beta(gpu, dn, golden):
    M, N, K = 32, 48, 64
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 43)
    C = np.zeros(M * N, np.float32)
    dn.check(dn.gemm_fp32(M, N, K, 2.0, A, K, B, N, 0.0, C, N))
    assert np.max(np.abs(C - golden["fp32_alpha2"])) <= fp32_tol(K)
    C = ref_uniform(M * N, 44)
    dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.5, C, N))
    assert np.max(np.abs(C - golden["fp32_beta05"])) <= fp32_tol(K)


def test_config1_host_and_device(gpu, dn, golden):
    torch = gpu
    M, N, K = 1, 4096, 4096
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 123)
    C = np.zeros(M * N, np.float32)
    dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.0, C, N))
    assert np.max(np.abs(C - golden["config1"])) <= fp32_tol(K)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.zeros(M * N, device="cuda")
    s = torch.cuda.current_stream()
    dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, K, N, N), dA, dB, dC, s))
    torch.cuda.synchronize()
    assert np.max(np.abs(dC.cpu().numpy() - golden["config1"])) <= fp32_tol(K)


@pytest.mark.parametrize("shape", C2_SHAPES)
def test_config2(gpu, dn, golden, shape):
    M, N, K = shape
    A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)
    dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.5, C, N))
    assert np.max(np.abs(C - golden[f"config2_{M}x{N}x{K}"])) <= fp32_tol(K)


def test_config2_device_api_deterministic(gpu, dn, golden):
    torch = gpu
    M, N, K = 7, 4093, 1024
    A, B, C0 = ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    outs = []
    for _ in range(3):
        dC = torch.from_numpy(C0.copy()).cuda()
        dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, K, N, N, 1.0, 0.5), dA, dB, dC,
                              torch.cuda.current_stream()))
        torch.cuda.synchronize()
        outs.append(dC.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))
    assert np.max(np.abs(outs[0] - golden[f"config2_{M}x{N}x{K}"])) <= fp32_tol(K)


@pytest.mark.parametrize("M", range(1, 9))
@pytest.mark.parametrize("N,K", [(1009, 1000), (33, 1023), (128, 7), (257, 4099), (200, 40000)])
def test_fp32_small_m_edges(gpu, dn, orc, M, N, K):
    A, B, C = ref_uniform(M * K, 1), ref_uniform(K * N, 2), ref_uniform(M * N, 3)
    ref = C.copy()
    orc.gemm_f32(M, N, K, 1.5, A, K, B, N, -0.25, ref, N)
    dn.check(dn.gemm_fp32(M, N, K, 1.5, A, K, B, N, -0.25, C, N))
    assert np.max(np.abs(C - ref)) <= fp32_tol(K)


def test_fp32_strides_unaligned_and_nan_c(gpu, dn, orc):
    torch = gpu
    M, N, K = 5, 300, 513
    lda, ldb, ldc = K + 3, N + 5, N + 7
    A = ref_uniform(M * lda, 4)
    Bbig = ref_uniform(K * ldb + 1, 5)
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(Bbig).cuda()[1:]            # 4-byte aligned only: scalar path
    dC = torch.full((M * ldc,), float("nan"), device="cuda")   # beta == 0 never reads C
    dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, lda, ldb, ldc), dA, dB, dC,
                          torch.cuda.current_stream()))
    torch.cuda.synchronize()
    ref = np.zeros(M * ldc, np.float32)
    orc.gemm_f32(M, N, K, 1.0, A, lda, np.ascontiguousarray(Bbig[1:]), ldb, 0.0, ref, ldc)
    got = dC.cpu().numpy().reshape(M, ldc)
    assert np.max(np.abs(got[:, :N] - ref.reshape(M, ldc)[:, :N])) <= fp32_tol(K)
    assert np.all(np.isnan(got[:, N:]))               # padding columns untouched


def cblas(dn):
    lib = ctypes.CDLL(dn.BLAS_PATH)
    lib.cblas_sgemm.argtypes = [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_void_p, ctypes.c_int,
                                                     ctypes.c_void_p, ctypes.c_int, ctypes.c_float,
                                                     ctypes.c_void_p, ctypes.c_int]
    lib.sgemm_.argtypes = [ctypes.c_void_p] * 13
    return lib


def cblas_operands(order, ta, tb, M, N, K):
    if order == 101:
        a_rows, a_cols = (K, M) if ta == 112 else (M, K)
        b_rows, b_cols = (N, K) if tb == 112 else (K, N)
        return a_rows, a_cols, b_rows, b_cols, a_cols, b_cols, N
    a_rows, a_cols = (M, K) if ta == 112 else (K, M)
    b_rows, b_cols = (K, N) if tb == 112 else (N, K)
    return a_rows, a_cols, b_rows, b_cols, a_cols, b_cols, M


@pytest.mark.parametrize("size", CBLAS_SIZES)
def test_cblas_against_reference(gpu, dn, golden, size):
    lib = cblas(dn)
    M, N, K = size
    for order in (101, 102):
        for ta in (111, 112):
            for tb in (111, 112):
                a_rows, a_cols, b_rows, b_cols, lda, ldb, ldc = cblas_operands(order, ta, tb, M, N, K)
                A = ref_uniform(a_rows * a_cols, 42)
                B = ref_uniform(b_rows * b_cols, 123)
                C = ref_uniform(M * N, 77)
                lib.cblas_sgemm(order, ta, tb, M, N, K, 1.0, A.ctypes.data, lda, B.ctypes.data,
                                ldb, 0.5, C.ctypes.data, ldc)
                exp = golden[f"cblas_{order}_{ta}_{tb}_{M}x{N}x{K}"]
                assert np.max(np.abs(C - exp)) <= fp32_tol(K), (order, ta, tb)
    A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)
    lib.cblas_sgemm(101, 111, 111, M, N, K, 2.5, A.ctypes.data, K, B.ctypes.data, N, -0.3,
                    C.ctypes.data, N)
    assert np.max(np.abs(C - golden[f"cblas_ab_{M}x{N}x{K}"])) <= K * 5e-5
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 123)
    C = np.zeros(M * N, np.float32)
    ta, tb = ctypes.c_char(b"N"), ctypes.c_char(b"N")
    m_, n_, k_ = ctypes.c_int(M), ctypes.c_int(N), ctypes.c_int(K)
    al, be = ctypes.c_float(1.0), ctypes.c_float(0.0)
    lda_, ldb_, ldc_ = ctypes.c_int(M), ctypes.c_int(K), ctypes.c_int(M)
    lib.sgemm_(*(ctypes.addressof(x) for x in (ta, tb, m_, n_, k_, al)), A.ctypes.data,
               ctypes.addressof(lda_), B.ctypes.data, ctypes.addressof(ldb_),
               ctypes.addressof(be), C.ctypes.data, ctypes.addressof(ldc_))
    assert np.max(np.abs(C - golden[f"fortran_{M}x{N}x{K}"])) <= fp32_tol(K)


# ------------------------------------------------ oneDNN entry (col-major) ---
COLMAJOR_CASES = [
    # M, N, K, transa, transb, lda_pad, ldb_pad, ldc_pad, alpha, beta, bias
    (4096, 1, 4096, "T", "N", 0, 0, 0, 1.0, 0.0, True),      # inner product, batch 1
    (1009, 7, 1024, "T", "N", 0, 0, 0, 1.0, 0.5, True),      # small batch, prime OC
    (2039, 3, 1024, "N", "N", 5, 0, 3, 0.75, 1.0, True),
    (257, 5, 96, "N", "T", 3, 1, 2, 1.0, 0.0, False),
    (300, 7, 128, "T", "T", 0, 4, 0, 1.0, -0.5, True),
    (64, 33, 40, "N", "N", 0, 0, 0, 1.0, 1.0, True),         # M > 8 rows in the row-major view
    (256, 256, 256, "N", "N", 0, 0, 0, 1.0, 0.0, True),
]


@pytest.mark.parametrize("case", COLMAJOR_CASES)
def test_sgemm_colmajor_matches_oracle(gpu, dn, orc, case):
    """dnnopt_sgemm_colmajor (host arrays) and dnnopt_cuda_sgemm_colmajor
    (device tensors) against the oracle's restatement of the oneDNN entry."""
    from tests.test_oracle_colmajor import operands
    torch = gpu
    M, N, K, ta, tb, pa, pb, pc, alpha, beta, with_bias = case
    A, lda, B, ldb, C, ldc = operands(M, N, K, ta, tb, pa, pb, pc)
    bias = ref_uniform(M, 5) if with_bias else None
    ref = C.copy()
    assert orc.sgemm_colmajor(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, ref, ldc, bias) == 0
    host = C.copy()
    dn.check(dn.sgemm_colmajor(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, host, ldc, bias))
    assert np.max(np.abs(host - ref)) <= fp32_tol(K)
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C))
    dbias = torch.from_numpy(bias).cuda() if with_bias else None
    s = torch.cuda.current_stream()
    dn.check(dn.cuda_sgemm_colmajor(ta, tb, M, N, K, alpha, dA, lda, dB, ldb, beta, dC, ldc, dbias, s))
    torch.cuda.synchronize()
    out = dC.cpu().numpy()
    assert np.max(np.abs(out - ref)) <= fp32_tol(K)
    # Padding between columns of C is left alone.
    for j in range(N):
        assert np.array_equal(out[j * ldc + M:(j + 1) * ldc], C[j * ldc + M:(j + 1) * ldc])


def test_host_entry_keeps_c_padding(gpu, dn, orc):
    """Host-pointer calls stage C's whole span (rows padded to ldc); with
    beta == 0 the padding must still come back unchanged."""
    M, N, K, ldc = 5, 257, 96, 260
    A, B = ref_uniform(M * K, 1), ref_uniform(K * N, 2)
    C = ref_uniform(M * ldc, 3)
    ref = C.copy()
    orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.0, ref, ldc)
    out = C.copy()
    dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.0, out, ldc))
    assert np.max(np.abs(out - ref)) <= fp32_tol(K)
    for m in range(M):
        assert np.array_equal(out[m * ldc + N:(m + 1) * ldc], C[m * ldc + N:(m + 1) * ldc])


def test_sgemm_colmajor_k0_and_overlapping_ldc(gpu, dn, orc):
    torch = gpu
    # K == 0: C scaled by beta (cleared for beta == 0, NaN included), bias added; bit-exact.
    M, N, ldc = 37, 5, 40
    for beta in (0.0, 1.0, 2.0):
        C = ref_uniform(ldc * N, 3)
        C[1] = np.nan if beta == 0.0 else C[1]
        bias = ref_uniform(M, 4)
        ref = C.copy()
        orc.sgemm_colmajor("N", "N", M, N, 0, 1.0, None, M, None, 1, beta, ref, ldc, bias)
        dC = torch.from_numpy(C).cuda()
        dn.check(dn.cuda_sgemm_colmajor("N", "N", M, N, 0, 1.0, None, M, None, 1, beta, dC, ldc,
                                        torch.from_numpy(bias).cuda(), torch.cuda.current_stream()))
        torch.cuda.synchronize()
        assert np.array_equal(dC.cpu().numpy().view(np.uint32), ref.view(np.uint32)), beta
    # ldc < M: the temporary-buffer path with its column-by-column copy-back.
    for (M, N, K, ldc, beta) in [(6, 4, 9, 4, 0.5), (20, 9, 33, 12, 0.0), (300, 3, 64, 128, 1.0)]:
        from tests.test_oracle_colmajor import operands
        A, lda, B, ldb, _, _ = operands(M, N, K, "N", "N")
        C = ref_uniform((N - 1) * ldc + M, 11)
        bias = ref_uniform(M, 12)
        ref = C.copy()
        orc.sgemm_colmajor("N", "N", M, N, K, 1.0, A, lda, B, ldb, beta, ref, ldc, bias)
        host = C.copy()
        dn.check(dn.sgemm_colmajor("N", "N", M, N, K, 1.0, A, lda, B, ldb, beta, host, ldc, bias))
        assert np.max(np.abs(host - ref)) <= fp32_tol(K), (M, N, K, ldc)


def test_cblas_256_all_orders(gpu, dn, orc):
    from tests.test_oracle_golden import cblas_by_oracle
    lib = cblas(dn)
    M = N = K = 256
    for order in (101, 102):
        for ta in (111, 112):
            for tb in (111, 112):
                a_rows, a_cols, b_rows, b_cols, lda, ldb, ldc = cblas_operands(order, ta, tb, M, N, K)
                A = ref_uniform(a_rows * a_cols, 42)
                B = ref_uniform(b_rows * b_cols, 123)
                C = ref_uniform(M * N, 77)
                ref = C.copy()
                cblas_by_oracle(orc, order, ta, tb, M, N, K, 1.0, A, lda, B, ldb, 0.5, ref, ldc)
                lib.cblas_sgemm(order, ta, tb, M, N, K, 1.0, A.ctypes.data, lda, B.ctypes.data,
                                ldb, 0.5, C.ctypes.data, ldc)
                assert np.max(np.abs(C - ref)) <= fp32_tol(K), (order, ta, tb)


@pytest.mark.parametrize("M,N,K,beta", [(5, 777, 1024, 0.5), (1, 4096, 4096, 0.0), (8, 300, 8000, -1.0),
                                         (3, 64, 30, 0.0),
                                         # register-resident dot form, 3-4 chunks per lane (M <= 2)
                                         (2, 4096, 4096, 0.5), (1, 1001, 3072, 1.0), (2, 37, 2052, 0.0),
                                         (1, 3, 4092, 0.5)])
def test_fp32_transposed_b_small_m(gpu, dn, orc, M, N, K, beta):
    """op(B) = B^T (B stored N x K): the dot-form kernels."""
    torch = gpu
    A, Bt, C0 = ref_uniform(M * K, 21), ref_uniform(N * K, 22), ref_uniform(M * N, 23)
    ref = C0.copy()
    orc.gemm_f32(M, N, K, 1.0, A, K, np.ascontiguousarray(Bt.reshape(N, K).T).ravel(), N, beta,
                 ref, N)
    dC = torch.from_numpy(C0.copy()).cuda()
    dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, K, K, N, 1.0, beta, trans_b=1),
                          torch.from_numpy(A).cuda(), torch.from_numpy(Bt).cuda(), dC,
                          torch.cuda.current_stream()))
    torch.cuda.synchronize()
    assert np.max(np.abs(dC.cpu().numpy() - ref)) <= fp32_tol(K)


@pytest.mark.parametrize("M,N,K,beta,ta,tb", [
    (9, 4096, 1024, 0.5, 0, 0), (16, 1009, 2048, 0.0, 0, 0), (33, 777, 300, 1.0, 0, 1),
    (64, 2048, 512, -0.5, 1, 0), (40, 130, 1000, 0.0, 1, 1), (128, 515, 96, 0.5, 0, 0),
    # N <= 64: 64-column tiles
    (200, 64, 300, 0.5, 0, 1), (37, 33, 129, 0.0, 1, 0), (16, 48, 1024, 1.0, 0, 0),
    # N <= 64 with >= 128 rows per SM: 128 x 64 tiles (conv3d's im2col GEMM)
    (20000, 64, 300, 0.5, 0, 1), (19000, 50, 129, 0.0, 1, 0), (20011, 37, 1000, 1.0, 0, 0),
    (19000, 64, 200, 0.0, 1, 1)])
def test_fp32_simt_small_m_bands(gpu, dn, orc, M, N, K, beta, ta, tb):
    """M from 9 up on the general SIMT kernel (16/32/64-row tiles, K split
    over a cluster), every transposition."""
    torch = gpu
    A, B, C0 = ref_uniform(M * K, 31), ref_uniform(K * N, 32), ref_uniform(M * N, 33)
    ref = C0.copy()
    orc.gemm_f32(M, N, K, 1.0, A, K, B, N, beta, ref, N)
    Ad = np.ascontiguousarray(A.reshape(M, K).T).ravel() if ta else A
    Bd = np.ascontiguousarray(B.reshape(K, N).T).ravel() if tb else B
    d = dn.desc(M, N, K, M if ta else K, K if tb else N, N, 1.0, beta, ta, tb)
    assert dn.plan_describe(dn.KIND_F32, d).startswith("gemm_simt")
    dC = torch.from_numpy(C0.copy()).cuda()
    dn.check(dn.cuda_gemm("f32", d, torch.from_numpy(Ad).cuda(), torch.from_numpy(Bd).cuda(), dC,
                          torch.cuda.current_stream()))
    torch.cuda.synchronize()
    assert np.max(np.abs(dC.cpu().numpy() - ref)) <= fp32_tol(K)


# ----------------------------------------------------------------- Conv3D ---
def _conv3d_shapes():
    from tests.test_oracle_conv3d import CONV3D_SHAPES
    # + a shape whose BF16 GEMM takes the tcgen05 kernel (K = 432, OC = 64, M = 1024),
    # + batch / stride / uneven padding with IC a multiple of 16 (the convert-once
    # input and 16-byte chunk im2col of the BF16 and INT8 paths)
    # + stride-1 shapes of the implicit tcgen05 conv: 32 / 64 / 128-byte
    # channel chunks (IC 32, 64, 96, 128 in INT8 and BF16), tiles ragged in
    # every dimension (batch, OW 11 and 130, OC 24 and 300: two channel tiles
    # with the filter streamed), asymmetric kernels and padding.
    return CONV3D_SHAPES + [(1, 16, 4, 16, 16, 64, 3, 3, 3, 1, 1, 1, 1, 1, 1),
                            (2, 32, 4, 9, 9, 24, 3, 3, 3, 2, 2, 2, 1, 1, 1),
                            (1, 48, 3, 7, 7, 16, 1, 3, 3, 1, 1, 1, 0, 1, 1),
                            (1, 64, 4, 14, 14, 64, 3, 3, 3, 1, 1, 1, 1, 1, 1),
                            (2, 32, 3, 9, 11, 24, 3, 3, 3, 1, 1, 1, 1, 1, 1),
                            (1, 96, 2, 6, 6, 300, 1, 3, 3, 1, 1, 1, 0, 1, 1),
                            (3, 128, 2, 5, 5, 40, 3, 1, 3, 1, 1, 1, 1, 0, 1),
                            (1, 16, 6, 7, 7, 16, 5, 3, 3, 1, 1, 1, 2, 1, 1),
                            (1, 32, 1, 2, 130, 32, 1, 1, 3, 1, 1, 1, 0, 0, 1),
                            # padded width 72: a window of all 3 x 3 taps would
                            # exceed 256 rows, so one window per filter row
                            (1, 32, 3, 4, 70, 32, 3, 3, 3, 1, 1, 1, 1, 1, 1)]


@pytest.mark.parametrize("p", _conv3d_shapes())
@pytest.mark.parametrize("precision", [0, 1, 2])
def test_conv3d_matches_oracle(gpu, dn, orc, p, precision):
    """dnnopt_conv3d (host arrays) and dnnopt_cuda_conv3d (device tensors)
    against the oracle: FP32 within 1e-5*K, BF16 within FP32 accumulation of
    the bf16 products (and the reference test's K*1e-2 of the exact result),
    INT8 bit for bit (deterministic quantisation, exact int32 sums)."""
    from tests.test_oracle_conv3d import conv3d_f64, conv3d_operands
    torch = gpu
    inp, flt, bias, n_out = conv3d_operands(p)
    K = p[1] * p[6] * p[7] * p[8]
    for post_op, b in ((0, None), (1, bias), (2, bias)):
        ref = np.zeros(n_out, np.float32)
        r64 = orc.conv3d(precision, p, inp, flt, b, ref, post_op, want64=True)
        host = np.full(n_out, np.nan, np.float32)
        dn.check(dn.conv3d(precision, p, inp, flt, b, host, post_op), "conv3d")
        dC = torch.full((n_out,), float("nan"), device="cuda")
        dn.check(dn.cuda_conv3d(precision, p, torch.from_numpy(inp).cuda(), torch.from_numpy(flt).cuda(),
                                None if b is None else torch.from_numpy(b).cuda(), dC, post_op,
                                torch.cuda.current_stream()), "cuda_conv3d")
        torch.cuda.synchronize()
        dev = dC.cpu().numpy()
        for got in (host, dev):
            if precision == 0:
                assert np.max(np.abs(got - ref)) <= fp32_tol(K), (p, post_op)
            elif precision == 1:
                assert np.max(np.abs(got - r64)) <= fp32_tol(K), (p, post_op)
                assert np.max(np.abs(got - conv3d_f64(p, inp, flt, b, post_op))) < K * 1e-2
            else:
                assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (p, post_op)


def test_saxpy(gpu, dn):
    X, Y = ref_uniform(1000, 1), ref_uniform(2000, 2)
    exp = Y.copy()
    exp[::2] = exp[::2] + np.float32(0.75) * X[:1000]
    dn.check(dn.saxpy(1000, 0.75, X, 1, Y, 2))
    assert np.max(np.abs(Y - exp)) <= 1e-6


# ------------------------------------------------------------------ INT8 ----
@pytest.mark.parametrize("shape", INT8_SHAPES + [(4, 11008, 4096)])
def test_int8_native_bitexact(gpu, dn, golden, shape):
    M, N, K = shape
    A, B = int8_uniform(M * K, 42), int8_uniform(N * K, 123)
    C = np.zeros(M * N, np.int32)
    dn.check(dn.gemm_int8_int8int8int32(M, N, K, A, K, B, K, C, N))
    key = "config3" if shape == (4, 11008, 4096) else f"s8_{M}x{N}x{K}"
    assert np.array_equal(C, golden[key])


def test_int8_edges_bitexact(gpu, dn, orc):
    torch = gpu
    for (M, N, K, lda, ldb, ldc, off) in [(1, 1009, 4096, 4096, 4096, 1009, 0),
                                          (7, 513, 300, 301, 305, 520, 1),
                                          (8, 64, 16, 16, 16, 64, 0),
                                          (12, 200, 777, 777, 777, 200, 0),
                                          (2, 5000, 127, 128, 127, 5000, 3),
                                          (8, 1000, 8192, 8192, 8192, 1000, 0),
                                          (3, 3001, 4112, 4112, 4128, 3001, 0),
                                          (6, 17, 64, 80, 64, 17, 0),
                                          # general dp4a tiles: split-K clusters, byte-wise
                                          # loads for unaligned rows, K below one word
                                          (100, 300, 1000, 1001, 1003, 300, 1),
                                          (64, 64, 4096, 4096, 4096, 64, 0),
                                          (200, 1000, 64, 64, 64, 1000, 0),
                                          (17, 33, 3, 3, 3, 33, 0),
                                          (130, 70, 1730, 1732, 1736, 72, 0)]:
        A = int8_uniform(M * lda, 7)
        Bb = int8_uniform(N * ldb + off, 8)
        ref = np.zeros(M * ldc, np.int32)
        orc.gemm_s8s32(M, N, K, A, lda, np.ascontiguousarray(Bb[off:]), ldb, ref, ldc)
        dA = torch.from_numpy(A).cuda()
        dB = torch.from_numpy(Bb).cuda()[off:]
        dC = torch.zeros(M * ldc, dtype=torch.int32, device="cuda")
        dn.check(dn.cuda_gemm("s8s32", dn.desc(M, N, K, lda, ldb, ldc), dA, dB, dC,
                              torch.cuda.current_stream()))
        torch.cuda.synchronize()
        got = dC.cpu().numpy().reshape(M, ldc)[:, :N]
        assert np.array_equal(got, ref.reshape(M, ldc)[:, :N]), (M, N, K)


# Both dot-form kernels with A in registers, forced through autotune-cache
# entries: the bulk-copy ring (dense rows: one copy per stage; padded rows: one
# per row) and the register-load form, on int8 (bit-exact) and on FP32 / BF16
# with B stored N x K.
@pytest.mark.parametrize("kernel", [7, 11])
@pytest.mark.parametrize("case", [
    ("s8s32", 4, 11008, 4096, 4096, 30), ("s8s32", 1, 1009, 4096, 4096, 7),
    ("s8s32", 8, 1000, 8192, 8192, 300), ("s8s32", 3, 3001, 4112, 4128, 150),
    ("s8s32", 6, 17, 64, 64, 5), ("s8s32", 2, 777, 512, 528, 296),
    ("f32", 3, 1000, 1024, 1024, 296), ("f32", 8, 257, 2048, 2052, 64),
    ("bf16f32", 5, 999, 2048, 2048, 148), ("bf16f32", 2, 4096, 4096, 4104, 296)])
def test_rows_kernels_forced(gpu, dn, orc, tmp_path, kernel, case):
    kind_name, M, N, K, ldb, grid = case
    torch = gpu
    mt = 1 if M <= 1 else 2 if M <= 2 else 4 if M <= 4 else 8
    kind = {"s8s32": dn.KIND_S8S32, "f32": dn.KIND_F32, "bf16f32": dn.KIND_BF16F32}[kind_name]
    _force_plan(dn, tmp_path, f"rows_{kernel}_{kind_name}_{M}_{N}.bin", kind, M, N, K, K, ldb, N, 0, 1, 1,
                (kernel, grid, 0, mt))
    s = torch.cuda.current_stream()
    if kind_name == "s8s32":
        A, Bb = int8_uniform(M * K, 17), int8_uniform(N * ldb, 18)
        ref = np.zeros(M * N, np.int32)
        orc.gemm_s8s32(M, N, K, A, K, Bb, ldb, ref, N)
        dC = torch.zeros(M * N, dtype=torch.int32, device="cuda")
        dn.check(dn.cuda_gemm("s8s32", dn.desc(M, N, K, K, ldb, N), torch.from_numpy(A).cuda(),
                              torch.from_numpy(Bb).cuda(), dC, s))
        torch.cuda.synchronize()
        assert np.array_equal(dC.cpu().numpy(), ref)
        return
    if kind_name == "f32":
        A, Bb, C0 = ref_uniform(M * K, 17), ref_uniform(N * ldb, 18), ref_uniform(M * N, 19)
        Bt = np.ascontiguousarray(Bb.reshape(N, ldb)[:, :K].T).reshape(-1)
        ref = C0.copy()
        orc.gemm_f32(M, N, K, 1.0, A, K, Bt, N, 0.5, ref, N)
        dC = torch.from_numpy(C0.copy()).cuda()
        dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, K, ldb, N, 1.0, 0.5, 0, 1), torch.from_numpy(A).cuda(),
                              torch.from_numpy(Bb).cuda(), dC, s))
        torch.cuda.synchronize()
        assert np.max(np.abs(dC.cpu().numpy() - ref)) <= fp32_tol(K)
        return
    rng = np.random.default_rng(20)
    Ab = bf16_bits(rng.standard_normal(M * K).astype(np.float32))
    Bb = bf16_bits(rng.standard_normal(N * ldb).astype(np.float32))
    Bt = np.ascontiguousarray(Bb.reshape(N, ldb)[:, :K].T).reshape(-1)
    ref = np.zeros(M * N, np.float32)
    r64 = orc.gemm_bf16f32(M, N, K, 1.0, Ab, K, Bt, N, 0.0, ref, N, want64=True)
    dC = torch.zeros(M * N, device="cuda")
    dn.check(dn.cuda_gemm("bf16f32", dn.desc(M, N, K, K, ldb, N, 1.0, 0.0, 0, 1),
                          torch.from_numpy(Ab.view(np.int16)).cuda(), torch.from_numpy(Bb.view(np.int16)).cuda(),
                          dC, s))
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    assert np.max(np.abs(got - r64)) <= 2e-6 * K * max(1.0, float(np.max(np.abs(r64))))


@pytest.mark.parametrize("shape", [(1, 128, 64), (7, 13, 5), (5, 7, 11), (4, 1009, 1024),
                                   (8, 4096, 512), (32, 48, 64), (13, 17, 19)])
def test_int8_fp32_api_bitexact(gpu, dn, orc, shape):
    M, N, K = shape
    for alpha, beta in [(1.0, 0.0), (1.5, 0.5)]:
        A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 43), ref_uniform(M * N, 44)
        ref = C.copy()
        orc.gemm_int8_f32api(M, N, K, alpha, A, K, B, N, beta, ref, N)
        dn.check(dn.gemm_int8(M, N, K, alpha, A, K, B, N, beta, C, N))
        assert np.array_equal(C.view(np.uint32), ref.view(np.uint32)), (alpha, beta)
        Cf = np.zeros(M * N, np.float32)
        orc.gemm_f32(M, N, K, alpha, A, K, B, N, 0.0, Cf, N)
        if beta == 0.0:
            assert np.max(np.abs(C - Cf)) < K * 2e-2   # reference test bound


# ------------------------------------------------------------------ BF16 ----
def _bf16_case(dn, orc, torch, M, N, K, alpha=1.0, beta=0.0, ldc=None, seed=42, b_layout="kn"):
    """b_layout: "kn" (B is K x N, ldb = N), "nk" (B is N x K, trans_b, ldb = K),
    "kn_pad1" (K x N with ldb = N + 1: rows not 16-byte aligned)."""
    ldc = ldc or N
    A32 = np.random.default_rng(seed).standard_normal(M * K).astype(np.float32)
    B32 = np.random.default_rng(seed + 81).standard_normal(K * N).astype(np.float32)
    A, B = bf16_bits(A32), bf16_bits(B32)
    C0 = ref_uniform(M * ldc, 5)
    ref = C0.copy()
    ref64 = orc.gemm_bf16f32(M, N, K, alpha, A, K, B, N, beta, ref, ldc, want64=True)
    if b_layout == "nk":
        Bdev, ldb, tb = np.ascontiguousarray(B.reshape(K, N).T).reshape(-1), K, 1
    elif b_layout == "kn_pad1":
        Bp = np.zeros((K, N + 1), np.uint16)
        Bp[:, :N] = B.reshape(K, N)
        Bdev, ldb, tb = Bp.reshape(-1), N + 1, 0
    else:
        Bdev, ldb, tb = B, N, 0
    dA = torch.from_numpy(A.view(np.int16)).cuda()
    dB = torch.from_numpy(Bdev.view(np.int16)).cuda()
    dC = torch.from_numpy(C0.copy()).cuda()
    dn.check(dn.cuda_gemm("bf16f32", dn.desc(M, N, K, K, ldb, ldc, alpha, beta, 0, tb), dA, dB, dC,
                          torch.cuda.current_stream()))
    torch.cuda.synchronize()
    got = dC.cpu().numpy().reshape(M, ldc)
    r64 = ref64.reshape(M, N)
    err = np.abs(got[:, :N] - r64)
    assert np.all(err <= 1e-2 * np.maximum(1.0, np.abs(r64)))        # BASELINE bound
    assert np.max(err) <= 2e-6 * K * max(1.0, float(np.max(np.abs(r64))))  # FP32 accumulation
    if ldc > N:
        assert np.array_equal(got[:, N:], C0.reshape(M, ldc)[:, N:])
    return got


# General tcgen05 GEMM (both operands by TMA): M > 8 int8 (kind::i8, exact
# int32 sums, so bit-identical to the oracle) and BF16 with N > 256
# (kind::f16), B as [K, N] (MN-major operand) or [N, K] (K-major).  Cases cover
# one and many 128 x 256 tiles, K split across CTAs (ticketed in-order
# reduction), K not a multiple of the 128-byte K-block (TMA zero fill), M and
# N not multiples of the tile, padded ldc, beta != 0.
@pytest.mark.parametrize("M,N,K,ldc", [
    (2048, 2048, 2048, None), (64, 4096, 4096, None), (300, 1000, 4096, 1004), (129, 257, 160, None),
    (9, 4096, 1024, None), (200, 1000, 64, None), (1000, 64, 1728, None), (777, 333, 4112, None)])
def test_gemm_tc_int8_bitexact(gpu, dn, orc, M, N, K, ldc):
    torch = gpu
    ldc = ldc or N
    d = dn.desc(M, N, K, K, K, ldc)
    assert dn.plan_describe(dn.KIND_S8S32, d).startswith("gemm_tcgen05"), dn.plan_describe(dn.KIND_S8S32, d)
    A, B = int8_uniform(M * K, 31), int8_uniform(N * K, 32)
    ref = np.zeros(M * ldc, np.int32)
    orc.gemm_s8s32(M, N, K, A, K, B, K, ref, ldc)
    dC = torch.full((M * ldc,), 7, dtype=torch.int32, device="cuda")
    for _ in range(2):   # the split-K tickets must be left at zero for the second call
        dn.check(dn.cuda_gemm("s8s32", d, torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), dC,
                              torch.cuda.current_stream()))
        torch.cuda.synchronize()
        got = dC.cpu().numpy().reshape(M, ldc)
        assert np.array_equal(got[:, :N], ref.reshape(M, ldc)[:, :N]), (M, N, K)
        assert np.all(got[:, N:] == 7)


@pytest.mark.parametrize("M,N,K", [(64, 512, 1024), (130, 300, 256), (1000, 4096, 512)])
def test_gemm_tc_int8_fp32_api_bitexact(gpu, dn, orc, M, N, K):
    """The FP32-API gemm_int8 (absmax quantisation) on the tcgen05 kernel's
    dequantising epilogue, bit-exact against the oracle's restatement."""
    for alpha, beta in [(1.0, 0.0), (1.5, 0.5)]:
        A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 43), ref_uniform(M * N, 44)
        ref = C.copy()
        orc.gemm_int8_f32api(M, N, K, alpha, A, K, B, N, beta, ref, N)
        dn.check(dn.gemm_int8(M, N, K, alpha, A, K, B, N, beta, C, N))
        assert np.array_equal(C.view(np.uint32), ref.view(np.uint32)), (M, N, K, alpha, beta)


@pytest.mark.parametrize("M,N,K,alpha,beta,ldc,layout", [
    (64, 4096, 4096, 1.0, 0.0, None, "kn"), (16, 4096, 4096, 1.0, 0.0, None, "kn"),
    (300, 1000, 512, 1.0, 0.5, None, "kn"), (200, 600, 1024, 2.0, 0.0, None, "nk"),
    (9, 4093, 768, 1.0, -1.0, 4100, "nk"), (1024, 1024, 1024, 1.0, 0.0, None, "kn"),
    (129, 320, 104, 0.5, 0.25, None, "kn"), (513, 2000, 2048, 1.0, 0.0, None, "nk")])
def test_gemm_tc_bf16(gpu, dn, orc, M, N, K, alpha, beta, ldc, layout):
    ldc_ = ldc or N
    ldb = K if layout == "nk" else N
    d = dn.desc(M, N, K, K, ldb, ldc_, alpha, beta, 0, 1 if layout == "nk" else 0)
    assert dn.plan_describe(dn.KIND_BF16F32, d).startswith("gemm_tcgen05"), dn.plan_describe(dn.KIND_BF16F32, d)
    _bf16_case(dn, orc, gpu, M, N, K, alpha, beta, ldc, b_layout=layout)


def test_bf16_config4_full(gpu, dn, orc):
    d = dn.desc(65536, 64, 256, 256, 64, 64)
    assert dn.plan_describe(dn.KIND_BF16F32, d) == "gemm_bf16_tcgen05"
    _bf16_case(dn, orc, gpu, 65536, 64, 256)


@pytest.mark.parametrize("M,N,K,alpha,beta,ldc", [
    (128, 64, 256, 1.0, 0.0, None), (200, 64, 256, 1.0, 0.0, None), (1000, 16, 64, 2.0, 0.0, None),
    (333, 48, 100, 1.0, 0.5, None), (4096, 256, 128, 0.5, 0.0, None), (257, 128, 320, 1.0, -1.0, 132),
    (129, 80, 8, 1.0, 0.0, None), (9, 64, 256, 1.0, 0.0, None),
    # One and two waves of 128-row tiles on 148 SMs.
    (18944, 64, 256, 1.0, 0.5, None), (37888, 48, 64, 1.0, 0.0, None),
    # A partial last round of tiles (one and two CTAs per SM), ragged last tile.
    (25600, 48, 320, 1.0, 0.0, None), (25563, 64, 256, 1.0, 0.5, None), (51195, 64, 128, 2.0, 0.0, None)])
def test_bf16_tcgen05_shapes(gpu, dn, orc, M, N, K, alpha, beta, ldc):
    _bf16_case(dn, orc, gpu, M, N, K, alpha, beta, ldc)


# B operand paths of the tcgen05 kernel: MN-major TMA (1-4 chunks of 64
# columns, ragged N), K-major TMA (trans_b) and the element gather (B rows not
# 16-byte aligned).
@pytest.mark.parametrize("M,N,K,beta,b_layout", [
    (1000, 40, 256, 0.0, "kn"), (777, 200, 192, 0.5, "kn"), (512, 256, 64, 0.0, "kn"),
    (300, 24, 136, 0.0, "kn"), (4096, 64, 256, 0.0, "nk"), (333, 48, 104, 0.5, "nk"),
    (257, 200, 64, 0.0, "nk"), (2000, 64, 256, 0.0, "kn_pad1"), (129, 36, 72, 0.5, "kn_pad1"),
    # deep K: B does not fit shared memory whole; aligned operands stream
    # through the general tcgen05 GEMM, unaligned ones run K in chunks
    # accumulating into C
    (2000, 64, 1728, 0.5, "nk"), (1500, 128, 2056, 0.0, "kn"), (777, 200, 1032, 0.5, "kn_pad1")])
def test_bf16_tcgen05_b_layouts(gpu, dn, orc, M, N, K, beta, b_layout):
    ldb = {"kn": N, "nk": K, "kn_pad1": N + 1}[b_layout]
    d = dn.desc(M, N, K, K, ldb, N, 1.0, beta, 0, int(b_layout == "nk"))
    want = "gemm_tcgen05" if K > 1024 and b_layout != "kn_pad1" else "gemm_bf16_tcgen05"
    assert dn.plan_describe(dn.KIND_BF16F32, d).split(" ")[0] == want
    _bf16_case(dn, orc, gpu, M, N, K, 1.0, beta, b_layout=b_layout)


@pytest.mark.parametrize("shape", [(1, 4096, 512), (7, 1009, 1024), (8, 64, 256), (65, 300, 77),
                                   (300, 300, 300)])
def test_bf16_other_paths(gpu, dn, orc, shape):
    M, N, K = shape
    _bf16_case(dn, orc, gpu, M, N, K, 1.0, 0.25)


@pytest.mark.parametrize("shape", [(1, 4096, 4096), (8, 1000, 2048), (2, 300, 8192), (5, 77, 96),
                                   (3, 4096, 4096), (12, 500, 256)])
def test_bf16_transposed_b(gpu, dn, orc, shape):
    """B stored N x K (weights as [out, in]): the register-resident dot form
    for M <= 8 with aligned rows, the SIMT kernel otherwise."""
    M, N, K = shape
    d = dn.desc(M, N, K, K, K, N, 1.0, 0.25, 0, 1)
    if M <= 8:
        assert dn.plan_describe(dn.KIND_BF16F32, d).startswith("gemv_rows_dot")
    _bf16_case(dn, orc, gpu, M, N, K, 1.0, 0.25, b_layout="nk")


@pytest.mark.parametrize("shape", GEMM_SHAPES)
def test_bf16_fp32_api(gpu, dn, orc, golden, shape):
    M, N, K = shape
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 42)
    C = np.zeros(M * N, np.float32)
    dn.check(dn.gemm_bf16(M, N, K, 1.0, A, K, B, N, 0.0, C, N))
    assert np.max(np.abs(C - golden[f"fp32_{M}x{N}x{K}"])) < K * 2e-3     # reference bound
    ref = np.zeros(M * N, np.float32)
    r64 = orc.gemm_bf16f32(M, N, K, 1.0, bf16_bits(A), K, bf16_bits(B), N, 0.0, ref, N,
                           want64=True)
    assert np.max(np.abs(C - r64)) <= 1e-5 * K


# ------------------------------------------------------------------- FP8 ----
def test_fp8_reference_codec_api(gpu, dn, orc, golden):
    M, N, K = 5, 37, 64
    enc4 = lambda x: orc.table("refe4m3", "from_f32", x)  # noqa: E731
    enc5 = lambda x: orc.table("refe5m2", "from_f32", x)  # noqa: E731
    A4, A5, B5 = enc4(ref_uniform(M * K, 42)), enc5(ref_uniform(M * K, 42)), enc5(ref_uniform(K * N, 123))
    C = np.zeros(M * N, np.float32)
    dn.check(dn.gemm_fp8_e4m3(M, N, K, 1.0, A4, K, B5, N, 0.0, C, N))
    assert np.max(np.abs(C - golden["fp8_e4m3_5x37x64"])) <= fp32_tol(K)
    C = np.zeros(M * N, np.float32)
    dn.check(dn.gemm_fp8_e5m2(M, N, K, 1.0, A5, K, B5, N, 0.0, C, N))
    assert np.max(np.abs(C - golden["fp8_e5m2_5x37x64"])) <= fp32_tol(K)
    # gemm_fp8 (FP32 API): the reference's FP8-hardware branch = encode, then e4m3 GEMM.
    for (M, N, K) in [(5, 37, 64), (33, 70, 90)]:
        A, B = ref_uniform(M * K, 1), ref_uniform(K * N, 2)
        ref = np.zeros(M * N, np.float32)
        orc.gemm_refe4m3_e5m2(M, N, K, 1.0, enc4(A), K, enc5(B), N, 0.0, ref, N)
        C = np.zeros(M * N, np.float32)
        dn.check(dn.gemm_fp8(M, N, K, 1.0, A, K, B, N, 0.0, C, N))
        assert np.max(np.abs(C - ref)) <= fp32_tol(K)


def e4m3_problem(orc, M, N, K, seed_a=42, seed_w=123):
    A = bf16_bits(np.random.default_rng(seed_a).standard_normal(M * K).astype(np.float32))
    W = (np.random.default_rng(seed_w).standard_normal(N * K) * 0.02).astype(np.float32)
    q, s = orc.quantize_e4m3_rows(N, K, W, K)
    return A, q, s


def check_e4m3(got_bits, ref64):
    got = bf16_to_f32(got_bits).astype(np.float64)
    err = np.abs(got - ref64)
    assert np.all(err <= 2.0 ** -7 * np.abs(ref64) + 1e-4 * np.max(np.abs(ref64)))


@pytest.mark.parametrize("shape", [(8, 512, 1024), (1, 300, 8192), (3, 1000, 1000), (8, 28672, 8192),
                                   (16, 256, 512), (20, 64, 96)])
def test_e4m3_decode_ffn(gpu, dn, orc, shape):
    torch = gpu
    M, N, K = shape
    A, q, s = e4m3_problem(orc, M, N, K)
    C = np.zeros(M * N, np.uint16)
    ref64 = orc.gemm_e4m3bf16(M, N, K, A, K, q, K, s, C, N)
    dA = torch.from_numpy(A.view(np.int16)).cuda()
    dW = torch.from_numpy(q).cuda()
    ds = torch.from_numpy(s).cuda()
    dC = torch.zeros(M * N, dtype=torch.int16, device="cuda")
    dn.check(dn.cuda_gemm("e4m3bf16", dn.desc(M, N, K, K, K, N), dA, dW, dC,
                          torch.cuda.current_stream(), scale=ds))
    torch.cuda.synchronize()
    check_e4m3(dC.cpu().numpy().view(np.uint16), ref64)
    # Host API on a small case.
    if M * N <= 8192:
        Ch = np.zeros(M * N, np.uint16)
        dn.check(dn.gemm_e4m3_bf16(M, N, K, A, K, q, K, s, Ch, N))
        check_e4m3(Ch, ref64)


# ------------------------------------------- fused all-gather, one GPU ----
def test_peer_wait_times_out_and_recovers(gpu, dn):
    """A flag that nothing sets: the bounded wait gives up after its limit,
    the stream reports KERNEL_TIMEOUT, and the device keeps working."""
    torch = gpu
    flags = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream()
    dn.check(dn.cuda_peer_wait(flags, 2, 1, 200000, s))         # 0.2 s limit
    assert dn.stream_status(s) == dn.KERNEL_TIMEOUT
    assert dn.stream_status(s) == dn.SUCCESS                     # cleared
    flags[1] = 1
    dn.check(dn.cuda_peer_wait(flags, 2, 1, 200000, s))
    assert dn.stream_status(s) == dn.SUCCESS
    flags[0] = 5                                                 # a later epoch also passes
    dn.check(dn.cuda_peer_wait(flags, 2, 1, 200000, s))
    assert dn.stream_status(s) == dn.SUCCESS


@pytest.mark.parametrize("M,N,K", [(8, 28672, 8192), (3, 1024, 1024)])
def test_fused_allgather_single_rank(gpu, dn, orc, M, N, K):
    """world = 1: the fused entry point writes the same bits as the plain
    e4m3 GEMM into buffer (call & 1), raises its own flag to the call number
    and advances the device-side counter -- eagerly and from a CUDA graph
    replayed with unchanged arguments."""
    torch = gpu
    from dnnopt_b200.sharded import _cuda_view
    A, q, s = e4m3_problem(orc, M, N, K)
    dA = torch.from_numpy(A.view(np.int16)).cuda()
    dW, ds = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    st = torch.cuda.Stream()
    plain = torch.zeros(M * N, dtype=torch.int16, device="cuda")
    dn.check(dn.cuda_gemm("e4m3bf16", dn.desc(M, N, K, K, K, N), dA, dW, plain, st, scale=ds))
    out_bytes = 8 * N * 2
    base = dn.peer_alloc(256 + 2 * out_bytes)
    try:
        ag = dn.AllGatherDesc()
        ag.world, ag.rank = 1, 0
        ag.out[0], ag.flags[0], ag.seq, ag.out_stride = base + 256, base, base + 64, out_bytes
        d = dn.desc(M, N, K, K, K, N)
        words = _cuda_view(base, (128,)).view(torch.int32)      # flags at 0, counter at 64 bytes
        bufs = [_cuda_view(base + 256 + p * out_bytes, (M * N,)) for p in (0, 1)]
        with torch.cuda.stream(st):
            for call in (1, 2, 3):
                dn.check(dn.cuda_gemm_e4m3bf16_allgather(d, dA, dW, ds, ag, st))
                assert dn.stream_status(st) == dn.SUCCESS
                assert torch.equal(bufs[call & 1], plain), call
                assert words[0].item() == call and words[16].item() == call
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                dn.check(dn.cuda_gemm_e4m3bf16_allgather(d, dA, dW, ds, ag, st))
                dn.check(dn.cuda_gemm_e4m3bf16_allgather(d, dA, dW, ds, ag, st))
            bufs[0].zero_(); bufs[1].zero_()
            st.synchronize()
            start = words[16].item()
            graph.replay()
            graph.replay()
            assert dn.stream_status(st) == dn.SUCCESS
            assert words[16].item() == start + 4 and words[0].item() == start + 4
            assert torch.equal(bufs[0], plain) and torch.equal(bufs[1], plain)
            del graph
    finally:
        torch.cuda.synchronize()
        dn.peer_free(base)


# -------------------------------------------------------- runtime paths ----
def test_plan_selection_on_device(gpu, dn):
    assert dn.plan_describe(dn.KIND_F32, dn.desc(1, 4096, 4096, 4096, 4096, 4096)).startswith(
        "gemv_kn_splitk mt=1 vec4=1 splits=16")
    assert dn.plan_describe(dn.KIND_S8S32, dn.desc(4, 11008, 4096, 4096, 4096, 11008)).startswith(
        "gemv_rows_dot mt=4 vec=1")


@pytest.mark.parametrize("splits", [2, 5, 8, 16])
def test_cluster_variant_forced(gpu, dn, orc, tmp_path, splits):
    """The cluster (DSMEM-reduction) variant, forced through an autotune-cache
    entry, against the oracle on a prime-N shape and an aligned shape."""
    for (M, N, K, vec) in [(3, 2039, 1024, 0), (8, 1024, 2048, 1)]:
        kchunk = ((K + splits - 1) // splits + 7) // 8 * 8
        se = (K + kchunk - 1) // kchunk
        mt = 1 if M <= 1 else 2 if M <= 2 else 4 if M <= 4 else 8
        h = plan_key(0, M, N, K, K, N, N, 0, 0, vec)
        path = tmp_path / f"cl_{splits}_{M}.bin"
        path.write_bytes(plan_file_bytes([(h, (6, se, kchunk, mt))]))
        assert dn.lib.dnnopt_autotune_load(str(path).encode()) == 1
        d = dn.desc(M, N, K, K, N, N, 1.0, 0.5)
        assert dn.plan_describe(dn.KIND_F32, d).startswith(("gemv_kn_", "gemv_panel"))  # heuristic view
        A, B, C = ref_uniform(M * K, 5), ref_uniform(K * N, 6), ref_uniform(M * N, 7)
        ref = C.copy()
        orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.5, ref, N)
        dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.5, C, N))
        assert np.max(np.abs(C - ref)) <= fp32_tol(K), (M, N, K, splits)


def _force_plan(dn, tmp_path, name, kind, M, N, K, lda, ldb, ldc, ta, tb, vec, entry):
    """Load an autotune-cache file holding one plan for this exact call."""
    h = plan_key(kind, M, N, K, lda, ldb, ldc, ta, tb, vec)
    path = tmp_path / name
    path.write_bytes(plan_file_bytes([(h, tuple(entry))]))
    assert dn.lib.dnnopt_autotune_load(str(path).encode()) == 1


# Column-slab kernel through a forced plan: the sweep shapes (FP32 now plans
# row panels for them), and shapes outside its heuristic range (tiny N, K over
# several 1024-row passes, K not a multiple of the 32-row step, transposed A,
# padded C).
@pytest.mark.parametrize("M,N,K,alpha,beta,ta,ldc,force", [
    (2, 1009, 1024, 1.0, 0.5, 0, None, 8), (7, 4093, 1024, 1.0, 0.5, 0, None, 16),
    (5, 2039, 1000, 2.0, 0.0, 0, None, 16), (8, 600, 2048, 1.0, -1.0, 0, 604, 8),
    (1, 7, 5, 1.0, 0.5, 0, None, 8), (3, 100, 3000, 1.0, 0.25, 0, None, 8),
    (4, 520, 1030, 0.5, 0.5, 1, None, 8), (6, 9000, 33, 1.0, 0.0, 0, None, 8),
    (1, 1024, 4097, 1.0, 0.5, 1, 1030, 8), (1, 7, 5, 1.0, 0.5, 0, None, 16),
    (3, 100, 3000, 1.0, 0.25, 0, None, 16), (7, 4093, 1024, 1.0, 0.5, 1, 4100, 16),
    (8, 1030, 2000, 1.0, 0.0, 0, None, 16)])
def test_slab_kernel(gpu, dn, orc, tmp_path, M, N, K, alpha, beta, ta, ldc, force):
    """force = 0: heuristic plan (must be the slab kernel); 8 / 16: slab width
    forced through an autotune-cache entry."""
    ldc = ldc or N
    lda = M if ta else K
    mt = 1 if M <= 1 else 2 if M <= 2 else 4 if M <= 4 else 8
    vec = 1 if N % 4 == 0 else 0
    if force:
        _force_plan(dn, tmp_path, f"slab_{M}_{N}_{K}_{force}.bin", 0, M, N, K, lda, N, ldc, ta, 0, vec,
                    (9, force, 0, mt))
    else:
        assert dn.plan_describe(dn.KIND_F32, dn.desc(M, N, K, lda, N, ldc, alpha, beta, ta, 0)) \
            .startswith(f"gemv_kn_slab mt={mt} w=")
    A, B = ref_uniform(M * K, 11), ref_uniform(K * N, 12)   # A is K x M when ta
    C0 = ref_uniform(M * ldc, 13)
    Ar = np.ascontiguousarray(A.reshape(K, M).T).reshape(-1) if ta else A
    ref_full = C0.reshape(M, ldc).copy()
    tmp = ref_full[:, :N].copy().reshape(-1)
    orc.gemm_f32(M, N, K, alpha, Ar, K, B, N, beta, tmp, N)
    ref_full[:, :N] = tmp.reshape(M, N)
    dA, dB, dC = (gpu.from_numpy(x).cuda() for x in (A, B, C0.copy()))
    dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, lda, N, ldc, alpha, beta, ta, 0), dA, dB, dC,
                          gpu.cuda.current_stream()))
    gpu.cuda.synchronize()
    got = dC.cpu().numpy().reshape(M, ldc)
    assert np.max(np.abs(got[:, :N] - ref_full[:, :N])) <= fp32_tol(K), (M, N, K)
    assert np.array_equal(got[:, N:], C0.reshape(M, ldc)[:, N:])


# Row-panel kernel (FP32, B K x N): heuristic shapes, then every panel width
# and K-range count forced through an autotune-cache entry on prime N, K not a
# multiple of the 32-row stage, K ranges that leave the last CTA short, M = 1..8,
# transposed A, padded C, beta = 0 over NaN, and a B base that is only 4-byte
# aligned (every row segment then starts mid-chunk).
PANEL_CASES = [
    (2, 1009, 1024, 1.0, 0.5, 0, None, 0, 0, 0), (7, 4093, 1024, 1.0, 0.5, 0, None, 0, 0, 0),
    (5, 2039, 1000, 2.0, 0.0, 0, None, 0, 0, 0), (8, 600, 2048, 1.0, -1.0, 0, 604, 0, 0, 0),
    (1, 4093, 1024, 1.0, 0.0, 0, None, 0, 0, 0), (3, 513, 777, 0.5, 0.25, 1, 520, 0, 0, 1),
]
for _w in (64, 128):
    for _s in (1, 2, 4, 8):
        PANEL_CASES += [(7, 1031, 999, 1.0, 0.5, 0, None, _w, _s, 0),
                        (4, 300, 520, 1.5, 0.0, 1, 301, _w, _s, 1),
                        (8, 2039, 1024, 1.0, 0.5, 0, 2048, _w, _s, 1)]
PANEL_CASES += [(6, 9000, 33, 1.0, 0.5, 0, None, 128, 1, 0), (1, 5, 70, 1.0, 0.5, 0, None, 128, 2, 0),
                (2, 4096, 2048, 1.0, 0.5, 0, None, 128, 8, 1), (5, 131, 4096, 1.0, 0.5, 1, None, 128, 8, 0)]


@pytest.mark.parametrize("M,N,K,alpha,beta,ta,ldc,w,splits,boff", PANEL_CASES)
def test_panel_kernel(gpu, dn, orc, tmp_path, M, N, K, alpha, beta, ta, ldc, w, splits, boff):
    """w = 0: heuristic plan (must be the panel kernel); else (w, splits)
    forced.  boff = 1 offsets B's base by one float."""
    ldc = ldc or N
    lda = M if ta else K
    mt = 1 if M <= 1 else 2 if M <= 2 else 4 if M <= 4 else 8
    Bbuf = ref_uniform(K * N + 1, 12)
    Bhost = Bbuf[boff:boff + K * N]
    vec = 1 if (N % 4 == 0 and boff == 0) else 0
    d = dn.desc(M, N, K, lda, N, ldc, alpha, beta, ta, 0)
    if w:
        _force_plan(dn, tmp_path, f"panel_{M}_{N}_{K}_{w}_{splits}_{boff}.bin", 0, M, N, K, lda, N, ldc, ta,
                    0, vec, (10, w, splits, mt))
    else:
        assert dn.plan_describe(dn.KIND_F32, d).startswith(f"gemv_panel mt={mt} w="), (M, N, K)
    A = ref_uniform(M * K, 11)   # K x M when ta
    C0 = ref_uniform(M * ldc, 13)
    if beta == 0.0:
        C0[::3] = np.nan         # never read when beta == 0
    Ar = np.ascontiguousarray(A.reshape(K, M).T).reshape(-1) if ta else A
    tmp = np.ascontiguousarray(C0.reshape(M, ldc)[:, :N]).reshape(-1).copy()
    tmp = np.nan_to_num(tmp) if beta == 0.0 else tmp
    orc.gemm_f32(M, N, K, alpha, Ar, K, Bhost.copy(), N, beta, tmp, N)
    dA, dC = gpu.from_numpy(A).cuda(), gpu.from_numpy(C0.copy()).cuda()
    dBbuf = gpu.from_numpy(Bbuf).cuda()
    dB = dBbuf[boff:boff + K * N]
    dn.check(dn.cuda_gemm("f32", d, dA, dB, dC, gpu.cuda.current_stream()))
    gpu.cuda.synchronize()
    got = dC.cpu().numpy().reshape(M, ldc)
    assert np.max(np.abs(got[:, :N] - tmp.reshape(M, N))) <= fp32_tol(K), (M, N, K, w, splits)
    assert np.array_equal(got[:, N:], C0.reshape(M, ldc)[:, N:], equal_nan=True)
    # Deterministic: a second call gives the same bits.
    dC2 = gpu.from_numpy(C0.copy()).cuda()
    dn.check(dn.cuda_gemm("f32", d, dA, dB, dC2, gpu.cuda.current_stream()))
    gpu.cuda.synchronize()
    assert np.array_equal(dC2.cpu().numpy().view(np.uint32), dC.cpu().numpy().view(np.uint32))


def test_panel_kernel_bias_through_onednn_entry(gpu, dn, orc):
    """The oneDNN entry with both operands untransposed maps onto a small-M
    K x N GEMM with the bias in the epilogue: C (OC x batch, column-major) =
    W (OC x K) x X (K x batch) + bias."""
    from tests.test_oracle_colmajor import operands
    torch = gpu
    M, N, K = 1000, 3, 512     # OC, batch, K
    A, lda, B, ldb, C, ldc = operands(M, N, K, "N", "N", 0, 0, 0)
    bias = ref_uniform(M, 5)
    assert dn.plan_describe(dn.KIND_F32, dn.desc(N, M, K, ldb, lda, ldc)).startswith("gemv_panel")
    ref = C.copy()
    assert orc.sgemm_colmajor("N", "N", M, N, K, 1.0, A, lda, B, ldb, 0.5, ref, ldc, bias) == 0
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C))
    s = torch.cuda.current_stream()
    dn.check(dn.cuda_sgemm_colmajor("N", "N", M, N, K, 1.0, dA, lda, dB, ldb, 0.5, dC, ldc,
                                    torch.from_numpy(bias).cuda(), s))
    torch.cuda.synchronize()
    assert np.max(np.abs(dC.cpu().numpy() - ref)) <= fp32_tol(K)


def test_autotune_roundtrip(gpu, dn, orc, tmp_path):
    M, N, K = 3, 2053, 1000     # a shape no other test plans
    A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)
    ref = C.copy()
    orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.5, ref, N)
    dn.check(dn.lib.dnnopt_autotune_enable(1))
    try:
        before = dn.lib.dnnopt_autotune_entries()
        dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.5, C, N))
        assert dn.lib.dnnopt_autotune_entries() == before + 1
        assert np.max(np.abs(C - ref)) <= fp32_tol(K)
        path = str(tmp_path / "tune.bin").encode()
        n = dn.lib.dnnopt_autotune_save(path)
        assert n >= 1 and dn.lib.dnnopt_autotune_load(path) == n
    finally:
        dn.lib.dnnopt_autotune_enable(0)


def test_injected_faults_leave_device_usable(gpu, dn, orc):
    M, N, K = 2, 1009, 1024
    A, B = ref_uniform(M * K, 1), ref_uniform(K * N, 2)
    for site in (1, 2, 3):
        C = np.zeros(M * N, np.float32)
        dn.check(dn.lib.dnnopt_debug_inject_fault(site, 1))
        assert dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.0, C, N) == dn.INJECTED_FAULT
        assert dn.lib.dnnopt_get_last_error() == dn.INJECTED_FAULT
        dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.0, C, N))
        ref = np.zeros(M * N, np.float32)
        orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.0, ref, N)
        assert np.max(np.abs(C - ref)) <= fp32_tol(K)


def test_launch_counter_counts_kernels(gpu, dn):
    A, B = ref_uniform(4 * 64, 1), ref_uniform(64 * 512, 2)
    C = np.zeros(4 * 512, np.float32)
    n0 = dn.launch_count()
    dn.check(dn.gemm_fp32(4, 512, 64, 1.0, A, 64, B, 512, 0.0, C, 512))
    assert dn.launch_count() == n0 + 1
