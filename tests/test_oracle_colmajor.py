"""The oracle's restatement of the oneDNN integration entry (CPU only).

`oracle_sgemm_colmajor` restates dnnopt_sgemm from the reference's
integration/onednn/0001-dnnopt-integration.patch:243-365.  Its GEMM core is
the naive FP32 GEMM that test_oracle_golden pins bit for bit against the
reference's gemm_naive_fp32; these tests pin the wrapper around it: the
column-major/row-major duality on the shapes and tolerance of the reference's
own tests/integration/test_dispatch_logic.cpp, the bias pass, the K == 0
branch and the ldc < M temporary-buffer path.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import ref_uniform

# tests/integration/test_dispatch_logic.cpp:139-149 (M, N, K, transa, transb).
DISPATCH_SHAPES = [(1, 256, 1024, "N", "N"), (256, 1024, 1, "T", "N"), (4, 256, 1024, "N", "N"),
                   (32, 256, 256, "N", "N"), (32, 256, 512, "N", "N"), (32, 512, 256, "N", "N"),
                   (8, 512, 512, "N", "N"), (8, 512, 1376, "N", "N"), (256, 256, 256, "N", "N")]


def colmajor_f64(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, bias=None):
    """Column-major alpha*op(A)*op(B) + beta*C (+ bias[i]) in float64."""
    a = A.astype(np.float64)
    b = B.astype(np.float64)
    # Column-major X (rows x cols, ld) is X.reshape(cols, ld)[:, :rows].T.
    opa = a[:M * lda].reshape(M, lda)[:, :K] if ta == "T" else a[:K * lda].reshape(K, lda)[:, :M].T
    opb = b[:K * ldb].reshape(K, ldb)[:, :N] if tb == "T" else b[:N * ldb].reshape(N, ldb)[:, :K].T
    out = C.astype(np.float64).copy()
    prod = alpha * (opa @ opb)
    for j in range(N):
        c0 = beta * out[j * ldc:j * ldc + M] if beta != 0 else 0.0
        v = prod[:, j] + c0
        if bias is not None:
            v = v + bias[:M]
        out[j * ldc:j * ldc + M] = v
    return out


def operands(M, N, K, ta, tb, lda_pad=0, ldb_pad=0, ldc_pad=0, seed=7):
    lda = (K if ta == "T" else M) + lda_pad
    ldb = (N if tb == "T" else K) + ldb_pad
    ldc = M + ldc_pad
    A = ref_uniform(lda * (M if ta == "T" else K), seed)
    B = ref_uniform(ldb * (K if tb == "T" else N), seed + 1)
    C = ref_uniform(ldc * N, seed + 2)
    return A, lda, B, ldb, C, ldc


@pytest.mark.parametrize("M,N,K,ta,tb", DISPATCH_SHAPES)
def test_dispatch_shapes_within_reference_tolerance(orc, M, N, K, ta, tb):
    A, lda, B, ldb, _, ldc = operands(M, N, K, ta, tb)
    C = np.zeros(ldc * N, np.float32)
    assert orc.sgemm_colmajor(ta, tb, M, N, K, 1.0, A, lda, B, ldb, 0.0, C, ldc) == 0
    ref = colmajor_f64(ta, tb, M, N, K, 1.0, A, lda, B, ldb, 0.0, np.zeros(ldc * N, np.float32), ldc)
    assert np.max(np.abs(C - ref)) < K * 2e-5      # test_dispatch_logic.cpp:245


@pytest.mark.parametrize("ta,tb", [("N", "N"), ("T", "N"), ("N", "T"), ("T", "T")])
def test_transposes_padding_bias(orc, ta, tb):
    M, N, K = 37, 6, 53
    A, lda, B, ldb, C, ldc = operands(M, N, K, ta, tb, 3, 2, 5)
    bias = ref_uniform(M, 99)
    ref = colmajor_f64(ta, tb, M, N, K, 0.75, A, lda, B, ldb, 0.5, C, ldc, bias)
    assert orc.sgemm_colmajor(ta, tb, M, N, K, 0.75, A, lda, B, ldb, 0.5, C, ldc, bias) == 0
    assert np.max(np.abs(C - ref)) < 1e-5 * K


def test_k0_scales_and_adds_bias(orc):
    M, N, ldc = 5, 3, 8
    C = ref_uniform(ldc * N, 3)
    C[0] = np.nan                              # beta == 0 clears, NaN included (memset)
    bias = ref_uniform(M, 4)
    out = C.copy()
    assert orc.sgemm_colmajor("N", "N", M, N, 0, 1.0, None, M, None, 1, 0.0, out, ldc, bias) == 0
    for j in range(N):
        for i in range(ldc):
            want = np.float32(bias[i]) if i < M else C[j * ldc + i]
            assert out[j * ldc + i] == want or (np.isnan(want) and np.isnan(out[j * ldc + i]))
    out = C.copy()
    out[0] = 1.0
    assert orc.sgemm_colmajor("N", "N", M, N, 0, 1.0, None, M, None, 1, 2.0, out, ldc, None) == 0
    assert out[0] == np.float32(2.0) and out[M] == C[M]


def test_ldc_below_m_copy_back_order(orc):
    """ldc < M: the GEMM runs on an N x M scratch that is copied back row by
    row (later columns overwrite earlier ones), then the bias is added per
    (i, j) pair (patch:330-362)."""
    M, N, K, ldc = 6, 4, 9, 4
    A, lda, B, ldb, _, _ = operands(M, N, K, "N", "N")
    C = ref_uniform((N - 1) * ldc + M, 11)
    bias = ref_uniform(M, 12)
    want = C.astype(np.float64).copy()
    tmp = np.array([[C[r * ldc + c] for c in range(M)] for r in range(N)], np.float64)
    a = A.astype(np.float64).reshape(K, lda)[:, :M].T        # op(A), M x K
    b = B.astype(np.float64).reshape(N, ldb)[:, :K].T        # op(B), K x N
    tmp = (a @ b).T + 0.5 * tmp                              # row r = column j of C
    for r in range(N):
        for c in range(M):
            want[r * ldc + c] = tmp[r, c]
    for j in range(N):
        for i in range(M):
            want[j * ldc + i] += bias[i]
    out = C.copy()
    assert orc.sgemm_colmajor("N", "N", M, N, K, 1.0, A, lda, B, ldb, 0.5, out, ldc, bias) == 0
    assert np.max(np.abs(out - want)) < 1e-5 * K


def test_packed_and_empty(orc):
    C = np.ones(4, np.float32)
    assert orc.sgemm_colmajor("P", "N", 2, 2, 2, 1.0, None, 2, None, 2, 0.0, C, 2) == -1
    assert orc.sgemm_colmajor("N", "N", 0, 2, 2, 1.0, None, 2, None, 2, 0.0, C, 2) == 0
    assert np.all(C == 1.0)


def test_library_entry_argument_errors(dn):
    """Host-side checks of dnnopt_sgemm_colmajor that need no device."""
    C = np.ones(4, np.float32)
    assert dn.sgemm_colmajor("P", "N", 2, 2, 2, 1.0, None, 2, None, 2, 0.0, C, 2) == dn.NOT_SUPPORTED
    assert dn.sgemm_colmajor("n", "p", 2, 2, 2, 1.0, None, 2, None, 2, 0.0, C, 2) == dn.NOT_SUPPORTED
    assert dn.sgemm_colmajor("N", "N", 0, 2, 2, 1.0, None, 2, None, 2, 0.0, C, 2) == dn.SUCCESS
    assert dn.sgemm_colmajor("N", "N", 2, 0, 2, 1.0, None, 2, None, 2, 0.0, C, 2) == dn.SUCCESS
    assert dn.sgemm_colmajor("N", "N", -1, 2, 2, 1.0, None, 2, None, 2, 0.0, C, 2) == dn.INVALID_VALUE
    A = np.ones(4, np.float32)
    assert dn.sgemm_colmajor("N", "N", 2, 2, 2, 1.0, A, 1, A, 2, 0.0, C, 2) == dn.INVALID_VALUE  # lda < M
    assert dn.sgemm_colmajor("N", "N", 2, 2, 2, 1.0, None, 2, A, 2, 0.0, C, 2) == dn.INVALID_VALUE
    assert np.all(C == 1.0)
