"""Pins the CPU oracle against the reference's own outputs (CPU only).

The fixture tests/golden/reference_outputs.npz was produced by the reference's
code (tests/golden/make_golden.py); inputs are regenerated from seeds.  The
oracle restatements of gemm_naive_fp32, cblas_sgemm/sgemm_,
gemm_int8_int8int8int32, the fp8 API and the scalar codecs must reproduce those
outputs bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import bf16_bits, bf16_to_f32, int8_uniform, ref_uniform

GEMM_SHAPES = [(1, 1, 1), (4, 4, 4), (8, 8, 8), (16, 16, 16), (32, 32, 32), (64, 64, 64),
               (1, 128, 64), (7, 13, 5), (3, 3, 1000), (128, 1, 768), (1, 1000, 2048),
               (5, 7, 11), (13, 17, 19), (127, 127, 127)]
CBLAS_SIZES = [(4, 4, 4), (16, 16, 16), (32, 64, 48), (7, 13, 11), (1, 64, 32)]
C2_SHAPES = [(m, n, 1024) for m in (2, 3, 5, 7) for n in (1009, 2039, 4093)]
INT8_SHAPES = [(1, 1, 1), (4, 37, 67), (3, 129, 1000), (8, 64, 4096), (5, 7, 11), (13, 17, 19)]


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("shape", GEMM_SHAPES)
def test_fp32_naive_bitexact(orc, golden, shape):
    M, N, K = shape
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 42)
    C = np.zeros(M * N, np.float32)
    orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.0, C, N)
    assert bits_equal(C, golden[f"fp32_{M}x{N}x{K}"])


def test_fp32_alpha_beta_bitexact(orc, golden):
    M, N, K = 32, 48, 64
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 43)
    C = np.zeros(M * N, np.float32)
    orc.gemm_f32(M, N, K, 2.0, A, K, B, N, 0.0, C, N)
    assert bits_equal(C, golden["fp32_alpha2"])
    C = ref_uniform(M * N, 44)
    orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.5, C, N)
    assert bits_equal(C, golden["fp32_beta05"])


def test_config1_config2_bitexact(orc, golden):
    M, N, K = 1, 4096, 4096
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 123)
    C = np.zeros(M * N, np.float32)
    orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.0, C, N)
    assert bits_equal(C, golden["config1"])
    for (M, N, K) in C2_SHAPES:
        A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)
        orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.5, C, N)
        assert bits_equal(C, golden[f"config2_{M}x{N}x{K}"]), (M, N, K)


def cblas_by_oracle(orc, order, ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc):
    """The reference's cblas reduction (src/blas/cblas_sgemm.cpp:67-143) with
    materialised transposes, evaluated by the oracle's naive GEMM."""
    def rowmajor(ta_, tb_, M_, N_, K_, A_, lda_, B_, ldb_):
        a = A_.reshape(-1, lda_)
        b = B_.reshape(-1, ldb_)
        a = np.ascontiguousarray(a[:K_, :M_].T) if ta_ else np.ascontiguousarray(a[:M_, :K_])
        b = np.ascontiguousarray(b[:N_, :K_].T) if tb_ else np.ascontiguousarray(b[:K_, :N_])
        orc.gemm_f32(M_, N_, K_, alpha, a.ravel(), K_, b.ravel(), N_, beta, C, ldc)
    if order == 101:
        rowmajor(ta != 111, tb != 111, M, N, K, A, lda, B, ldb)
    else:
        rowmajor(tb != 111, ta != 111, N, M, K, B, ldb, A, lda)


@pytest.mark.parametrize("size", CBLAS_SIZES)
def test_cblas_bitexact(orc, golden, size):
    M, N, K = size
    for order in (101, 102):
        for ta in (111, 112):
            for tb in (111, 112):
                if order == 101:
                    a_rows, a_cols = (K, M) if ta == 112 else (M, K)
                    b_rows, b_cols = (N, K) if tb == 112 else (K, N)
                    lda, ldb, ldc = a_cols, b_cols, N
                else:
                    a_rows, a_cols = (M, K) if ta == 112 else (K, M)
                    b_rows, b_cols = (K, N) if tb == 112 else (N, K)
                    lda, ldb, ldc = a_cols, b_cols, M
                A = ref_uniform(a_rows * a_cols, 42)
                B = ref_uniform(b_rows * b_cols, 123)
                C = ref_uniform(M * N, 77)
                cblas_by_oracle(orc, order, ta, tb, M, N, K, 1.0, A, lda, B, ldb, 0.5, C, ldc)
                assert bits_equal(C, golden[f"cblas_{order}_{ta}_{tb}_{M}x{N}x{K}"]), (order, ta, tb)


@pytest.mark.parametrize("shape", INT8_SHAPES + [(4, 11008, 4096)])
def test_int8_native_bitexact(orc, golden, shape):
    M, N, K = shape
    A, B = int8_uniform(M * K, 42), int8_uniform(N * K, 123)
    C = np.zeros(M * N, np.int32)
    orc.gemm_s8s32(M, N, K, A, K, B, K, C, N)
    key = "config3" if shape == (4, 11008, 4096) else f"s8_{M}x{N}x{K}"
    assert np.array_equal(C, golden[key])


def test_reference_fp8_codecs_bitexact(orc, golden):
    b = np.arange(256)
    for codec, key in (("refe4m3", "ref_e4m3_decode"), ("refe5m2", "ref_e5m2_decode")):
        assert bits_equal(orc.table(codec, "to_f32", b), golden[key]), codec
    sweep = golden["codec_sweep"]
    assert np.array_equal(orc.table("refe4m3", "from_f32", sweep), golden["ref_e4m3_encode"])
    assert np.array_equal(orc.table("refe5m2", "from_f32", sweep), golden["ref_e5m2_encode"])
    assert np.array_equal(bf16_bits(sweep), golden["ref_bf16_encode"])
    assert np.array_equal(
        np.array([orc.lib.oracle_bf16_from_f32(float(v)) for v in sweep], np.uint16),
        golden["ref_bf16_encode"])


def test_fp8_api_bitexact(orc, golden):
    M, N, K = 5, 37, 64
    enc4 = lambda x: orc.table("refe4m3", "from_f32", x)  # noqa: E731
    enc5 = lambda x: orc.table("refe5m2", "from_f32", x)  # noqa: E731
    A4, A5 = enc4(ref_uniform(M * K, 42)), enc5(ref_uniform(M * K, 42))
    B5 = enc5(ref_uniform(K * N, 123))
    C = np.zeros(M * N, np.float32)
    orc.gemm_refe4m3_e5m2(M, N, K, 1.0, A4, K, B5, N, 0.0, C, N)
    assert bits_equal(C, golden["fp8_e4m3_5x37x64"])
    C = np.zeros(M * N, np.float32)
    orc.gemm_refe5m2_e5m2(M, N, K, 1.0, A5, K, B5, N, 0.0, C, N)
    assert bits_equal(C, golden["fp8_e5m2_5x37x64"])


def test_ocp_e4m3_codec_against_torch(orc):
    """The OCP E4M3FN restatement agrees with torch.float8_e4m3fn (an
    independent implementation) on every code and on an RNE sweep."""
    torch = pytest.importorskip("torch")
    codes = np.arange(256, dtype=np.uint8)
    mine = orc.table("e4m3fn", "to_f32", codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(theirs)
    assert np.array_equal(np.isnan(mine), nan)
    assert bits_equal(mine[~nan], theirs[~nan])
    sweep = np.concatenate([ref_uniform(20000, 9) * 500, ref_uniform(2000, 10) * 0.02,
                            np.float32(2.0) ** np.arange(-12, 9, dtype=np.float32)]).astype(np.float32)
    sweep = sweep[np.abs(sweep) <= 448]
    ours = orc.table("e4m3fn", "from_f32", sweep)
    ref = torch.from_numpy(sweep).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)


def test_bf16_oracle_within_reference_tolerance(orc):
    """gemm_bf16_bf16bf16f32 restatement vs FP64 of the same bf16 inputs, and vs
    the reference test's bound K*2e-3 against the FP32 naive GEMM
    (tests/test_gemm_correctness.cpp:126-137)."""
    M, N, K = 33, 64, 256
    A32, B32 = ref_uniform(M * K, 42), ref_uniform(K * N, 43)
    A, B = bf16_bits(A32), bf16_bits(B32)
    C = np.zeros(M * N, np.float32)
    c64 = orc.gemm_bf16f32(M, N, K, 1.0, A, K, B, N, 0.0, C, N, want64=True)
    assert np.max(np.abs(C - c64)) <= 1e-5 * K
    Cf = np.zeros(M * N, np.float32)
    orc.gemm_f32(M, N, K, 1.0, A32, K, B32, N, 0.0, Cf, N)
    assert np.max(np.abs(C - Cf)) < K * 2e-3
    assert np.array_equal(bf16_to_f32(A), bf16_to_f32(bf16_bits(bf16_to_f32(A))))


def test_int8_f32api_within_reference_tolerance(orc):
    """FP32-API int8 restatement vs the reference test bound K*2e-2
    (tests/test_gemm_correctness.cpp:139-151)."""
    for (M, N, K) in [(1, 128, 64), (7, 13, 5), (5, 7, 11), (32, 48, 64)]:
        A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 42)
        C = np.zeros(M * N, np.float32)
        orc.gemm_int8_f32api(M, N, K, 1.0, A, K, B, N, 0.0, C, N)
        Cf = np.zeros(M * N, np.float32)
        orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.0, Cf, N)
        assert np.max(np.abs(C - Cf)) < K * 2e-2


def test_e4m3_quantization_roundtrip(orc):
    """Config-5 weight preparation: scale = absmax/448 per row, every code is a
    finite e4m3 value and dequantised rows stay within half an e4m3 ulp."""
    N, K = 64, 512
    W = (np.random.default_rng(123).standard_normal(N * K) * 0.02).astype(np.float32)
    q, s = orc.quantize_e4m3_rows(N, K, W, K)
    assert not np.any((q & 0x7F) == 0x7F)
    dec = orc.table("e4m3fn", "to_f32", np.arange(256))[q].reshape(N, K) * s[:, None]
    err = np.abs(dec - W.reshape(N, K))
    assert np.all(err <= np.abs(W.reshape(N, K)) * 2.0 ** -4 + s[:, None] * 2.0 ** -10)
