"""Generate tests/golden/reference_outputs.npz from the reference's own code.

Run in a container that has the reference tree (it builds oracle/_ref from the
reference sources with oracle/Makefile):

    make -C oracle && python tests/golden/make_golden.py

Every expected output in the fixture is produced by calling the reference's
functions (oracle/_ref/libdnnopt_ref.so, compiled from xuefenghao5121/DNN-Opt
src/ on x86 where gemm_fp32 resolves to gemm_naive_fp32).  Inputs are NOT
stored: they are regenerated from seeds with oracle.oracle.ref_uniform (the
reference tests' std::mt19937 + uniform_real(-1, 1) stream, checked here
against the reference's own generator) and oracle.oracle.int8_uniform.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle.oracle import int8_uniform, load_ref, ref_uniform  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden", "reference_outputs.npz")

# tests/test_gemm_correctness.cpp:159-182 shapes whose outputs are small.
GEMM_SHAPES = [(1, 1, 1), (4, 4, 4), (8, 8, 8), (16, 16, 16), (32, 32, 32), (64, 64, 64),
               (1, 128, 64), (7, 13, 5), (3, 3, 1000), (128, 1, 768), (1, 1000, 2048),
               (5, 7, 11), (13, 17, 19), (127, 127, 127)]
# tests/test_cblas.cpp:340-348 sizes (256^3 is checked against the oracle at test time).
CBLAS_SIZES = [(4, 4, 4), (16, 16, 16), (32, 64, 48), (7, 13, 11), (1, 64, 32)]
# BASELINE config 2.
C2_SHAPES = [(m, n, 1024) for m in (2, 3, 5, 7) for n in (1009, 2039, 4093)]
INT8_SHAPES = [(1, 1, 1), (4, 37, 67), (3, 129, 1000), (8, 64, 4096), (5, 7, 11), (13, 17, 19)]


def p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def main() -> None:
    ref = load_ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libdnnopt_ref.so is missing: run `make -C oracle` with the "
                         "reference tree present")
    out: dict[str, np.ndarray] = {}

    # Generator pin: numpy's MT19937 stream == the reference tests' generator.
    for seed in (42, 43, 44, 77, 123):
        a = np.zeros(4099, np.float32)
        ref.ref_fill_random(p(a), a.size, seed)
        assert np.array_equal(a, ref_uniform(a.size, seed)), seed

    # gemm_fp32 (kAuto -> gemm_naive_fp32 on x86), alpha=1, beta=0, C zeroed.
    for (M, N, K) in GEMM_SHAPES:
        A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 42)
        C = np.zeros(M * N, np.float32)
        ref.ref_gemm_fp32(M, N, K, 1.0, p(A), K, p(B), N, 0.0, p(C), N)
        out[f"fp32_{M}x{N}x{K}"] = C

    # alpha/beta cases (tests/test_gemm_correctness.cpp:185-225).
    M, N, K = 32, 48, 64
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 43)
    C = np.zeros(M * N, np.float32)
    ref.ref_gemm_fp32(M, N, K, 2.0, p(A), K, p(B), N, 0.0, p(C), N)
    out["fp32_alpha2"] = C
    C = ref_uniform(M * N, 44)
    ref.ref_gemm_fp32(M, N, K, 1.0, p(A), K, p(B), N, 0.5, p(C), N)
    out["fp32_beta05"] = C

    # cblas_sgemm / sgemm_ (tests/test_cblas.cpp), seeds 42/123/77.
    for (M, N, K) in CBLAS_SIZES:
        for order in (101, 102):
            for ta in (111, 112):
                for tb in (111, 112):
                    # Stored shapes: row-major op(A) M x K; col-major A M x K (ld = rows).
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
                    ref.cblas_sgemm(order, ta, tb, M, N, K, 1.0, p(A), lda, p(B), ldb, 0.5, p(C), ldc)
                    out[f"cblas_{order}_{ta}_{tb}_{M}x{N}x{K}"] = C
        # alpha=2.5, beta=-0.3 row-major NN.
        A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)
        ref.cblas_sgemm(101, 111, 111, M, N, K, 2.5, p(A), K, p(B), N, -0.3, p(C), N)
        out[f"cblas_ab_{M}x{N}x{K}"] = C
        # Fortran sgemm_ (column-major NN, alpha 1, beta 0, C zeroed).
        A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 123)
        C = np.zeros(M * N, np.float32)
        args = [ctypes.c_char(b"N"), ctypes.c_char(b"N"), ctypes.c_int(M), ctypes.c_int(N),
                ctypes.c_int(K), ctypes.c_float(1.0)]
        lda_, ldb_, ldc_ = ctypes.c_int(M), ctypes.c_int(K), ctypes.c_int(M)
        beta = ctypes.c_float(0.0)
        ref.sgemm_(ctypes.byref(args[0]), ctypes.byref(args[1]), ctypes.byref(args[2]),
                   ctypes.byref(args[3]), ctypes.byref(args[4]), ctypes.byref(args[5]), p(A),
                   ctypes.byref(lda_), p(B), ctypes.byref(ldb_), ctypes.byref(beta), p(C),
                   ctypes.byref(ldc_))
        out[f"fortran_{M}x{N}x{K}"] = C

    # BASELINE config 1 and config 2 (A seed 42, B seed 123, C seed 77).
    M, N, K = 1, 4096, 4096
    A, B = ref_uniform(M * K, 42), ref_uniform(K * N, 123)
    C = np.zeros(M * N, np.float32)
    ref.ref_gemm_fp32(M, N, K, 1.0, p(A), K, p(B), N, 0.0, p(C), N)
    out["config1"] = C
    for (M, N, K) in C2_SHAPES:
        A, B, C = ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)
        ref.ref_gemm_fp32(M, N, K, 1.0, p(A), K, p(B), N, 0.5, p(C), N)
        out[f"config2_{M}x{N}x{K}"] = C

    # gemm_int8_int8int8int32: B is [N, K].  A seed 42, B seed 123.
    for (M, N, K) in INT8_SHAPES + [(4, 11008, 4096)]:
        A, B = int8_uniform(M * K, 42), int8_uniform(N * K, 123)
        C = np.zeros(M * N, np.int32)
        ref.ref_gemm_int8_int8int8int32(M, N, K, p(A), K, p(B), K, p(C), N)
        key = "config3" if (M, N, K) == (4, 11008, 4096) else f"s8_{M}x{N}x{K}"
        out[key] = C

    # Scalar codecs over every byte / a float sweep.
    bytes_ = np.arange(256, dtype=np.uint8)
    out["ref_e4m3_decode"] = np.array([ref.ref_e4m3_to_f32(int(b)) for b in bytes_], np.float32)
    out["ref_e5m2_decode"] = np.array([ref.ref_e5m2_to_f32(int(b)) for b in bytes_], np.float32)
    sweep = np.concatenate([
        ref_uniform(2000, 5) * 4,
        np.float32(2.0) ** np.arange(-20, 20, dtype=np.float32),
        -(np.float32(2.0) ** np.arange(-20, 20, dtype=np.float32)),
        np.array([0.0, -0.0, 448.0, 500.0, 57344.0, 1e6, -1e6, 1e-8, 0.9375, 0.96875], np.float32),
    ]).astype(np.float32)
    out["codec_sweep"] = sweep
    out["ref_e4m3_encode"] = np.array([ref.ref_e4m3_from_f32(float(v)) for v in sweep], np.uint8)
    out["ref_e5m2_encode"] = np.array([ref.ref_e5m2_from_f32(float(v)) for v in sweep], np.uint8)
    out["ref_bf16_encode"] = np.array([ref.ref_bf16_from_f32(float(v)) for v in sweep], np.uint16)

    # FP8 API (gemm_fp8.cpp): reference codecs, then gemm_fp32.
    M, N, K = 5, 37, 64
    A = np.array([ref.ref_e4m3_from_f32(float(v)) for v in ref_uniform(M * K, 42)], np.uint8)
    Be = np.array([ref.ref_e5m2_from_f32(float(v)) for v in ref_uniform(K * N, 123)], np.uint8)
    Ae = np.array([ref.ref_e5m2_from_f32(float(v)) for v in ref_uniform(M * K, 42)], np.uint8)
    C = np.zeros(M * N, np.float32)
    ref.ref_gemm_fp8_e4m3(M, N, K, 1.0, p(A), K, p(Be), N, 0.0, p(C), N)
    out["fp8_e4m3_5x37x64"] = C
    C = np.zeros(M * N, np.float32)
    ref.ref_gemm_fp8_e5m2(M, N, K, 1.0, p(Ae), K, p(Be), N, 0.0, p(C), N)
    out["fp8_e5m2_5x37x64"] = C

    np.savez_compressed(OUT, **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {OUT}: {len(out)} arrays, {total / 1024:.0f} KiB uncompressed")


if __name__ == "__main__":
    main()
