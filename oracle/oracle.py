"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the CPU oracle.

``liboracle.so`` (oracle.c) restates the reference's arithmetic; the optional
``_ref/libdnnopt_ref.so`` is the reference's own portable code compiled from
its sources (see Makefile).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may use this module, as the checker or the timed
CPU baseline -- never as the product path.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libdnnopt_ref.so")

_I, _F, _P, _SZ = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


def _p(a):
    return None if a is None else a.ctypes.data_as(_P)


def load_oracle():
    lib = ctypes.CDLL(ORACLE_SO)
    lib.oracle_bf16_from_f32.argtypes = [_F]
    lib.oracle_bf16_from_f32.restype = ctypes.c_uint16
    lib.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
    lib.oracle_bf16_to_f32.restype = _F
    for n in ("e4m3fn", "refe4m3", "refe5m2"):
        getattr(lib, f"oracle_{n}_to_f32").argtypes = [ctypes.c_uint8]
        getattr(lib, f"oracle_{n}_to_f32").restype = _F
        getattr(lib, f"oracle_{n}_from_f32").argtypes = [_F]
        getattr(lib, f"oracle_{n}_from_f32").restype = ctypes.c_uint8
    sig = [_I, _I, _I, _F, _P, _I, _P, _I, _F, _P, _I]
    for n in ("oracle_gemm_f32_naive", "oracle_gemm_int8_f32api", "oracle_gemm_refe4m3_refe5m2",
              "oracle_gemm_refe5m2_refe5m2"):
        getattr(lib, n).argtypes = sig
    lib.oracle_gemm_f32_f64.argtypes = sig + [_P, _I]
    lib.oracle_gemm_s8s32.argtypes = [_I, _I, _I, _P, _I, _P, _I, _P, _I, _I]
    lib.oracle_gemm_bf16f32.argtypes = sig + [_P, _I]
    lib.oracle_gemm_e4m3bf16.argtypes = [_I, _I, _I, _P, _I, _P, _I, _P, _P, _I, _P, _I]
    lib.oracle_quantize_e4m3_rows.argtypes = [_I, _I, _P, _I, _P, _P, _I]
    _L = ctypes.c_int64
    lib.oracle_sgemm_colmajor.argtypes = [ctypes.c_char, ctypes.c_char, _L, _L, _L, _F, _P, _L, _P,
                                          _L, _F, _P, _L, _P]
    lib.oracle_sgemm_colmajor.restype = _I
    lib.oracle_conv3d.argtypes = [_I, _P, _P, _P, _P, _P, _I, _P]
    return lib


def load_ref():
    """The reference's own code (None when oracle/_ref was not built)."""
    if not os.path.exists(REF_SO):
        return None
    lib = ctypes.CDLL(REF_SO)
    sig = [_I, _I, _I, _F, _P, _I, _P, _I, _F, _P, _I]
    for n in ("ref_gemm_fp32_naive", "ref_gemm_fp32", "ref_gemm_bf16", "ref_gemm_int8",
              "ref_gemm_fp8_e4m3", "ref_gemm_fp8_e5m2", "ref_gemm_fp8"):
        getattr(lib, n).argtypes = sig
    lib.ref_gemm_fp32_naive_mt.argtypes = sig + [_I]
    lib.ref_gemm_int8_int8int8int32.argtypes = [_I, _I, _I, _P, _I, _P, _I, _P, _I]
    lib.ref_gemm_int8_int8int8int32_mt.argtypes = [_I, _I, _I, _P, _I, _P, _I, _P, _I, _I]
    lib.cblas_sgemm.argtypes = [_I, _I, _I, _I, _I, _I, _F, _P, _I, _P, _I, _F, _P, _I]
    lib.sgemm_.argtypes = [_P] * 13
    lib.ref_conv3d.argtypes = [_I, _P, _P, _P, _P, _P, _I]
    lib.ref_fill_random.argtypes = [_P, _SZ, ctypes.c_uint]
    lib.ref_bf16_from_f32.argtypes = [_F]
    lib.ref_bf16_from_f32.restype = ctypes.c_uint16
    for n in ("e4m3", "e5m2"):
        getattr(lib, f"ref_{n}_to_f32").argtypes = [ctypes.c_uint8]
        getattr(lib, f"ref_{n}_to_f32").restype = _F
        getattr(lib, f"ref_{n}_from_f32").argtypes = [_F]
        getattr(lib, f"ref_{n}_from_f32").restype = ctypes.c_uint8
    lib.ref_has_fp8_support.restype = _I
    return lib


# ---- seeded generators -------------------------------------------------------
def ref_uniform(n: int, seed: int) -> np.ndarray:
    """std::mt19937(seed) + std::uniform_real_distribution<float>(-1, 1), as in
    the reference tests (tests/test_gemm_correctness.cpp:20-24): libstdc++
    draws one 32-bit word per float, scales by 2^-32 and maps to [-1, 1)."""
    bg = np.random.MT19937()
    bg._legacy_seeding(seed)
    raw = bg.random_raw(n).astype(np.uint64)
    s = raw.astype(np.float32) / np.float32(2.0 ** 32)
    s = np.where(s >= 1, np.nextafter(np.float32(1), np.float32(0)), s).astype(np.float32)
    return (np.float32(-1) + np.float32(2) * s).astype(np.float32)


def int8_uniform(n: int, seed: int) -> np.ndarray:
    """int8 i.i.d. uniform integers in [-127, 127]."""
    return np.random.default_rng(seed).integers(-127, 128, size=n, dtype=np.int16).astype(np.int8)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round-to-nearest-even (reference gemm_types.h:18-24)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---- oracle wrappers ------------------------------------------------------------
class Oracle:
    def __init__(self):
        self.lib = load_oracle()

    def gemm_f32(self, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc):
        self.lib.oracle_gemm_f32_naive(M, N, K, alpha, _p(A), lda, _p(B), ldb, beta, _p(C), ldc)

    def sgemm_colmajor(self, transa, transb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, bias=None):
        return self.lib.oracle_sgemm_colmajor(transa.encode(), transb.encode(), M, N, K, alpha, _p(A),
                                              lda, _p(B), ldb, beta, _p(C), ldc, _p(bias))

    def conv3d(self, precision, params, inp, flt, bias, out, post_op=0, want64=False):
        """params: the 15 ints N, IC, ID, IH, IW, OC, KD, KH, KW, strides, pads."""
        p = np.asarray(params, np.int32)
        out64 = np.zeros(out.size, np.float64) if want64 else None
        self.lib.oracle_conv3d(precision, _p(p), _p(inp), _p(flt), _p(bias), _p(out), post_op, _p(out64))
        return out64

    def gemm_f32_f64(self, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, threads=8):
        out = np.zeros(M * N, np.float64)
        self.lib.oracle_gemm_f32_f64(M, N, K, alpha, _p(A), lda, _p(B), ldb, beta, _p(C), ldc,
                                     _p(out), threads)
        return out

    def gemm_s8s32(self, M, N, K, A, lda, B, ldb, C, ldc, threads=8):
        self.lib.oracle_gemm_s8s32(M, N, K, _p(A), lda, _p(B), ldb, _p(C), ldc, threads)

    def gemm_bf16f32(self, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, want64=False, threads=8):
        out = np.zeros(M * N, np.float64) if want64 else None
        self.lib.oracle_gemm_bf16f32(M, N, K, alpha, _p(A), lda, _p(B), ldb, beta, _p(C), ldc,
                                     _p(out), threads)
        return out

    def gemm_int8_f32api(self, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc):
        self.lib.oracle_gemm_int8_f32api(M, N, K, alpha, _p(A), lda, _p(B), ldb, beta, _p(C), ldc)

    def gemm_e4m3bf16(self, M, N, K, A, lda, W, ldw, scale, C, ldc, want64=True, threads=8):
        out = np.zeros(M * N, np.float64) if want64 else None
        self.lib.oracle_gemm_e4m3bf16(M, N, K, _p(A), lda, _p(W), ldw, _p(scale), _p(C), ldc,
                                      _p(out), threads)
        return out

    def quantize_e4m3_rows(self, N, K, W, ldw, threads=8):
        q = np.zeros(N * K, np.uint8)
        s = np.zeros(N, np.float32)
        self.lib.oracle_quantize_e4m3_rows(N, K, _p(W), ldw, _p(q), _p(s), threads)
        return q, s

    def gemm_refe4m3_e5m2(self, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc):
        self.lib.oracle_gemm_refe4m3_refe5m2(M, N, K, alpha, _p(A), lda, _p(B), ldb, beta, _p(C), ldc)

    def gemm_refe5m2_e5m2(self, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc):
        self.lib.oracle_gemm_refe5m2_refe5m2(M, N, K, alpha, _p(A), lda, _p(B), ldb, beta, _p(C), ldc)

    def table(self, codec: str, direction: str, values: np.ndarray) -> np.ndarray:
        fn = getattr(self.lib, f"oracle_{codec}_{direction}")
        if direction == "to_f32":
            return np.array([fn(int(v)) for v in values], np.float32)
        return np.array([fn(float(v)) for v in values], np.uint8)
