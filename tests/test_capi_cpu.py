"""C ABI checks that need no GPU: exported symbols, argument validation and
the reference's early-return semantics, plan selection, autotune-cache files,
thread-count plumbing.  (No kernel is launched here.)"""
from __future__ import annotations

import ctypes
import os
import struct
import subprocess

import numpy as np
import pytest

from tests.conftest import fnv1a64, plan_file_bytes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def test_every_declared_function_is_exported(dn):
    names = dn.declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(dn.lib, n)]
    assert not missing, missing


def test_cpp_mirror_symbols_exported(dn):
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", dn.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    for sig in [
        "dnnopt::gemm_fp32(int, int, int, float, float const*, int, float const*, int, float, float*, int)",
        "dnnopt::gemm_fp32(int, int, int, float, float const*, int, float const*, int, float, float*, int, dnnopt::GemmAlgo)",
        "dnnopt::gemm_bf16(int, int, int, float, float const*, int, float const*, int, float, float*, int)",
        "dnnopt::gemm_bf16_bf16bf16f32(int, int, int, float, dnnopt::bfloat16_t const*, int, dnnopt::bfloat16_t const*, int, float, float*, int)",
        "dnnopt::gemm_int8(int, int, int, float, float const*, int, float const*, int, float, float*, int)",
        "dnnopt::gemm_int8_int8int8int32(int, int, int, signed char const*, int, signed char const*, int, int*, int)",
        "dnnopt::gemm_fp8_e4m3(int, int, int, float, dnnopt::fp8_e4m3_t const*, int, dnnopt::fp8_e5m2_t const*, int, float, float*, int)",
        "dnnopt::gemm_fp8_e5m2(int, int, int, float, dnnopt::fp8_e5m2_t const*, int, dnnopt::fp8_e5m2_t const*, int, float, float*, int)",
        "dnnopt::gemm_fp8(int, int, int, float, float const*, int, float const*, int, float, float*, int)",
        "dnnopt::has_fp8_support()",
        "dnnopt::gemm_set_num_threads(int)",
        "dnnopt::gemm_get_num_threads()",
    ]:
        assert sig in out, sig
    # Only the public surface is exported (no CUDA runtime symbols leak).
    raw = subprocess.run(["nm", "-D", "--defined-only", dn.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    for line in raw.splitlines():
        name = line.split()[-1]
        assert name.startswith("dnnopt_") or name.startswith("_ZN6dnnopt"), name


def test_blas_library_exports(dn):
    blas = ctypes.CDLL(dn.BLAS_PATH)
    for n in ("cblas_sgemm", "cblas_saxpy", "sgemm_", "SGEMM", "openblas_set_num_threads",
              "openblas_get_num_threads", "blas_set_num_threads", "omp_set_num_threads_blas"):
        assert hasattr(blas, n), n
    blas.openblas_set_num_threads(6)
    assert blas.openblas_get_num_threads() == 6
    blas.openblas_set_num_threads(0)


def test_status_strings(dn):
    assert dn.status_string(dn.SUCCESS) == "success"
    assert dn.status_string(dn.INVALID_VALUE) == "invalid value"
    assert dn.status_string(dn.KERNEL_TIMEOUT) == "in-kernel wait timed out"
    assert dn.status_string(99) == "unknown status"


def test_reference_early_return_is_success(dn):
    # M, N or K == 0 returns silently in the reference (src/gemm/gemm.cpp:180);
    # here it is a successful no-op that touches nothing (no device needed).
    C = np.full(4, 7.0, np.float32)
    for (M, N, K) in [(0, 4, 4), (4, 0, 4), (4, 4, 0)]:
        assert dn.gemm_fp32(M, N, K, 1.0, None, 4, None, 4, 0.0, C, 4) == dn.SUCCESS
        assert dn.gemm_int8_int8int8int32(M, N, K, None, 4, None, 4, C, 4) == dn.SUCCESS
    assert np.all(C == 7.0)


def test_invalid_arguments(dn):
    A = np.zeros(64, np.float32)
    B = np.zeros(64, np.float32)
    C = np.zeros(64, np.float32)
    assert dn.gemm_fp32(-1, 4, 4, 1.0, A, 4, B, 4, 0.0, C, 4) == dn.INVALID_VALUE
    assert dn.gemm_fp32(4, 4, 8, 1.0, A, 4, B, 4, 0.0, C, 4) == dn.INVALID_VALUE   # lda < K
    assert dn.gemm_fp32(4, 8, 4, 1.0, A, 4, B, 4, 0.0, C, 8) == dn.INVALID_VALUE   # ldb < N
    assert dn.gemm_fp32(4, 4, 4, 1.0, A, 4, B, 4, 0.0, C, 3) == dn.INVALID_VALUE   # ldc < N
    assert dn.gemm_fp32(4, 4, 4, 1.0, None, 4, B, 4, 0.0, C, 4) == dn.INVALID_VALUE
    # int8: B is N x K, so ldb must cover K.
    a8 = np.zeros(64, np.int8)
    c32 = np.zeros(64, np.int32)
    assert dn.gemm_int8_int8int8int32(2, 8, 8, a8, 8, a8, 4, c32, 8) == dn.INVALID_VALUE
    assert dn.cuda_gemm("f32", dn.desc(4, 4, 4, 3, 4, 4, trans_a=1), A, B, C) == dn.INVALID_VALUE
    # e4m3 needs its scale vector.
    assert dn.gemm_e4m3_bf16(2, 4, 4, np.zeros(8, np.uint16), 4, np.zeros(16, np.uint8), 4,
                             None, np.zeros(8, np.uint16), 4) == dn.INVALID_VALUE
    assert dn.saxpy(4, 1.0, A, -1, C, 1) == dn.INVALID_VALUE
    assert dn.saxpy(0, 1.0, None, 1, None, 1) == dn.SUCCESS


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device status")
def test_no_device_status(dn):
    A = np.ones(16, np.float32)
    C = np.zeros(16, np.float32)
    assert dn.gemm_fp32(4, 4, 4, 1.0, A, 4, A, 4, 0.0, C, 4) == dn.NO_DEVICE
    assert dn.lib.dnnopt_get_last_error() == dn.NO_DEVICE


def test_cpp_mirror_records_status(dn):
    fn = getattr(dn.lib, "_ZN6dnnopt9gemm_fp32EiiifPKfiS1_ifPfi")
    fn.restype = None
    fn.argtypes = [ctypes.c_int] * 3 + [ctypes.c_float, ctypes.c_void_p, ctypes.c_int,
                                        ctypes.c_void_p, ctypes.c_int, ctypes.c_float,
                                        ctypes.c_void_p, ctypes.c_int]
    fn(-3, 4, 4, 1.0, None, 4, None, 4, 0.0, None, 4)
    assert dn.lib.dnnopt_get_last_error() == dn.INVALID_VALUE
    fn(0, 4, 4, 1.0, None, 4, None, 4, 0.0, None, 4)
    assert dn.lib.dnnopt_get_last_error() == dn.SUCCESS


def test_plan_selection_without_device(dn):
    # Dispatch classes of the reference's shape router (src/gemm/gemm.cpp:168-455).
    s = dn.plan_describe(dn.KIND_F32, dn.desc(1, 4096, 4096, 4096, 4096, 4096))
    assert s.startswith("gemv_kn_splitk mt=1 vec4=1"), s
    # The irregular-N sweep (K = 1024): 64-column row panels, K in 4 ranges
    # of 256 rows, reduced by the last CTA of each panel.
    s = dn.plan_describe(dn.KIND_F32, dn.desc(7, 4093, 1024, 1024, 4093, 4093, beta=0.5))
    assert s == "gemv_panel mt=8 w=64 splits=4 ctas=256", s
    s = dn.plan_describe(dn.KIND_F32, dn.desc(2, 1009, 1024, 1024, 1009, 1009))
    assert s == "gemv_panel mt=2 w=64 splits=4 ctas=64", s
    s = dn.plan_describe(dn.KIND_F32, dn.desc(3, 2039, 600, 600, 2039, 2039))
    assert s == "gemv_panel mt=4 w=64 splits=2 ctas=64", s   # 600 rows: 2 ranges of 304
    # Other encodings of the same shapes keep the whole-K column slabs.
    s = dn.plan_describe(dn.KIND_BF16F32, dn.desc(7, 4093, 1024, 1024, 4093, 4093, beta=0.5))
    assert s == "gemv_kn_slab mt=8 w=8 ctas=512", s
    s = dn.plan_describe(dn.KIND_BF16F32, dn.desc(3, 2039, 1024, 1024, 2039, 2039))
    assert s == "gemv_kn_slab mt=4 w=16 ctas=128", s   # M <= 4 from 1536 columns on: 16 wide
    # Deeper K: split-K, one wave of resident CTAs, at most 16 splits.
    s = dn.plan_describe(dn.KIND_F32, dn.desc(7, 4093, 4096, 4096, 4093, 4093, beta=0.5))
    assert s.startswith("gemv_kn_splitk mt=8 vec4=0 splits=13 kchunk=320"), s   # prime N: scalar loads
    s = dn.plan_describe(dn.KIND_F32, dn.desc(2, 1009, 4096, 4096, 1009, 1009))
    assert s.startswith("gemv_kn_splitk mt=2 vec4=0 splits=16 kchunk=256"), s
    s = dn.plan_describe(dn.KIND_S8S32, dn.desc(4, 11008, 4096, 4096, 4096, 11008))
    assert s.startswith("gemv_rows_dot mt=4 vec=1"), s
    s = dn.plan_describe(dn.KIND_S8S32, dn.desc(4, 11008, 4100, 4100, 4100, 11008))
    assert s.startswith("gemv_nk_dot mt=4 vec=0"), s      # rows not 16-byte aligned
    s = dn.plan_describe(dn.KIND_E4M3BF16, dn.desc(8, 28672, 8192, 8192, 8192, 28672))
    assert s.startswith("gemv_nk_dot mt=8"), s
    s = dn.plan_describe(dn.KIND_F32, dn.desc(127, 127, 127, 127, 127, 127))
    assert s == "gemm_simt bm=64 bn=128 splits=2 kchunk=64", s      # 2 tiles: K split, two 32-deep slices per CTA
    s = dn.plan_describe(dn.KIND_F32, dn.desc(16, 4096, 4096, 4096, 4096, 4096))
    assert s == "gemm_simt bm=16 bn=128 splits=8 kchunk=512", s      # M 9-16: 16-row tiles
    s = dn.plan_describe(dn.KIND_F32, dn.desc(25088, 64, 1728, 1728, 1728, 64, trans_b=1))
    assert s == "gemm_simt bm=128 bn=64 splits=2 kchunk=864", s     # conv3d im2col GEMM: 128 x 64 tiles
    s = dn.plan_describe(dn.KIND_F32, dn.desc(3, 64, 32, 3, 32, 64, trans_a=1, trans_b=1))
    assert s.startswith("gemv_rows_dot"), s
    s = dn.plan_describe(dn.KIND_F32, dn.desc(3, 64, 30, 3, 30, 64, trans_a=1, trans_b=1))
    assert s.startswith("gemv_nk_dot"), s                 # K not a multiple of 4
    # Split-K keeps at least 64 K-rows per split.
    s = dn.plan_describe(dn.KIND_F32, dn.desc(2, 64, 100, 100, 64, 64))
    assert "splits=1 " in s, s


def test_autotune_cache_files(dn, tmp_path):
    p = str(tmp_path / "cache.bin").encode()
    n = dn.lib.dnnopt_autotune_save(p)
    assert n >= 0
    with open(p, "rb") as f:
        head = f.read(16)
    assert head[:8] == b"DNNAUTO\x00"
    assert struct.unpack("<II", head[8:16]) == (5, n)
    assert dn.lib.dnnopt_autotune_load(p) == n
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"DNNAUTO\x00" + struct.pack("<II", 3, 0))   # reference v3 file: rejected
    assert dn.lib.dnnopt_autotune_load(str(bad).encode()) == -1
    bad.write_bytes(plan_file_bytes([(1, (0, 1, 8, 1))], version=4))   # mistyped-basis keys: rejected
    assert dn.lib.dnnopt_autotune_load(str(bad).encode()) == -1
    bad.write_bytes(b"garbage")
    assert dn.lib.dnnopt_autotune_load(str(bad).encode()) == -1
    assert dn.lib.dnnopt_autotune_load(b"/nonexistent/file") == -1


def _saved_keys(dn, path):
    assert dn.lib.dnnopt_autotune_save(str(path).encode()) >= 0
    raw = path.read_bytes()
    n = struct.unpack("<I", raw[12:16])[0]
    return [struct.unpack("<Q", raw[16 + 28 * i:24 + 28 * i])[0] for i in range(n)]


def test_autotune_cache_is_lru_of_256(dn, tmp_path):
    """The plan cache keeps the 256 most recently used plans, like the
    reference's ShapeCache (include/dnnopt/autotune/shape_cache.h:139-146):
    inserting past the capacity evicts the least recently used key, and
    re-inserting a key refreshes it.  Saved files list keys least recent
    first, so a load restores the order."""
    base = 1 << 40
    first = [(base + i, (0, 1, 8, 1)) for i in range(300)]
    f1 = tmp_path / "many.bin"
    f1.write_bytes(plan_file_bytes(first))
    assert dn.lib.dnnopt_autotune_load(str(f1).encode()) == 300
    assert dn.lib.dnnopt_autotune_entries() == 256
    keys = _saved_keys(dn, tmp_path / "s1.bin")
    assert keys == [base + i for i in range(44, 300)]
    # Refresh the oldest survivor, then insert a new key: the next oldest goes.
    f2 = tmp_path / "two.bin"
    f2.write_bytes(plan_file_bytes([(base + 44, (0, 2, 8, 1)), (base + 1000, (0, 1, 8, 1))]))
    assert dn.lib.dnnopt_autotune_load(str(f2).encode()) == 2
    keys = _saved_keys(dn, tmp_path / "s2.bin")
    assert len(keys) == 256
    assert base + 45 not in keys and keys[-2:] == [base + 44, base + 1000]
    assert keys[0] == base + 46


def test_plan_key_hash_is_fnv1a():
    """Known-answer values of 64-bit FNV-1a for the key helper that the GPU
    tests use to force plans (a forced plan is found only when the library
    hashes its keys the same way)."""
    for b, want in ((b"", 0xCBF29CE484222325), (b"a", 0xAF63DC4C8601EC8C),
                    (b"foobar", 0x85944171F73967E8)):
        assert fnv1a64(b) == want


def test_thread_count_plumbing(dn):
    dn.lib.dnnopt_gemm_set_num_threads(12)
    assert dn.lib.dnnopt_gemm_get_num_threads() == 12
    dn.lib.dnnopt_gemm_set_num_threads(0)
    assert dn.lib.dnnopt_gemm_get_num_threads() == 1
    assert dn.has_fp8_support()


def test_fault_injection_control(dn):
    assert dn.lib.dnnopt_debug_inject_fault(9, 1) == dn.INVALID_VALUE
    assert dn.lib.dnnopt_debug_inject_fault(2, 0) == dn.SUCCESS


def test_product_library_does_not_link_oracle(dn):
    out = subprocess.run(["ldd", dn.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in out and "dnnopt_ref" not in out
    strings = open(dn.LIB_PATH, "rb").read()
    assert b"oracle_gemm" not in strings and b"ref_gemm_fp32" not in strings
