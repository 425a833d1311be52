"""The drop-in header's storage types (include/dnnopt/gemm/gemm_types.h)
convert to and from float exactly as the reference's do
(include/dnnopt/gemm/gemm_types.h:14-200 of the reference): a small C++ shim
compiled against the header here is checked bit for bit against the golden
outputs of the reference's own codecs (all 256 decodes of each fp8 type, the
2,090-value encode sweep, bf16 rounding) and, on extra values (signed zeros,
infinities, NaN, subnormals, the saturation edges), against the oracle's
restatement, which the golden outputs pin."""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SHIM = r'''
#include "dnnopt/gemm/gemm_types.h"
extern "C" {
float e4m3_to_f32(unsigned char b) { return float(dnnopt::fp8_e4m3_t(b, true)); }
float e5m2_to_f32(unsigned char b) { return float(dnnopt::fp8_e5m2_t(b, true)); }
unsigned char e4m3_from_f32(float f) { dnnopt::fp8_e4m3_t x; x = f; return x.raw_bits; }
unsigned char e5m2_from_f32(float f) { return dnnopt::fp8_e5m2_t(f).raw_bits; }
unsigned short bf16_from_f32(float f) { return dnnopt::bfloat16_t(f).raw_bits; }
}
'''


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    d = tmp_path_factory.mktemp("hdr")
    src, lib = d / "shim.cpp", d / "libshim.so"
    src.write_text(SHIM)
    subprocess.run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"),
                    str(src), "-o", str(lib)], check=True)
    h = ctypes.CDLL(str(lib))
    for n in ("e4m3_to_f32", "e5m2_to_f32"):
        getattr(h, n).restype, getattr(h, n).argtypes = ctypes.c_float, [ctypes.c_ubyte]
    for n in ("e4m3_from_f32", "e5m2_from_f32"):
        getattr(h, n).restype, getattr(h, n).argtypes = ctypes.c_ubyte, [ctypes.c_float]
    h.bf16_from_f32.restype, h.bf16_from_f32.argtypes = ctypes.c_ushort, [ctypes.c_float]
    return h


def _bits(x):
    return np.asarray(x, np.float32).view(np.uint32)


def test_decodes_match_reference(shim, golden):
    for fn, key in ((shim.e4m3_to_f32, "ref_e4m3_decode"), (shim.e5m2_to_f32, "ref_e5m2_decode")):
        got = np.array([fn(b) for b in range(256)], np.float32)
        assert np.array_equal(_bits(got), _bits(golden[key])), key


def test_encodes_match_reference(shim, golden):
    sweep = golden["codec_sweep"]
    for fn, key in ((shim.e4m3_from_f32, "ref_e4m3_encode"), (shim.e5m2_from_f32, "ref_e5m2_encode")):
        got = np.array([fn(float(v)) for v in sweep], np.uint8)
        assert np.array_equal(got, golden[key]), key
    got = np.array([shim.bf16_from_f32(float(v)) for v in sweep], np.uint16)
    assert np.array_equal(got, golden["ref_bf16_encode"])


def test_encode_edges_match_oracle(shim, orc):
    edges = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 2.0 ** -6, 2.0 ** -7,
                      2.0 ** -9, 2.0 ** -14, 2.0 ** -16, 2.0 ** -17, 0.9375, 0.94, 1.0, 448.0,
                      57344.0, 65536.0, 3.4e38, -3.4e38, 1.5 * 2.0 ** -8], np.float32)
    rng = np.random.default_rng(5)
    vals = np.concatenate([edges, (rng.standard_normal(4000) * 10.0 ** rng.uniform(-8, 6, 4000))
                           .astype(np.float32)])
    for fn, codec in ((shim.e4m3_from_f32, "refe4m3"), (shim.e5m2_from_f32, "refe5m2")):
        got = np.array([fn(float(v)) for v in vals], np.uint8)
        assert np.array_equal(got, orc.table(codec, "from_f32", vals)), codec
