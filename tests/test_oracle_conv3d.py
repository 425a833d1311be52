"""Pins the oracle's Conv3D restatement (CPU only).

oracle_conv3d restates dnnopt::conv3d_fp32 / conv3d_bf16 / conv3d_int8
(reference src/conv/conv3d.cpp).  On this x86 host the reference's own
conv3d_fp32 (built from its sources into oracle/_ref) is im2col3d plus its
naive GEMM, so the FP32 restatement must match it bit for bit, bias and
post-ops included.  The BF16 and INT8 entries fall back to FP32 on x86, so
their restatements are checked the way the reference's own
tests/test_conv3d_correctness.cpp checks the ARM paths: against a float64
direct convolution with its tolerances (K*1e-2 for BF16, K*5e-2 for INT8).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import load_ref, ref_uniform

# tests/test_conv3d_correctness.cpp:227-237: N, IC, ID, IH, IW, OC, KD, KH, KW, strides, pads.
CONV3D_SHAPES = [
    (1, 1, 3, 3, 3, 1, 3, 3, 3, 1, 1, 1, 1, 1, 1),
    (1, 3, 3, 8, 8, 4, 3, 3, 3, 1, 1, 1, 1, 1, 1),
    (1, 3, 4, 8, 8, 4, 3, 3, 3, 2, 2, 2, 1, 1, 1),
    (1, 16, 5, 16, 16, 32, 3, 3, 3, 1, 1, 1, 1, 1, 1),
    (1, 8, 8, 14, 14, 16, 5, 3, 3, 1, 1, 1, 2, 1, 1),
    (2, 4, 4, 8, 8, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1),
]


def out_dims(p):
    N, IC, ID, IH, IW, OC, KD, KH, KW, sd, sh, sw, pd, ph, pw = p
    return ((ID + 2 * pd - KD) // sd + 1, (IH + 2 * ph - KH) // sh + 1, (IW + 2 * pw - KW) // sw + 1)


def conv3d_operands(p, seed=42):
    N, IC, ID, IH, IW, OC, KD, KH, KW = p[:9]
    inp = ref_uniform(N * ID * IH * IW * IC, seed)
    flt = ref_uniform(OC * KD * KH * KW * IC, seed + 81)
    bias = ref_uniform(OC, seed + 7)
    OD, OH, OW = out_dims(p)
    return inp, flt, bias, N * OD * OH * OW * OC


def conv3d_f64(p, inp, flt, bias=None, post_op=0, quant=False):
    """Direct NDHWC convolution in float64 (INT8: on the quantised values)."""
    N, IC, ID, IH, IW, OC, KD, KH, KW, sd, sh, sw, pd, ph, pw = p
    OD, OH, OW = out_dims(p)
    x = inp.astype(np.float64).reshape(N, ID, IH, IW, IC)
    w = flt.astype(np.float64).reshape(OC, KD, KH, KW, IC)
    xp = np.zeros((N, ID + 2 * pd, IH + 2 * ph, IW + 2 * pw, IC))
    xp[:, pd:pd + ID, ph:ph + IH, pw:pw + IW, :] = x
    out = np.zeros((N, OD, OH, OW, OC))
    for kd in range(KD):
        for kh in range(KH):
            for kw in range(KW):
                patch = xp[:, kd:kd + sd * OD:sd, kh:kh + sh * OH:sh, kw:kw + sw * OW:sw, :]
                out += np.einsum("ndhwc,oc->ndhwo", patch, w[:, kd, kh, kw, :])
    if bias is not None:
        out += bias.astype(np.float64)
    if post_op == 1:
        out = np.maximum(out, 0)
    elif post_op == 2:
        out = np.clip(out, 0, 6)
    return out.ravel()


@pytest.mark.parametrize("p", CONV3D_SHAPES)
@pytest.mark.parametrize("post_op,with_bias", [(0, False), (1, True), (2, True)])
def test_fp32_bitexact_with_reference(orc, p, post_op, with_bias):
    ref = load_ref()
    if ref is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    inp, flt, bias, n_out = conv3d_operands(p)
    b = bias if with_bias else None
    got = np.zeros(n_out, np.float32)
    orc.conv3d(0, p, inp, flt, b, got, post_op)
    want = np.zeros(n_out, np.float32)
    pp = np.asarray(p, np.int32)
    ref.ref_conv3d(0, pp.ctypes.data, inp.ctypes.data, flt.ctypes.data,
                   None if b is None else b.ctypes.data, want.ctypes.data, post_op)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    K = p[1] * p[6] * p[7] * p[8]
    assert np.max(np.abs(got - conv3d_f64(p, inp, flt, b, post_op))) < K * 5e-5   # reference test bound


@pytest.mark.parametrize("p", CONV3D_SHAPES)
def test_bf16_int8_within_reference_tolerance(orc, p):
    inp, flt, bias, n_out = conv3d_operands(p)
    K = p[1] * p[6] * p[7] * p[8]
    exact = conv3d_f64(p, inp, flt, bias, 1)
    out = np.zeros(n_out, np.float32)
    r64 = orc.conv3d(1, p, inp, flt, bias, out, 1, want64=True)
    assert np.max(np.abs(out - exact)) < K * 1e-2                  # test_conv3d_correctness.cpp:138
    assert np.max(np.abs(out - r64)) <= 1e-5 * K                   # FP32 accumulation of bf16 products
    out8 = np.zeros(n_out, np.float32)
    orc.conv3d(2, p, inp, flt, bias, out8, 1)
    assert np.max(np.abs(out8 - exact)) < K * 5e-2                 # test_conv3d_correctness.cpp:169


def test_int8_quantisation_restated(orc):
    """INT8: the integer sums on the quantised tensors, dequantised with
    s_in * s_f, equal the oracle bit for bit (the float64 sums of small
    integers are exact)."""
    p = CONV3D_SHAPES[3]
    inp, flt, bias, n_out = conv3d_operands(p, seed=5)
    s_in = np.float32(np.max(np.abs(inp)) / np.float32(127))
    s_f = np.float32(np.max(np.abs(flt)) / np.float32(127))
    q = lambda x, s: np.clip(np.round(x * (np.float32(1) / s)), -128, 127)   # noqa: E731
    # np.round is half-to-even; roundf is half-away: no value here sits on .5 exactly
    acc = conv3d_f64(p, q(inp, s_in).astype(np.float32), q(flt, s_f).astype(np.float32))
    want = (acc.astype(np.float32) * (s_in * s_f)).astype(np.float32)
    out8 = np.zeros(n_out, np.float32)
    orc.conv3d(2, p, inp, flt, None, out8, 0)
    assert np.array_equal(out8, want)


def test_library_conv3d_argument_errors(dn):
    """Host-side checks of dnnopt_conv3d that need no device."""
    o = np.zeros(4, np.float32)
    ok = (1, 1, 3, 3, 3, 1, 3, 3, 3, 1, 1, 1, 1, 1, 1)
    assert dn.conv3d(3, ok, o, o, None, o) == dn.INVALID_VALUE             # precision
    assert dn.conv3d(0, ok, o, o, None, o, 3) == dn.INVALID_VALUE          # post-op
    assert dn.conv3d(0, (0,) + ok[1:], o, o, None, o) == dn.SUCCESS        # N = 0: no-op
    assert dn.conv3d(0, ok[:9] + (0, 1, 1) + ok[12:], o, o, None, o) == dn.INVALID_VALUE   # stride 0
    assert dn.conv3d(0, ok[:12] + (-1, 1, 1), o, o, None, o) == dn.INVALID_VALUE          # negative pad
    big = (1, 1, 2, 2, 2, 1, 11, 11, 11, 1, 1, 1, 5, 5, 5)                  # 1331 taps > 1024
    assert dn.conv3d(0, big, o, o, None, o) == dn.NOT_SUPPORTED
    assert dn.conv3d(0, ok, None, o, None, o) == dn.INVALID_VALUE
    assert np.all(o == 0)
