"""The allocation-free entry point, dnnopt_cuda_gemm_f32_noalloc.

Callers whose device memory belongs to a framework's caching allocator,
serving loops that allow no allocation after warm-up, and runtimes with a
memory budget fixed at start-up cannot let a library call cudaMalloc.  This
entry point takes its split-K scratch from a fixed device array inside the
library instead.  The test calls it through the C ABI twice in a row per shape
and compares each result with dnnopt_cuda_gemm_f32 (which uses the per-stream
workspace) within the FP32 tolerance of the parity suite, 1e-5 * K.  It also
checks the limits: requests beyond the scratch capacity and shapes outside the
small-M class are refused with a status, before anything runs on the GPU.

The file is named to be collected last; it passes alone in a fresh process
(the first call performs the per-device set-up) and after the other tests.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import ref_uniform

pytestmark = pytest.mark.gpu

SHAPES = [(1, 4096, 4096), (2, 1009, 1024), (7, 4093, 1024), (5, 300, 513), (8, 131072, 64)]


def test_noalloc_matches_allocating_entry_point(torch_cuda, dn):
    torch = torch_cuda
    s = torch.cuda.current_stream()
    for (M, N, K) in SHAPES:
        A, B, C0 = ref_uniform(M * K, 11), ref_uniform(K * N, 12), ref_uniform(M * N, 13)
        d = dn.desc(M, N, K, K, N, N, 1.25, 0.5)
        dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
        want = torch.from_numpy(C0.copy()).cuda()
        dn.check(dn.cuda_gemm("f32", d, dA, dB, want, s), "allocating entry point")
        for call in range(2):
            got = torch.from_numpy(C0.copy()).cuda()
            dn.check(dn.cuda_gemm("f32_noalloc", d, dA, dB, got, s), "no-alloc entry point")
            torch.cuda.synchronize()
            err = float((got - want).abs().max().item())
            assert err <= 1e-5 * K, (M, N, K, call, err)


def test_noalloc_limits(torch_cuda, dn):
    torch = torch_cuda
    s = torch.cuda.current_stream()
    buf = torch.zeros(16, device="cuda")
    # More than 1024 strips of 128 columns does not fit the fixed ticket array.
    assert dn.cuda_gemm("f32_noalloc", dn.desc(1, 131073, 4, 4, 131073, 131073), buf, buf, buf,
                        s) == dn.EXCEEDS_SCRATCH
    # Outside the small-M streaming class.
    assert dn.cuda_gemm("f32_noalloc", dn.desc(9, 64, 4, 4, 64, 64), buf, buf, buf,
                        s) == dn.NOT_SUPPORTED
    assert dn.cuda_gemm("f32_noalloc", dn.desc(2, 64, 4, 4, 4, 64, trans_b=1), buf, buf, buf,
                        s) == dn.NOT_SUPPORTED
    assert dn.cuda_gemm("f32_noalloc", dn.desc(2, 64, 4, 3, 64, 64), buf, buf, buf,
                        s) == dn.INVALID_VALUE
    assert dn.cuda_gemm("f32_noalloc", dn.desc(0, 64, 4, 4, 64, 64), None, None, None,
                        s) == dn.SUCCESS
