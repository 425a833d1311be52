"""The allocation-free entry point, dnnopt_cuda_gemm_f32_noalloc.

Callers whose device memory belongs to a framework's caching allocator,
serving loops that allow no allocation after warm-up, and runtimes with a
memory budget fixed at start-up cannot let a library call cudaMalloc.  This
entry point takes its split-K scratch from a fixed device array inside the
library instead.  The test calls it through the C ABI twice in a row per shape
and checks each result against the CPU oracle (the reference's naive FP32
restatement) and against dnnopt_cuda_gemm_f32 (which uses the per-stream
workspace) within the FP32 tolerance of the parity suite, 1e-5 * K; the two
calls must also agree bit for bit, since they share the array and the plan.
It also checks the limits: requests beyond the scratch capacity and shapes
outside the small-M class are refused with a status, before anything runs on
the GPU.

The file is named to be collected last; it passes alone in a fresh process
(the first call performs the per-device set-up) and after the other tests.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import ref_uniform

pytestmark = pytest.mark.gpu

# Deep K (16 splits), the config-2 class, a wide-N shape, odd sizes, and
# 1024 strips of 128 columns (the ticket array's capacity).
SHAPES = [(1, 4096, 4096), (2, 1009, 1024), (7, 4093, 1024), (5, 300, 513), (8, 131072, 64),
          (3, 8192, 2048)]


def test_noalloc_matches_oracle_and_allocating_entry_point(torch_cuda, dn, orc):
    torch = torch_cuda
    s = torch.cuda.current_stream()
    for (M, N, K) in SHAPES:
        A, B, C0 = ref_uniform(M * K, 11), ref_uniform(K * N, 12), ref_uniform(M * N, 13)
        ref = C0.copy()
        orc.gemm_f32(M, N, K, 1.25, A, K, B, N, 0.5, ref, N)
        d = dn.desc(M, N, K, K, N, N, 1.25, 0.5)
        dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
        want = torch.from_numpy(C0.copy()).cuda()
        dn.check(dn.cuda_gemm("f32", d, dA, dB, want, s), "allocating entry point")
        torch.cuda.synchronize()
        want = want.cpu().numpy()
        results = []
        for call in range(2):
            got = torch.from_numpy(C0.copy()).cuda()
            dn.check(dn.cuda_gemm("f32_noalloc", d, dA, dB, got, s), "no-alloc entry point")
            torch.cuda.synchronize()
            got = got.cpu().numpy()
            results.append(got)
            assert np.max(np.abs(got - ref)) <= 1e-5 * K, (M, N, K, call, "oracle")
            assert np.max(np.abs(got - want)) <= 1e-5 * K, (M, N, K, call, "allocating path")
        assert np.array_equal(results[0], results[1]), (M, N, K)


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
