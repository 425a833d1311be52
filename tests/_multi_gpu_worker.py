"""Worker for tests/test_multi_gpu.py: one rank (one GPU) of the N-sharded
config-5 GEMM.  Checks, on every rank, that the fused GEMM + all-gather
(peer-memory stores inside the GEMM kernel) returns exactly the NCCL-mode
result on three consecutive calls (both output parities), and that both are
within the FP8 tolerance of the FP32-dequantised oracle."""
from __future__ import annotations

import datetime
import importlib.util
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = os.path.join(ROOT, "dnn-opt_b200")


def main() -> int:
    spec = importlib.util.spec_from_file_location("dnnopt_b200", os.path.join(PKG, "__init__.py"),
                                                  submodule_search_locations=[PKG])
    dn = importlib.util.module_from_spec(spec)
    sys.modules["dnnopt_b200"] = dn
    spec.loader.exec_module(dn)
    from dnnopt_b200.sharded import ShardedE4M3Gemm
    from oracle.oracle import Oracle, bf16_bits, bf16_to_f32

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    ok = True
    orc = Oracle()
    for (M, N, K) in [(8, 28672, 8192), (5, 1024 * world, 1024)]:
        A = bf16_bits(np.random.default_rng(42).standard_normal(M * K).astype(np.float32))
        W = (np.random.default_rng(123).standard_normal(N * K) * 0.02).astype(np.float32)
        q, s = orc.quantize_e4m3_rows(N, K, W, K)
        fused = ShardedE4M3Gemm(dist, N, K, rank, world, mode="fused")
        nccl = ShardedE4M3Gemm(dist, N, K, rank, world, mode="nccl")
        r0, r1 = fused.rows()
        dA = torch.from_numpy(A.view(np.int16).reshape(M, K)).cuda()
        dW = torch.from_numpy(q.reshape(N, K)[r0:r1].copy()).cuda()
        ds = torch.from_numpy(s[r0:r1].copy()).cuda()
        want = nccl.forward(dA, dW, ds).clone()
        for _ in range(3):
            got = fused.forward(dA, dW, ds)
            st = dn.stream_status(torch.cuda.current_stream())
            ok = ok and st == dn.SUCCESS and torch.equal(got, want)
        C = np.zeros(M * N, np.uint16)
        ref64 = orc.gemm_e4m3bf16(M, N, K, A, K, q, K, s, C, N).reshape(-1)
        g = bf16_to_f32(want.cpu().numpy().view(np.uint16).reshape(-1)).astype(np.float64)
        ok = ok and bool(np.all(np.abs(g - ref64) <= 2.0 ** -7 * np.abs(ref64) + 1e-4 * np.max(np.abs(ref64))))
        torch.cuda.synchronize()
        fused.close()
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    ok = int(flag.item()) == 1
    dist.destroy_process_group()
    if rank == 0:
        print("multi-gpu fused all-gather:", "ok" if ok else "MISMATCH", flush=True)
    return 0 if ok else 3


if __name__ == "__main__":
    sys.exit(main())
