"""Worker for tests/test_sharded_cpu.py: one gloo rank of the N-sharded
config-5 GEMM host logic, with the oracle standing in for the GPU kernel."""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PKG = os.path.join(ROOT, "dnn-opt_b200")


class _FakeLib:
    """Stands in for the C ABI in the fused mode's host logic: addresses are
    per-rank integers, IPC handles carry the address, and the fused GEMM call
    records its descriptors."""

    MAX_RANKS = 8

    def __init__(self, mod, rank):
        self.mod, self.rank = mod, rank
        self.AllGatherDesc, self.desc = mod.AllGatherDesc, mod.desc
        self.calls, self.closed, self.freed = [], [], []

    def check(self, st, what=""):
        assert st == 0, (st, what)

    def peer_alloc(self, nbytes):
        self.nbytes = nbytes
        return (self.rank + 1) << 40

    def ipc_handle(self, address):
        return address.to_bytes(8, "little") + bytes(56)

    def ipc_open(self, handle):
        assert len(handle) == 64
        return int.from_bytes(handle[:8], "little")

    def ipc_close(self, address):
        self.closed.append(address)

    def peer_free(self, address):
        self.freed.append(address)

    def cuda_gemm_e4m3bf16_allgather(self, d, A, W, s, ag, stream):
        self.calls.append((d.M, d.N, d.K, d.ldc, ag.world, ag.rank, ag.seq, ag.out_stride,
                           [ag.out[q] for q in range(ag.world)],
                           [ag.flags[q] for q in range(ag.world)]))
        return 0


def fused_host_logic(mod, rank, world) -> bool:
    """Peer-address exchange, constant per-call arguments (device-side call
    numbering) and the returned buffer's parity in the fused mode."""
    from dnnopt_b200.sharded import FLAG_BYTES, SEQ_OFFSET, ShardedE4M3Gemm
    M, N, K = 8, 128 * world * 3, 256
    fake = _FakeLib(mod, rank)
    sh = ShardedE4M3Gemm(dist, N, K, rank, world, mode="fused", lib=fake,
                         view=lambda address, shape: (address, shape))
    bases = [(q + 1) << 40 for q in range(world)]
    ok = sh.peer_base == bases and fake.nbytes == FLAG_BYTES + 2 * 8 * N * 2
    A = torch.zeros((M, K), dtype=torch.int16)
    for call in range(1, 4):
        address, shape = sh.forward_fused(A, None, None, stream=0)
        parity = call & 1
        m, n, k, ldc, w, r, seq, stride, outs, flags = fake.calls[-1]
        ok = ok and (m, n, k, ldc, w, r) == (M, N // world, K, N, world, rank)
        ok = ok and seq == bases[rank] + SEQ_OFFSET and stride == 8 * N * 2
        ok = ok and outs == [b + FLAG_BYTES for b in bases] and flags == bases
        ok = ok and address == bases[rank] + FLAG_BYTES + parity * 8 * N * 2 and shape == (M, N)
    sh.close()
    ok = ok and sorted(fake.closed) == sorted(b for q, b in enumerate(bases) if q != rank)
    ok = ok and fake.freed == [bases[rank]]
    return ok


def dead_rank(rank, world) -> int:
    """The last rank joins the group and leaves before the all-gather (between
    calls, with nothing in flight); every other rank must get an error from
    the collective within the short process-group timeout instead of hanging.
    Exit 0 = this rank behaved as expected."""
    import datetime
    from dnnopt_b200.sharded import ShardedE4M3Gemm
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == world - 1:
        return 0                      # leaves without a word
    M, N, K = 2, 128 * world, 64

    def compute(A_t, W_t, s_t, C_t):
        C_t.zero_()

    sh = ShardedE4M3Gemm(dist, N, K, rank, world, compute=compute)
    try:
        sh.forward(torch.zeros((M, K), dtype=torch.int16), None, None)
    except Exception as e:            # gloo: connection closed or timed out
        print(f"rank {rank}: peer loss detected: {type(e).__name__}", flush=True)
        return 0
    return 3


def main() -> None:
    spec = importlib.util.spec_from_file_location("dnnopt_b200", os.path.join(PKG, "__init__.py"),
                                                  submodule_search_locations=[PKG])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["dnnopt_b200"] = mod
    spec.loader.exec_module(mod)
    from dnnopt_b200.sharded import ShardedE4M3Gemm
    from oracle.oracle import Oracle, bf16_bits

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if os.environ.get("MODE") == "dead_rank":
        sys.exit(dead_rank(rank, world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    if os.environ.get("MODE") == "fused":
        ok = fused_host_logic(mod, rank, world)
        flag = torch.tensor([1 if ok else 0])
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        dist.destroy_process_group()
        sys.exit(0 if int(flag.item()) == 1 else 3)
    M, N, K = int(os.environ["M"]), int(os.environ["N"]), int(os.environ["K"])
    orc = Oracle()
    A = bf16_bits(np.random.default_rng(42).standard_normal(M * K).astype(np.float32))
    W = (np.random.default_rng(123).standard_normal(N * K) * 0.02).astype(np.float32)
    q, s = orc.quantize_e4m3_rows(N, K, W, K)

    def compute(A_t, W_t, s_t, C_t):
        m, n = A_t.shape[0], W_t.shape[0]
        out = np.zeros(m * n, np.uint16)
        orc.gemm_e4m3bf16(m, n, K, A_t.numpy().view(np.uint16).ravel(), K,
                          W_t.numpy().ravel(), K, s_t.numpy(), out, n, want64=False)
        C_t.copy_(torch.from_numpy(out.view(np.int16).reshape(m, n)))

    sh = ShardedE4M3Gemm(dist, N, K, rank, world, compute=compute)
    r0, r1 = sh.rows()
    Wl = torch.from_numpy(q.reshape(N, K)[r0:r1].copy())
    sl = torch.from_numpy(s[r0:r1].copy())
    out = sh.forward(torch.from_numpy(A.view(np.int16).reshape(M, K)), Wl, sl)
    full = np.zeros(M * N, np.uint16)
    orc.gemm_e4m3bf16(M, N, K, A, K, q, K, s, full, N, want64=False)
    ok = np.array_equal(out.numpy().view(np.uint16).ravel(), full)
    flag = torch.tensor([1 if ok else 0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 1 else 3)


if __name__ == "__main__":
    main()
