"""N-sharded decode-FFN weight GEMM over torch.distributed.

One process per GPU.  The weight matrix W [N, K] (OCP e4m3, K contiguous) and
its per-row scales are split by output rows: rank r owns rows
[bounds[r], bounds[r+1]).  Each rank computes its column block of
C[M, N] = A[M, K] x W^T through the C ABI (dnnopt_cuda_gemm_e4m3bf16), and the
blocks are assembled on every rank with one all-gather (NCCL over NVLink on
GPUs, gloo in the CPU tests) followed by a [G, M, n] -> [M, G*n] interleave.

The reference has no multi-device code at all (it is single-process CPU);
this module is the B200 build's own data-parallel layer for the one config
that shards.
"""
from __future__ import annotations

from typing import Callable, Optional


def shard_bounds(N: int, world: int, align: int = 128) -> list[int]:
    """Row boundaries of the N-split: equal shares rounded up to `align` rows
    (the kernels' natural tile), the last shard taking the remainder."""
    if world < 1:
        raise ValueError("world must be >= 1")
    per = -(-N // world)
    per = -(-per // align) * align
    b = [min(N, r * per) for r in range(world)] + [N]
    return b


class ShardedE4M3Gemm:
    """Holds this rank's weight shard and runs the sharded GEMM + all-gather.

    `compute(A, W_shard, scale_shard, C_shard)` fills C_shard [M, n_r]
    (bf16 bits as int16); the default calls the C ABI on the current CUDA
    stream.  Equal shard sizes are required for the collective (the configs
    use N divisible by 128 * world)."""

    def __init__(self, dist, N: int, K: int, rank: int, world: int,
                 compute: Optional[Callable] = None, group=None):
        self.dist, self.N, self.K = dist, N, K
        self.rank, self.world, self.group = rank, world, group
        self.bounds = shard_bounds(N, world)
        sizes = {self.bounds[r + 1] - self.bounds[r] for r in range(world)}
        if len(sizes) != 1:
            raise ValueError(f"N={N} does not split evenly over {world} ranks in 128-row tiles")
        self.n_local = sizes.pop()
        self.compute = compute or self._compute_cuda

    def rows(self) -> tuple[int, int]:
        return self.bounds[self.rank], self.bounds[self.rank + 1]

    def _compute_cuda(self, A, W, s, C):
        import torch
        import dnnopt_b200 as dn
        M = A.shape[0]
        d = dn.desc(M, self.n_local, self.K, self.K, self.K, self.n_local)
        dn.check(dn.cuda_gemm("e4m3bf16", d, A, W, C, torch.cuda.current_stream(), scale=s),
                 "e4m3 shard GEMM")

    def forward(self, A, W_shard, s_shard, C_local=None, gathered=None, out=None):
        """A: [M, K] bf16 bits (int16).  Returns C [M, N] (int16 bf16 bits)."""
        import torch
        M = A.shape[0]
        if C_local is None:
            C_local = torch.empty((M, self.n_local), dtype=torch.int16, device=A.device)
        self.compute(A, W_shard, s_shard, C_local)
        if gathered is None:
            gathered = torch.empty((self.world, M, self.n_local), dtype=torch.int16, device=A.device)
        if self.world == 1:
            gathered[0].copy_(C_local)
        elif hasattr(self.dist, "all_gather_into_tensor") and A.is_cuda:
            self.dist.all_gather_into_tensor(gathered, C_local, group=self.group)
        else:
            # Byte views: some backends (gloo) have no 16-bit integer type.
            parts = list(gathered.view(torch.uint8).unbind(0))
            self.dist.all_gather(parts, C_local.view(torch.uint8), group=self.group)
        if out is None:
            out = torch.empty((M, self.N), dtype=torch.int16, device=A.device)
        out.view(M, self.world, self.n_local).copy_(gathered.permute(1, 0, 2))
        return out
