"""N-sharded decode-FFN weight GEMM over torch.distributed.

One process per GPU.  The weight matrix W [N, K] (OCP e4m3, K contiguous) and
its per-row scales are split by output rows: rank r owns rows
[bounds[r], bounds[r+1]).  Each rank computes its column block of
C[M, N] = A[M, K] x W^T, and every rank ends up with the whole C.  Two ways:

* ``mode="fused"`` (the B200 path): one C-ABI call,
  dnnopt_cuda_gemm_e4m3bf16_allgather, whose GEMM epilogue stores each
  finished column block straight into every rank's output buffer (peer memory
  mapped through CUDA IPC, NVLink stores) and raises a per-rank flag; the
  stream then waits (bounded) for every rank's flag.  No collective library
  is involved and the transfer overlaps the tiles still computing.  Calls are
  numbered on the device, so the arguments never change and the call can be
  captured in a CUDA graph; output buffers alternate by call parity so that a
  rank one call ahead never overwrites a buffer its peers may still read.
* ``mode="nccl"``: the shard GEMM (dnnopt_cuda_gemm_e4m3bf16) followed by an
  NCCL all-gather and a [G, M, n] -> [M, G*n] interleave (gloo in the CPU
  tests); kept as the library-collective comparison.

The reference has no multi-device code at all (it is single-process CPU);
this module is the B200 build's own data-parallel layer for the one config
that shards.
"""
from __future__ import annotations

from typing import Callable, Optional

FLAG_BYTES = 256          # flag array + call counter at the start of each rank's buffer
SEQ_OFFSET = 64           # this rank's device-side call counter (local use only)


def shard_bounds(N: int, world: int, align: int = 128) -> list[int]:
    """Row boundaries of the N-split: equal shares rounded up to `align` rows
    (the kernels' natural tile), the last shard taking the remainder."""
    if world < 1:
        raise ValueError("world must be >= 1")
    per = -(-N // world)
    per = -(-per // align) * align
    b = [min(N, r * per) for r in range(world)] + [N]
    return b


class _DeviceArray:
    """Zero-copy view of library-owned device memory for torch.as_tensor."""

    def __init__(self, address: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (address, False), "version": 3,
                                         "strides": None, "stream": None}


def _cuda_view(address: int, shape: tuple):
    import torch
    return torch.as_tensor(_DeviceArray(address, shape, "<i2"), device="cuda")


class ShardedE4M3Gemm:
    """Holds this rank's weight shard and runs the sharded GEMM + all-gather.

    Equal shard sizes are required (the configs use N divisible by
    128 * world).  `lib` is the dnnopt_b200 module (replaceable in host-logic
    tests); `compute` overrides the shard GEMM of the NCCL mode; `view`
    turns (address, shape) into the returned output (default: a torch CUDA
    tensor over the library buffer)."""

    def __init__(self, dist, N: int, K: int, rank: int, world: int,
                 compute: Optional[Callable] = None, group=None, mode: str = "nccl",
                 max_rows: int = 8, lib=None, view: Optional[Callable] = None):
        if mode not in ("nccl", "fused"):
            raise ValueError(f"unknown mode {mode!r}")
        self.dist, self.N, self.K = dist, N, K
        self.rank, self.world, self.group = rank, world, group
        self.mode = mode
        self.bounds = shard_bounds(N, world)
        sizes = {self.bounds[r + 1] - self.bounds[r] for r in range(world)}
        if len(sizes) != 1:
            raise ValueError(f"N={N} does not split evenly over {world} ranks in 128-row tiles")
        self.n_local = sizes.pop()
        self.compute = compute or self._compute_cuda
        self._lib = lib
        self._view = view or _cuda_view
        self.base = None
        self.peer_base: list[int] = []
        self.calls = 0
        self._ag = None
        self._descs = {}
        if mode == "fused":
            if world > self.dn.MAX_RANKS:
                raise ValueError(f"at most {self.dn.MAX_RANKS} ranks")
            self.max_rows = max_rows
            self.out_bytes = max_rows * N * 2
            self._setup_peers()

    @property
    def dn(self):
        if self._lib is None:
            import dnnopt_b200
            self._lib = dnnopt_b200
        return self._lib

    def rows(self) -> tuple[int, int]:
        return self.bounds[self.rank], self.bounds[self.rank + 1]

    # ---- fused mode -------------------------------------------------------
    def _exchange(self, handle: bytes) -> list[bytes]:
        """All-gather of this rank's 64-byte IPC handle."""
        import torch
        backend = self.dist.get_backend(self.group) if hasattr(self.dist, "get_backend") else "gloo"
        dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
        mine = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
        parts = [torch.empty(64, dtype=torch.uint8, device=dev) for _ in range(self.world)]
        self.dist.all_gather(parts, mine, group=self.group)
        return [bytes(p.cpu().tolist()) for p in parts]

    def _setup_peers(self) -> None:
        dn = self.dn
        self.base = dn.peer_alloc(FLAG_BYTES + 2 * self.out_bytes)
        handles = self._exchange(dn.ipc_handle(self.base))
        self.peer_base = [self.base if q == self.rank else dn.ipc_open(handles[q])
                          for q in range(self.world)]
        ag = dn.AllGatherDesc()
        ag.world, ag.rank = self.world, self.rank
        for q in range(self.world):
            ag.out[q] = self.peer_base[q] + FLAG_BYTES
            ag.flags[q] = self.peer_base[q]
        ag.seq = self.base + SEQ_OFFSET
        ag.out_stride = self.out_bytes
        self._ag = ag                          # the same arguments for every call
        self.dist.barrier(group=self.group)   # every rank has mapped every buffer

    def out_address(self, q: int, parity: int) -> int:
        return self.peer_base[q] + FLAG_BYTES + parity * self.out_bytes

    def forward_fused(self, A, W_shard, s_shard, stream=None):
        """A: [M, K] bf16 bits (int16), M <= max_rows.  Returns C [M, N]
        (int16 bf16 bits), a view of this rank's output buffer that stays valid
        until the call after next.  The c-th execution of the call (counting
        from 1, graph replays included) writes buffer c & 1; this method counts
        its own invocations to pick the view it returns."""
        dn = self.dn
        M = A.shape[0]
        if M > self.max_rows:
            raise ValueError(f"M={M} exceeds max_rows={self.max_rows}")
        d = self._descs.get(M)
        if d is None:
            d = self._descs[M] = dn.desc(M, self.n_local, self.K, self.K, self.K, self.N)
        if stream is None:
            import torch
            stream = torch.cuda.current_stream()
        dn.check(dn.cuda_gemm_e4m3bf16_allgather(d, A, W_shard, s_shard, self._ag, stream),
                 "fused e4m3 all-gather GEMM")
        self.calls += 1
        return self.output(self.calls & 1, M)

    def output(self, parity: int, M: int | None = None):
        """View of this rank's output buffer `parity` (the result of calls
        with that parity)."""
        return self._view(self.out_address(self.rank, parity), (M or self.max_rows, self.N))

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after a barrier, so
        no peer still writes into it)."""
        if self.mode != "fused" or self.base is None:
            return
        self.dist.barrier(group=self.group)
        for q, b in enumerate(self.peer_base):
            if q != self.rank:
                self.dn.ipc_close(b)
        self.dn.peer_free(self.base)
        self.base, self.peer_base = None, []

    # ---- NCCL mode --------------------------------------------------------
    def _compute_cuda(self, A, W, s, C):
        import torch
        dn = self.dn
        M = A.shape[0]
        d = dn.desc(M, self.n_local, self.K, self.K, self.K, self.n_local)
        dn.check(dn.cuda_gemm("e4m3bf16", d, A, W, C, torch.cuda.current_stream(), scale=s),
                 "e4m3 shard GEMM")

    def forward(self, A, W_shard, s_shard, C_local=None, gathered=None, out=None):
        """A: [M, K] bf16 bits (int16).  Returns C [M, N] (int16 bf16 bits)."""
        if self.mode == "fused":
            return self.forward_fused(A, W_shard, s_shard)
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
            # Byte views: NCCL has no 16-bit integer type.
            self.dist.all_gather_into_tensor(gathered.view(torch.uint8), C_local.view(torch.uint8),
                                             group=self.group)
        else:
            # Byte views: gloo has no 16-bit integer type either.
            parts = list(gathered.view(torch.uint8).unbind(0))
            self.dist.all_gather(parts, C_local.view(torch.uint8), group=self.group)
        if out is None:
            out = torch.empty((M, self.N), dtype=torch.int16, device=A.device)
        out.view(M, self.world, self.n_local).copy_(gathered.permute(1, 0, 2))
        return out
