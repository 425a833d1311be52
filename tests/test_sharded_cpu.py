"""Multi-rank host logic of the N-sharded config-5 GEMM on CPU (gloo).

Two (or four) processes each own a row block of the e4m3 weights, compute
their column block of C (the oracle stands in for the GPU kernel) and
assemble the full C with one all-gather; every rank must hold exactly the
single-process result."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds(dn):
    from dnnopt_b200.sharded import shard_bounds
    assert shard_bounds(28672, 1) == [0, 28672]
    assert shard_bounds(28672, 8) == [r * 3584 for r in range(9)]
    assert shard_bounds(1000, 3) == [0, 384, 768, 1000]
    with pytest.raises(ValueError):
        shard_bounds(10, 0)


def _run_ranks(world, **extra):
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()),
               WORLD_SIZE=str(world), CUDA_VISIBLE_DEVICES="", **extra)
    procs = [subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "_sharded_worker.py")],
                              env=dict(env, RANK=str(r)), stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(world)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    codes = [p.returncode for p in procs]
    assert codes == [0] * world, (codes, outs)


@pytest.mark.parametrize("world,N", [(2, 512), (4, 1024)])
def test_sharded_allgather_matches_single_process(dn, world, N):
    _run_ranks(world, M="8", N=str(N), K="256")


@pytest.mark.parametrize("world", [2, 4])
def test_fused_mode_host_logic(dn, world):
    """Fused mode: IPC-handle exchange maps every rank's buffer, every call
    passes the same arguments (the device numbers the calls), the returned
    view alternates buffers by parity, close() unmaps the peers and frees the
    own buffer."""
    _run_ranks(world, MODE="fused")


@pytest.mark.parametrize("world", [2, 3])
def test_dead_rank_detected(dn, world):
    """Failure detection on the host: a rank that leaves between calls makes
    the others' next all-gather fail within the process-group timeout."""
    _run_ranks(world, MODE="dead_rank")


def test_uneven_split_rejected(dn):
    from dnnopt_b200.sharded import ShardedE4M3Gemm
    with pytest.raises(ValueError):
        ShardedE4M3Gemm(None, 1000, 64, 0, 3)
