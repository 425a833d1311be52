"""Shared fixtures for the dnnopt B200 test suite.

CPU tests (-m "not gpu"): the oracle against the reference's golden outputs,
the C ABI's exports and host-side behaviour, multi-rank host logic on gloo.
GPU tests (-m gpu): the CUDA path through the C ABI against the oracle and the
golden fixtures.
"""
from __future__ import annotations

import importlib.util
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_outputs.npz")
PKG_DIR = os.path.join(ROOT, "dnn-opt_b200")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _ensure_built() -> None:
    lib = os.path.join(PKG_DIR, "lib", "libdnnopt_b200.so")
    orc = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-j8", "-C", PKG_DIR], check=True)
    if not os.path.exists(orc):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)


def load_dnnopt():
    """Import dnn-opt_b200/__init__.py as module `dnnopt_b200`."""
    if "dnnopt_b200" in sys.modules:
        return sys.modules["dnnopt_b200"]
    _ensure_built()
    spec = importlib.util.spec_from_file_location(
        "dnnopt_b200", os.path.join(PKG_DIR, "__init__.py"),
        submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["dnnopt_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


# Autotune-cache files ("DNNAUTO" v5): a plan key is the 64-bit FNV-1a hash
# (offset basis 14695981039346656037, prime 1099511628211) of ten
# little-endian int64 fields; an entry is the key plus (kernel id, p0, p1, mt,
# time_us).
PLAN_FILE_VERSION = 5


def fnv1a64(data: bytes) -> int:
    h = 14695981039346656037
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def plan_key(kind, M, N, K, lda, ldb, ldc, ta, tb, vec):
    import struct
    return fnv1a64(struct.pack("<10q", kind, M, N, K, lda, ldb, ldc, ta, tb, vec))


def plan_file_bytes(entries, version=PLAN_FILE_VERSION):
    """entries: [(key, (kernel, p0, p1, mt))], least recently used first."""
    import struct
    out = b"DNNAUTO\x00" + struct.pack("<II", version, len(entries))
    for key, e in entries:
        out += struct.pack("<Q", key) + struct.pack("<iiiif", *e, 0.0)
    return out


@pytest.fixture(scope="session")
def dn():
    return load_dnnopt()


@pytest.fixture(scope="session")
def orc():
    _ensure_built()
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def torch_cuda():
    """torch with a CUDA device; GPU tests skip cleanly on CPU-only hosts."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch
