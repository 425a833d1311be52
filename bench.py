#!/usr/bin/env python
"""Benchmark of the B200 small-M / irregular-N / tall-skinny GEMM path.

Headline workload: the FP32 small-batch
irregular-N sweep -- 12 GEMMs per step, M in {2,3,5,7} x N in {1009, 2039,
4093} (primes), K=1024, alpha=1, beta=0.5 -- run through the C ABI
(dnnopt_cuda_gemm_f32) and replayed as one CUDA graph per input set.  Three
input sets rotate (351 MB > the 126 MB L2), so every step reads from HBM.

Metric: GFLOP/s (2*M*N*K per GEMM summed over the sweep).  `e2e` is the same
metric through the reference-signature host API (dnnopt_gemm_fp32) with
pinned host buffers, copies included.  `per_config` adds configs 1, 3, 4, 5
(and the N-sharded config 5 when run on several GPUs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Multi-GPU: launched with torchrun, one rank per GPU; the sweep runs as
independent replicas (the reference and BASELINE shard only config 5, which
is reported under per_config.c5_sharded), value = all ranks' flops / max time.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "dnn-opt_b200")
sys.path.insert(0, ROOT)

C2_SHAPES = [(m, n, 1024) for m in (2, 3, 5, 7) for n in (1009, 2039, 4093)]
METRIC = "GFLOP/s (TOPS int8/fp8) and % of HBM/tensor roofline per shape vs reference CPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
N_SETS = 3
SWEEP_STREAMS = 12
# One workload string for both arms, so their lines name the same config.
WORKLOAD = ("C2 FP32 sweep: M{2,3,5,7} x N{1009,2039,4093} x K1024, alpha=1, beta=0.5 "
            "(12 GEMMs per step)")


def load_dnnopt():
    if "dnnopt_b200" in sys.modules:
        return sys.modules["dnnopt_b200"]
    spec = importlib.util.spec_from_file_location("dnnopt_b200", os.path.join(PKG, "__init__.py"),
                                                  submodule_search_locations=[PKG])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["dnnopt_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, source="fallback")


def lpt_assignment(sizes, n_streams):
    """Longest-processing-time assignment of independent jobs to streams:
    returns (issue order, stream index per job), largest job first, each onto
    the stream with the fewest bytes so far."""
    order = sorted(range(len(sizes)), key=lambda i: -sizes[i])
    load = [0] * n_streams
    stream_of = {}
    for i in order:
        k = min(range(n_streams), key=lambda j: load[j])
        stream_of[i] = k
        load[k] += sizes[i]
    return order, stream_of


def rotating_sets(bytes_per_set, floor=3):
    """Input sets to rotate between timed calls: at least `floor` and at least
    ~3x the 126 MB L2 in all (384 MB), so that no call finds its operands in
    L2 left over from an earlier call."""
    return max(floor, -(-384_000_000 // int(bytes_per_set)))


def gemm_bytes(M, N, K, beta, eb=4):
    return eb * (M * K + K * N + M * N * (2 if beta != 0 else 1))


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "window": "warm-up pre-roll + timed region"}


# ------------------------------------------------------------ reference arm --
def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_sweep_runner():
    """Returns (run_once, kind, sample, cores): one pass of the config-2 sweep
    on the host with the reference's own code (oracle/_ref) when it was built,
    else the oracle port, using every host thread (column slices)."""
    from oracle.oracle import Oracle, load_ref, ref_uniform
    threads = cpu_threads()
    data = []
    for (M, N, K) in C2_SHAPES:
        data.append((M, N, K, ref_uniform(M * K, 42), ref_uniform(K * N, 123), ref_uniform(M * N, 77)))
    ref = load_ref()
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if ref is not None:
        def run_once():
            for (M, N, K, A, B, C0) in data:
                C = C0.copy()
                ref.ref_gemm_fp32_naive_mt(M, N, K, 1.0, p(A), K, p(B), N, 0.5, p(C), N, threads)
        kind = "reference"
        sample = ("full config-2 sweep (12 GEMMs) per step through the reference's "
                  "gemm_fp32 (x86 portable path = gemm_naive_fp32), column slices on all host threads")
    else:
        orc = Oracle()
        # The oracle's naive restatement is single-threaded per call.
        def run_once():
            for (M, N, K, A, B, C0) in data:
                C = C0.copy()
                orc.gemm_f32(M, N, K, 1.0, A, K, B, N, 0.5, C, N)
        kind, threads = "port", 1
        sample = "full config-2 sweep per step through the oracle port (1 thread)"
    return run_once, kind, sample, threads


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    run_once, kind, sample, cores = reference_sweep_runner()
    flops = sum(2.0 * M * N * K for (M, N, K) in C2_SHAPES)
    for _ in range(args.warmup):
        run_once()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run_once()
    dt = (time.perf_counter() - t0) / args.steps
    v = flops / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded uniform[-1,1], reference test generator)",
        "config": {"workload": WORKLOAD},
        "cpu_baseline": {"value": v, "unit": "GFLOP/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": v, "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """Bounded CPU sample for the GPU arm's cpu_baseline (rank 0, N=1)."""
    run_once, kind, sample, cores = reference_sweep_runner()
    flops = sum(2.0 * M * N * K for (M, N, K) in C2_SHAPES)
    run_once()
    reps, t0 = 0, time.perf_counter()
    while reps < 2 or (time.perf_counter() - t0 < 10.0 and reps < 20):
        run_once()
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": flops / dt / 1e9, "unit": "GFLOP/s", "cores": cores, "kind": kind,
            "sample": sample + f"; {reps} sweeps timed"}


# ------------------------------------------------------------------ GPU arm --
def make_sweep_sets(torch, dev):
    from oracle.oracle import ref_uniform  # seeded generator only
    sets = []
    for s in range(N_SETS):
        items = []
        for (M, N, K) in C2_SHAPES:
            A = torch.from_numpy(ref_uniform(M * K, 42 + s)).to(dev)
            B = torch.from_numpy(ref_uniform(K * N, 123 + s)).to(dev)
            C = torch.from_numpy(ref_uniform(M * N, 77 + s)).to(dev)
            items.append((M, N, K, A, B, C))
        sets.append(items)
    return sets


def time_graphs(torch, graphs, steps, warmup, stream, dist=None):
    for i in range(warmup):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        graphs[i % len(graphs)].replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    return ms / steps


def capture(torch, stream, fn):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


# DRAM bytes (read + write) of one C2 sweep, summed over its 12 launches of
# the row-panel GEMV, from one ncu capture:  ncu --clock-control none --metrics
# dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum --csv
# -k regex:gemv -s 12 -c 12 python bench.py --profile c2 --reps 2
# (C and the split partials are written into L2 and leave it after the launch,
# so writes read 0).
C2_DRAM_BYTES_PER_STEP = 117_945_344


def bench_single(torch, dn, stream, fn_list, bytes_per_call, flops_per_call, iters=30):
    """Per-call device time of rotating calls: one CUDA graph holds 4 rounds
    over `fn_list` (so graph-launch overhead is amortised), replayed `iters`
    times between CUDA events on `stream`."""
    rounds = 4
    g = capture(torch, stream, lambda: [f() for _ in range(rounds) for f in fn_list])
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (iters * rounds * len(fn_list))
    return {"us_per_call": us, "GB_s": bytes_per_call / us / 1e3, "TFLOP_s": flops_per_call / us / 1e6}


def per_config(torch, dn, stream, pk, world, rank, dist):
    from oracle.oracle import bf16_bits, int8_uniform, ref_uniform
    out = {}
    s = stream
    # C1: FP32 1 x 4096 x 4096.
    M, N, K = 1, 4096, 4096
    ns = rotating_sets(gemm_bytes(M, N, K, 0.0))
    As = [torch.from_numpy(ref_uniform(M * K, 42 + i)).cuda() for i in range(ns)]
    Bs = [torch.from_numpy(ref_uniform(K * N, 123 + i)).cuda() for i in range(ns)]
    Cs = [torch.zeros(M * N, device="cuda") for _ in range(ns)]
    d = dn.desc(M, N, K, K, N, N)
    for i in range(ns):
        dn.check(dn.cuda_gemm("f32", d, As[i], Bs[i], Cs[i], s))
    fns = [lambda i=i: dn.cuda_gemm("f32", d, As[i], Bs[i], Cs[i], s) for i in range(ns)]
    r = bench_single(torch, dn, s, fns, gemm_bytes(M, N, K, 0.0), 2.0 * M * N * K)
    out["c1_fp32_1x4096x4096"] = {"GFLOP_s": r["TFLOP_s"] * 1e3, "us": r["us_per_call"],
                                  "GB_s": r["GB_s"], "hbm_frac": r["GB_s"] / pk["hbm_gbs"],
                                  "input_sets": ns, "kernel": dn.plan_describe(dn.KIND_F32, d)}
    del As, Bs, Cs
    # The oneDNN entry on an inner-product pattern: column-major C (OC x batch)
    # = W^T-stored weights x activations + bias, through dnnopt_cuda_sgemm_colmajor.
    M, N, K = 4096, 1, 4096
    ns = rotating_sets(4 * (M * K + K * N + M * N))
    Ws = [torch.from_numpy(ref_uniform(M * K, 52 + i)).cuda() for i in range(ns)]
    Xs = [torch.from_numpy(ref_uniform(K * N, 133 + i)).cuda() for i in range(ns)]
    Ys = [torch.zeros(M * N, device="cuda") for _ in range(ns)]
    bias = torch.from_numpy(ref_uniform(M, 7)).cuda()
    fns = [lambda i=i: dn.cuda_sgemm_colmajor("T", "N", M, N, K, 1.0, Ws[i], K, Xs[i], K, 0.0, Ys[i], M,
                                              bias, s) for i in range(ns)]
    for f in fns:
        dn.check(f())
    r = bench_single(torch, dn, s, fns, 4 * (M * K + K * N + M * N + M), 2.0 * M * N * K)
    out["onednn_sgemm_T_N_4096x1x4096_bias"] = {
        "GFLOP_s": r["TFLOP_s"] * 1e3, "us": r["us_per_call"], "GB_s": r["GB_s"],
        "hbm_frac": r["GB_s"] / pk["hbm_gbs"],
        "kernel": dn.plan_describe(dn.KIND_F32, dn.desc(N, M, K, K, K, M, trans_b=1)) + " + bias epilogue"}
    del Ws, Xs, Ys
    # Conv3D (the in-tree caller of the BF16 / INT8 GEMMs), a video layer:
    # N=1, IC=64, 8x56x56, OC=64, 3x3x3, stride 1, pad 1, bias + relu.
    cp = (1, 64, 8, 56, 56, 64, 3, 3, 3, 1, 1, 1, 1, 1, 1)
    nin, nflt, nout = 8 * 56 * 56 * 64, 64 * 27 * 64, 8 * 56 * 56 * 64
    cin = torch.from_numpy(ref_uniform(nin, 3)).cuda()
    cflt = torch.from_numpy(ref_uniform(nflt, 4)).cuda()
    cbias = torch.from_numpy(ref_uniform(64, 5)).cuda()
    cout = torch.zeros(nout, device="cuda")
    flops = 2.0 * nout * 27 * 64
    for prec, name in ((0, "fp32"), (1, "bf16"), (2, "int8")):
        fns = [lambda prec=prec: dn.cuda_conv3d(prec, cp, cin, cflt, cbias, cout, dn.POSTOP_RELU, s)]
        dn.check(fns[0](), "conv3d")
        r = bench_single(torch, dn, s, fns, 4 * (nin + nflt + nout), flops, iters=10)
        out[f"conv3d_{name}_1x64x8x56x56_oc64_k3"] = {
            "TFLOP_s": r["TFLOP_s"], "us": r["us_per_call"],
            "note": {"fp32": "SIMT implicit GEMM gathering A from the input, bias/relu in its epilogue",
                     "bf16": "padded BF16 copy + implicit tcgen05 kind::f16 conv (window boxes), bias/relu in its epilogue",
                     "int8": "cooperative absmax/quantised padded copy + implicit tcgen05 kind::i8 conv, "
                             "dequant/bias/relu in its epilogue"}[name]}
    del cin, cflt, cbias, cout
    # C3: INT8 4 x 11008 x 4096, B is [N, K].
    M, N, K = 4, 11008, 4096
    ns = rotating_sets(M * K + N * K + 4 * M * N)
    As = [torch.from_numpy(int8_uniform(M * K, 42 + i)).cuda() for i in range(ns)]
    Bs = [torch.from_numpy(int8_uniform(N * K, 123 + i)).cuda() for i in range(ns)]
    Cs = [torch.zeros(M * N, dtype=torch.int32, device="cuda") for _ in range(ns)]
    d = dn.desc(M, N, K, K, K, N)
    for i in range(ns):
        dn.check(dn.cuda_gemm("s8s32", d, As[i], Bs[i], Cs[i], s))
    fns = [lambda i=i: dn.cuda_gemm("s8s32", d, As[i], Bs[i], Cs[i], s) for i in range(ns)]
    r = bench_single(torch, dn, s, fns, M * K + N * K + 4 * M * N, 2.0 * M * N * K)
    out["c3_int8_4x11008x4096"] = {"TOPS": r["TFLOP_s"], "us": r["us_per_call"], "GB_s": r["GB_s"],
                                   "hbm_frac": r["GB_s"] / pk["hbm_gbs"], "input_sets": ns,
                                   "kernel": dn.plan_describe(dn.KIND_S8S32, d)}
    del As, Bs, Cs
    # C4: BF16 65536 x 64 x 256 -> FP32.
    M, N, K = 65536, 64, 256
    ns = rotating_sets(2 * (M * K + K * N) + 4 * M * N)
    rng = np.random.default_rng(42)
    As = [torch.from_numpy(bf16_bits(rng.standard_normal(M * K).astype(np.float32)).view(np.int16)).cuda()
          for _ in range(ns)]
    Bs = [torch.from_numpy(bf16_bits(rng.standard_normal(K * N).astype(np.float32)).view(np.int16)).cuda()
          for _ in range(ns)]
    Cs = [torch.zeros(M * N, device="cuda") for _ in range(ns)]
    d = dn.desc(M, N, K, K, N, N)
    for i in range(ns):
        dn.check(dn.cuda_gemm("bf16f32", d, As[i], Bs[i], Cs[i], s))
    fns = [lambda i=i: dn.cuda_gemm("bf16f32", d, As[i], Bs[i], Cs[i], s) for i in range(ns)]
    r = bench_single(torch, dn, s, fns, 2 * (M * K + K * N) + 4 * M * N, 2.0 * M * N * K)
    out["c4_bf16_65536x64x256"] = {"TFLOP_s": r["TFLOP_s"], "us": r["us_per_call"], "GB_s": r["GB_s"],
                                   "hbm_frac": r["GB_s"] / pk["hbm_gbs"], "input_sets": ns,
                                   "tensor_frac": r["TFLOP_s"] / pk["bf16_tflops"],
                                   "kernel": dn.plan_describe(dn.KIND_BF16F32, d)}
    del As, Bs, Cs
    # Small-M BF16 on the general tcgen05 GEMM (B [K, N], K split across the
    # CTAs of a thread-block cluster): the M >= 9 band above the GEMV kernels.
    for M in (64, 16):
        N, K = 4096, 4096
        byts = 2 * (M * K + K * N) + 4 * M * N
        ns = rotating_sets(byts)
        As = [torch.randn(M * K, device="cuda").to(torch.bfloat16).view(torch.int16) for _ in range(ns)]
        Bs = [torch.randn(K * N, device="cuda").to(torch.bfloat16).view(torch.int16) for _ in range(ns)]
        Cs = [torch.zeros(M * N, device="cuda") for _ in range(ns)]
        d = dn.desc(M, N, K, K, N, N)
        for i in range(ns):
            dn.check(dn.cuda_gemm("bf16f32", d, As[i], Bs[i], Cs[i], s))
        fns = [lambda i=i: dn.cuda_gemm("bf16f32", d, As[i], Bs[i], Cs[i], s) for i in range(ns)]
        r = bench_single(torch, dn, s, fns, byts, 2.0 * M * N * K)
        out[f"bf16_{M}x{N}x{K}"] = {"TFLOP_s": r["TFLOP_s"], "us": r["us_per_call"], "GB_s": r["GB_s"],
                                    "hbm_frac": r["GB_s"] / pk["hbm_gbs"], "input_sets": ns,
                                    "kernel": dn.plan_describe(dn.KIND_BF16F32, d)}
        del As, Bs, Cs
    # C5: e4m3 decode-FFN 8 x 28672 x 8192 (W 235 MB > L2).
    M, N, K = 8, 28672, 8192
    A = torch.from_numpy(bf16_bits(np.random.default_rng(42).standard_normal(M * K)
                                   .astype(np.float32)).view(np.int16)).cuda()
    g = torch.Generator(device="cuda").manual_seed(123)
    Wf = torch.randn((N, K), device="cuda", generator=g) * 0.02
    scale = (Wf.abs().amax(dim=1) / 448.0).clamp_min(1e-30)
    W = (Wf / scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
    del Wf
    C = torch.zeros(M * N, dtype=torch.int16, device="cuda")
    d = dn.desc(M, N, K, K, K, N)
    dn.check(dn.cuda_gemm("e4m3bf16", d, A, W, C, s, scale=scale))
    fns = [lambda: dn.cuda_gemm("e4m3bf16", d, A, W, C, s, scale=scale)]
    r = bench_single(torch, dn, s, fns, N * K + 4 * N + 2 * M * K + 2 * M * N, 2.0 * M * N * K, iters=10)
    out["c5_e4m3_8x28672x8192"] = {"TFLOP_s": r["TFLOP_s"], "us": r["us_per_call"], "GB_s": r["GB_s"],
                                   "hbm_frac": r["GB_s"] / pk["hbm_gbs"],
                                   "kernel": dn.plan_describe(dn.KIND_E4M3BF16, d)}
    # C5 N-sharded over the ranks (BASELINE: 1/2/4/8 GPUs): the fused GEMM +
    # all-gather (peer-memory stores inside the GEMM kernel), the shard GEMM
    # followed by an NCCL all-gather, the shard GEMM alone, and the full GEMM
    # on one GPU, all timed the same way, so that speed-up and efficiency
    # against one GPU come from one run.
    def queued_us(call, n=100):
        """Device time per call of n back-to-back calls: the stream first
        spins for ~20 ms so that the host has queued every call before the
        first event (an eager Python call costs more host time than the GPU
        work at 4-8 ranks), max over ranks."""
        for _ in range(3):
            call(0)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(40_000_000)
        e0.record()
        for i in range(n):
            call(i)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / n], device="cuda")
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) * 1e3

    full_us = queued_us(lambda i: dn.check(dn.cuda_gemm("e4m3bf16", d, A, W, C, s, scale=scale)))
    sharded = {"ranks": world, "full_1gpu_us": full_us,
               "timing": "device time per call, 100 calls queued behind a GPU sleep, max over ranks"}
    if world == 1:
        sharded.update({"us": full_us, "speedup_vs_1gpu": 1.0, "efficiency": 1.0,
                        "kernel": dn.plan_describe(dn.KIND_E4M3BF16, d)})
    else:
        from dnnopt_b200.sharded import ShardedE4M3Gemm  # noqa: E402
        Am = A.view(M, K)
        res = {}
        for mode in ("fused", "nccl"):
            sh = ShardedE4M3Gemm(dist, N, K, rank, world, mode=mode)
            r0, r1 = sh.rows()
            sl = scale[r0:r1].contiguous()
            # Rotating copies of the weight shard, > 256 MB in all, so that no
            # call finds its shard in the 126 MB L2.
            n_copies = 1 + (256 << 20) // ((r1 - r0) * K)
            Ws = [W[r0:r1].clone() for _ in range(n_copies)]
            bufs = {}
            if mode == "nccl":
                bufs = dict(C_local=torch.empty((M, sh.n_local), dtype=torch.int16, device="cuda"),
                            gathered=torch.empty((world, M, sh.n_local), dtype=torch.int16, device="cuda"),
                            out=torch.empty((M, N), dtype=torch.int16, device="cuda"))
            holder = {}

            def call(i, sh=sh, Ws=Ws, sl=sl, bufs=bufs, holder=holder, n_copies=n_copies):
                holder["out"] = sh.forward(Am, Ws[i % n_copies], sl, **bufs)
            res[mode] = (queued_us(call), holder["out"].reshape(-1).clone())
            if mode == "fused":
                ok_status = dn.stream_status(torch.cuda.current_stream()) == dn.SUCCESS
                # The shard GEMM alone (no all-gather), same rotating shards.
                ds = dn.desc(M, r1 - r0, K, K, K, r1 - r0)
                Cl = torch.empty(M * (r1 - r0), dtype=torch.int16, device="cuda")
                shard_us = queued_us(lambda i: dn.check(dn.cuda_gemm("e4m3bf16", ds, A, Ws[i % n_copies], Cl, s,
                                                                     scale=sl)))
            sh.close()
            del Ws
        us = res["fused"][0]
        sharded.update({
            "us": us, "TFLOP_s": 2.0 * M * N * K / us / 1e6,
            "speedup_vs_1gpu": full_us / us, "efficiency": full_us / us / world,
            "GB_s_per_gpu": (N * K / world + 4 * N / world + 2 * M * K + 2 * M * N) / us / 1e3,
            "kernel": "gemm_e4m3_tcgen05 with peer-memory all-gather epilogue + bounded flag wait",
            "nccl_allgather_us": res["nccl"][0], "nccl_speedup_vs_1gpu": full_us / res["nccl"][0],
            "shard_gemm_alone_us": shard_us,
            "matches_nccl_path": bool(torch.equal(res["fused"][1], res["nccl"][1])) and ok_status,
            "shard_plan": dn.plan_describe(dn.KIND_E4M3BF16, dn.desc(M, N // world, K, K, K, N // world))})
    out["c5_sharded"] = sharded
    return out


def run_profile(args):
    """Runs one config's kernel `--reps` times on rotating inputs and exits
    (the command that ncu captures; prints no bench line)."""
    import torch
    from oracle.oracle import bf16_bits, int8_uniform, ref_uniform
    dn = load_dnnopt()
    torch.cuda.set_device(0)
    s = torch.cuda.current_stream()
    name = args.profile
    calls = []
    if name == "c2":
        for items in make_sweep_sets(torch, torch.device("cuda", 0)):
            for (M, N, K, A, B, C) in items:
                d = dn.desc(M, N, K, K, N, N, 1.0, 0.5)
                calls.append(lambda d=d, A=A, B=B, C=C: dn.cuda_gemm("f32", d, A, B, C, s))
    elif name == "c1":
        M, N, K = 1, 4096, 4096
        d = dn.desc(M, N, K, K, N, N)
        for i in range(N_SETS):
            A = torch.from_numpy(ref_uniform(M * K, 42 + i)).cuda()
            B = torch.from_numpy(ref_uniform(K * N, 123 + i)).cuda()
            C = torch.zeros(M * N, device="cuda")
            calls.append(lambda A=A, B=B, C=C: dn.cuda_gemm("f32", d, A, B, C, s))
    elif name == "simt64":
        M, N, K = 64, 4096, 4096
        d = dn.desc(M, N, K, K, N, N)
        for i in range(N_SETS):
            A = torch.from_numpy(ref_uniform(M * K, 42 + i)).cuda()
            B = torch.from_numpy(ref_uniform(K * N, 123 + i)).cuda()
            C = torch.zeros(M * N, device="cuda")
            calls.append(lambda A=A, B=B, C=C: dn.cuda_gemm("f32", d, A, B, C, s))
    elif name in ("conv3d_fp32", "conv3d_bf16", "conv3d_int8"):
        # The bench's Conv3D layer (BF16 / INT8: operand prep + implicit tcgen05 conv).
        cp = (1, 64, 8, 56, 56, 64, 3, 3, 3, 1, 1, 1, 1, 1, 1)
        nin, nflt, nout = 8 * 56 * 56 * 64, 64 * 27 * 64, 8 * 56 * 56 * 64
        cin = torch.from_numpy(ref_uniform(nin, 3)).cuda()
        cflt = torch.from_numpy(ref_uniform(nflt, 4)).cuda()
        cbias = torch.from_numpy(ref_uniform(64, 5)).cuda()
        cout = torch.zeros(nout, device="cuda")
        prec = {"conv3d_fp32": 0, "conv3d_bf16": 1, "conv3d_int8": 2}[name]
        calls.append(lambda: dn.cuda_conv3d(prec, cp, cin, cflt, cbias, cout, dn.POSTOP_RELU, s))
    elif name == "onednn":
        M, N, K = 4096, 1, 4096
        bias = torch.from_numpy(ref_uniform(M, 7)).cuda()
        for i in range(N_SETS):
            W = torch.from_numpy(ref_uniform(M * K, 52 + i)).cuda()
            X = torch.from_numpy(ref_uniform(K * N, 133 + i)).cuda()
            Y = torch.zeros(M * N, device="cuda")
            calls.append(lambda W=W, X=X, Y=Y: dn.cuda_sgemm_colmajor("T", "N", M, N, K, 1.0, W, K, X, K,
                                                                      0.0, Y, M, bias, s))
    elif name == "c3":
        M, N, K = 4, 11008, 4096
        d = dn.desc(M, N, K, K, K, N)
        for i in range(N_SETS):
            A = torch.from_numpy(int8_uniform(M * K, 42 + i)).cuda()
            B = torch.from_numpy(int8_uniform(N * K, 123 + i)).cuda()
            C = torch.zeros(M * N, dtype=torch.int32, device="cuda")
            calls.append(lambda A=A, B=B, C=C: dn.cuda_gemm("s8s32", d, A, B, C, s))
    elif name == "c4":
        M, N, K = 65536, 64, 256
        d = dn.desc(M, N, K, K, N, N)
        rng = np.random.default_rng(42)
        for i in range(N_SETS):
            A = torch.from_numpy(bf16_bits(rng.standard_normal(M * K).astype(np.float32)).view(np.int16)).cuda()
            B = torch.from_numpy(bf16_bits(rng.standard_normal(K * N).astype(np.float32)).view(np.int16)).cuda()
            C = torch.zeros(M * N, device="cuda")
            calls.append(lambda A=A, B=B, C=C: dn.cuda_gemm("bf16f32", d, A, B, C, s))
    elif name == "tc_i8":
        # The general tcgen05 GEMM (kind::i8) on int8 2048^3, B stored [N, K].
        M, N, K = 2048, 2048, 2048
        d = dn.desc(M, N, K, K, K, N)
        C = torch.zeros(M * N, dtype=torch.int32, device="cuda")
        for i in range(4):
            A = torch.randint(-127, 128, (M * K,), dtype=torch.int8, device="cuda")
            B = torch.randint(-127, 128, (N * K,), dtype=torch.int8, device="cuda")
            calls.append(lambda A=A, B=B: dn.cuda_gemm("s8s32", d, A, B, C, s))
    elif name == "tc_bf16_small":
        # The general tcgen05 GEMM on small-M BF16 64 x 4096 x 4096 (B [K, N]):
        # K split across the CTAs of a thread-block cluster.
        M, N, K = 64, 4096, 4096
        d = dn.desc(M, N, K, K, N, N)
        for i in range(N_SETS):
            A = torch.randn(M * K, device="cuda").to(torch.bfloat16).view(torch.int16)
            B = torch.randn(K * N, device="cuda").to(torch.bfloat16).view(torch.int16)
            C = torch.zeros(M * N, device="cuda")
            calls.append(lambda A=A, B=B, C=C: dn.cuda_gemm("bf16f32", d, A, B, C, s))
    elif name == "c5":
        M, N, K = 8, 28672, 8192
        d = dn.desc(M, N, K, K, K, N)
        A = torch.from_numpy(bf16_bits(np.random.default_rng(42).standard_normal(M * K)
                                       .astype(np.float32)).view(np.int16)).cuda()
        g = torch.Generator(device="cuda").manual_seed(123)
        Wf = torch.randn((N, K), device="cuda", generator=g) * 0.02
        scale = (Wf.abs().amax(dim=1) / 448.0).clamp_min(1e-30)
        W = (Wf / scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
        del Wf
        C = torch.zeros(M * N, dtype=torch.int16, device="cuda")
        calls.append(lambda: dn.cuda_gemm("e4m3bf16", d, A, W, C, s, scale=scale))
    else:
        raise SystemExit(f"unknown profile config {name}")
    for r in range(args.reps):
        for c in calls:
            dn.check(c(), name)
    torch.cuda.synchronize()
    print(f"profile {name}: {args.reps} x {len(calls)} calls ok")


def run_gpu_arm(args):
    import torch
    import torch.distributed as dist
    dn = load_dnnopt()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    use_dist = world > 1
    if use_dist:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(device=dev)
    pk = peaks()
    torch.cuda.set_stream(stream)

    sets = make_sweep_sets(torch, dev)
    flops = sum(2.0 * M * N * K for (M, N, K) in C2_SHAPES)
    bytes_step = sum(gemm_bytes(M, N, K, 0.5) for (M, N, K) in C2_SHAPES)
    # The 12 GEMMs are independent: issue them on SWEEP_STREAMS streams forked
    # from and joined back into `stream`, so their latencies overlap; each
    # stream has its own library workspace.  Streams are loaded by bytes,
    # largest GEMM first onto the least-loaded stream (longest-processing-time
    # order), so that no stream carries much more than its share.
    side = [torch.cuda.Stream(device=dev) for _ in range(args.streams)]
    order, stream_of = lpt_assignment([gemm_bytes(M, N, K, 0.5) for (M, N, K) in C2_SHAPES], args.streams)

    def sweep(items, streams):
        if streams is None or len(streams) == 1:
            streams = [stream]
            for (M, N, K, A, B, C) in items:
                dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, K, N, N, 1.0, 0.5), A, B, C,
                                      streams[0]), "sweep GEMM")
            return
        fork = torch.cuda.Event()
        fork.record(stream)
        for st in streams:
            st.wait_event(fork)
        for i in order:
            (M, N, K, A, B, C) = items[i]
            dn.check(dn.cuda_gemm("f32", dn.desc(M, N, K, K, N, N, 1.0, 0.5), A, B, C,
                                  streams[stream_of[i]]), "sweep GEMM")
        for st in streams:
            join = torch.cuda.Event()
            join.record(st)
            stream.wait_event(join)

    for items in sets:      # first calls size the workspaces and plans (not capturable)
        sweep(items, side)
        sweep(items, None)
    torch.cuda.synchronize()
    n0 = dn.launch_count()
    graphs = [capture(torch, stream, lambda it=items: sweep(it, side)) for items in sets]
    launches_per_step = (dn.launch_count() - n0) // len(sets)
    serial_graphs = [capture(torch, stream, lambda it=items: sweep(it, None)) for items in sets]

    clocks = ClockSampler(local)
    clocks.start()
    t_end = time.time() + 0.6           # pre-roll under load so the sampler sees it
    while time.time() < t_end:
        for g in graphs:
            g.replay()
        torch.cuda.synchronize()
    ms = time_graphs(torch, graphs, args.steps, max(args.warmup, 3), stream, dist if use_dist else None)
    clk = clocks.stop()
    value = flops * world / (ms * 1e-3) / 1e9

    # Dominant kernel: the row-panel GEMV, all 12 launches of a step.
    achieved = bytes_step / (ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": C2_DRAM_BYTES_PER_STEP,
                "traffic_unit": "bytes per step (12 launches), ncu dram__bytes_read.sum + dram__bytes_write.sum",
                "algorithmic_bytes_per_step": bytes_step,
                "kernel": "gemv_panel_kernel (12 launches per step, algorithmic bytes / step time; plan of the "
                          "largest GEMM: " + dn.plan_describe(dn.KIND_F32, dn.desc(7, 4093, 1024, 1024, 4093, 4093,
                                                                                 1.0, 0.5)) + ")",
                "peak_source": pk["source"]}

    # e2e: reference-signature host API, pinned host buffers, copies inside.
    from oracle.oracle import ref_uniform
    host = []
    for (M, N, K) in C2_SHAPES:
        A = torch.from_numpy(ref_uniform(M * K, 42)).pin_memory()
        B = torch.from_numpy(ref_uniform(K * N, 123)).pin_memory()
        C = torch.from_numpy(ref_uniform(M * N, 77)).pin_memory()
        host.append((M, N, K, A.numpy(), B.numpy(), C.numpy()))
    dn.check(dn.set_stream(stream))
    for (M, N, K, A, B, C) in host:
        dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.5, C, N))
    e2e_steps = max(5, min(args.steps, 50))
    if use_dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for (M, N, K, A, B, C) in host:
            dn.check(dn.gemm_fp32(M, N, K, 1.0, A, K, B, N, 0.5, C, N))
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if use_dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    h2d = sum(4 * (M * K + K * N + M * N) for (M, N, K) in C2_SHAPES)
    d2h = sum(4 * M * N for (M, N, K) in C2_SHAPES)
    dn.check(dn.set_stream(None))

    extra = {}
    ms_serial = time_graphs(torch, serial_graphs, max(20, args.steps // 2), 3, stream)
    extra["c2_sweep_one_stream"] = {
        "us_per_step": ms_serial * 1e3, "GFLOP_s": flops / (ms_serial * 1e-3) / 1e9,
        "GB_s": bytes_step / (ms_serial * 1e-3) / 1e9,
        "note": "same 12 GEMMs serialised on one stream (latency-bound per launch)"}
    if not args.no_per_config:
        extra.update(per_config(torch, dn, stream, pk, world, rank, dist if use_dist else None))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded uniform[-1,1], the reference tests' std::mt19937 stream)",
            "config": {
                "workload": WORKLOAD,
                "api": f"dnnopt_cuda_gemm_f32 (device pointers); the 12 independent GEMMs on {args.streams} "
                       "streams (largest first onto the least-loaded stream) forked/joined inside one CUDA "
                       "graph per input set",
                "l2": f"{N_SETS} rotating input sets ({N_SETS * bytes_step / 1e6:.0f} MB > 126 MB L2)",
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            },
            "e2e": {"value": flops * world / e2e_s / 1e9, "unit": "GFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "dnnopt_gemm_fp32 (reference signature), pinned host buffers"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "per_config": extra,
        }
        print(json.dumps(line), flush=True)
    for g in graphs:
        del g
    if use_dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["dnnopt", "reference"], default="dnnopt")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--streams", type=int, default=SWEEP_STREAMS,
                    help="streams the 12 independent sweep GEMMs are spread over")
    ap.add_argument("--no-per-config", action="store_true", help="skip the per-config section")
    ap.add_argument("--profile", choices=["c1", "c2", "c3", "c4", "c5", "onednn", "simt64", "tc_i8",
                                         "conv3d_fp32", "conv3d_bf16", "conv3d_int8", "tc_bf16_small"],
                    help="run one config's kernel --reps times for an ncu capture, no bench line")
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    if args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
