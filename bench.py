#!/usr/bin/env python
"""Headline benchmark: strict-FP32 SGEMM TFLOP/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N == 1: one step = one sgblasSgemm of BASELINE configs[1], 4096^3 NN
(column-major, lda=ldb=ldc=4096, alpha=1, beta=0), inputs resident in HBM.
The 256 MiB L2 flush before each step is outside the step's CUDA events.

N > 1 (torchrun, one rank per GPU): one step = one sgblasMgSgemm of BASELINE
configs[4], 32768 x 32768 x 8192 NN split into N column blocks, A broadcast
from rank 0 by NCCL inside the step; inputs are > L2 on every rank. value =
whole-job FLOPs / max over ranks of the timed region (strong scaling).

Printed keys beyond the base contract: e2e (the same metric through the C ABI
with pinned host inputs copied in and C copied out every step, copies
pipelined against compute), roofline (FP32 FMA pipe peak = SMs x 128 lanes x
2 x SM clock sampled during the run), cpu_baseline (the reference's only CPU
SGEMM arithmetic -- the FP64 oracle loop of tests/cuda/correctness.cu -- on a
column sample, all host threads), cublas_pedantic (cublasGemmEx with
CUBLAS_COMPUTE_32F_PEDANTIC on the same buffers), clocks, gpu_launches.

--impl reference: the reference's CPU path on the host cores (the reference
has no CPU SGEMM; its oracle loop restated in oracle/ is used, "kind": "port").
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import pathlib
import re
import statistics
import subprocess
import sys
import time

# Strict FP32 everywhere (cuBLAS would otherwise be free to use TF32), except
# for the TF32 lane (--math tf32), whose comparison is cuBLAS's own TF32 mode.
if "tf32" not in sys.argv:
    os.environ.setdefault("NVIDIA_TF32_OVERRIDE", "0")

ROOT = pathlib.Path(__file__).resolve().parent
METRIC = "strict-FP32 SGEMM TFLOP/s at 4096³ NN vs cuBLAS pedantic and FP32 FMA peak"
UNIT = "TFLOP/s"
FP32_LANES_PER_SM = 128
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--size", type=int, default=4096, help="N=1 square size (4096 headline)")
    ap.add_argument("--shape", type=str, default=None,
                    help="N=1 M,N,K (default: --size cubed); e.g. 8192,8192,256 for config 4")
    ap.add_argument("--beta", type=float, default=0.0, help="N=1 beta (config 4 uses 1)")
    ap.add_argument("--alpha", type=float, default=1.0, help="N=1 alpha (config 3 uses 1.5)")
    ap.add_argument("--op", choices=["NN", "NT", "TN", "TT"], default="NN",
                    help="N=1 transpose modes of A and B")
    ap.add_argument("--pad", type=int, default=0,
                    help="N=1 leading dimensions = stored rows + PAD (config 3 uses 13)")
    ap.add_argument("--math", choices=["fp32", "tf32"], default="fp32",
                    help="N=1: fp32 (the strict default) or the TF32 tensor-core lane "
                         "(SGBLAS_MATH_TF32; compared with CUBLAS_COMPUTE_32F_FAST_TF32)")
    ap.add_argument("--batch", type=int, default=1,
                    help="N=1: matrices per call (sgblasSgemmStridedBatched when > 1)")
    ap.add_argument("--no-flush", action="store_true",
                    help="N=1: back-to-back calls without the L2 flush (latency of small calls)")
    ap.add_argument("--back-to-back", type=int, default=0, metavar="R",
                    help="N=1: R calls between one pair of events per step, no L2 flush (the "
                         "reference benchmark's protocol, bench/benchmark.cu:290-307); the R "
                         "calls are captured once in a CUDA graph and replayed, for ours and "
                         "for cuBLAS alike, so that no host overhead sits between them")
    ap.add_argument("--rotate", action="store_true",
                    help="N=1: cold-cache lane of the reference's protocol (docs/benchmarking.md:82): "
                         "cycle through copies of A, B, C whose total exceeds twice the L2, no "
                         "flush; cuBLAS gets the same rotation")
    ap.add_argument("--no-allgather", action="store_true",
                    help="N>1: skip the lane that also gathers C on every rank each step")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="report the launch estimate instead of tracing one extra call (for "
                         "runs under ncu, which owns the profiling interface)")
    ap.add_argument("--no-sharded-n1", action="store_true",
                    help="N=1: skip the config-5 (32768 x 32768 x 8192) single-GPU line")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    return ap.parse_args()


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        # median of the busy samples (the region is bracketed by idle time)
        busy = [s for s in sm if s >= 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "busy_samples": len(busy)}


def smi_index(torch, dev: int) -> str:
    props = torch.cuda.get_device_properties(dev)
    bus = getattr(props, "pci_bus_id", None)
    dom = getattr(props, "pci_domain_id", None)
    did = getattr(props, "pci_device_id", None)
    if bus is not None and dom is not None and did is not None:
        return f"{dom:08x}:{bus:02x}:{did:02x}.0"
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        return vis.split(",")[dev]
    return str(dev)


class NearGpu:
    """Binds this thread to the CPUs of the NUMA node the GPU hangs off
    (sysfs local_cpulist) while pinned host buffers are allocated and first
    touched, so that the kernel places them next to the GPU's PCIe link; the
    previous affinity is restored on exit. A no-op where the node is unknown."""

    def __init__(self, torch, dev: int):
        self.cpus = None
        props = torch.cuda.get_device_properties(dev)
        ids = [getattr(props, f, None) for f in ("pci_domain_id", "pci_bus_id", "pci_device_id")]
        if None in ids or not hasattr(os, "sched_setaffinity"):
            return
        try:
            text = open(f"/sys/bus/pci/devices/{ids[0]:04x}:{ids[1]:02x}:{ids[2]:02x}.0/"
                        "local_cpulist").read().strip()
        except OSError:
            return
        cpus = set()
        for part in text.split(","):
            if "-" in part:
                lo, hi = part.split("-")
                cpus.update(range(int(lo), int(hi) + 1))
            elif part:
                cpus.add(int(part))
        self.cpus = cpus & os.sched_getaffinity(0) or None
        self.text = text

    def __enter__(self):
        self.saved = os.sched_getaffinity(0) if self.cpus else None
        if self.cpus:
            os.sched_setaffinity(0, self.cpus)
        return self

    def __exit__(self, *exc):
        if self.saved:
            os.sched_setaffinity(0, self.saved)

    def describe(self) -> str:
        return (f"pinned host buffers allocated from the GPU's NUMA node (CPUs {self.text})"
                if self.cpus else "pinned host buffers allocated without NUMA binding")


# ---------------------------------------------------------------------------
class Cublas:
    """cublasGemmEx with CUBLAS_COMPUTE_32F_PEDANTIC (comparison lane only)."""

    def __init__(self, tf32: bool = False):
        self.lib = None
        for name in ("libcublas.so.12", "libcublas.so"):
            try:
                self.lib = ctypes.CDLL(name)
                break
            except OSError:
                continue
        if self.lib is None:
            raise OSError("libcublas not found")
        self.h = ctypes.c_void_p()
        assert self.lib.cublasCreate_v2(ctypes.byref(self.h)) == 0
        # CUBLAS_PEDANTIC_MATH, or CUBLAS_TF32_TENSOR_OP_MATH for the TF32 lane
        assert self.lib.cublasSetMathMode(self.h, 3 if tf32 else 2) == 0
        self.compute = 77 if tf32 else 69   # CUBLAS_COMPUTE_32F_FAST_TF32 / _32F_PEDANTIC
        ver = ctypes.c_int()
        self.lib.cublasGetVersion_v2(self.h, ctypes.byref(ver))
        self.version = ver.value
        f = self.lib.cublasGemmEx
        vp, ip = ctypes.c_void_p, ctypes.c_int
        f.argtypes = [vp, ip, ip, ip, ip, ip, vp, vp, ip, ip, vp, ip, ip, vp, vp, ip, ip, ip, ip]

    def set_stream(self, stream) -> None:
        self.lib.cublasSetStream_v2(self.h, ctypes.c_void_p(stream.cuda_stream))

    def sgemm(self, ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc) -> int:
        al = ctypes.c_float(alpha)
        be = ctypes.c_float(beta)
        return self.lib.cublasGemmEx(self.h, ta, tb, m, n, k, ctypes.byref(al), a, 0, lda, b, 0,
                                     ldb, ctypes.byref(be), c, 0, ldc, self.compute, -1)

    def sgemm_strided_batched(self, ta, tb, m, n, k, alpha, a, lda, sa, b, ldb, sb, beta, c, ldc,
                              sc, count) -> int:
        f = self.lib.cublasGemmStridedBatchedEx
        vp, ip, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
        f.argtypes = [vp, ip, ip, ip, ip, ip, vp, vp, ip, ip, ll, vp, ip, ip, ll, vp, vp, ip, ip,
                      ll, ip, ip, ip]
        al = ctypes.c_float(alpha)
        be = ctypes.c_float(beta)
        return f(self.h, ta, tb, m, n, k, ctypes.byref(al), a, 0, lda, sa, b, 0, ldb, sb,
                 ctypes.byref(be), c, 0, ldc, sc, count, self.compute, -1)


def profile_traffic(name: str):
    """DRAM bytes per launch recorded from an ncu capture (profiles/<name>)."""
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch\s*[:=]\s*([0-9.eE+]+)", path.read_text())
    return float(m.group(1)) if m else None


def own_launches(torch, fn):
    """Kernels of this library that fn() launches, counted from the CUDA
    activity trace of torch.profiler over one extra call outside the timed
    region (names in the sgblas namespace: the product kernels and the operand
    copies). Nothing is timed under the profiler. None if it cannot trace."""
    try:
        from torch.profiler import ProfilerActivity, profile
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        return sum(1 for e in prof.events()
                   if e.device_type == torch.autograd.DeviceType.CUDA and "sgblas" in e.name)
    except Exception:  # noqa: BLE001  (no CUPTI: the caller reports its own estimate)
        return None


def fp32_peak_tflops(sms: int, mhz: float) -> float:
    return sms * FP32_LANES_PER_SM * 2 * mhz * 1e6 / 1e12


# ---------------------------------------------------------------------------
def cpu_baseline(a, b, m, n, k, lda, ldb, budget_s: float) -> dict:
    """The oracle loop (FP32 in, FP64 accumulate) on a column sample of the
    workload, all host threads; rate extrapolated per column."""
    import numpy as np

    import oracle

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    c = np.zeros(m * threads, dtype=np.float32)
    t0 = time.perf_counter()
    oracle.sgemm_cpu(0, 0, m, k, 1.0, a, lda, b, ldb, 0.0, c, m, 0, threads, threads)
    t_one = time.perf_counter() - t0
    rounds = max(1, min(int(budget_s / max(t_one, 1e-3)), n // threads))
    cols = rounds * threads
    c = np.zeros(m * cols, dtype=np.float32)
    t0 = time.perf_counter()
    oracle.sgemm_cpu(0, 0, m, k, 1.0, a, lda, b, ldb, 0.0, c, m, 0, cols, threads)
    dt = time.perf_counter() - t0
    rate = 2.0 * m * k * cols / dt / 1e12
    # One thread, the reference's loop order exactly (column, row, k).
    c1 = np.zeros(m * n, dtype=np.float32)    # column j is written at c1[j * m]
    t0 = time.perf_counter()
    one_cols = 0
    while one_cols < n and (one_cols == 0 or time.perf_counter() - t0 < budget_s / 4):
        oracle.sgemm_cpu(0, 0, m, k, 1.0, a, lda, b, ldb, 0.0, c1, m, one_cols, one_cols + 1, 1)
        one_cols += 1
    dt1 = time.perf_counter() - t0
    return {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"columns 0..{cols - 1} of C ({cols}/{n}) of the {m}x{n}x{k} NN workload, "
                      f"FP64-accumulated oracle loop of tests/cuda/correctness.cu:373-392, "
                      f"{dt:.1f} s, rate extrapolated per column",
            "seconds": dt, "cpu_model": cpu_model(),
            "single_thread": {"value": 2.0 * m * k * one_cols / dt1 / 1e12, "unit": UNIT,
                              "cores": 1, "seconds": dt1,
                              "sample": f"{one_cols} columns of C, one thread, the reference "
                                        "loop order (column, row, k)"}}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
def sampled_parity(torch, a, b, c, m, n, k, lda, ldb, ldc, alpha=1.0, count=4096, seed=0,
                   full_cols=(0, -1)) -> dict:
    """Sampled check of an NN product with beta = 0 against an FP64
    restatement of the oracle loop (tests/cuda/correctness.cu:373-392): C at
    `count` random entries plus every row of the columns in full_cols (-1:
    the last column), within the north-star bound 2*max(K,2)*2^-24*mag,
    mag = |alpha| * sum |a*b|. Runs after timing, on the GPU in FP64 (torch
    reductions; nothing of this library is involved)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    rows = torch.randint(0, m, (count,), generator=g).to(a.device)
    cols = torch.randint(0, n, (count,), generator=g).to(a.device)
    av = a[: lda * k].view(k, lda)
    bv = b[: ldb * n].view(n, ldb)[:, :k]
    cv = c[: ldc * n].view(n, ldc)
    ar = av[:, rows].double().T            # count x k
    bc = bv[cols].double()                 # count x k
    ref = alpha * (ar * bc).sum(1)
    mag = abs(alpha) * (ar.abs() * bc.abs()).sum(1)
    got = cv[cols, rows].double()
    ratio = ((got - ref).abs() / (2.0 * max(k, 2) * 2.0 ** -24 * mag).clamp_min(1e-300)).max()
    worst = float(ratio)
    finite = bool(torch.isfinite(got).all())
    a64 = av[:, :m].double()               # k x m
    checked = count
    for j in full_cols:
        j = n - 1 if j < 0 else j
        col = bv[j].double()
        ref = alpha * (a64.T @ col)
        mag = abs(alpha) * (a64.abs().T @ col.abs())
        got = cv[j, :m].double()
        worst = max(worst, float(((got - ref).abs() /
                                  (2.0 * max(k, 2) * 2.0 ** -24 * mag).clamp_min(1e-300)).max()))
        finite = finite and bool(torch.isfinite(got).all())
        checked += m
    del a64
    return {"checked": checked, "max_ratio": worst, "ok": finite and worst <= 1.0,
            "method": f"{count} random entries + every row of columns {list(full_cols)}, FP64, "
                      "bound 2*max(K,2)*2^-24*|alpha|*sum|a*b|"}


def sharded_n1(torch, sg, steps: int, warmup: int) -> dict:
    """BASELINE configs[4] on one GPU: 32768 x 32768 x 8192 NN, alpha 1, beta
    0, one sgblasSgemm per step (what the sharded path runs with one rank);
    inputs (6 GiB) larger than L2. The denominator of the multi-GPU scaling."""
    M, N, K = 32768, 32768, 8192
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    a = torch.empty(M * K, device="cuda").uniform_(-1.0, 1.0, generator=gen)
    b = torch.empty(K * N, device="cuda").uniform_(-1.0, 1.0, generator=gen)
    c = torch.empty(M * N, device="cuda")
    stream = torch.cuda.Stream()
    h = sg.Handle()
    h.set_stream(stream)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            h.sgemm(0, 0, M, N, K, 1.0, a, M, b, K, 0.0, c, M)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    with torch.cuda.stream(stream):
        for i in range(steps):
            ev[i][0].record(stream)
            h.sgemm(0, 0, M, N, K, 1.0, a, M, b, K, 0.0, c, M)
            ev[i][1].record(stream)
    torch.cuda.synchronize()
    secs = sum(s.elapsed_time(e) for s, e in ev) / 1e3
    h.close()
    parity = sampled_parity(torch, a, b, c, M, N, K, M, K, M)
    del a, b, c
    torch.cuda.empty_cache()
    return {"value": 2.0 * M * N * K * steps / secs / 1e12, "unit": UNIT,
            "ms_per_step": 1e3 * secs / steps, "steps": steps, "warmup": warmup,
            "workload": f"sgemm NN {M}x{N}x{K} alpha=1 beta=0 on one GPU (BASELINE configs[4] "
                        "unsharded); inputs larger than L2", "parity": parity}


# ---------------------------------------------------------------------------
def run_reference(args) -> None:
    """--impl reference: the reference's CPU path (oracle port) on host cores."""
    import numpy as np

    import oracle

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps = args.steps if args.steps is not None else 5
    warmup = args.warmup if args.warmup is not None else 1
    m = n = k = args.size
    rng = np.random.default_rng(1)
    a = rng.uniform(-1.0, 1.0, m * k).astype(np.float32)
    b = rng.uniform(-1.0, 1.0, k * n).astype(np.float32)
    threads = len(os.sched_getaffinity(0))
    cols = threads          # one column per thread per step (a bounded sample)
    c = np.zeros(m * cols, dtype=np.float32)
    for _ in range(warmup):
        oracle.sgemm_cpu(0, 0, m, k, 1.0, a, m, b, k, 0.0, c, m, 0, cols, threads)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        oracle.sgemm_cpu(0, 0, m, k, 1.0, a, m, b, k, 0.0, c, m, 0, cols, threads)
        times.append(time.perf_counter() - t0)
    rate = 2.0 * m * k * cols * steps / sum(times) / 1e12
    sample = (f"{cols} columns of C per step of the {m}^3 NN workload ({threads} threads, one "
              f"column each), FP64-accumulated oracle loop of tests/cuda/correctness.cu:373-392")
    out = {"metric": METRIC, "value": rate, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
           "steps": steps, "warmup": warmup, "ms_per_step": 1e3 * sum(times) / steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic",
           "config": {"workload": f"sgemm NN {m}x{n}x{k} column-major alpha=1 beta=0 "
                                  "(BASELINE configs[1]); per step a column sample"},
           "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference has no CPU SGEMM (src/sgemm_host.cpp:26-27 returns "
                   "NOT_SUPPORTED); its only CPU GEMM arithmetic is the FP64 oracle loop"}
    emit(json.dumps(out))


# ---------------------------------------------------------------------------
def run_single(args) -> None:
    import numpy as np
    import torch

    import sgblas_b200 as sg

    steps = args.steps if args.steps is not None else 200
    warmup = max(3, args.warmup if args.warmup is not None else 20)
    dev = 0
    torch.cuda.set_device(dev)
    props = torch.cuda.get_device_properties(dev)
    sms = props.multi_processor_count
    if args.shape:
        m, n, k = (int(v) for v in args.shape.split(","))
    else:
        m = n = k = args.size
    beta, alpha = args.beta, args.alpha
    ta, tb = int(args.op[0] == "T"), int(args.op[1] == "T")
    # column-major; ld = stored rows + pad (tight by default)
    lda = (k if ta else m) + args.pad
    ldb = (n if tb else k) + args.pad
    ldc = m + args.pad
    a_cols, b_cols = (m if ta else k), (k if tb else n)
    batch = args.batch
    plain = (ta, tb, args.pad, alpha, batch) == (0, 0, 0, 1.0, 1)   # the configs' NN layout
    flops = 2.0 * m * n * k * batch
    sa, sb, sc = lda * a_cols, ldb * b_cols, ldc * n     # batch strides (elements)

    rng = np.random.default_rng(1)
    ha = rng.uniform(-1.0, 1.0, sa * batch).astype(np.float32)
    hb = rng.uniform(-1.0, 1.0, sb * batch).astype(np.float32)
    hc = np.random.default_rng(2).uniform(-1.0, 1.0, sc * batch).astype(np.float32)
    da = torch.from_numpy(ha).cuda()
    db = torch.from_numpy(hb).cuda()
    dc = torch.from_numpy(hc).cuda()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    stream = torch.cuda.Stream()
    h = sg.Handle()
    h.set_stream(stream)
    tf32 = args.math == "tf32"
    if tf32:
        h.set_math_mode(sg.SGBLAS_MATH_TF32)
        plain = False

    # --rotate: workspace sets (A, B, C) used in turn, step by step.
    rot = []
    if args.rotate:
        l2 = getattr(props, "L2_cache_size", 126 << 20)
        set_bytes = 4 * (da.numel() + db.numel() + dc.numel())
        count = min(64, max(2, -(-2 * l2 // set_bytes)))
        rot = [(da, db, dc)] + [(da.clone(), db.clone(), dc.clone()) for _ in range(count - 1)]
        args.no_flush = True
    cur = [0]

    def operands():
        return rot[cur[0] % len(rot)] if rot else (da, db, dc)

    def launch():
        a_, b_, c_ = operands()
        if batch == 1:
            h.sgemm(ta, tb, m, n, k, alpha, a_, lda, b_, ldb, beta, c_, ldc)
        else:
            h.sgemm_strided_batched(ta, tb, m, n, k, alpha, a_, lda, sa, b_, ldb, sb, beta, c_,
                                    ldc, sc, batch)

    reps = max(1, args.back_to_back)
    if args.back_to_back:
        args.no_flush = True

    def flush_l2():
        if not args.no_flush:
            flush.zero_()

    with torch.cuda.stream(stream):
        for i in range(warmup):
            cur[0] = i
            flush_l2()
            launch()
    torch.cuda.synchronize()

    def capture(fn):
        # The R back-to-back calls as one CUDA graph (set-up done by warm-up).
        graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(reps):
                fn()
        torch.cuda.synchronize()
        return graph

    graph = capture(launch) if args.back_to_back else None
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    with ClockSampler(smi_index(torch, dev)) as clk:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(steps):
                cur[0] = i
                flush_l2()
                ev[i][0].record(stream)
                if graph is not None:
                    graph.replay()
                else:
                    launch()
                ev[i][1].record(stream)
        torch.cuda.synchronize()
    times_ms = [s.elapsed_time(e) for s, e in ev]
    total_s = sum(times_ms) / 1e3 / reps      # per call
    value = flops * steps / total_s / 1e12
    clocks = clk.summary()
    if sg.get_device_errors() != 0:
        raise RuntimeError("device error flags raised during the bench")
    per_step = None
    if not args.no_launch_count:
        with torch.cuda.stream(stream):
            per_step = own_launches(torch, launch)
    if per_step is None:
        launches, launches_method = steps * reps, "estimate: one product kernel per call"
    else:
        launches = steps * per_step
        launches_method = (f"{per_step} sgblas kernel(s) per step, counted on one extra "
                           "untimed step with the torch.profiler CUDA trace")

    mhz = clocks["sm_mhz"] or 1965.0
    peak = fp32_peak_tflops(sms, mhz)
    peak_source = (f"{sms} SMs x {FP32_LANES_PER_SM} FP32 lanes x 2 x {mhz:.0f} MHz "
                   f"(median of {clocks.get('busy_samples', 0)} busy SM-clock samples of "
                   f"{clocks.get('samples', 0)} taken during the timed region); "
                   "MEASURED_PEAKS.json has no FP32 CUDA-core figure")
    if tf32:
        measured = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
            if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        bf16 = measured.get("bf16_tflops", 1590.0)
        peak = bf16 / 2.0
        peak_source = (f"dense TF32 = half the dense BF16 tensor rate; BF16 {bf16:g} TFLOP/s "
                       + ("measured (MEASURED_PEAKS.json bf16_tflops, burst)"
                          if "bf16_tflops" in measured else "fallback"))
    # DRAM bytes per launch from an ncu capture of this workload
    traffic = None
    if not args.no_flush and (ta, tb, args.pad, batch, beta) == (0, 0, 0, 1, 0.0):
        traffic = profile_traffic(("tf32" if tf32 else "sgemm") + f"_nn_{m}x{n}x{k}.md")
    roofline = {"bound": "tensor" if tf32 else "fp32_fma", "achieved": value, "peak": peak,
                "unit": UNIT, "frac": value / peak, "traffic": traffic,
                "peak_source": peak_source,
                "frac_of_max_clock": value / (peak if tf32 else fp32_peak_tflops(sms, 1965.0)),
                "algorithmic_flops_per_launch": flops,
                "algorithmic_bytes_per_launch":
                    4.0 * batch * (m * k + k * n + m * n * (2 if beta else 1)),
                "hbm_gbs_algorithmic": 4.0 * batch * (m * k + k * n + m * n * (2 if beta else 1)) /
                                       (total_s / steps) / 1e9}

    out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": steps,
           "warmup": warmup, "ms_per_step": 1e3 * total_s / steps, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None,
           "vs_published_a100": value / 17.736,
           "dtype": "tf32" if tf32 else "f32", "data": "synthetic",
           "config": {"workload": (f"strided batch of {batch} x " if batch > 1 else "") +
                                  ("TF32 tensor-core " if tf32 else "") +
                                  f"sgemm {args.op} {m}x{n}x{k} column-major alpha={alpha:g} "
                                  f"beta={beta:g}" + (f" ld=rows+{args.pad}" if args.pad else "") +
                                  (" (BASELINE configs[1])"
                                   if plain and (m, n, k, beta) == (4096, 4096, 4096, 0.0) else ""),
                      "m": m, "n": n, "k": k, "lda": lda, "ldb": ldb, "ldc": ldc,
                      "inputs": "uniform[-1,1) float32 (numpy seeds 1: A,B; 2: C)",
                      "l2": (f"rotated over {len(rot)} copies of A, B, C "
                             f"({len(rot) * 4 * (da.numel() + db.numel() + dc.numel()) >> 20} MiB, "
                             "over twice the L2), no flush" if rot else
                             "not flushed: back-to-back calls" if args.no_flush else
                             "flushed before every timed step (256 MiB write outside the "
                             "step's CUDA events)")},
           "calls_per_event_pair": reps,
           "launch": ("the calls of a step replayed as one CUDA graph" if args.back_to_back
                      else "one call per step from the host"),
           "roofline": roofline, "clocks": clocks, "gpu_launches": launches,
           "gpu_launches_method": launches_method,
           "device": props.name}

    if not args.no_cublas:
        try:
            cb = Cublas(tf32=tf32)
            cb.set_stream(stream)
            # cuBLAS writes its own copies of C (ours are checked afterwards)
            c2 = [x[2].clone() for x in rot] if rot else [dc.clone()]

            def cublas_call():
                a_, b_, _ = operands()
                c_ = c2[cur[0] % len(c2)]
                if batch == 1:
                    return cb.sgemm(ta, tb, m, n, k, alpha, a_.data_ptr(), lda, b_.data_ptr(),
                                    ldb, beta, c_.data_ptr(), ldc)
                return cb.sgemm_strided_batched(ta, tb, m, n, k, alpha, a_.data_ptr(), lda, sa,
                                                b_.data_ptr(), ldb, sb, beta, c_.data_ptr(), ldc,
                                                sc, batch)

            with torch.cuda.stream(stream):
                for i in range(warmup):
                    cur[0] = i
                    st = cublas_call()
            torch.cuda.synchronize()
            assert st == 0
            cgraph = capture(cublas_call) if args.back_to_back else None
            cev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(steps)]
            with torch.cuda.stream(stream):
                for i in range(steps):
                    cur[0] = i
                    flush_l2()
                    cev[i][0].record(stream)
                    if cgraph is not None:
                        cgraph.replay()
                    else:
                        st = cublas_call()
                    cev[i][1].record(stream)
            torch.cuda.synchronize()
            assert st == 0
            cval = flops * steps * reps / (sum(s.elapsed_time(e) for s, e in cev) / 1e3) / 1e12
            out["cublas_tf32" if tf32 else "cublas_pedantic"] = {
                "value": cval, "unit": UNIT, "ratio": value / cval, "version": cb.version,
                "call": ("cublasGemmEx" if batch == 1 else "cublasGemmStridedBatchedEx") +
                        (" CUDA_R_32F x3, CUBLAS_COMPUTE_32F_FAST_TF32, CUBLAS_TF32_TENSOR_OP_MATH"
                         if tf32 else " CUDA_R_32F x3, CUBLAS_COMPUTE_32F_PEDANTIC, "
                                      "CUBLAS_PEDANTIC_MATH, NVIDIA_TF32_OVERRIDE=0")}
            del c2
        except (OSError, AssertionError) as e:
            out["cublas_pedantic"] = {"unavailable": str(e)}

    if plain and beta == 0.0:
        out["parity"] = sampled_parity(torch, da, db, dc, m, n, k, lda, ldb, ldc)
    if not args.no_e2e and plain:
        # At least 40 steps, so that the first upload and the last download,
        # which nothing overlaps, weigh little in the steady-state rate.
        out["e2e"] = e2e_single(torch, sg, ha, hb, hc, beta, m, n, k, max(40, steps // 4), warmup)
    if not args.no_sharded_n1 and plain and (m, n, k, beta) == (4096, 4096, 4096, 0.0):
        out["sharded_n1"] = sharded_n1(torch, sg, 3, 3)
    if not args.no_cpu_baseline and plain:
        out["cpu_baseline"] = cpu_baseline(ha, hb, m, n, k, lda, ldb, args.cpu_seconds)
    h.close()
    emit(json.dumps(out))


def e2e_single(torch, sg, ha, hb, hc, beta, m, n, k, steps, warmup) -> dict:
    """The metric through the public C ABI with host buffers: each step copies
    A and B (and C when beta != 0) from pinned host memory, runs sgblasSgemm
    and copies C back. Two device buffer sets; copies of step i+1 overlap the
    SGEMM of step i."""
    near = NearGpu(torch, torch.cuda.current_device())
    with near:
        pa = torch.from_numpy(ha).pin_memory()
        pb = torch.from_numpy(hb).pin_memory()
        pc_in = torch.from_numpy(hc).pin_memory() if beta != 0.0 else None
        pc = torch.empty(m * n, dtype=torch.float32).pin_memory()
    sets = [(torch.empty(m * k, device="cuda"), torch.empty(k * n, device="cuda"),
             torch.empty(m * n, device="cuda")) for _ in range(2)]
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    h = sg.Handle()
    h.set_stream(s_comp)
    in_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]

    def run(count):
        for i in range(count):
            j = i % 2
            da, db, dc = sets[j]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(comp_done[j])     # set j free for new inputs
                da.copy_(pa, non_blocking=True)
                db.copy_(pb, non_blocking=True)
                in_done[j].record(s_in)
            s_comp.wait_event(in_done[j])
            if i >= 2:
                s_comp.wait_event(out_done[j])        # C of step i-2 has left
            if pc_in is not None:                     # C is an input too
                with torch.cuda.stream(s_comp):
                    dc.copy_(pc_in, non_blocking=True)
            h.sgemm(0, 0, m, n, k, 1.0, da, m, db, k, beta, dc, m)
            comp_done[j].record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[j])
                pc.copy_(dc, non_blocking=True)
                out_done[j].record(s_out)

    run(warmup)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    run(steps)
    s_in.wait_stream(s_out)
    end.record(s_in)
    torch.cuda.synchronize()
    secs = start.elapsed_time(end) / 1e3
    h.close()
    return {"value": 2.0 * m * n * k * steps / secs / 1e12, "unit": UNIT,
            "h2d_bytes_per_step": 4 * (m * k + k * n + (m * n if pc_in is not None else 0)),
            "d2h_bytes_per_step": 4 * m * n,
            "steps": steps, "pipelining": "2 buffer sets; H2D, SGEMM and D2H on 3 streams",
            "host_memory": near.describe()}


# ---------------------------------------------------------------------------
def run_sharded(args) -> None:
    """N ranks: config 5, 32768 x 32768 x 8192 NN, columns split across ranks,
    A broadcast from rank 0 inside every step (sgblasMgSgemm)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import sgblas_b200 as sg
    from sgblas_b200.mg import check_consistent, exchange_unique_id, panel_plan, shard_columns

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    steps = args.steps if args.steps is not None else 5
    warmup = max(3, args.warmup if args.warmup is not None else 3)
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    M, N, K = 32768, 32768, 8192
    _, n_loc = shard_columns(N, world, rank)
    flops = 2.0 * M * N * K
    check_consistent(dict(transa=0, transb=0, m=M, k=K, alpha=1.0, beta=0.0, lda=M, root=0))
    mg = sg.MgHandle(world, rank, exchange_unique_id(sg.mg_unique_id), local)
    stream = torch.cuda.Stream()
    mg.set_stream(stream)

    gen = torch.Generator(device="cuda")
    gen.manual_seed(5 + rank)
    # A exists on the root only; the call sends it to the other ranks' staging.
    a = torch.empty(M * K, device="cuda").uniform_(-1.0, 1.0, generator=gen) if rank == 0 \
        else None
    b = torch.empty(K * n_loc, device="cuda").uniform_(-1.0, 1.0, generator=gen)
    c = torch.empty(M * n_loc, device="cuda")

    def step():
        mg.sgemm(0, 0, M, n_loc, K, 1.0, a, M, 0, b, K, 0.0, c, M)

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            step()
    torch.cuda.synchronize()
    dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    with ClockSampler(smi_index(torch, local)) as clk:
        torch.cuda.synchronize()
        dist.barrier()
        with torch.cuda.stream(stream):
            for i in range(steps):
                ev[i][0].record(stream)
                step()
                ev[i][1].record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    local_s = sum(s.elapsed_time(e) for s, e in ev) / 1e3
    t = torch.tensor([local_s], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_s = float(t.item())
    value = flops * steps / total_s / 1e12
    clocks = clk.summary()
    allc = [None] * world
    dist.all_gather_object(allc, clocks)
    errors = sg.get_device_errors()
    # Launches: one more (untimed) step on every rank under the profiler's
    # CUDA trace; C is recomputed with the same values.
    per_step = None
    if not args.no_launch_count:
        with torch.cuda.stream(stream):
            per_step = own_launches(torch, step)
    counts = [None] * world
    dist.all_gather_object(counts, per_step)
    # Parity of the timed steps' C (outside the timed region): one more call
    # with no columns of its own delivers A to every rank (C untouched), then
    # each rank checks its shard against FP64.
    a_full = a if rank == 0 else torch.empty(M * K, device="cuda")
    with torch.cuda.stream(stream):
        mg.sgemm(0, 0, M, 0, K, 1.0, a_full, M, 0, b, K, 0.0, c, M)
    torch.cuda.synchronize()
    mine = sampled_parity(torch, a_full, b, c, M, n_loc, K, M, K, M, seed=rank)
    parities = [None] * world
    dist.all_gather_object(parities, mine)
    parity = {"checked": sum(x["checked"] for x in parities),
              "max_ratio": max(x["max_ratio"] for x in parities),
              "ok": all(x["ok"] for x in parities),
              "method": "every rank: " + mine["method"] + "; A delivered by a further call"}
    # With the C all-gather: every step also assembles the whole C (ldc == M,
    # equal column blocks) on every rank with sgblasMgAllGather, after the
    # product; same timing rules.
    gathered = None
    if N % world == 0 and not args.no_allgather:
        full = torch.empty(M * N, device="cuda")
        a_only = a if rank == 0 else None

        def step_gather():
            mg.sgemm(0, 0, M, n_loc, K, 1.0, a_only, M, 0, b, K, 0.0, c, M)
            mg.all_gather(c, full, M * n_loc)

        with torch.cuda.stream(stream):
            step_gather()
        torch.cuda.synchronize()
        dist.barrier()
        gev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
        with torch.cuda.stream(stream):
            for i in range(steps):
                gev[i][0].record(stream)
                step_gather()
                gev[i][1].record(stream)
        torch.cuda.synchronize()
        gt = torch.tensor([sum(s_.elapsed_time(e_) for s_, e_ in gev) / 1e3], dtype=torch.float64)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        # the gathered C against this rank's block of it
        blk = full.view(N, M)[rank * n_loc:(rank + 1) * n_loc]
        same = bool(torch.equal(blk, c.view(n_loc, M)))
        flags = torch.tensor([1 if same else 0], dtype=torch.int64)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        gathered = {"value": flops * steps / float(gt.item()) / 1e12, "unit": UNIT,
                    "ms_per_step": 1e3 * float(gt.item()) / steps, "steps": steps,
                    "blocks_match": bool(flags.item()),
                    "what": "each step: the sharded product, then sgblasMgAllGather of C "
                            f"({4 * M * N >> 20} MiB assembled on every rank); max over ranks"}
        del full
    del a, b, c, a_full
    torch.cuda.empty_cache()

    e2e = None
    if not args.no_e2e:
        e2e = e2e_sharded(torch, dist, sg, mg, rank, M, n_loc, K, flops, max(2, steps // 2))
    mg.close()
    props = torch.cuda.get_device_properties(local)
    sms = props.multi_processor_count
    mhz = statistics.median([x["sm_mhz"] for x in allc if x["sm_mhz"]] or [1965.0])
    peak = world * fp32_peak_tflops(sms, mhz)
    if rank == 0:
        if errors != 0:
            raise RuntimeError("device error flags raised during the bench")
        reasons = sorted({r for x in allc for r in x["reasons"]})
        out = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
               "warmup": warmup, "ms_per_step": 1e3 * total_s / steps, "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
               "config": {"workload": f"sharded sgemm NN {M}x{N}x{K} (BASELINE configs[4]), "
                                      f"B and C split into {world} column blocks, "
                                      "A (1 GiB) sent from rank 0 to every rank in every step",
                          "m": M, "n": N, "k": K,
                          "parallelism": f"column-shard x{world}", "l2": "inputs larger than L2",
                          "broadcast": "A sent along a chain of ranks by copy engines in row "
                                       "panels (512, 1024, 2048, ~4096 rows), each rank "
                                       "computing a panel's rows as it arrives"},
               "parity": parity,
               "with_allgather": gathered,
               "roofline": {"bound": "fp32_fma", "achieved": value, "peak": peak, "unit": UNIT,
                            "frac": value / peak, "traffic": None,
                            "peak_source": f"{world} x {sms} SMs x 128 lanes x 2 x {mhz:.0f} MHz "
                                           "(median sampled SM clock)"},
               "clocks": {"sm_mhz": mhz, "sm_max_mhz": max((x["sm_max_mhz"] or 0) for x in allc),
                          "reasons": reasons},
               "gpu_launches": (steps * max(counts) if None not in counts
                                else steps * len(panel_plan(M, K, world))),
               "gpu_launches_note": ("per rank (the largest count over ranks): sgblas kernels "
                                     "of one extra untimed step, torch.profiler CUDA trace"
                                     if None not in counts else
                                     "estimate per rank: one product kernel per row panel of A "
                                     "per step"),
               "e2e": e2e}
        emit(json.dumps(out))
    dist.barrier()
    dist.destroy_process_group()


def e2e_sharded(torch, dist, sg, mg, rank, M, n_loc, K, flops, steps) -> dict:
    """Config 5 through the C ABI from host memory: every step rank 0 copies
    A in, every rank copies its B shard in, runs sgblasMgSgemm and copies its
    C shard out. Two buffer sets overlap the copies of step i+1 with step i."""
    near = NearGpu(torch, torch.cuda.current_device())
    with near:
        pa = torch.empty(M * K).uniform_(-1.0, 1.0).pin_memory() if rank == 0 else None
        pb = torch.empty(K * n_loc).uniform_(-1.0, 1.0).pin_memory()
        pc = torch.empty(M * n_loc).pin_memory()
    sets = [(torch.empty(M * K, device="cuda") if rank == 0 else None,
             torch.empty(K * n_loc, device="cuda"), torch.empty(M * n_loc, device="cuda"))
            for _ in range(2)]
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    mg.set_stream(s_comp)
    in_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]

    def run(count):
        for i in range(count):
            j = i % 2
            da, db, dc = sets[j]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(comp_done[j])
                if pa is not None:
                    da.copy_(pa, non_blocking=True)
                db.copy_(pb, non_blocking=True)
                in_done[j].record(s_in)
            s_comp.wait_event(in_done[j])
            if i >= 2:
                s_comp.wait_event(out_done[j])
            mg.sgemm(0, 0, M, n_loc, K, 1.0, da, M, 0, db, K, 0.0, dc, M)
            comp_done[j].record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[j])
                pc.copy_(dc, non_blocking=True)
                out_done[j].record(s_out)

    run(2)
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    run(steps)
    s_in.wait_stream(s_out)
    end.record(s_in)
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end) / 1e3], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {"value": flops * steps / float(t.item()) / 1e12, "unit": UNIT,
            "h2d_bytes_per_step": 4 * (M * K + K * 32768), "d2h_bytes_per_step": 4 * M * 32768,
            "steps": steps,
            "pipelining": "2 buffer sets per rank; H2D, broadcast+SGEMM and D2H on 3 streams; "
                          "bytes are whole-job totals (A once on rank 0, B and C over all ranks)",
            "host_memory": near.describe()}


_RESULT_FD = None


def emit(line: str) -> None:
    """Writes the one result line to the process's real stdout (everything
    else -- NCCL's banner, library messages -- was redirected to stderr)."""
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (line + "\n").encode())


def main():
    global _RESULT_FD
    # Keep stdout for the single JSON line: libraries that print (NCCL's
    # version banner under NCCL_DEBUG=VERSION) go to stderr instead.
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    args = parse_args()
    sys.path.insert(0, str(ROOT))
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.gpus > 1:
        if world == 1:
            raise SystemExit("--gpus > 1 must be launched with torchrun (one rank per GPU)")
        run_sharded(args)
    else:
        run_single(args)


if __name__ == "__main__":
    main()
