#!/usr/bin/env python
"""bench.py — throughput of the dense FP32 contraction hot path on B200.

Workload (default, `--workload linear`): the linear-layer GEMM configuration
m=8192 (per GPU), k=4096, n=11008, lda=4128, ldb=ldc=11040, A ~ N(0,1),
B ~ N(0, 1/64) (std 1/sqrt(4096)), C ~ N(0,1), alpha=0.5, beta=1, strict FP32
(3xTF32 on tcgen05). One step = one pass of the hot path over one batch:
split prepass + tcgen05 GEMM; with N > 1 GPUs each rank owns 8192 rows of A and C
(weak scaling) and B is broadcast from rank 0 over NVLink by NCCL inside the step,
in column panels overlapped with the per-panel GEMM.

Prints ONE JSON line (rank 0). `--impl reference` times the reference's own CPU
gemm_f32 (oracle/_ref, built from the reference sources) on the same configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mfb|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP32 GEMM TFLOPS (N=2048/8192) at 1/2/4/8 B200, % of roofline; GEMV GB/s"

WORKLOADS = {
    # name: (m per GPU, n, k, lda, ldb, ldc, alpha, beta, description); A, C ~ N(0,1), B ~ N(0, 1/64)
    "linear": (8192, 11008, 4096, 4096 + 32, 11008 + 32, 11008 + 32, 0.5, 1.0,
               "linear-layer GEMM m=8192/GPU k=4096 n=11008, lda=4128 ldb=ldc=11040, alpha=0.5 beta=1"),
    "linear_m2048": (2048, 11008, 4096, 4096 + 32, 11008 + 32, 11008 + 32, 0.5, 1.0,
                     "linear-layer GEMM with m=2048/GPU (profiling size; B alone exceeds L2)"),
    "square8192": (8192, 8192, 8192, 8192, 8192, 8192, 1.0, 0.0, "square GEMM 8192^3, alpha=1 beta=0"),
    "square2048": (2048, 2048, 2048, 2048, 2048, 2048, 1.0, 0.0, "square GEMM 2048^3, alpha=1 beta=0"),
    "longk512": (512, 512, 65536, 65536, 512, 512, 1.0, 0.0,
                 "long-K GEMM m=n=512 k=65536 (4 SM-pair tiles: K shared among the SMs), alpha=1 beta=0"),
    "c5": (32768, 32768, 32768, 32768, 32768, 32768, 1.0, 0.0,
           "square GEMM 32768^3 rows split across GPUs (32768 rows total), B broadcast"),
}


L2_BYTES = 126 * 10**6
FLUSH_BYTES = 512 << 20


def link_roofline(torch, h2d_bytes, d2h_bytes, ms_per_step, nbytes=256 << 20, reps=3):
    """PCIe bound of an end-to-end step: pinned host<->device copy rates measured here (each
    direction alone, CUDA events), and the step time those rates allow for the step's bytes."""
    h = torch.empty(nbytes // 4, dtype=torch.float32, pin_memory=True)
    d = torch.empty(nbytes // 4, dtype=torch.float32, device="cuda")
    rates = {}
    for name, fn in (("h2d_gbs", lambda: d.copy_(h, non_blocking=True)),
                     ("d2h_gbs", lambda: h.copy_(d, non_blocking=True))):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        rates[name] = nbytes * reps / (e0.elapsed_time(e1) / 1e3) / 1e9
    bound = max(h2d_bytes / rates["h2d_gbs"], d2h_bytes / rates["d2h_gbs"]) / 1e6
    return {"h2d_gbs": rates["h2d_gbs"], "d2h_gbs": rates["d2h_gbs"], "bound_ms": bound,
            "ms_per_step": ms_per_step, "frac": bound / ms_per_step if ms_per_step > 0 else None,
            "basis": "max(h2d bytes / h2d rate, d2h bytes / d2h rate), rates of 256 MiB pinned copies "
                     "each direction alone"}


def read_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def read_profile_traffic(kernel_tag: str):
    """DRAM bytes per launch recorded from an ncu capture in profiles/ (a 'traffic_bytes_per_launch' line)."""
    path = os.path.join(ROOT, "profiles", f"{kernel_tag}.md")
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", text)
    return float(m.group(1)) if m else None


class ClockSampler:
    """Samples SM clock, power and throttle reasons through NVML (read-only) every 10 ms
    while the timed region runs, on a background thread."""

    # nvmlClocksEventReason bits (nvml.h): the ones a run must report.
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []
        self.error = None
        self._stop = None
        self._thread = None

    def _handle(self, nv):
        # Match the CUDA device to its NVML handle by PCI bus id (CUDA_VISIBLE_DEVICES may renumber).
        import torch
        props = torch.cuda.get_device_properties(self.cuda_index)
        want = getattr(props, "pci_bus_id", None)
        for i in range(nv.nvmlDeviceGetCount()):
            h = nv.nvmlDeviceGetHandleByIndex(i)
            if want is None:
                return h
            pci = nv.nvmlDeviceGetPciInfo(h)
            if (pci.bus, pci.device, pci.domain) == (want, getattr(props, "pci_device_id", pci.device),
                                                     getattr(props, "pci_domain_id", pci.domain)):
                return h
        return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception as exc:  # sampling is reported, never required
            self.error = f"nvml unavailable: {exc}"
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((float(sm), pw, int(rs)))
                except Exception as exc:
                    self.error = str(exc)
                    return
                self._stop.wait(0.01)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": getattr(self, "max_mhz", None),
                    "reasons": [self.error or "no samples"], "samples": 0}
        reasons = sorted({name for (_, _, r) in self.samples for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_max": max(p for _, p, _ in self.samples), "source": "NVML, 10 ms period"}


def cpu_reference_sample(m, n, k, lda, ldb, ldc, alpha, beta, rows, reps, warm=1, seed=20261001):
    """Times the reference's compiled gemm_f32 on `rows` rows of the workload; returns TFLOPS."""
    import oracle
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((rows, lda), dtype=np.float32)
    b = (rng.standard_normal((k, ldb), dtype=np.float32) / 64.0).astype(np.float32)
    c = rng.standard_normal((rows, ldc), dtype=np.float32)
    impl = "reference" if oracle.reference_available() else "restatement"
    times = []
    for i in range(warm + reps):
        cc = c.copy()
        t0 = time.perf_counter()
        oracle.gemm_f32(rows, n, k, a, lda, b, ldb, cc, ldc, alpha, beta, impl=impl)
        dt = time.perf_counter() - t0
        if i >= warm:
            times.append(dt)
    flops = 2.0 * rows * n * k
    info = oracle.reference_info() if impl == "reference" else {"worker_count": 1, "gemm_kernel_name": "port"}
    med = statistics.median(times)
    return {
        "tflops": flops / med / 1e12,
        "cores": int(info["worker_count"]),
        "kind": "reference" if impl == "reference" else "port",
        "kernel": info["gemm_kernel_name"],
        "seconds_per_rep": med,
        "rows": rows,
    }


def run_reference_arm(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    m, n, k, lda, ldb, ldc, alpha, beta, desc = wl
    rows = min(m, args.ref_rows)
    import oracle
    if not oracle.reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libmfref_cpu.so was not built "
                          "(build() compiles it where the reference sources exist)"}))
        return 0
    steps = []
    rng = np.random.default_rng(20261001)
    a = rng.standard_normal((rows, lda), dtype=np.float32)
    b = (rng.standard_normal((k, ldb), dtype=np.float32) / 64.0).astype(np.float32)
    c = rng.standard_normal((rows, ldc), dtype=np.float32)
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle.gemm_f32(rows, n, k, a, lda, b, ldb, c, ldc, alpha, beta, impl="reference")
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            steps.append(dt)
    total = sum(steps)
    tflops = 2.0 * rows * n * k * len(steps) / total / 1e12
    info = oracle.reference_info()
    sample = (f"{rows} of the {m} rows per step (full n={n}, k={k}); reference gemm_f32 "
              f"({info['gemm_kernel_name']}) compiled from the reference sources; pool of {info['worker_count']} "
              f"threads, rows split into ~8 chunks by the reference (grain m/8)")
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": desc, "rows_per_step_sample": rows, "precision": "fp32 (CPU FMA)"},
        "cpu_baseline": {"value": tflops, "unit": "TFLOPS", "cores": info["worker_count"], "kind": "reference",
                         "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


class SampledCheck:
    """Oracle check of one seeded 64 x 64 block of this rank's C, run after the timed region
    (the reference's benchmark validates its timed product the same way,
    benchmarks/bench_gemm_fair.cpp:76-95,153,157).

    Before the first step it keeps C's starting values on the sampled rows. After the timed
    steps it writes them back, makes every rank but the broadcast root forget B (NaN), runs
    one more step of the same operator (so the sampled columns of B reach this rank through
    the broadcast) and compares the block with the oracle's gemm_f32 on the same inputs and
    with an FP64 product. Gates: strict FP32 ||C - C64||_F / ||C64||_F <= max(1e-6, that
    error of gemm_f32 itself) and max |C - C_gemm_f32| <= 1e-5 k max|A| max|B|; TF32
    ||C - C_gemm_f32||_F / ||C_gemm_f32||_F <= 5e-3."""

    SIZE = 64

    def __init__(self, torch, m, n, k, C, rank):
        rng = np.random.default_rng(20261001 + rank)
        self.rows = np.sort(rng.choice(m, size=min(self.SIZE, m), replace=False))
        # the sampled columns are the same on every rank
        self.cols = np.sort(np.random.default_rng(20261001).choice(n, size=min(self.SIZE, n), replace=False))
        self.rows_dev = torch.from_numpy(self.rows).to(C.device)
        self.cols_dev = torch.from_numpy(self.cols).to(C.device)
        self.c0_rows = C.index_select(0, self.rows_dev).clone()  # (rows, n) on the device
        self.k = k

    def run(self, torch, op, A, B, B_buf, C, alpha, beta, strict, rank, src=0):
        import oracle
        C.index_copy_(0, self.rows_dev, self.c0_rows)
        a_s = A.index_select(0, self.rows_dev).cpu().numpy()                      # (64, k)
        b_s = B.index_select(1, self.cols_dev).cpu().numpy()                      # (k, 64)
        c0 = self.c0_rows.index_select(1, self.cols_dev).cpu().numpy()            # (64, 64)
        if rank != src:
            B_buf.fill_(float("nan"))  # only the broadcast can bring B to this rank
        if C.is_cuda:
            torch.cuda.synchronize()
        op(A, B, C, alpha, beta)
        if C.is_cuda:
            torch.cuda.synchronize()
        got = C.index_select(0, self.rows_dev).index_select(1, self.cols_dev).cpu().numpy()
        r, s = a_s.shape[0], b_s.shape[1]
        ref32 = oracle.gemm_f32_sampled(np.arange(r), np.arange(s), s, self.k, a_s, self.k, np.ascontiguousarray(b_s),
                                        s, c_in=c0, alpha=alpha, beta=beta)
        ref64 = alpha * (a_s.astype(np.float64) @ b_s.astype(np.float64))
        if beta != 0.0:
            ref64 += beta * c0.astype(np.float64)
        finite = bool(np.isfinite(got).all())
        max_abs = oracle.max_abs(got, ref32) if finite else float("inf")
        if strict:
            err = oracle.normwise_rel(got, ref64) if finite else float("inf")
            oracle_err = oracle.normwise_rel(ref32, ref64)
            gate = max(1e-6, oracle_err)
            bound = oracle.elementwise_bound(self.k, float(np.abs(a_s).max()), float(np.abs(b_s).max()))
            ok = finite and err <= gate and max_abs <= bound
        else:
            err = oracle.normwise_rel(got, ref32) if finite else float("inf")
            oracle_err = oracle.normwise_rel(ref32, ref64)
            gate, bound = 5e-3, float("inf")
            ok = finite and err <= gate
        return [err, gate, max_abs, bound, oracle_err, 1.0 if ok else 0.0]

    @staticmethod
    def summarize(per_rank, strict):
        """Worst rank of the per-rank results (lists from run())."""
        worst = max(range(len(per_rank)), key=lambda i: (per_rank[i][5] == 0.0, per_rank[i][0] / per_rank[i][1]))
        err, gate, max_abs, bound, oracle_err, _ = per_rank[worst]
        return {"ok": all(r[5] == 1.0 for r in per_rank), "ranks": len(per_rank), "worst_rank": worst,
                "normwise": err, "normwise_vs": "fp64" if strict else "gemm_f32", "gate": gate,
                "max_abs_vs_gemm_f32": max_abs, "elementwise_bound": bound if strict else None,
                "gemm_f32_vs_fp64": oracle_err,
                "block": "64 seeded rows of each rank x 64 seeded columns, after the timed steps, one more step "
                         "from C's starting values with B known only to the broadcast root"}


AUX_WORKLOADS = {
    # GEMV / skinny GEMM: A 16384 x 16384 ~ U[-1,1], x 16384 x n ~ N(0,1), alpha 1, beta 0.
    "gemv_n1": ("gemv", 1), "gemv_n4": ("gemv", 4), "gemv_n8": ("gemv", 8), "gemv_n16": ("gemv", 16),
    # conv2d forward, stride 1, pad 1, 3x3: (N, C, H, W, K); x ~ U[-1,1], w ~ N(0, 2/fan_in), bias 0.
    "conv_c4a": ("conv", (8, 3, 32, 32, 16)), "conv_c4b": ("conv", (256, 64, 56, 56, 64)),
    # conv2d backward of the same shape: input, weight and bias gradients per step
    "conv_c4b_bwd": ("conv_bwd", (256, 64, 56, 56, 64)),
    # strided-batched GEMM (batch_matmul): (batch, m, n, k); A, B ~ U[-1,1], alpha 1, beta 0.
    "bmm_b16_2048": ("bmm", (16, 2048, 2048, 2048)),
    # column covariance of X (rows x cols) ~ N(1, 1): (rows, cols)
    "cov_65536x2048": ("cov", (65536, 2048)),
}


GRAPH_WORKLOADS = ("conv_c4a",)


def tf32_mma_fields(mf, device, achieved, strict):
    """The TF32 MMA rate measured on this GPU after the timed region (N = 256 MMAs from reused
    shared-memory operands: the tensor pipe's own ceiling, above the bf16/2 derivation) and the
    achieved rate as a fraction of it (strict = 3 TF32 passes)."""
    try:
        peak = mf.probe_tf32_mma_tflops(256, device)
    except Exception as exc:  # diagnostic only
        return {"peak_tf32_mma_measured": f"failed: {exc}"}
    frac = achieved / (peak / (3.0 if strict else 1.0)) if achieved and peak > 0 else None
    return {"peak_tf32_mma_measured": peak, "frac_vs_tf32_mma_measured": frac}


def run_aux_workload(args):
    """GEMV and conv2d workloads: one GPU per process (N > 1 runs independent replicas)."""
    import torch
    import matrixflash_pro_b200 as mf
    import oracle

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    kind, shape = AUX_WORKLOADS[args.workload]
    gen = torch.Generator(device="cuda").manual_seed(20261001 + rank)
    peaks, peak_src = read_peaks()
    strict = args.precision == "fp32"
    prec = mf.GemmPrecision.fp32 if strict else mf.GemmPrecision.tf32
    if kind == "gemv":
        n = shape
        m = k = 16384
        A = torch.rand((m, k), device="cuda", generator=gen) * 2 - 1
        X = torch.randn((k, n), device="cuda", generator=gen)
        Y = torch.empty((m, n), device="cuda")
        work = 4.0 * (m * k + k * n + m * n)  # algorithmic bytes per step
        unit, metric_unit = "GB/s", 1e9
        desc = f"GEMV/skinny GEMM A 16384x16384 x B 16384x{n}, alpha 1, beta 0 (A alone is 1 GiB > L2)"

        def step():
            mf.gemv(A, X, Y)

        host = [torch.empty_like(A, device="cpu").pin_memory(), torch.empty_like(X, device="cpu").pin_memory()]
        host[0].copy_(A)
        host[1].copy_(X)
        y_host = torch.empty_like(Y, device="cpu").pin_memory()

        def e2e_step():
            A.copy_(host[0], non_blocking=True)
            X.copy_(host[1], non_blocking=True)
            step()
            y_host.copy_(Y, non_blocking=True)

        h2d, d2h = (A.numel() + X.numel()) * 4, Y.numel() * 4
        roof = {"bound": "hbm", "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "peak_basis": f"hbm_gbs of {peak_src} MEASURED_PEAKS.json",
                "kernel": f"gemv_tile_kernel (TMA-fed, {1 if n == 1 else 4 if n <= 4 else 8 if n <= 8 else 16}-column "
                          f"variant, n={n})"}
        launches = 1

        def cpu_sample():
            rows = 2048
            a = A[:rows].cpu().numpy()
            x = X.cpu().numpy()
            c = np.zeros((rows, n), np.float32)
            impl = "reference" if oracle.reference_available() else "restatement"
            oracle.gemm_f32(rows, n, k, a, k, x, n, c, n, 1.0, 0.0, impl=impl)
            t0 = time.perf_counter()
            for _ in range(3):
                oracle.gemm_f32(rows, n, k, a, k, x, n, c, n, 1.0, 0.0, impl=impl)
            dt = (time.perf_counter() - t0) / 3
            info = oracle.reference_info() if impl == "reference" else {"worker_count": 1}
            return {"value": 4.0 * (rows * k + k * n + rows * n) / dt / 1e9, "unit": "GB/s",
                    "cores": info["worker_count"], "kind": "reference" if impl == "reference" else "port",
                    "sample": f"{rows} of the 16384 rows, full k and n, gemm_f32, mean of 3"}
    elif kind == "bmm":
        nb, m, n, k = shape
        A = torch.rand((nb, m, k), device="cuda", generator=gen) * 2 - 1
        B = torch.rand((nb, k, n), device="cuda", generator=gen) * 2 - 1
        C = torch.empty((nb, m, n), device="cuda")
        work = 2.0 * nb * m * n * k
        unit, metric_unit = "TFLOPS", 1e12
        desc = f"strided-batched GEMM {nb} x ({m}x{k} @ {k}x{n}), alpha 1, beta 0 (operands 3 x {nb * m * k * 4 >> 20} MiB)"
        opts = mf.GemmOptions(precision=prec)

        def step():
            mf.sgemm_strided_batched(A, B, C, 1.0, 0.0, opts)

        host = [torch.empty_like(A, device="cpu").pin_memory(), torch.empty_like(B, device="cpu").pin_memory()]
        host[0].copy_(A)
        host[1].copy_(B)
        c_host = torch.empty_like(C, device="cpu").pin_memory()

        def e2e_step():
            A.copy_(host[0], non_blocking=True)
            B.copy_(host[1], non_blocking=True)
            step()
            c_host.copy_(C, non_blocking=True)

        h2d, d2h = (A.numel() + B.numel()) * 4, C.numel() * 4
        passes = 6.0 if strict else 2.0
        roof = {"bound": "tensor", "peak": peaks["bf16_tflops"] / passes, "unit": "TFLOP/s",
                "peak_basis": f"bf16_tflops/{int(passes)} of {peak_src} MEASURED_PEAKS.json",
                "kernel": "tc_persistent_kernel<GemmProblem> over the batch (time includes the split prepass)"}
        launches = 3

        def cpu_sample():
            rows = 256
            a = A[0, :rows].cpu().numpy()
            b = B[0].cpu().numpy()
            c = np.zeros((rows, n), np.float32)
            impl = "reference" if oracle.reference_available() else "restatement"
            oracle.gemm_f32(rows, n, k, a, k, b, n, c, n, 1.0, 0.0, impl=impl)
            t0 = time.perf_counter()
            oracle.gemm_f32(rows, n, k, a, k, b, n, c, n, 1.0, 0.0, impl=impl)
            dt = time.perf_counter() - t0
            info = oracle.reference_info() if impl == "reference" else {"worker_count": 1}
            return {"value": 2.0 * rows * n * k / dt / 1e12, "unit": "TFLOPS", "cores": info["worker_count"],
                    "kind": "reference" if impl == "reference" else "port",
                    "sample": f"{rows} rows of batch entry 0, gemm_f32 (the reference batches through cuBLAS only)"}
    elif kind == "cov":
        rows, cols = shape
        X = torch.randn((rows, cols), device="cuda", generator=gen) + 1.0
        work = 2.0 * cols * cols * rows  # the centered product X_c^T X_c
        unit, metric_unit = "TFLOPS", 1e12
        desc = f"covariance of a {rows}x{cols} matrix (X_c^T X_c / (rows-1); X is {rows * cols * 4 >> 20} MiB)"

        def step():
            mf.covariance(X, prec)

        x_host = torch.empty_like(X, device="cpu").pin_memory()
        x_host.copy_(X)
        out_host = torch.empty((cols, cols), pin_memory=True)

        def e2e_step():
            X.copy_(x_host, non_blocking=True)
            out_host.copy_(mf.covariance(X, prec), non_blocking=True)

        h2d, d2h = X.numel() * 4, cols * cols * 4
        passes = 6.0 if strict else 2.0
        roof = {"bound": "tensor", "peak": peaks["bf16_tflops"] / passes, "unit": "TFLOP/s",
                "peak_basis": f"bf16_tflops/{int(passes)} of {peak_src} MEASURED_PEAKS.json",
                "kernel": "mean GEMV + tc_persistent_kernel (trans_a, centering fused in the split prepass)"}
        launches = 6  # fill, GEMV partial + finish, split A, split B, GEMM

        def cpu_sample():
            sample_rows = 4096
            xs = X[:sample_rows].cpu().numpy()
            impl = "reference" if oracle.reference_available() else "restatement"
            oracle.covariance_f32(xs, impl=impl)
            t0 = time.perf_counter()
            oracle.covariance_f32(xs, impl=impl)
            dt = time.perf_counter() - t0
            info = oracle.reference_info() if impl == "reference" else {"worker_count": 1}
            return {"value": 2.0 * cols * cols * sample_rows / dt / 1e12, "unit": "TFLOPS",
                    "cores": info["worker_count"], "kind": "reference" if impl == "reference" else "port",
                    "sample": f"first {sample_rows} rows: oracle centering + the reference's gemm_f32"}
    elif kind == "conv_bwd":
        nb, c, h, w, kf = shape
        x = torch.rand((nb, c, h, w), device="cuda", generator=gen) * 2 - 1
        wt = torch.randn((kf, c, 3, 3), device="cuda", generator=gen) * float(np.sqrt(2.0 / (c * 9)))
        g = torch.randn((nb, kf, h, w), device="cuda", generator=gen)
        work = 2 * 2.0 * nb * kf * h * w * c * 9  # dx and dw: one forward-sized contraction each
        unit, metric_unit = "TFLOPS", 1e12
        desc = f"conv2d backward (dx, dw, db) NCHW {nb}x{c}x{h}x{w}, {kf} 3x3 filters, stride 1, pad 1"

        def step():
            mf.conv2d_input_backward(g, x, wt, 1, 1, prec)
            mf.conv2d_weight_backward(g, x, wt, 1, 1, prec)
            mf.conv2d_bias_backward(g)

        g_h = torch.empty_like(g, device="cpu").pin_memory()
        x_h = torch.empty_like(x, device="cpu").pin_memory()
        g_h.copy_(g)
        x_h.copy_(x)

        def e2e_step():
            g.copy_(g_h, non_blocking=True)
            x.copy_(x_h, non_blocking=True)
            dx = mf.conv2d_input_backward(g, x, wt, 1, 1, prec)
            dw = mf.conv2d_weight_backward(g, x, wt, 1, 1, prec)
            mf.conv2d_bias_backward(g)
            dx.cpu()
            dw.cpu()

        h2d, d2h = (g.numel() + x.numel()) * 4, (x.numel() + wt.numel()) * 4
        passes = 6.0 if strict else 2.0
        roof = {"bound": "tensor", "peak": peaks["bf16_tflops"] / passes, "unit": "TFLOP/s",
                "peak_basis": f"bf16_tflops/{int(passes)} of {peak_src} MEASURED_PEAKS.json",
                "kernel": "dx: tc_persistent_kernel<ConvProblem> on flipped filters; dw: tc_persistent_kernel"
                          "<ConvWgradProblem> split over positions + fixed-order reduce (time includes prepasses)"}
        launches = 10  # dx: 2 prepasses + GEMM; dw: 2 prepasses + GEMM + reduce; db: 1 (+ the output allocation)

        def cpu_sample():
            xs, gs, ws = x[:1].cpu().numpy(), g[:1].cpu().numpy(), wt.cpu().numpy()
            t0 = time.perf_counter()
            oracle.conv2d_input_backward(gs, ws, xs.shape, 1, 1)
            oracle.conv2d_weight_backward(gs, xs, ws.shape, 1, 1)
            dt = time.perf_counter() - t0
            return {"value": 2 * 2.0 * kf * h * w * c * 9 / dt / 1e12, "unit": "TFLOPS", "cores": 1, "kind": "port",
                    "sample": "1 image, single-thread restatements of the reference's backward kernels"}
    else:
        nb, c, h, w, kf = shape
        x = torch.rand((nb, c, h, w), device="cuda", generator=gen) * 2 - 1
        wt = torch.randn((kf, c, 3, 3), device="cuda", generator=gen) * float(np.sqrt(2.0 / (c * 9)))
        bias = torch.zeros(kf, device="cuda")
        y = torch.empty((nb, kf, h, w), device="cuda")
        work = 2.0 * nb * kf * h * w * c * 9  # algorithmic FLOPs per step
        unit, metric_unit = "TFLOPS", 1e12
        desc = f"conv2d forward NCHW {nb}x{c}x{h}x{w}, {kf} 3x3 filters, stride 1, pad 1"

        def step():
            mf.conv2d_into(x, wt, bias, y, 1, 1, prec)

        x_h = torch.empty_like(x, device="cpu").pin_memory()
        x_h.copy_(x)
        y_h = torch.empty_like(y, device="cpu").pin_memory()

        def e2e_step():
            x.copy_(x_h, non_blocking=True)
            step()
            y_h.copy_(y, non_blocking=True)

        h2d, d2h = x.numel() * 4, y.numel() * 4
        passes = 6.0 if strict else 2.0
        roof = {"bound": "tensor", "peak": peaks["bf16_tflops"] / passes, "unit": "TFLOP/s",
                "peak_basis": f"bf16_tflops/{int(passes)} of {peak_src} MEASURED_PEAKS.json",
                "kernel": "tc_persistent_kernel<ConvProblem> (implicit GEMM; time includes the layout prepass)"}
        launches = 3

        def cpu_sample():
            xs = x[:1].cpu().numpy()
            ws = wt.cpu().numpy()
            bs = bias.cpu().numpy()
            t0 = time.perf_counter()
            oracle.conv2d_f32(xs, ws, bs, 1, 1)
            dt = time.perf_counter() - t0
            return {"value": 2.0 * kf * h * w * c * 9 / dt / 1e12, "unit": "TFLOPS", "cores": 1, "kind": "port",
                    "sample": "1 image, single-thread restatement of conv2d_kernel (the reference has no CPU conv)"}

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    mf.sync()
    # Launch-bound workloads (a few microseconds of GPU work per step) replay the K timed steps as
    # one captured CUDA graph, so the host's Python/ctypes call overhead is not what is timed.
    use_graph = args.workload in GRAPH_WORKLOADS
    graph = None
    if use_graph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()  # per-stream scratch, if any, exists before capture
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):  # the stream whose library scratch exists
            for _ in range(args.steps):
                step()
        graph.replay()  # warm replay
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        e0.record()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(args.steps):
                step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    mf.sync()
    value = work * args.steps / (ms / 1e3) / metric_unit
    roof.update({"achieved": value, "frac": value / roof["peak"], "traffic": read_profile_traffic(
        f"{args.workload}_{args.precision}" if kind in ("conv", "conv_bwd") else args.workload)})
    if roof["bound"] == "tensor" and rank == 0:
        roof.update(tf32_mma_fields(mf, local, value, strict))
    e2e = None
    if args.e2e_steps > 0:
        e2e_step()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        s1.record()
        torch.cuda.synchronize()
        e2e = {"value": work * args.e2e_steps / (s0.elapsed_time(s1) / 1e3) / metric_unit, "unit": unit,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": args.e2e_steps,
               "link": link_roofline(torch, h2d, d2h, s0.elapsed_time(s1) / args.e2e_steps)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_sample()
        except Exception as exc:
            cpu = {"value": None, "unit": unit, "cores": None, "kind": None, "sample": f"failed: {exc}"}
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value * world, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": desc, "precision": args.precision, "parallelism": f"{world} independent replicas",
                       "l2": "inputs larger than L2 every step" if not use_graph
                       else "launch-bound workload: inputs fit in L2; the K steps replay as one CUDA graph",
                       "cuda_graph": use_graph},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches * args.steps,
            "clocks": clocks.summary()}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mfb", "reference"], default="mfb")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(AUX_WORKLOADS), default="linear")
    ap.add_argument("--precision", choices=["fp32", "tf32"], default="fp32")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the oracle check of a sampled block of C")
    ap.add_argument("--ref-rows", type=int, default=2048, help="rows per reference-arm step (bounded sample)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload in AUX_WORKLOADS:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm is defined for the GEMM "
                              "workloads (the reference's CPU path for this path is gemm_f32)"}))
            return 0
        return run_aux_workload(args)
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference_arm(args, wl)

    import torch
    import torch.distributed as dist
    import matrixflash_pro_b200 as mf
    from matrixflash_pro_b200.distributed import RowSplitGemm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    m_total, n, k, lda, ldb, ldc, alpha, beta, desc = wl
    if args.workload == "c5":
        m = -(-m_total // world)  # strong scaling: the rows of one product split across ranks
        scaling = "strong"
    else:
        m = m_total               # weak scaling: m rows per GPU
        scaling = "weak"
    precision = mf.GemmPrecision.fp32 if args.precision == "fp32" else mf.GemmPrecision.tf32

    gen = torch.Generator(device="cuda").manual_seed(20261001 + rank)
    A_buf = torch.randn((m, lda), device="cuda", generator=gen)
    B_buf = torch.randn((k, ldb), device="cuda", generator=torch.Generator(device="cuda").manual_seed(7)) / 64.0
    C_buf = torch.randn((m, ldc), device="cuda", generator=gen)
    A, B, C = A_buf[:, :k], B_buf[:, :n], C_buf[:, :n]
    op = RowSplitGemm(m, n, k, lda, ldb, ldc, precision)
    check = SampledCheck(torch, m, n, k, C, rank) if not args.no_check else None

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        op(A, B, C, alpha, beta)
    torch.cuda.synchronize()
    mf.sync()
    # one more warm-up step, timed, to tell short steps from long ones (see the timed loop)
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0.record()
    op(A, B, C, alpha, beta)
    w1.record()
    torch.cuda.synchronize()
    t_warm = torch.tensor([w0.elapsed_time(w1)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_warm, op=dist.ReduceOp.MAX)  # every rank takes the same branch
    short_steps = float(t_warm.item()) < 1.0

    # ---------------------------------------------------------------- timed region (device)
    # Bytes one step touches: A, B, C (read and written) and the operand planes of the prepass.
    planes = 2 if precision == mf.GemmPrecision.fp32 else 1
    footprint = 4 * (m * lda + k * ldb + 2 * m * ldc) + 4 * planes * (m * (k + 3) + k * (n + 3))
    flush = footprint < 2 * L2_BYTES  # otherwise the inputs exceed L2 every step
    flush_buf = torch.empty(FLUSH_BYTES // 4, device="cuda") if flush else None
    stream = torch.cuda.current_stream()
    kernel_ms = 0.0
    step_events = []
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        kernel_records = []
        for _ in range(args.steps):
            # The GEMM kernels' own time, for the roofline, comes from CUDA events around each
            # GEMM launch. An event between the prepass and the GEMM keeps the GEMM from
            # launching programmatically behind the prepass: measured 4-8% of a 2048^3 step,
            # noise on a 3 ms step. Short steps (under 1 ms) therefore run clean and each is
            # followed by an untimed twin that carries the events, under the same flush,
            # clocks and power state; long steps carry the events themselves, since a twin per
            # step would double their power draw and bring on the power cap. Every timed step
            # is bracketed by its own events and `value` sums those.
            if flush:
                flush_buf.zero_()  # a write larger than L2 before each step
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            op(A, B, C, alpha, beta, time_kernels=not short_steps)
            s1.record(stream)
            step_events.append((s0, s1))
            if short_steps:
                if flush:
                    flush_buf.zero_()
                op(A, B, C, alpha, beta, time_kernels=True)
            kernel_records.extend(op.kernel_events)
        torch.cuda.synchronize()
        barrier()
    elapsed_ms = sum(a.elapsed_time(b) for a, b in step_events)
    kernel_ms = sum(a.elapsed_time(b) for a, b in kernel_records)
    mf.sync()  # raises on a device-side timeout

    t = torch.tensor([elapsed_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    flops_per_rank_step = 2.0 * m * n * k
    value = world * flops_per_rank_step * args.steps / (max_ms / 1e3) / 1e12

    # ---------------------------------------------------------------- end to end (host buffers)
    e2e = None
    if args.e2e_steps > 0:
        A_h = torch.empty((m, lda), dtype=torch.float32, pin_memory=True)
        B_h = torch.empty((k, ldb), dtype=torch.float32, pin_memory=True)
        C_h = torch.empty((m, ldc), dtype=torch.float32, pin_memory=True)
        A_h.copy_(A_buf)
        B_h.copy_(B_buf)
        C_h.copy_(C_buf)
        A_hv, B_hv, C_hv = A_h[:, :k], B_h[:, :n], C_h[:, :n]
        opts = mf.GemmOptions(precision=precision)
        # mfb_sgemm_host streams rows of A and C through the GPU in panels (copies overlap the
        # GEMM) and returns C into the same pinned host matrix. B: from host on one GPU; with
        # several, rank 0 copies it in and broadcasts it over NVLink, as RowSplitGemm takes it.
        h2d = 4 * (m * k + (m * n if beta != 0.0 else 0) + (k * n if rank == 0 else 0))
        d2h = 4 * m * n

        def e2e_step():
            if world == 1:
                mf.sgemm_host(A_hv, B_hv, C_hv, alpha, beta, opts)
                return
            if rank == 0:
                B_buf.copy_(B_h, non_blocking=True)
            dist.broadcast(B_buf, src=0)
            mf.sgemm_host(A_hv, B, C_hv, alpha, beta, opts)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t2 = torch.tensor([s0.elapsed_time(s1)], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        e2e_ms = float(t2.item())
        e2e = {"value": world * flops_per_rank_step * args.e2e_steps / (e2e_ms / 1e3) / 1e12, "unit": "TFLOPS",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": args.e2e_steps,
               "path": "mfb_sgemm_host on pinned host A/B/C (row panels of A and C copied in and C copied out "
                       "on copy streams while the GEMM of the previous panel runs)"
                       + ("" if world == 1 else "; B copied in on rank 0 and broadcast (NCCL)"),
               "link": link_roofline(torch, h2d, d2h, e2e_ms / args.e2e_steps)}

    # ---------------------------------------------------------------- oracle check (every rank)
    strict = precision == mf.GemmPrecision.fp32
    check_line = None
    if check is not None:
        try:
            res = check.run(torch, op, A, B, B_buf, C, alpha, beta, strict, rank)
        except Exception as exc:  # reported as a failed check; every rank still joins the gather
            print(f"rank {rank}: oracle check failed to run: {exc}", file=sys.stderr)
            res = [float("inf"), 0.0, float("inf"), 0.0, float("nan"), 0.0]
        mine = torch.tensor(res, device="cuda", dtype=torch.float64)
        if world > 1:
            gathered = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(gathered, mine)
        else:
            gathered = [mine]
        check_line = SampledCheck.summarize([g.cpu().tolist() for g in gathered], strict)

    # ---------------------------------------------------------------- roofline of the GEMM kernel
    peaks, peak_src = read_peaks()
    passes = 6.0 if strict else 2.0   # TF32 runs at half the bf16 rate; strict = 3 TF32 passes
    # Short loops of ~3-5 ms steps run at full clocks (see "clocks"): burst denominator. Long steps
    # (the 32768^3 case: ~0.4 s each, seconds in total) run into the 1000 W power cap: sustained.
    peak_burst = peaks["bf16_tflops"] / passes
    peak_sust = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]) / passes
    long_run = max_ms / args.steps > 50.0 or max_ms > 1000.0
    peak_used = peak_sust if long_run else peak_burst
    gemm_flops = flops_per_rank_step * args.steps
    achieved = gemm_flops / (kernel_ms / 1e3) / 1e12 if kernel_ms > 0 else None
    launches_gemm = op.gemm_launches_per_step() * args.steps
    tag = f"gemm_{'3xtf32' if strict else 'tf32'}_{args.workload}"
    traffic = read_profile_traffic(tag)
    basis = "bf16_tflops_sustained" if long_run else "bf16_tflops"
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_used, "unit": "TFLOP/s",
                "frac": (achieved / peak_used) if achieved else None, "traffic": traffic,
                "kernel": "tc_pair_kernel / tc_persistent_kernel (tcgen05 kind::tf32, "
                          + ("3xTF32" if strict else "1xTF32") + ")"
                          + (" + streamk_reduce_kernel (the last tiles share K among the SMs; the timed GEMM "
                             "phase includes this fix-up)" if op.plan.stream_k and world == 1 else ""),
                "peak_basis": f"{basis}/{int(passes)} of {peak_src} MEASURED_PEAKS.json "
                              f"({'sustained: long steps hit the power cap' if long_run else 'burst: short steps'}; "
                              "TF32 = bf16/2, strict = 3 TF32 passes)",
                "peak_burst": peak_burst, "peak_sustained": peak_sust,
                "kernel_ms_per_launch": kernel_ms / max(1, launches_gemm),
                "kernel_timing": ("CUDA events around each GEMM launch of an untimed twin that follows every "
                                  "timed step (steps under 1 ms)" if short_steps else
                                  "CUDA events around each GEMM launch of the timed steps"),
                "flops_per_launch": gemm_flops / max(1, launches_gemm)}
    if rank == 0:
        roofline.update(tf32_mma_fields(mf, local, achieved, strict))

    # ---------------------------------------------------------------- CPU baseline (rank 0, N=1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            rows = 1024 if args.workload in ("linear", "square8192") else min(256, m)
            r = cpu_reference_sample(m, n, k, lda, ldb, ldc, alpha, beta, rows, reps=3)
            cpu = {"value": r["tflops"], "unit": "TFLOPS", "cores": r["cores"], "kind": r["kind"],
                   "sample": f"{rows} rows x n={n} x k={k} of the same workload, 1 warm-up + median of 3 "
                             f"({r['seconds_per_rep']:.2f} s each), gemm_f32 kernel {r['kernel']}, "
                             f"nproc={os.cpu_count()}"}
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "TFLOPS", "cores": None, "kind": None, "sample": f"failed: {exc}"}

    clk = clocks.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": desc, "m_per_gpu": m, "n": n, "k": k, "lda": lda, "ldb": ldb, "ldc": ldc,
                       "precision": "strict fp32 (3xTF32 tcgen05)" if strict else "tf32 (tcgen05)",
                       "parallelism": f"row-split x{world}" + (", B broadcast by NCCL in column panels" if world > 1
                                                               else ""),
                       "l2": (f"step footprint {footprint / 2**20:.0f} MiB < 2 x L2: L2 flushed by a "
                              f"{FLUSH_BYTES >> 20} MiB write between steps, each step timed alone by CUDA "
                              "events" if flush else
                              f"step footprint {footprint / 2**20:.0f} MiB, larger than L2 (126 MB) every step; "
                              "each step timed alone by CUDA events"),
                       "global_batch": m * world, "seq_len": None,
                       "b_panels": op.sched.panels if world > 1 else None,
                       "panels_capped_at_end": ([i for i, c in enumerate(op.capped) if c] if world > 1 else None)},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": op.launches_per_step() * args.steps, "clocks": clk, "check": check_line,
        }
        print(json.dumps(line))
    op.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if check_line is not None and not check_line["ok"]:
        print(f"oracle check failed: {check_line}", file=sys.stderr)
        return 3
    return 0


if __name__ == "__main__":
    sys.exit(main())
