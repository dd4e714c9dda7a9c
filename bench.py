#!/usr/bin/env python
"""Batched SPD Cholesky-solve benchmark (one JSON line on rank 0).

A step is one fused pass of the hot path over one batch: Cholesky factor +
forward/back substitution + log-determinant of B SPD matrices (k x k,
float32), i.e. the work of mlx_addons.linalg's ``solve`` plus ``logdet_spd``
on the same A, through the C ABI entry ``b2c_posv``. The default workload is
the headline configuration: B = 10,000 matrices per GPU, k = 64, one
right-hand side (A = G G^T / 64 + I, G ~ N(0, 1), b ~ N(0, 1), generated on
the device from a seed).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2_k64]
  torchrun --nproc-per-node N bench.py --gpus N ...        (one rank per GPU)
  python bench.py --impl reference ...                      (CPU reference arm)

Timing: W untimed warm-up launches, then EXACTLY K launches captured in one
CUDA graph and replayed between CUDA events on the launching stream, with a
barrier + synchronize on both sides; the time is the max over ranks, and each
rank's time is printed too. A 2 ms device-side sleep queued before the start
event keeps host delays out of the window. Inputs
rotate through enough buffer sets that the bytes touched between two reads of
the same set exceed twice the L2 size. Every rank processes its own B
matrices (weak scaling, no collective on the data path). SM clocks and
throttle reasons are sampled through NVML during the timed region.

e2e: the same metric through the public API (mlx_addons_b200.linalg
.cho_solve_logdet) with pinned HOST inputs: host->device copy of A and b,
the kernel, device->host copy of x and logdet, every step, host-timed.

cpu_baseline (rank 0, N = 1): the reference's own kernel code compiled for
the host (oracle/_ref), all host threads, on a bounded sample of the same
workload; LAPACK spotrf + spotrs is reported beside it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "SPD solves/sec at k=64,B=10K on 1/2/4/8 B200; % of HBM/FP32 roofline"
UNIT = "solves/s"
WORKLOADS = {
    # headline; the reference README publishes this workload (B = 10,000,
    # k = 64, one right-hand side): 29.62 ms on an Apple M3 Max
    "c2_k64": dict(B=10_000, k=64, m=1, eps=1.0, pub_ms=29.62),
    "c1_k16": dict(B=10_000, k=16, m=1, eps=1.0),
    "c3_k5": dict(B=1_000_000, k=5, m=4, eps=0.1),
    "c4_k256": dict(B=1_000, k=256, m=8, eps=1.0),
    "c5_k512": dict(B=8_000, k=512, m=1, eps=1.0),
}
# The reference README's own solve tables (M3 Max, README.md:94-109), on its
# benchmark's inputs (benchmarks/bench_linalg.py:16-25: A = G G^T + k I,
# b ~ N(0, 1), one right-hand side): the published GPU time is the baseline
# of each line (vs_baseline = published ms / measured ms).
for _k, _B, _ms in ((5, 10_000, 0.63), (15, 10_000, 0.97), (30, 10_000, 2.20), (48, 10_000, 10.51),
                    (64, 10_000, 29.62), (80, 10_000, 66.64), (128, 1_000, 14.4), (256, 1_000, 59.9),
                    (512, 1_000, 222.3)):
    WORKLOADS[f"readme_k{_k}_b{_B // 1000}k"] = dict(B=_B, k=_k, m=1, eps=float(_k), div=1.0, pub_ms=_ms)
del _k, _B, _ms


def algo_bytes(k, m, op="posv"):
    """HBM bytes of one matrix. posv: A read once, b read, x and logdet
    written. gesv: A and b read, x written. qr: A read, Q and R written."""
    if op == "gesv":
        return 4 * (k * k + 2 * k * m)
    if op == "qr":
        return 4 * 3 * k * k
    if op == "seq3":  # A read three times, L written, b read, x written, logdet written
        return 4 * (4 * k * k + 2 * k * m + 1)
    if op == "slogdet":
        return 4 * (k * k + 2)
    if op == "trsm":  # the lower triangle of L read, b read, x written
        return 4 * (k * (k + 1) // 2 + 2 * k * m)
    return 4 * (k * k + 2 * k * m + 1)


def algo_flops(k, m, op="posv"):
    """LAWN 41 counts. posv: potrf k^3/3 + k^2/2 + k/6 and two triangular
    solves 2 k^2 m. gesv: getrf 2k^3/3 - k^2/2 + 5k/6 and 2 k^2 m. qr: geqrf
    4k^3/3 + 2k^2 + 14k/3 and orgqr 4k^3/3 (square)."""
    if op == "gesv":
        return 2 * k ** 3 / 3 - k ** 2 / 2 + 5 * k / 6 + 2 * k * k * m
    if op == "qr":
        return 8 * k ** 3 / 3 + 2 * k ** 2 + 14 * k / 3
    if op == "seq3":
        return 3 * (k ** 3 / 3 + k ** 2 / 2 + k / 6) + 2 * k * k * m
    if op == "slogdet":
        return 2 * k ** 3 / 3 - k ** 2 / 2 + 5 * k / 6
    if op == "trsm":
        return k * k * m
    return k ** 3 / 3 + k ** 2 / 2 + k / 6 + 2 * k * k * m


# The general-matrix rows (solve_lu, qr) reuse the configurations' B, k, m on
# A = G ~ N(0, 1) (non-symmetric; LU pivots, QR reflects every column).
OP_METRICS = {
    "posv": (METRIC, UNIT),
    "gesv": ("general (partial-pivot LU) solves/sec, solve_lu", "solves/s"),
    "qr": ("Householder QR factorizations/sec (Q and R), qr", "factorizations/s"),
    "seq3": ("SPD solves/sec through the literal API sequence cholesky -> solve -> logdet_spd (3 calls)",
             "solves/s"),
    "slogdet": ("slogdet (sign, log|det|) per second, partial-pivot LU", "determinants/s"),
    "trsm": ("triangular solves/sec, triu_solve (L^T x = b with the lower factor)", "solves/s"),
}


# randomized_svd workloads: the reference's benchmark shapes
# (benchmarks/bench_svd.py:64-69), n_iter = 4, n_oversamples = 10.
RSVD_WORKLOADS = {
    "rsvd_10000x2048_k32": (10_000, 2048, 32),
    "rsvd_5000x1024_k64": (5_000, 1024, 64),
    "rsvd_2000x512_k32": (2_000, 512, 32),
    "rsvd_633x128_k32": (633, 128, 32),
}
# The reference README's M3 Max time for (10000, 2048), k = 32: 59 ms per call
# (src/mlx_addons/linalg/_svd.py:17).
RSVD_PUBLISHED_MS = {"rsvd_10000x2048_k32": 59.0, "rsvd_5000x1024_k64": 46.0, "rsvd_2000x512_k32": 12.0,
                     "rsvd_633x128_k32": 8.0}


def rsvd_flops_bytes(n, m, k, n_iter=4, p=10):
    """The products with X dominate: X Omega, 2 n_iter products in the power
    iteration and Q^T X, each 2 n m (k + p) flops and one read of X (4 n m
    bytes)."""
    passes = 2 + 2 * n_iter
    return passes * 2.0 * n * m * (k + p), passes * 4.0 * n * m


def kernel_name(op, k, m=1):
    if op == "trsm":
        return "trsm_kernel"
    if op == "gesv":
        return ("gesv_warp_kernel" if k <= 32 else "gesv_warp2_kernel" if k <= 64 else
                "gesv_cta_kernel" if k <= 224 or k > 864 else "gesv_blocked_kernel")
    if op == "qr":
        return "qr_warp_kernel" if k <= 32 else "qr_warp64_kernel" if k <= 64 else "qr_cta_kernel"
    if op == "slogdet":
        return ("slogdet_half_kernel" if k <= 16 else "slogdet_warp_kernel" if k <= 32 else
                "slogdet_cta_kernel" if k <= 224 or k > 864 else "slogdet_blocked_kernel")
    if 32 < k <= 64:
        return "posv_tile_kernel" if m <= 1 and os.environ.get("B2C_TILE_TIER", "1")[:1] != "0" \
            else "posv_warp64_kernel"
    dag, nb = os.environ.get("B2C_SMEM_DAG", ""), (k + 31) // 32
    if (nb >= 3 if dag == "all" else nb >= 7 or (3 <= nb <= 5 and m >= 2)) and k <= 256 and k % 4 == 0 and m <= 8 \
            and dag != "0":
        return "posv_dag_kernel"
    return ("posv_thread_db_kernel" if k <= 16 else "posv_seg_kernel" if k <= 32 else
            "posv_smem_kernel" if k <= 256 else
            "posv_blocked2_kernel" if k <= 9216 and os.environ.get("B2C_BLOCKED_LEGACY", "")[:1] != "1"
            else "posv_blocked_kernel")


def workload_text(op, B, k, m, eps):
    """The workload named the same way in the GPU and the reference arm."""
    return {"posv": f"batched SPD factor+solve+logdet, B={B} per GPU, k={k}, m={m}, eps={eps}",
            "gesv": f"batched general LU solve (solve_lu), B={B} per GPU, k={k}, m={m}, A ~ N(0,1)",
            "qr": f"batched Householder QR (qr), B={B} per GPU, k={k}, A ~ N(0,1)",
            "seq3": f"batched SPD cholesky + solve + logdet_spd as 3 API calls, B={B} per GPU, k={k}, m={m}, "
                    f"eps={eps}",
            "slogdet": f"batched slogdet (partial-pivot LU), B={B} per GPU, k={k}, A ~ N(0,1)",
            "trsm": f"batched triu_solve (L^T x = b), B={B} per GPU, k={k}, m={m}, L = tril(G)/sqrt(k) + |diag|"}[op]


def zero_copy_a_bytes(k):
    """Bytes of one k x k matrix that the zero-copy path pulls across PCIe:
    the k <= 64 tiers fetch the 16-byte chunks holding lower-triangle entries,
    i.e. ceil((floor(r/4) + 1) / 2) 32-byte sectors of row r; the other tiers
    read the whole lower-triangle block rows, counted here as all of A."""
    if k <= 64:
        return sum(-(-((r // 4) + 1) // 2) for r in range(k)) * 32
    return 4 * k * k


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measure_fp32_peak(dev):
    """FP32 FFMA peak of this GPU, measured: the best of 10 cuBLAS SGEMMs of
    8192^3 (TF32 disabled, 2 N^3 flops each) timed with CUDA events. The
    nominal figure is 148 SMs x 128 lanes x 2 x 1.965 GHz = 74.4 TFLOP/s."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        n = 8192
        a = torch.randn(n, n, device=dev)
        b = torch.randn(n, n, device=dev)
        c = torch.empty(n, n, device=dev)
        for _ in range(2):
            torch.mm(a, b, out=c)
        best = float("inf")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(10):
            e0.record()
            torch.mm(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e-3)
        del a, b, c
        return 2.0 * n ** 3 / best / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


FFMA_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # 74.4: 148 SMs x 128 FP32 lanes x 2 x 1.965 GHz


def roofline(B, k, m, op, per_launch, hbm_peak, peak_src, fp32_peak, traffic, kernel, config=None):
    """Roofline of one launch: the slower of the algorithmic bytes at the HBM
    peak and the algorithmic flops at the FP32 peak names the bound."""
    nbytes, flops = B * algo_bytes(k, m, op), B * algo_flops(k, m, op)
    gbs, tfs = nbytes / per_launch / 1e9, flops / per_launch / 1e12
    hbm_src = f"{peak_src} hbm_gbs (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback 6650 GB/s"
    fp32_src = "measured: best cuBLAS SGEMM 8192^3 (TF32 off) in this run"
    common = {"traffic": traffic,
              "traffic_source": (f"dram__bytes_read.sum + dram__bytes_write.sum per launch from the committed ncu "
                                 f"summary profiles/{op}_{config}_ncu.md (not measured in this run)")
              if traffic is not None else None,
              "bytes_per_matrix": algo_bytes(k, m, op), "flops_per_matrix": algo_flops(k, m, op),
              "kernel": kernel, "hbm_gbs": gbs, "hbm_frac": gbs / hbm_peak, "fp32_tflops": tfs,
              "fp32_peak_tflops": fp32_peak, "fp32_frac": tfs / fp32_peak if fp32_peak else None,
              "fp32_frac_of_nominal_ffma": tfs / FFMA_NOMINAL_TFLOPS}
    if fp32_peak and flops / (fp32_peak * 1e12) > nbytes / (hbm_peak * 1e9):
        return {"bound": "fp32", "achieved": tfs, "peak": fp32_peak, "unit": "TFLOP/s", "frac": tfs / fp32_peak,
                "peak_source": fp32_src, **common}
    return {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
            "peak_source": hbm_src, **common}


def profile_traffic(config, op="posv", kernel=None, overridden=False):
    """DRAM bytes per launch from the committed ncu summary of this workload,
    if any: only for the workload as named (no batch, k or m override) and
    only when the summary's title names the kernel that runs it."""
    path = os.path.join(ROOT, "profiles", f"{op}_{config}_ncu.md")
    if overridden or not os.path.exists(path):
        return None
    with open(path) as f:
        text = f.read()
    if kernel and kernel not in text.split("\n", 1)[0]:
        return None
    mt = re.search(r"dram_bytes_per_launch\s*=\s*([0-9.eE+]+)", text)
    return float(mt.group(1)) if mt else None


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    """Polls the SM clock and the clock-event reasons of one GPU through NVML
    on a background thread while the timed region runs."""

    def __init__(self, torch_device):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        self._h = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            self.error = f"{type(e).__name__}: {e}"

    def _run(self):
        nv = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(get_reasons(self._h))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.0005)

    def start(self):
        if self._h is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()

    def stop(self):
        if self._thr is not None:
            self._stop.set()
            self._thr.join()

    def summary(self):
        if self._h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "error": getattr(self, "error", "nvml unavailable")}
        names = [n for bit, n in _REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        med = float(np.median(self.samples)) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                "source": "NVML polled during the timed region"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def run_b2c(args, rank, world, local):
    import torch
    import torch.distributed as dist

    from mlx_addons_b200 import _lib
    import mlx_addons_b200.linalg as la

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    wl = WORKLOADS[args.config]
    B, k, m, eps = wl["B"], wl["k"], wl["m"], wl["eps"]
    if args.batch:
        B = args.batch
    if args.k:
        k = args.k
    if args.m:
        m = args.m
    lib = _lib.load()
    props = torch.cuda.get_device_properties(dev)
    l2 = int(getattr(props, "L2_cache_size", 126 << 20))
    set_bytes = B * k * k * 4 + B * k * m * 4
    nbuf = int(min(8, max(2, math.ceil(2 * l2 / set_bytes) + 1)))

    op = args.op
    if op == "qr":
        m = 0
        set_bytes = B * k * k * 4 * 3
        nbuf = int(min(8, max(2, math.ceil(2 * l2 / set_bytes) + 1)))

    if op == "seq3":  # L is written as well
        set_bytes = B * k * k * 4 * 2 + B * k * m * 4
        nbuf = int(min(8, max(2, math.ceil(2 * l2 / set_bytes) + 1)))
    if op == "slogdet":
        m = 0

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    As, bs, xs, lds, Ls = [], [], [], [], []
    for _ in range(nbuf):
        G = torch.randn((B, k, k), generator=gen, device=dev)
        if op == "trsm":  # a well-conditioned lower-triangular factor
            A = torch.tril(G) / math.sqrt(k)
            A.diagonal(dim1=1, dim2=2).abs_().add_(1.0)
            del G
        elif op in ("posv", "seq3"):
            A = torch.empty((B, k, k), device=dev)
            for lo in range(0, B, 4096):
                torch.bmm(G[lo:lo + 4096], G[lo:lo + 4096].transpose(1, 2), out=A[lo:lo + 4096])
            A.div_(wl.get("div", k))
            A.diagonal(dim1=1, dim2=2).add_(eps)
            del G
        else:
            A = G
        As.append(A)
        if op == "qr":  # xs: Q, lds: R
            xs.append(torch.empty((B, k, k), device=dev))
            lds.append(torch.empty((B, k, k), device=dev))
            continue
        if op == "slogdet":  # xs: sign, lds: log|det|
            xs.append(torch.empty((B,), device=dev))
            lds.append(torch.empty((B,), device=dev))
            continue
        if op == "seq3":
            Ls.append(torch.empty((B, k, k), device=dev))
        bs.append(torch.randn((B, k, m), generator=gen, device=dev))
        xs.append(torch.empty((B, k, m), device=dev))
        lds.append(torch.empty((B,), device=dev))
    ws_op = {"posv": _lib.OP_POSV, "gesv": _lib.OP_GESV, "qr": _lib.OP_QR, "seq3": _lib.OP_POSV,
             "slogdet": _lib.OP_SLOGDET, "trsm": _lib.OP_TRSM}[op]
    ws_bytes = int(lib.b2c_workspace_size(ws_op, B, k, m))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)

    def launch(i, stream_handle):
        j = i % nbuf
        if op == "posv":
            rc = lib.b2c_posv(As[j].data_ptr(), bs[j].data_ptr(), xs[j].data_ptr(), None, lds[j].data_ptr(),
                              B, k, m, ws.data_ptr(), ws_bytes, stream_handle)
        elif op == "gesv":
            rc = lib.b2c_gesv(As[j].data_ptr(), bs[j].data_ptr(), xs[j].data_ptr(), B, k, m, ws.data_ptr(),
                              ws_bytes, stream_handle)
        elif op == "seq3":  # L = cholesky(A); x = solve(A, b); ld = logdet_spd(A)
            rc = lib.b2c_potrf(As[j].data_ptr(), Ls[j].data_ptr(), None, B, k, None, 0, stream_handle)
            _lib.check(rc, "b2c_potrf")
            rc = lib.b2c_posv(As[j].data_ptr(), bs[j].data_ptr(), xs[j].data_ptr(), None, None, B, k, m,
                              ws.data_ptr(), ws_bytes, stream_handle)
            _lib.check(rc, "b2c_posv")
            rc = lib.b2c_potrf(As[j].data_ptr(), None, lds[j].data_ptr(), B, k, ws.data_ptr(), ws_bytes,
                               stream_handle)
        elif op == "slogdet":
            rc = lib.b2c_slogdet(As[j].data_ptr(), xs[j].data_ptr(), lds[j].data_ptr(), B, k, ws.data_ptr(),
                                 ws_bytes, stream_handle)
        elif op == "trsm":
            rc = lib.b2c_trsm(As[j].data_ptr(), bs[j].data_ptr(), xs[j].data_ptr(), B, k, m, 1, stream_handle)
        else:
            rc = lib.b2c_qr(As[j].data_ptr(), xs[j].data_ptr(), lds[j].data_ptr(), B, k, ws.data_ptr(),
                            ws_bytes, stream_handle)
        _lib.check(rc, "b2c_" + op)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            launch(i, stream.cuda_stream)
    torch.cuda.synchronize(dev)

    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(args.steps):
                launch(args.warmup + i, stream.cuda_stream)
        torch.cuda.synchronize(dev)

    sampler = ClockSampler(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    # a 2 ms device-side pre-roll (torch's sleep kernel, before the start
    # event) keeps the stream busy while the host enqueues the start event, the
    # K launches and the end event, so a late host thread (another rank, the
    # clock sampler) cannot open an idle gap inside the timed window
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(2e-3 * props.clock_rate * 1e3))
    e0.record(stream)
    if graph is not None:
        with torch.cuda.stream(stream):
            graph.replay()
    else:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                launch(args.warmup + i, stream.cuda_stream)
    e1.record(stream)
    e1.synchronize()
    sampler.stop()
    torch.cuda.synchronize(dev)
    elapsed = e0.elapsed_time(e1) / 1e3
    per_rank = [elapsed]
    if world > 1:
        t = torch.tensor([elapsed], device=dev, dtype=torch.float64)
        allt = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        per_rank = [float(x.item()) for x in allt]
        elapsed = max(per_rank)
        dist.barrier()
    del graph

    # the timed kernels did the work: sampled backward error of the last outputs
    j = (args.warmup + args.steps - 1) % nbuf
    idx = torch.randperm(B)[:16].to(dev)
    if op == "slogdet":
        A_ = As[j][idx].double()
        s_ref, l_ref = torch.linalg.slogdet(A_)
        check = {"sign_matches_float64": bool((xs[j][idx].double() == s_ref).all()),
                 "max_abs_logabsdet_error_vs_float64": float((lds[j][idx].double() - l_ref).abs().max()),
                 "finite": bool(torch.isfinite(lds[j]).all())}
    elif op == "qr":
        A_, Q_, R_ = (t[idx].double() for t in (As[j], xs[j], lds[j]))
        rec = torch.linalg.norm((Q_ @ R_ - A_).flatten(1), dim=1) / torch.linalg.norm(A_.flatten(1), dim=1)
        orth = (Q_.transpose(1, 2) @ Q_ - torch.eye(k, dtype=torch.float64, device=dev)).abs().amax()
        check = {"max_reconstruction_error": float(rec.max()), "max_orthogonality_error": float(orth),
                 "finite": bool(torch.isfinite(xs[j]).all() and torch.isfinite(lds[j]).all())}
    else:
        As_, bs_, xs_ = (t[idx].double() for t in (As[j], bs[j], xs[j]))
        S = (torch.tril(As_) + torch.tril(As_, -1).transpose(1, 2) if op in ("posv", "seq3") else
             As_.transpose(1, 2) if op == "trsm" else As_)
        r = torch.linalg.norm((S @ xs_ - bs_).flatten(1), dim=1) / (
            torch.linalg.norm(S.flatten(1), dim=1) * torch.linalg.norm(xs_.flatten(1), dim=1))
        check = {"max_backward_error": float(r.max()), "finite": bool(torch.isfinite(xs[j]).all())}

    # e2e through the public API with pinned host buffers
    e2e = None
    metric, unit = OP_METRICS[op]
    if not args.no_e2e:
        pcie = None
        A_h = As[0].cpu().pin_memory()
        b_h = bs[0].cpu().pin_memory() if op not in ("qr", "slogdet") else None
        call = {"posv": lambda: la.cho_solve_logdet(A_h, b_h), "gesv": lambda: (la.solve_lu(A_h, b_h),),
                "trsm": lambda: (la.triu_solve(A_h, b_h),),
                "qr": lambda: la.qr(A_h), "slogdet": lambda: la.slogdet(A_h),
                "seq3": lambda: (la.cholesky(A_h), la.solve(A_h, b_h), la.logdet_spd(A_h))}[op]
        call()  # warm the pinned pool and the streams
        n_e2e = int(max(3, min(args.steps, args.e2e_steps)))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            outs = call()
        t_e2e = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([t_e2e], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        pcie = None
        if op == "posv":
            # the pinned-copy ceiling of this box, and the staged path (copy
            # engine, pipelined chunks on two streams) beside the zero-copy one
            blk = torch.empty((32 << 20,), dtype=torch.float32, pin_memory=True)
            blk_d = torch.empty_like(blk, device=dev)
            blk_d.copy_(blk, non_blocking=True)
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(5):
                blk_d.copy_(blk, non_blocking=True)
            torch.cuda.synchronize(dev)
            copy_gbs = 5 * blk.numel() * 4 / (time.perf_counter() - t0) / 1e9
            del blk, blk_d
            staged = lambda: la._host_call(lambda a_, b_: la._posv_dev(a_, b_, True, False, True)[::2],  # noqa: E731
                                           [A_h, b_h])
            staged()
            n_st = max(3, n_e2e // 2)
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(n_st):
                staged()
            t_st = time.perf_counter() - t0
            cross = B * (zero_copy_a_bytes(k) + 4 * k * m)
            pcie = {"h2d_bytes_crossing_per_step": int(cross),
                    "d2h_bytes_crossing_per_step": int(B * 4 * (k * m + 1)),
                    "achieved_h2d_gbs": cross / (t_e2e / n_e2e) / 1e9,
                    "pinned_copy_gbs_measured": copy_gbs,
                    "frac_of_pinned_copy": cross / (t_e2e / n_e2e) / 1e9 / copy_gbs,
                    "note": "the zero-copy kernels read only the 32-byte sectors holding lower-triangle "
                            "entries of A (h2d_bytes_per_step counts the full tensors)",
                    "staged_copy_engine_path": {"value": B * n_st / t_st, "unit": unit,
                                                "what": "linalg._host_call: full A and b copied by the copy "
                                                        f"engine in {la._HOST_CHUNK_BYTES >> 20} MB chunks on two "
                                                        "streams, overlapping the kernels"}}
        api = {"posv": "cho_solve_logdet(host pinned A, b)", "gesv": "solve_lu(host pinned A, b)",
               "trsm": "triu_solve(host pinned L, b)",
               "qr": "qr(host pinned A)", "slogdet": "slogdet(host pinned A)",
               "seq3": "cholesky, solve, logdet_spd (host pinned A, b)"}[op]
        e2e = {"value": world * B * n_e2e / t_e2e, "unit": unit, "steps": n_e2e,
               "h2d_bytes_per_step": int(A_h.numel() * 4 + (b_h.numel() * 4 if b_h is not None else 0)),
               "d2h_bytes_per_step": int(sum(o.numel() * 4 for o in outs)),
               "api": "mlx_addons_b200.linalg." + api,
               "transfer": "pinned host buffers handed to the kernel (zero-copy): the inputs cross PCIe "
                           "inside the kernel every step and the outputs are written back to host memory"
                           + (" (the k<=64 tier reads only the lower-triangle chunks of A)" if op == "posv"
                              else "") + "; h2d bytes count the full input tensors",
               "timing": "host clock around blocking calls, max over ranks"}
        if pcie is not None:
            e2e["pcie"] = pcie

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0

    value = world * B * args.steps / elapsed
    per_launch = elapsed / args.steps
    hbm_peak, peak_src = load_peaks()
    fp32_peak = measure_fp32_peak(dev)
    traffic = profile_traffic(args.config, op, kernel_name(op, k, m), bool(args.batch or args.k or args.m))
    what = workload_text(op, B, k, m, eps)
    out = {
        "metric": metric,
        "value": value,
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_launch * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        # null where the reference publishes no number for this workload
        "vs_baseline": wl["pub_ms"] / (per_launch * 1e3) if (op == "posv" and "pub_ms" in wl) else None,
        "dtype": "f32",
        "data": (f"synthetic: per rank A = G G^T + {eps:g} I (the reference benchmark's make_spd), G ~ N(0,1), "
                 "b ~ N(0,1), seeded on the device" if "div" in wl else
                 "synthetic: per rank A = G G^T/k + eps I, G ~ N(0,1), b ~ N(0,1), seeded on the device")
        if op in ("posv", "seq3") else "synthetic: per rank A = G ~ N(0,1), b ~ N(0,1), seeded on the device",
        "config": {"workload": what, "op": op,
                   "name": args.config + (f" (batch overridden to {B})" if args.batch else ""),
                   "B_per_gpu": B, "k": k, "m": m, "parallelism": f"batch shards x{world}",
                   "l2": f"{nbuf} rotating input sets of {set_bytes / 1e6:.0f} MB (> 2 x L2 between reuses)",
                   "timing": "CUDA graph of K launches between CUDA events" if not args.no_graph
                   else "K direct launches between CUDA events",
                   "vs_baseline_ref": (f"Apple M3 Max, reference README.md:94-109 ({wl['pub_ms']} ms for B={B}, k={k})"
                                       if (op == "posv" and "pub_ms" in wl) else None)},
        "roofline": roofline(B, k, m, op, per_launch, hbm_peak, peak_src, fp32_peak, traffic,
                             kernel_name(op, k, m), args.config),
        "per_rank_ms_per_step": [t / args.steps * 1e3 for t in per_rank] if world > 1 else None,
        "gpu_launches": args.steps * (3 if op == "seq3" else 1),
        "clocks": sampler.summary(),
        "check": check,
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu:
        out["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds, op)
    print(json.dumps(out), flush=True)
    return 0


# ---------------------------------------------------------------------------
# CPU arms
# ---------------------------------------------------------------------------

def _cpu_sample(wl, n, op="posv"):
    from tests._data import general_batch, spd_batch
    if op == "trsm":
        G = general_batch(n, wl["k"], seed=99)
        L = np.tril(G) / np.float32(np.sqrt(wl["k"]))
        idx = np.arange(wl["k"])
        L[:, idx, idx] = np.abs(L[:, idx, idx]) + np.float32(1.0)
        b = np.random.default_rng(98).standard_normal((n, wl["k"], max(wl["m"], 1)), dtype=np.float32)
        return np.ascontiguousarray(L, dtype=np.float32), b
    if op in ("posv", "seq3"):
        if "div" in wl:  # the reference benchmark's A = G G^T + k I = k (G G^T / k + I)
            A, b = spd_batch(n, wl["k"], m=wl["m"], eps=1.0, seed=99)
            return A * np.float32(wl["k"]), b
        return spd_batch(n, wl["k"], m=wl["m"], eps=wl["eps"], seed=99)
    A = general_batch(n, wl["k"], seed=99)
    b = np.random.default_rng(98).standard_normal((n, wl["k"], max(wl["m"], 1)), dtype=np.float32)
    return A, b


def _ref_solver(k, op="posv"):
    """The reference's own CPU-runnable implementation of the path: its kernel
    code compiled for the host (oracle/_ref) where it exists and k is in the
    reference's GPU-kernel range, else the C restatement."""
    import oracle
    if op == "gesv":
        if oracle.ref_available() and k <= oracle.MAX_GPU_K:
            return "reference", (lambda A, b, nt: oracle.ref_lu_solve(A, b, nthreads=nt))
        return "port", (lambda A, b, nt: oracle.lu_solve(A, b, nthreads=nt))
    if op == "qr":
        if oracle.ref_available() and k <= oracle.QR_SHARED_K_MAX:
            return "reference", (lambda A, b, nt: oracle.ref_qr(A, nthreads=nt))
        return "port", (lambda A, b, nt: oracle.qr(A, nthreads=nt))
    if op == "trsm":
        if oracle.ref_available() and k <= oracle.MAX_GPU_K:
            return "reference", (lambda L, b, nt: oracle.ref_tri_solve(L, b, upper=True, nthreads=nt))
        return "port", (lambda L, b, nt: oracle.triu_solve(L, b, nthreads=nt))
    if op == "slogdet":  # the reference calls LAPACK getrf on the CPU stream: the restatement stands in
        return "port", (lambda A, b, nt: oracle.slogdet(A, nthreads=nt))
    if op == "seq3":
        if oracle.ref_available() and k <= oracle.MAX_GPU_K:
            return "reference", (lambda A, b, nt: (oracle.ref_cholesky_small(A, nthreads=nt),
                                                   oracle.ref_solve_small(A, b, nthreads=nt),
                                                   oracle.ref_cholesky_small(A, nthreads=nt)))
        return "port", (lambda A, b, nt: (oracle.cholesky(A, nthreads=nt), oracle.solve(A, b, nthreads=nt),
                                           oracle.logdet_spd(A, nthreads=nt)))
    if oracle.ref_available() and k <= oracle.MAX_GPU_K:
        # the fused kernel's x plus logdet = 2 sum log diag L from the L it writes
        # (the same outputs as one b2c_posv call)
        def ref(A, b, nt):
            x, L = oracle.ref_solve_small(A, b, nthreads=nt, return_L=True)
            return x, 2.0 * np.log(np.diagonal(L, axis1=1, axis2=2)).sum(-1)
        return "reference", ref
    return "port", (lambda A, b, nt: oracle.solve(A, b, return_logdet=True, nthreads=nt))


def _time_solver(fn, A, b, nt, seconds):
    fn(A, b, nt)
    n, t0 = 0, time.perf_counter()
    while True:
        fn(A, b, nt)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return n * A.shape[0] / el, n


def cpu_baseline(wl, seconds, op="posv"):
    import oracle
    nt = os.cpu_count() or 1
    kind, fn = _ref_solver(wl["k"], op)
    per = algo_bytes(wl["k"], wl["m"], op)
    n = int(max(64, min(wl["B"], (256 << 20) // per)))
    A, b = _cpu_sample(wl, n, op)
    value, reps = _time_solver(fn, A, b, nt, seconds)
    kname = {"posv": "fused cholesky_solve (+ logdet from its L)", "gesv": "LU solve", "qr": "Householder QR",
             "trsm": "triangular solve",
             "seq3": "cholesky, cholesky_solve and cholesky (logdet)", "slogdet": "LU slogdet"}[op]
    out = {"value": value, "unit": OP_METRICS[op][1], "cores": nt, "kind": kind,
           "sample": f"{n} matrices of the workload, {reps} passes, {seconds:.0f} s budget",
           "impl": f"reference {kname} kernel body on host threads" if kind == "reference"
           else "C restatement of the reference algorithm on host threads"}
    if op != "posv":
        return out
    try:
        lap, _ = _time_solver(lambda A_, b_, t_: oracle.lapack_posv(A_, b_, nthreads=t_), A, b, nt,
                              max(2.0, seconds / 4))
        out["lapack_spotrf_spotrs"] = {"value": lap, "unit": UNIT, "cores": nt}
    except Exception as e:  # noqa: BLE001
        out["lapack_spotrf_spotrs"] = {"error": str(e)}
    return out


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import oracle
    oracle.build() if not os.path.exists(oracle.ORC_LIB) else None
    wl = WORKLOADS[args.config]
    op = args.op
    metric, unit = OP_METRICS[op]
    nt = os.cpu_count() or 1
    kind, fn = _ref_solver(wl["k"], op)
    A1, b1 = _cpu_sample(wl, 64, op)
    fn(A1, b1, nt)
    t0 = time.perf_counter()
    fn(A1, b1, nt)
    per_matrix = max((time.perf_counter() - t0) / 64, 1e-9)
    target = min(1.0, max(0.01, 60.0 / max(1, args.steps + args.warmup)))
    n = int(max(32, min(wl["B"], target / per_matrix)))
    A, b = _cpu_sample(wl, n, op)
    for _ in range(args.warmup):
        fn(A, b, nt)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn(A, b, nt)
    el = time.perf_counter() - t0
    value = n * args.steps / el
    sample = f"{n} matrices of the workload per step (of B={wl['B']})"
    out = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": value / (wl["B"] / (wl["pub_ms"] * 1e-3)) if (op == "posv" and "pub_ms" in wl) else None,
        "dtype": "f32",
        "data": "synthetic: A = G G^T/k + eps I, G ~ N(0,1), b ~ N(0,1), numpy seed 99" if op in ("posv", "seq3")
        else "synthetic: A = G ~ N(0,1), b ~ N(0,1), numpy seed 99",
        "config": {"workload": workload_text(op, wl["B"], wl["k"], wl["m"], wl["eps"]), "op": op,
                   "name": args.config, "B_per_gpu": wl["B"], "k": wl["k"], "m": wl["m"],
                   "parallelism": "host threads", "sample": sample},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": unit, "cores": nt, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)
    return 0


def run_reference_rsvd(args, rank, world):
    """The reference algorithm on the host: the numpy restatement (the
    reference itself needs MLX), all host threads, full calls."""
    if rank != 0:
        return 0
    import oracle
    name = args.config if args.config in RSVD_WORKLOADS else "rsvd_10000x2048_k32"
    n, m, k = RSVD_WORKLOADS[name]
    X = np.random.default_rng(99).standard_normal((n, m)).astype(np.float32)
    for i in range(args.warmup):
        oracle.randomized_svd(X, k, random_state=i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        oracle.randomized_svd(X, k, random_state=i)
    el = time.perf_counter() - t0
    value = args.steps / el
    nt = os.cpu_count() or 1
    out = {"metric": f"randomized_svd calls/sec, X {n}x{m}, k={k}, n_iter=4, p=10", "value": value,
           "unit": "calls/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": RSVD_PUBLISHED_MS[name] / (el / args.steps * 1e3), "dtype": "f32",
           "data": "synthetic: X ~ N(0,1), numpy seed 99",
           "config": {"workload": f"randomized_svd of one {n}x{m} matrix, k={k}", "name": name, "op": "rsvd"},
           "impl": "reference",
           "cpu_baseline": {"value": value, "unit": "calls/s", "cores": nt, "kind": "port",
                            "sample": f"{args.steps} full calls"},
           "e2e": {"value": value, "unit": "calls/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


def run_rsvd(args, rank, world, local):
    """One step = one randomized_svd call (n_iter = 4, p = 10) on a CUDA X
    through the public API. Weak scaling: every rank factors its own X."""
    import torch
    import torch.distributed as dist
    import mlx_addons_b200.linalg as la

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    name = args.config if args.config in RSVD_WORKLOADS else "rsvd_10000x2048_k32"
    n, m, k = RSVD_WORKLOADS[name]
    gen = torch.Generator(device=dev).manual_seed(4321 + rank)
    Xs = [torch.randn((n, m), generator=gen, device=dev) for _ in range(2)]
    stream = torch.cuda.current_stream(dev)
    for i in range(max(1, args.warmup)):
        la.randomized_svd(Xs[i % 2], n_components=k, random_state=i)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    e0.record(stream)
    for i in range(args.steps):
        U, S, Vt = la.randomized_svd(Xs[i % 2], n_components=k, random_state=i)
    e1.record(stream)
    e1.synchronize()
    sampler.stop()
    elapsed = e0.elapsed_time(e1) / 1e3
    if world > 1:
        t = torch.tensor([elapsed], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    X0 = Xs[(args.steps - 1) % 2].double()
    S_ref = torch.linalg.svdvals(X0)[:k]
    check = {"max_rel_singular_value_error_vs_full_svd": float(((S.double() - S_ref).abs() / S_ref).max()),
             "finite": bool(torch.isfinite(U).all() and torch.isfinite(Vt).all())}
    e2e = None
    if not args.no_e2e:
        Xh = Xs[0].cpu().numpy()
        la.randomized_svd(Xh, n_components=k)
        n_e2e = int(max(3, min(args.steps, 10)))
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            Uh, Sh, Vth = la.randomized_svd(Xh, n_components=k)
        t_e2e = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([t_e2e], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        e2e = {"value": world * n_e2e / t_e2e, "unit": "calls/s", "steps": n_e2e,
               "h2d_bytes_per_step": int(Xh.nbytes), "d2h_bytes_per_step": int(Uh.nbytes + Sh.nbytes + Vth.nbytes),
               "api": "mlx_addons_b200.linalg.randomized_svd(numpy X) -> numpy (U, S, Vt)",
               "timing": "host clock around blocking calls, max over ranks"}
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    per = elapsed / args.steps
    flops, nbytes = rsvd_flops_bytes(n, m, k)
    hbm_peak, peak_src = load_peaks()
    out = {
        "metric": f"randomized_svd calls/sec, X {n}x{m}, k={k}, n_iter=4, p=10",
        "value": world * args.steps / elapsed, "unit": "calls/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": RSVD_PUBLISHED_MS[name] / (per * 1e3), "dtype": "f32",
        "data": "synthetic: X ~ N(0,1) seeded on the device, two inputs alternating",
        "config": {"workload": f"randomized_svd of one {n}x{m} float32 matrix per GPU, k={k}", "name": name,
                   "op": "rsvd", "l2": f"X is {4 * n * m / 1e6:.0f} MB, two alternating inputs",
                   "timing": "K API calls between CUDA events",
                   "vs_baseline_ref": "Apple M3 Max, reference _svd.py:14-17"},
        "roofline": {"bound": "hbm", "achieved": nbytes / per / 1e9, "peak": hbm_peak, "unit": "GB/s",
                     "frac": nbytes / per / 1e9 / hbm_peak, "traffic": None,
                     "peak_source": f"{peak_src} hbm_gbs (MEASURED_PEAKS.json)",
                     "bytes_per_call": nbytes, "flops_per_call": flops,
                     "kernel": "cuBLAS products with X (library); b2c_potrf / b2c_trsm in the thin QR",
                     "fp32_tflops": flops / per / 1e12},
        "gpu_launches": None,
        "clocks": sampler.summary(),
        "check": check,
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu:
        import oracle
        Xc = Xs[0].cpu().numpy()
        oracle.randomized_svd(Xc, k)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < args.cpu_seconds:
            oracle.randomized_svd(Xc, k, random_state=reps)
            reps += 1
        el = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": reps / el, "unit": "calls/s", "cores": os.cpu_count() or 1, "kind": "port",
                               "sample": f"{reps} full calls on the same {n}x{m} X",
                               "impl": "numpy restatement of the reference algorithm (LAPACK QR / SVD, "
                                       "OpenBLAS GEMM on all host threads)"}
    print(json.dumps(out), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["b2c", "reference"], default="b2c")
    ap.add_argument("--config", choices=list(WORKLOADS) + list(RSVD_WORKLOADS), default="c2_k64")
    ap.add_argument("--op", choices=list(OP_METRICS) + ["rsvd"], default="posv",
                    help="posv: the fused SPD solve (the headline); seq3: cholesky + solve + logdet_spd as "
                         "three calls; slogdet; gesv: solve_lu; qr: qr; rsvd: randomized_svd (configs rsvd_*)")
    ap.add_argument("--no-graph", action="store_true", help="direct launches instead of one CUDA graph")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--batch", type=int, default=0,
                    help="override B per GPU (small cases for profiler captures; not a bench line)")
    ap.add_argument("--k", type=int, default=0,
                    help="override k (profiler captures of other tiers; not a bench line)")
    ap.add_argument("--m", type=int, default=0,
                    help="override the right-hand sides per matrix (tier sweeps; not a bench line)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.steps < 1 or args.warmup < 0:
        ap.error("--steps >= 1 and --warmup >= 0")
    if args.op == "rsvd":
        if args.impl == "reference":
            return run_reference_rsvd(args, rank, world)
        return run_rsvd(args, rank, world, local)
    if args.config not in WORKLOADS:
        ap.error(f"--config {args.config} is a randomized_svd workload (use --op rsvd)")
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_b2c(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
