"""Benchmark of the Ozaki-scheme GEMM path on B200 (one JSON line on rank 0).

Workload (BASELINE.json headline, config "C3"): FP64 -> INT8 slices,
num_splits = 4, one GEMM with M = N = K = 8192, entries
x = (U(0,1) - 0.5) * exp(N(0,1)) from seed 2 (synthetic, generated on the
host).  One step = one public ``ozaki_matmul`` call: split of B by columns,
split of A by rows, fused cross-GEMM over the 16 slice pairs with the FP64
epilogue (``--config`` picks the other BASELINE.json configurations).

* ``value``: emulated TFLOPS = 2*M*N*K / step time, inputs resident in HBM
  (A and B are 512 MiB each, larger than L2, so no flush is needed).
* ``e2e``: the same metric through ``ozaki_matmul_from_host`` with the
  operands in pinned host memory: host->device copies of A and B and the
  device->host copy of C are inside the timed region.
* ``roofline``: the cross-GEMM kernel (CUDA events around its launch inside
  the timed steps, ``oz_profile_next_gemm``), int8 tensor ops (pairs * 2MNK)
  per launch over its duration, against the larger of 2x the measured dense
  bf16 peak and the int8 rate cuBLAS reaches on this GPU (``torch._int_mm``
  at 8192^3, measured in the same run).
* comparators in the same run: cuBLAS DGEMM / SGEMM of the input dtype, CPU
  ``torch.matmul`` in the input dtype on all host cores, and
  ``cpu_baseline`` = the CPU restatement of the reference (oracle/) on a
  bounded sample of the same workload.

Multi-GPU (torchrun, N > 1): ``bench_dist.py``.  By default A is sharded by
rows and B by column panels; every rank splits its own panel and the panels'
int8 slices are pulled from the peers over NVLink by copy engines
(``--transport p2p``), each block's GEMM starting on arrival.  The same run
also times the NCCL-broadcast layout (B on rank 0) and the gather of C to
rank 0, and checks a sample of C bit for bit against the oracle.  Total work
is fixed, so scaling is "strong".  ``--impl reference`` times the reference
algorithm's CPU restatement on the host cores (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = N = K = 8192
NUM_SPLITS = 4
WORKLOAD = ("C3: FP64->INT8 Ozaki num_splits=4, single GEMM M=N=K=8192, "
            "x=(U(0,1)-0.5)*exp(N(0,1)) seed 2")
METRIC = "emulated TFLOPS (2MNK/t), FP64->INT8 s=4 8192^3"


def make_inputs(seed: int = 2, m: int = M, n: int = N, k: int = K):
    """Host fp64 operands of the headline law; draw order A's U, A's N, B's U, B's N."""
    g = torch.Generator().manual_seed(seed)
    ua = torch.rand(m, k, generator=g, dtype=torch.float64)
    na = torch.randn(m, k, generator=g, dtype=torch.float64)
    ub = torch.rand(k, n, generator=g, dtype=torch.float64)
    nb = torch.randn(k, n, generator=g, dtype=torch.float64)
    return (ua - 0.5) * torch.exp(na), (ub - 0.5) * torch.exp(nb)


class ClockSampler:
    """SM clock / clock-event-reason sampling during the timed region.

    NVML (read-only queries) polled every 5 ms from a thread; nvidia-smi
    -lms 50 where NVML cannot be loaded.  The GPU is found by its PCI bus id,
    so CUDA_VISIBLE_DEVICES remapping does not matter.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.005

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.nvml = None
        self.samples = []            # (sm MHz, max MHz, reasons bitmask)
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            p = torch.cuda.get_device_properties(self.index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:  # noqa: BLE001 - fall back to the index
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        return pynvml, h

    def _poll(self):
        pv, h = self.nvml
        reasons = getattr(pv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pv.nvmlDeviceGetCurrentClocksThrottleReasons
        mx = pv.nvmlDeviceGetMaxClockInfo(h, pv.NVML_CLOCK_SM)
        while not self.stop.is_set():
            try:
                self.samples.append((pv.nvmlDeviceGetClockInfo(h, pv.NVML_CLOCK_SM), mx,
                                     int(reasons(h))))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.PERIOD_S)

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 5:
                time.sleep(0.001)
            self.samples.clear()
            return self
        except Exception:  # noqa: BLE001 - no NVML: nvidia-smi
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # the sampler is up (first sample read) before the timed region starts
            t0 = time.time()
            while not self.lines and time.time() - t0 < 10:
                time.sleep(0.01)
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.nvml is not None:
            self.stop.set()
            self.thread.join(timeout=2)
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        if self.nvml is not None:
            pv = self.nvml[0]
            bits = [pv.nvmlClocksThrottleReasonHwSlowdown,
                    pv.nvmlClocksThrottleReasonHwThermalSlowdown,
                    pv.nvmlClocksThrottleReasonSwThermalSlowdown,
                    pv.nvmlClocksThrottleReasonSwPowerCap]
            for mhz, mxx, r in self.samples:
                sm.append(float(mhz))
                mx = float(mxx)
                for nm, bit in zip(names, bits):
                    if r & bit:
                        reasons.add(nm)
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml"}
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def committed_traffic():
    """dram bytes per cross-GEMM launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as fh:
            return json.load(fh)
    return None


def cpu_baseline_sample(seconds_budget: float = 20.0):
    """The oracle (CPU restatement of the reference) on row/column samples."""
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ms = ns = 256
    a, b = make_inputs(seed=2, m=ms, n=ns, k=K)
    a, b = a.numpy(), b.numpy()
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        oracle.ozaki_matmul(a, b, NUM_SPLITS, "int8", "fp64")
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > seconds_budget or len(times) >= 5:
            break
    t = statistics.median(times)
    return {"value": 2.0 * ms * ns * K / t / 1e12, "unit": "TFLOPS", "cores": threads,
            "kind": "port",
            "sample": f"{ms}x{ns} block of C with full K={K} (A rows x B columns of the "
                      f"workload law), numpy oracle, median of {len(times)}"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ms = ns = 256
    a, b = make_inputs(seed=2, m=ms, n=ns, k=K)
    a, b = a.numpy(), b.numpy()
    for _ in range(args.warmup):
        oracle.ozaki_matmul(a, b, NUM_SPLITS, "int8", "fp64")
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.ozaki_matmul(a, b, NUM_SPLITS, "int8", "fp64")
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = 2.0 * ms * ns * K / dt / 1e12
    line = {"metric": METRIC, "value": v, "unit": "TFLOPS", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample": f"{ms}x{ns}x{K} per step"},
            "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": threads, "kind": "port",
                             "sample": f"{ms}x{ns} block of C, full K={K}, per step"},
            "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "the reference is Python/Triton and cannot run on the GPU box; this arm "
                    "times its CPU restatement (oracle/) with all host threads"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-dgemm", action="store_true")
    ap.add_argument("--root-discount", type=int, default=768,
                    help="multi-GPU root mode: rows of A moved off rank 0, which also splits B")
    ap.add_argument("--chunks", type=int, default=0,
                    help="multi-GPU root mode: column blocks B is split and broadcast in "
                         "(0 = auto)")
    ap.add_argument("--transport", default="p2p", choices=["p2p", "collective"],
                    help="multi-GPU sharded mode: how B's slices travel (copy-engine pulls "
                         "from mapped peer buffers, or one NCCL all-gather)")
    ap.add_argument("--dist", default="sharded", choices=["sharded", "root"],
                    help="multi-GPU data layout: A rows x B column panels with an all-gather "
                         "of B's slices (sharded), or B on rank 0 broadcast (root)")
    ap.add_argument("--alt-steps", type=int, default=5,
                    help="multi-GPU: timed steps of the other layout and of the gather of C "
                         "to rank 0 (0 = skip)")
    ap.add_argument("--config", default="C3", choices=sorted(CONFIGS),
                    help="benchmark configuration (C3 = the headline)")
    ap.add_argument("--num-splits", type=int, default=0, help="override the config's s")
    ap.add_argument("--graph", action="store_true",
                    help="1 GPU: time CUDA-graph replays of the step (launch-bound small configs)")
    ap.add_argument("--profile", action="store_true",
                    help="timed steps only (no e2e, DGEMM or CPU legs): the ncu command line")
    ap.add_argument("--emulate-rank", type=int, default=0, metavar="N",
                    help="1 GPU, diagnostic: one rank's GEMM phase of the N-GPU C3 p2p layout "
                         "with every column block present, per-block launches against the "
                         "one-launch peer GEMM")
    args = ap.parse_args()
    if args.emulate_rank:
        import bench_dist
        bench_dist.emulate_rank(args)
        return
    if args.profile:
        args.no_e2e = args.no_cpu_baseline = args.no_dgemm = True
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.gpus > 1:
        import bench_dist
        bench_dist.main(args)
        return
    run_single(args)


# the benchmark configurations of BASELINE.json (C3 is the headline)
CONFIGS = {
    "C1": dict(a=(256, 256), b=(256, 256), dtype=torch.float32, slice=torch.float16, s=2,
               law="uniform", seed=0,
               desc="FP32->FP16 Ozaki s=2, 256^3, U(-1,1) seed 0"),
    "C2": dict(a=(8192, 8192), b=(8192, 8192), dtype=torch.float32, slice=torch.float16, s=2,
               law="normal", seed=1, desc="FP32->FP16 Ozaki s=2, 8192^3, N(0,1) seed 1"),
    "C3": dict(a=(8192, 8192), b=(8192, 8192), dtype=torch.float64, slice=torch.int8, s=4,
               law=1.0, seed=2, desc=WORKLOAD),
    "C4": dict(a=(16, 1, 2048, 4096), b=(1, 8, 4096, 2048), dtype=torch.float64,
               slice=torch.float16, s=3, law="normal", seed=3,
               desc="FP64->FP16 Ozaki s=3, (16,1,2048,4096)x(1,8,4096,2048) -> 128 GEMMs, "
                    "N(0,1) seed 3"),
    "C5": dict(a=(16384, 16384), b=(16384, 16384), dtype=torch.float64, slice=torch.int8, s=4,
               law=4.0, seed=4,
               desc="FP64->INT8 Ozaki s=4, 16384^3, x=(U(0,1)-0.5)*exp(4 N(0,1)) seed 4"),
}
SLICE_NAME = {torch.int8: "int8", torch.float16: "fp16", torch.bfloat16: "bf16",
              torch.float32: "fp32"}
DTYPE_NAME = {torch.float64: "fp64", torch.float32: "fp32", torch.float16: "fp16",
              torch.bfloat16: "bf16"}


def config_inputs(cfg):
    """Host operands of a configuration from its seeded CPU generator."""
    g = torch.Generator().manual_seed(cfg["seed"])
    law = cfg["law"]
    if law == "uniform":
        a = torch.rand(cfg["a"], generator=g, dtype=torch.float64) * 2 - 1
        b = torch.rand(cfg["b"], generator=g, dtype=torch.float64) * 2 - 1
    elif law == "normal":
        a = torch.randn(cfg["a"], generator=g, dtype=torch.float64)
        b = torch.randn(cfg["b"], generator=g, dtype=torch.float64)
    else:   # (U(0,1) - 0.5) * exp(sigma N(0,1)); draw order A's U, A's N, B's U, B's N
        ua = torch.rand(cfg["a"], generator=g, dtype=torch.float64)
        na = torch.randn(cfg["a"], generator=g, dtype=torch.float64)
        ub = torch.rand(cfg["b"], generator=g, dtype=torch.float64)
        nb = torch.randn(cfg["b"], generator=g, dtype=torch.float64)
        a, b = (ua - 0.5) * torch.exp(law * na), (ub - 0.5) * torch.exp(law * nb)
    return a.to(cfg["dtype"]), b.to(cfg["dtype"])


def int8_tensor_rate(dev, n: int = 8192, reps: int = 10) -> float:
    """Dense int8 tensor rate cuBLAS reaches on this GPU (TOPS): torch._int_mm
    at n^3 (int8 x int8 -> int32), best of ``reps`` launches timed with CUDA
    events."""
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
    bt = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
    b = bt.t()                      # column-major B: the layout cuBLASLt takes natively
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    st = torch.cuda.current_stream(dev)
    for _ in range(reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        torch._int_mm(a, b)
        e1.record(st)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def cpu_native_matmul(a_h: torch.Tensor, b_h: torch.Tensor, budget_flops: float = 2.3e12):
    """CPU torch.matmul in the input dtype on all host cores: the whole
    product when it is at most ``budget_flops``, else a block of A's rows
    (full K and N) scaled to that budget."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    m, k = a_h.shape[-2:]
    n = b_h.shape[-1]
    bn = a_h.numel() // (m * k) if a_h.dim() > 2 else 1
    bn = max(bn, b_h.numel() // (k * n) if b_h.dim() > 2 else 1)
    full = 2.0 * bn * m * n * k
    if full <= budget_flops:
        a_s, b_s, sample = a_h, b_h, "the whole product"
        flops = full
    else:
        a2 = a_h.reshape(-1, m, k)[0]
        b2 = b_h.reshape(-1, k, n)[0]
        rows = max(64, int(m * budget_flops / (2.0 * m * n * k)))
        a_s, b_s = a2[:rows].contiguous(), b2
        flops = 2.0 * rows * n * k
        sample = f"{rows} rows of A (x full B) of one batch member"
    torch.matmul(a_s[..., :64, :], b_s)              # warm-up (threads, kernels)
    t0 = time.perf_counter()
    torch.matmul(a_s, b_s)
    dt = time.perf_counter() - t0
    return {"value": flops / dt / 1e12, "unit": "TFLOPS", "cores": threads,
            "dtype": str(a_h.dtype).replace("torch.", ""), "sample": sample,
            "seconds": dt}


def run_single(args):
    import math

    import ozaki_triton_b200 as oz
    from ozaki_triton_b200 import _lib

    name = args.config
    cfg = CONFIGS[name]
    s = args.num_splits or cfg["s"]
    sd, dt = cfg["slice"], cfg["dtype"]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    a_h, b_h = config_inputs(cfg)
    a = a_h.to(dev)
    b = b_h.to(dev)
    stream = torch.cuda.current_stream()
    Mm, Kk = a.shape[-2:]
    Nn = b.shape[-1]
    a_batch, b_batch = tuple(a.shape[:-2]), tuple(b.shape[:-2])
    full = tuple(torch.broadcast_shapes(a_batch, b_batch))
    BN = math.prod(full)
    BA, BB = math.prod(a_batch), math.prod(b_batch)
    residual = _lib.OZ_RESIDUAL_COMPAT if s <= 4 else _lib.OZ_RESIDUAL_EXACT
    lib = _lib.load()
    gemm_events = []
    # CUDA events for the GEMM launches of the timed steps, created up front
    # (torch creates the underlying event at its first record)
    ev_pool = []
    for _ in range(args.steps + 4):
        pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        for e in pair:
            e.record(stream)
        ev_pool.append(pair)
    torch.cuda.synchronize()

    def step(record: bool):
        """One public ozaki_matmul call; with ``record`` its cross-GEMM launch
        is bracketed by a pair of CUDA events (oz_profile_next_gemm)."""
        if record:
            e0, e1 = ev_pool[len(gemm_events)]
            lib.oz_profile_next_gemm(e0.cuda_event, e1.cuda_event)
            gemm_events.append((e0, e1))
        return oz.ozaki_matmul(a, b, num_splits=s, slice_dtype=sd)

    for _ in range(args.warmup):
        step(False)
    # the GEMM's CUDA events are recorded inside the timed region, except for
    # products short enough that the host's launch work sets the step time
    # (there the hook's own host work would be timed too): those take the
    # GEMM events from as many steps right after the timed region
    torch.cuda.synchronize()
    p0 = time.perf_counter()
    step(False)
    torch.cuda.synchronize()
    gemm_in_timed = (time.perf_counter() - p0) > 1e-3

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    graph = None
    if args.graph:
        # the whole step (both splits and the GEMM) captured once and replayed:
        # no host launch work per step (the GEMM time for the roofline comes
        # from event-timed steps outside the graph)
        for _ in range(3):
            step(True)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        n0 = _lib.load().oz_launch_count()
        with torch.cuda.graph(graph):
            step(False)
        graph_launches = _lib.load().oz_launch_count() - n0
        torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        launches0 = _lib.load().oz_launch_count()
        start.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(gemm_in_timed)
        end.record(stream)
        torch.cuda.synchronize()
        # the library's own kernels in the timed region (counted at launch;
        # a replayed graph launches the kernels it captured)
        launches = (_lib.load().oz_launch_count() - launches0 if graph is None
                    else graph_launches * args.steps)
    ms = start.elapsed_time(end) / args.steps
    if not gemm_events:
        for _ in range(args.steps):
            step(True)
        torch.cuda.synchronize()
    gemm_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in gemm_events)
    flops = 2.0 * BN * Mm * Nn * Kk
    value = flops / (ms * 1e-3) / 1e12
    pairs = s * s
    bf16_peak, hbm_peak, peak_src = peaks()
    # the tensor peak of the slice dtype: B200's dense int8 rate is twice its
    # bf16 rate, tf32 half; for int8 the rate cuBLAS reaches here is measured
    # too and the larger of the two is the denominator
    tensor_peak = 2.0 * bf16_peak if sd == torch.int8 else (bf16_peak if sd != torch.float32
                                                            else bf16_peak / 2.0)
    peak_note = {torch.int8: "2x", torch.float16: "1x", torch.bfloat16: "1x",
                 torch.float32: "0.5x"}[sd]
    int8_cublas = None
    if sd == torch.int8 and not args.no_dgemm:
        int8_cublas = int8_tensor_rate(dev)
        tensor_peak = max(tensor_peak, int8_cublas)
    achieved = pairs * flops / (gemm_ms * 1e-3) / 1e12

    # accuracy against an fp64 matmul, and the native GEMM of the input dtype
    rel_err = native_tflops = None
    if not args.no_dgemm:
        ref = torch.matmul(a.double(), b.double())
        c = step(False).reshape(ref.shape).double()
        rel_err = ((c - ref).norm() / ref.norm()).item()
        del ref, c
        torch.backends.cuda.matmul.allow_tf32 = False
        for _ in range(2):
            torch.matmul(a, b)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(3):
            torch.matmul(a, b)
        t1.record(stream)
        torch.cuda.synchronize()
        native_tflops = flops / (t0.elapsed_time(t1) / 3 * 1e-3) / 1e12

    # end to end through the public call with host operands
    e2e = None
    if not args.no_e2e:
        a_pin = a_h.pin_memory()
        b_pin = b_h.pin_memory()
        c_pin = torch.empty((*full, Mm, Nn), dtype=dt).pin_memory()

        def e2e_step():
            # the public host-operand call: copies pipelined with the splits/GEMMs
            oz.ozaki_matmul_from_host(a_pin, b_pin, num_splits=s, slice_dtype=sd, out=c_pin)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        e2e_steps = max(2, min(args.steps, 5))
        s0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = s0.elapsed_time(s1) / e2e_steps
        e2e = {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": a_h.numel() * a_h.element_size() +
               b_h.numel() * b_h.element_size(),
               "d2h_bytes_per_step": c_pin.numel() * c_pin.element_size()}

    traffic = committed_traffic() if name == "C3" and s == 4 else None
    clocks = clk.summary()
    cpu_native = None
    if not args.no_cpu_baseline:
        cpu_native = cpu_native_matmul(a_h, b_h)
    line = {
        "metric": METRIC if name == "C3" else f"emulated TFLOPS (2MNK/t), {cfg['desc']}",
        "value": value, "unit": "TFLOPS", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": SLICE_NAME[sd], "data": "synthetic",
        "config": {"workload": cfg["desc"], "name": name, "A": list(a.shape), "B": list(b.shape),
                   "num_splits": s, "slice_dtype": SLICE_NAME[sd],
                   "input_dtype": DTYPE_NAME[dt],
                   "residual": "compat" if residual == _lib.OZ_RESIDUAL_COMPAT else "exact",
                   "l2": "no flush: operands larger than the 126 MB L2" if a.numel() * a.element_size() > 126e6
                   else "operands smaller than L2 (small config)",
                   "parallelism": "1 GPU",
                   "launch": "CUDA graph replay" if graph is not None else "eager"},
        "roofline": {"bound": "tensor", "kernel": f"cross_gemm_kernel<{SLICE_NAME[sd]}>",
                     "achieved": achieved, "peak": tensor_peak, "unit": "TFLOP/s",
                     "frac": achieved / tensor_peak,
                     "peak_source": f"max of {peak_note} {peak_src} dense bf16 ({bf16_peak} TF/s, "
                                    "MEASURED_PEAKS.json; B200 dense int8 = 2x bf16, "
                                    "tf32 = 0.5x) and the int8 cuBLAS rate measured in this run",
                     "frac_of_2x_bf16": (achieved / (2.0 * bf16_peak)
                                         if sd == torch.int8 else None),
                     "int8_cublas_tops": int8_cublas,
                     "frac_of_int8_cublas": achieved / int8_cublas if int8_cublas else None,
                     "gemm_ms": gemm_ms,
                     "gemm_events": ("timed region" if gemm_in_timed and graph is None else
                                     f"{args.steps} steps after the timed region (launch-bound "
                                     "product or graph replay)"),
                     # the GEMM runs at the power cap: its time scaled to the
                     # maximum SM clock by the median clock sampled meanwhile
                     "gemm_ms_at_max_clock": (gemm_ms * clocks["sm_mhz"] / clocks["sm_max_mhz"]
                                              if clocks.get("sm_mhz") and clocks.get("sm_max_mhz")
                                              else None),
                     "traffic": traffic.get("cross_gemm_bytes_per_launch") if traffic else None},
        "rel_err_vs_fp64": rel_err,
        "native_gemm_tflops": native_tflops,
        "native_gemm": "cuBLAS DGEMM" if dt == torch.float64 else "cuBLAS SGEMM (no TF32)",
        "cpu_native_matmul": cpu_native,
        "reference_triton_b200": ("unavailable: the reference has no setup.py or "
                                  "pyproject.toml, so it cannot be installed for the GPU box, "
                                  "and its sources are not copied into this repository"),
        "clocks": clocks,
        "gpu_launches": launches,
        "e2e": e2e,
    }
    if not args.no_cpu_baseline and name == "C3":
        line["cpu_baseline"] = cpu_baseline_sample()
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
