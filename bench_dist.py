"""bench.py's multi-GPU leg (one process per GPU under torchrun).

Headline workload (config C3): FP64 -> INT8, num_splits = 4, M = N = K = 8192.
Default layout (``--dist sharded``): A sharded by row blocks and B by column
panels; every rank splits its own rows and panel and the panels' int8 slices
are all-gathered over NCCL (``dist.ozaki_matmul_sharded``).  ``--dist root``:
B lives on rank 0, which splits it in column blocks and broadcasts each
block's slices (``dist.ozaki_matmul_mrows``).  Total work is fixed: strong
scaling.  The step time is the max over ranks of
each rank's CUDA-event time, with a barrier and a device synchronise on both
sides of the timed region.
"""

from __future__ import annotations

import json
import os
import statistics
from datetime import timedelta

import torch
import torch.distributed as dist

from ozaki_triton_b200 import dist as ozd


def main(args):
    import bench  # workload recipe, clock sampler, peaks

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    M, N, K, S = bench.M, bench.N, bench.K, bench.NUM_SPLITS
    sharded = args.dist == "sharded"
    if sharded:
        rows = [b - a for a, b in (ozd.block_range(M, world, r) for r in range(world))]
        p0, p1 = ozd.column_panel(N, world, rank)
    else:
        # rank 0 also splits and broadcasts B: it takes fewer rows of A (about
        # the rows its B split is worth at this problem's per-row GEMM rate)
        rows = ozd.weighted_rows(M, world, root=0, root_discount=int(args.root_discount))
        p0, p1 = (0, N) if rank == 0 else (0, 0)
    lo = sum(rows[:rank])
    hi = lo + rows[rank]
    a_h, b_h = bench.make_inputs()
    a_loc = a_h[lo:hi].contiguous().to(dev)
    b = b_h[:, p0:p1].contiguous().to(dev) if (sharded or rank == 0) else None
    stream = torch.cuda.current_stream()
    gemm_ms = []

    class TimedBackend(ozd.Backend):
        """Records an event before the first GEMM launch of a step."""
        record = False
        first = None

        def gemm(self, *a, **kw):
            if self.record and self.first is None:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record(kw.get("stream") or torch.cuda.current_stream())
                self.first = e0
            return super().gemm(*a, **kw)

    be = TimedBackend()

    # root mode: B travels in column blocks (split of block c+1 overlaps the
    # broadcast of block c); one GEMM over all of N once B is complete
    b_blocks = args.chunks or None

    def run(a_dev, b_dev):
        if sharded:
            return ozd.ozaki_matmul_sharded(a_dev, b_dev, S, torch.int8, n=N, backend=be,
                                            transport=args.transport)
        return ozd.ozaki_matmul_mrows(a_dev, b_dev, S, torch.int8, backend=be, b_blocks=b_blocks)

    def step():
        c = run(a_loc, b)
        if be.record and be.first is not None:
            # the GEMM phase of a step: its first GEMM launch to the join of
            # every GEMM stream (the block GEMMs of the p2p transport overlap)
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(stream)
            gemm_ms.append((be.first, e1))
            be.first = None
        return c

    for _ in range(args.warmup):
        step()
    be.record = True
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with bench.ClockSampler(local) as clk:
        dist.barrier()
        torch.cuda.synchronize()
        launches0 = ozd._lib.load().oz_launch_count()
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        launches = ozd._lib.load().oz_launch_count() - launches0
        torch.cuda.synchronize()
        dist.barrier()
    ms_local = t0.elapsed_time(t1) / args.steps
    t = torch.tensor([ms_local], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    spans = [e0.elapsed_time(e1) for e0, e1 in gemm_ms]
    g_local = statistics.mean(spans)

    # end to end through the public sharded call with host operands: each
    # rank copies its A rows (rank 0 also B) in and its C rows out
    e2e = None
    if not args.no_e2e:
        a_pin = a_h[lo:hi].contiguous().pin_memory()
        b_pin = b_h[:, p0:p1].contiguous().pin_memory() if (sharded or rank == 0) else None
        c_pin = torch.empty((hi - lo, N), dtype=torch.float64).pin_memory()
        be.record = False

        def e2e_step():
            ad = a_pin.to(dev, non_blocking=True)
            bd = b_pin.to(dev, non_blocking=True) if b_pin is not None else None
            cd = run(ad, bd)
            c_pin.copy_(cd, non_blocking=True)

        for _ in range(2):
            e2e_step()
        dist.barrier()
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        n_e2e = max(2, min(args.steps, 5))
        s0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        te = torch.tensor([s0.elapsed_time(s1) / n_e2e], dtype=torch.float64, device=dev)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item())
        h2d = (hi - lo) * K * 8 + K * (p1 - p0) * 8
        e2e = {"value": 2.0 * M * N * K / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": M * K * 8 + K * N * 8,
               "d2h_bytes_per_step": M * N * 8, "h2d_bytes_rank": h2d}

    if rank == 0:
        flops = 2.0 * M * N * K
        bf16_peak, _, peak_src = bench.peaks()
        achieved = S * S * 2.0 * (hi - lo) * N * K / (g_local * 1e-3) / 1e12
        line = {
            "metric": bench.METRIC, "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": bench.WORKLOAD, "M": M, "N": N, "K": K, "num_splits": S,
                       "slice_dtype": "int8", "input_dtype": "fp64", "residual": "compat",
                       "l2": "no flush: operands larger than the 126 MB L2",
                       "parallelism": (f"A rows x B column panels over {world} GPUs, B "
                                       + ("slices pulled block by block over NVLink by copy "
                                          "engines, each block's GEMM started on arrival"
                                          if args.transport == "p2p" else
                                          "slices all-gathered over NCCL") if sharded else
                                       f"M-row sharding over {world} GPUs, B slices broadcast "
                                       "from rank 0 over NCCL in column blocks"),
                       "rows_per_rank": rows,
                       "b_panel_cols": ozd.block_width(N, world) if sharded else None,
                       "transport": (args.transport + (" (" + ozd.p2p_status() + ")"
                                                       if args.transport == "p2p" else ""))
                       if sharded else "broadcast",
                       "b_blocks": None if sharded else (b_blocks or "auto")},
            "roofline": {"bound": "tensor",
                         "kernel": "cross_gemm_kernel (rank 0 rows; span of the step's GEMMs)",
                         "achieved": achieved, "peak": 2.0 * bf16_peak, "unit": "TFLOP/s",
                         "frac": achieved / (2.0 * bf16_peak),
                         "peak_source": f"2x {peak_src} dense bf16; B200 dense int8 = 2x bf16",
                         "gemm_ms": g_local, "traffic": None},
            "clocks": clk.summary(),
            # rank 0's own kernels per step: transpose + split of B's panel (or
            # blocks), split of A's rows, the GEMM (NCCL kernels not counted)
            "gpu_launches": launches,     # rank 0's library kernels in the timed region
            "e2e": e2e,
        }
        print(json.dumps(line), flush=True)
    ozd.release_peer_buffers()
    dist.barrier()
    dist.destroy_process_group()
