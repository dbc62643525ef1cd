"""bench.py's multi-GPU leg (one process per GPU under torchrun).

Configurations (``--config``):

* C3 (default) and C5, one large GEMM.  Default layout (``--dist sharded``):
  A sharded by row blocks and B by column panels; every rank splits its own
  rows and panel, and the panels' int8 slices reach every rank
  (``dist.ozaki_matmul_sharded``: copy-engine pulls over NVLink with
  ``--transport p2p``, or one NCCL all-gather with ``collective``).
  ``--dist root``: B lives on rank 0, which splits it in column blocks and
  broadcasts each block's slices over NCCL (``dist.ozaki_matmul_mrows``).
  The same run also times the other layout and the gather of C's row blocks
  to rank 0 (``gather_to=0``), each for ``--alt-steps`` steps.
* C4, the broadcast batched product: contiguous ranges of the 128 output
  batches per rank (``dist.ozaki_matmul_batches``), no exchange at all.

Total work is fixed: strong scaling.  The step time is the max over ranks of
each rank's CUDA-event time, with a barrier and a device synchronise on both
sides of the timed region.  After the timed steps the run checks itself: a
sample of C's rows and columns, gathered from the ranks that own them, is
compared bit for bit (int8 slices) or within 1e-6 (float slices) with the
CPU oracle restatement of the reference on the same rows and columns; the
line carries ``parity_checked`` and the sample's relative error against an
fp64 product.
"""

from __future__ import annotations

import json
import math
import os
import statistics
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

from ozaki_triton_b200 import dist as ozd

SAMPLE = 24          # rows and columns of C checked against the oracle


def _sample_lines(total: int, k: int = SAMPLE) -> np.ndarray:
    """Fixed sample of line indices: both ends, the block boundaries of
    every 128 rows near the ends, and an even spread in between."""
    pick = {0, 1, 127, 128, total // 2, total - 2, total - 1}
    pick.update(np.linspace(0, total - 1, k - len(pick)).astype(int).tolist())
    out = sorted(x for x in pick if 0 <= x < total)
    return np.array(out[:k], dtype=np.int64)


def _timed(fn, steps: int, stream, sync_ranks=True):
    """Per-rank CUDA-event time of ``steps`` calls of fn, max over ranks (ms)."""
    if sync_ranks:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        fn()
    t1.record(stream)
    torch.cuda.synchronize()
    if sync_ranks:
        dist.barrier()
    t = torch.tensor([t0.elapsed_time(t1) / max(steps, 1)], dtype=torch.float64,
                     device=torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _check_rows_sample(c_local, lo, hi, rows, cols, a_h, b_h, s, slice_kind, dev):
    """Rank 0: the sampled entries of C, gathered from their owners, against
    the oracle (bit for bit for int8 slices) and an fp64 product."""
    import oracle

    ns, nc = len(rows), len(cols)
    mine = torch.zeros((ns, nc), dtype=torch.float64, device=dev)
    own = torch.zeros((ns,), dtype=torch.int32, device=dev)
    for i, r in enumerate(rows):
        if lo <= r < hi:
            mine[i] = c_local[r - lo][torch.as_tensor(cols, device=dev)].double()
            own[i] = 1
    world = dist.get_world_size()
    all_vals = [torch.zeros_like(mine) for _ in range(world)]
    all_own = [torch.zeros_like(own) for _ in range(world)]
    dist.all_gather(all_vals, mine)
    dist.all_gather(all_own, own)
    if dist.get_rank() != 0:
        return None
    got = np.zeros((ns, nc))
    owners = np.zeros(ns, dtype=int)
    for v, o in zip(all_vals, all_own):
        o = o.cpu().numpy().astype(bool)
        got[o] = v.cpu().numpy()[o]
        owners += o
    a_s = a_h[rows].numpy()
    b_s = b_h[:, cols].numpy()
    want = oracle.ozaki_matmul(a_s, b_s, s, slice_kind, "fp64")
    exact = a_s @ b_s
    rel = float(np.linalg.norm(got - exact) / np.linalg.norm(exact))
    if slice_kind == "int8":
        ok = bool((owners == 1).all() and np.array_equal(got.view(np.uint64),
                                                         want.view(np.uint64)))
        diff = float(np.abs(got - want).max())
    else:
        diff = float(np.linalg.norm(got - want) / np.linalg.norm(want))
        ok = bool((owners == 1).all() and diff < 1e-6)
    return {"parity_checked": ok, "sample": f"{ns} rows x {nc} columns of C",
            "vs_oracle": "bit-exact" if slice_kind == "int8" else "rel diff < 1e-6",
            "max_diff_vs_oracle": diff, "rel_err_vs_fp64_sample": rel}


def _gemm_config(name):
    import bench

    cfg = bench.CONFIGS[name]
    return cfg


def main(args):
    import bench  # workload recipe, clock sampler, peaks

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        if args.config == "C4":
            line = run_batches(args, rank, world, dev)
        else:
            line = run_rows(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        ozd.release_peer_buffers()
        dist.barrier()
        dist.destroy_process_group()


def run_rows(args, rank, world, dev):
    """C3 / C5: one GEMM, A by rows; B by column panels (sharded) or on rank 0."""
    import bench

    cfg = bench.CONFIGS[args.config]
    assert len(cfg["a"]) == 2, "row sharding takes a single GEMM"
    S = args.num_splits or cfg["s"]
    sd = cfg["slice"]
    slice_kind = bench.SLICE_NAME[sd]
    a_h, b_h = bench.config_inputs(cfg)
    M, K = a_h.shape
    N = b_h.shape[1]
    stream = torch.cuda.current_stream()

    def layout(kind):
        if kind == "sharded":
            rows = [b - a for a, b in (ozd.block_range(M, world, r) for r in range(world))]
            p0, p1 = ozd.column_panel(N, world, rank)
        else:
            # rank 0 also splits and broadcasts B: it takes fewer rows of A
            rows = ozd.weighted_rows(M, world, root=0, root_discount=int(args.root_discount))
            p0, p1 = (0, N) if rank == 0 else (0, 0)
        lo = sum(rows[:rank])
        return rows, lo, lo + rows[rank], p0, p1

    gemm_spans = []

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

    def make_step(kind, transport, gather):
        rows, lo, hi, p0, p1 = layout(kind)
        a_loc = a_h[lo:hi].contiguous().to(dev)
        b_loc = (b_h[:, p0:p1].contiguous().to(dev)
                 if (kind == "sharded" or rank == 0) else None)

        def step():
            if kind == "sharded":
                c = ozd.ozaki_matmul_sharded(a_loc, b_loc, S, sd, n=N, backend=be,
                                             transport=transport,
                                             gather_to=0 if gather else None)
            else:
                c = ozd.ozaki_matmul_mrows(a_loc, b_loc, S, sd, backend=be,
                                           b_blocks=args.chunks or None,
                                           gather_to=0 if gather else None)
            if be.record and be.first is not None:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record(stream)
                gemm_spans.append((be.first, e1))
                be.first = None
            return c
        return step, (rows, lo, hi, p0, p1), a_loc, b_loc

    main_kind = args.dist
    step, (rows, lo, hi, p0, p1), a_loc, b_loc = make_step(main_kind, args.transport, False)
    for _ in range(args.warmup):
        step()
    be.record = True
    with bench.ClockSampler(local_index(dev)) as clk:
        launches0 = ozd._lib.load().oz_launch_count()
        ms = _timed(step, args.steps, stream)
        launches = ozd._lib.load().oz_launch_count() - launches0
    be.record = False
    g_local = statistics.mean(e0.elapsed_time(e1) for e0, e1 in gemm_spans)
    c_last = step()
    torch.cuda.synchronize()
    check = _check_rows_sample(c_last, lo, hi, _sample_lines(M), _sample_lines(N), a_h, b_h, S,
                               slice_kind, dev)
    del c_last

    # the other layout, and the gather of C to rank 0, in the same run
    alt = {}
    n_alt = args.alt_steps
    if world > 1 and n_alt > 0:
        for name, (kind, transport, gather) in {
                "gathered_to_rank0": (main_kind, args.transport, True),
                ("root_broadcast" if main_kind == "sharded" else "sharded_p2p"):
                (("root", "p2p", False) if main_kind == "sharded" else ("sharded", "p2p", False)),
        }.items():
            st2, _, _, _ = make_step(kind, transport, gather)
            for _ in range(2):
                st2()
            t = _timed(st2, n_alt, stream)
            alt[name] = {"value": 2.0 * M * N * K / (t * 1e-3) / 1e12, "ms_per_step": t,
                         "steps": n_alt,
                         "layout": {"root": "B on rank 0, slices broadcast over NCCL in column "
                                            "blocks",
                                    "sharded": f"A rows x B column panels ({transport})"}[kind]
                         + (", then C's row blocks sent to rank 0 (NCCL point-to-point)"
                            if gather else "")}
            del st2
            torch.cuda.empty_cache()

    # end to end through the public sharded call with host operands: each
    # rank copies its A rows and its B panel in and its C rows out
    e2e = None
    if not args.no_e2e:
        a_pin = a_h[lo:hi].contiguous().pin_memory()
        b_pin = b_h[:, p0:p1].contiguous().pin_memory() if b_loc is not None else None
        c_pin = torch.empty((hi - lo, N), dtype=a_h.dtype).pin_memory()

        def e2e_step():
            ad = a_pin.to(dev, non_blocking=True)
            bd = b_pin.to(dev, non_blocking=True) if b_pin is not None else None
            if main_kind == "sharded":
                cd = ozd.ozaki_matmul_sharded(ad, bd, S, sd, n=N, transport=args.transport)
            else:
                cd = ozd.ozaki_matmul_mrows(ad, bd, S, sd, b_blocks=args.chunks or None)
            c_pin.copy_(cd, non_blocking=True)

        for _ in range(2):
            e2e_step()
        n_e2e = max(2, min(args.steps, 5))
        e2e_ms = _timed(e2e_step, n_e2e, stream)
        es = a_h.element_size()
        e2e = {"value": 2.0 * M * N * K / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": (M * K + K * N) * es,
               "d2h_bytes_per_step": M * N * es,
               "h2d_bytes_rank0": ((hi - lo) * K + K * (p1 - p0)) * es}

    if rank != 0:
        return None
    flops = 2.0 * M * N * K
    bf16_peak, _, peak_src = bench.peaks()
    tensor_peak = 2.0 * bf16_peak if sd == torch.int8 else bf16_peak
    achieved = S * S * 2.0 * (hi - lo) * N * K / (g_local * 1e-3) / 1e12
    metric = bench.METRIC if args.config == "C3" else \
        f"emulated TFLOPS (2MNK/t), {cfg['desc']}"
    return {
        "metric": metric, "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOPS",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": slice_kind, "data": "synthetic",
        "config": {"workload": cfg["desc"], "name": args.config, "M": M, "N": N, "K": K,
                   "num_splits": S, "slice_dtype": slice_kind,
                   "input_dtype": bench.DTYPE_NAME[cfg["dtype"]],
                   "residual": "compat" if S <= 4 else "exact",
                   "l2": "no flush: operands larger than the 126 MB L2",
                   "parallelism": (f"A rows x B column panels over {world} GPUs, B's slices "
                                   + ("pulled block by block over NVLink by copy engines, each "
                                      "block's GEMM started on arrival"
                                      if args.transport == "p2p" else
                                      "all-gathered over NCCL") if main_kind == "sharded" else
                                   f"M-row sharding over {world} GPUs, B's slices broadcast "
                                   "from rank 0 over NCCL in column blocks"),
                   "result": "C left row-sharded (rank r holds its rows); the gathered "
                             "figure is under alt_layouts",
                   "rows_per_rank": rows,
                   "b_panel_cols": ozd.block_width(N, world) if main_kind == "sharded" else None,
                   "transport": (args.transport + (" (" + ozd.p2p_status() + ")"
                                                   if args.transport == "p2p" else ""))
                   if main_kind == "sharded" else "broadcast"},
        "roofline": {"bound": "tensor",
                     "kernel": "cross_gemm_kernel (rank 0 rows; span of the step's GEMMs)",
                     "achieved": achieved, "peak": tensor_peak, "unit": "TFLOP/s",
                     "frac": achieved / tensor_peak,
                     "peak_source": f"{'2x' if sd == torch.int8 else '1x'} {peak_src} dense "
                                    "bf16; B200 dense int8 = 2x bf16",
                     "gemm_ms": g_local, "traffic": None},
        **(check or {}),
        "alt_layouts": alt,
        "clocks": clk.summary(),
        # rank 0's own kernels in the timed region (NCCL kernels not counted)
        "gpu_launches": launches,
        "e2e": e2e,
    }


def run_batches(args, rank, world, dev):
    """C4: contiguous ranges of the broadcast batch per rank, no exchange."""
    import bench
    import oracle

    cfg = bench.CONFIGS["C4"]
    S = args.num_splits or cfg["s"]
    sd = cfg["slice"]
    slice_kind = bench.SLICE_NAME[sd]
    a_h, b_h = bench.config_inputs(cfg)
    a = a_h.to(dev)
    b = b_h.to(dev)
    M, K = a.shape[-2:]
    N = b.shape[-1]
    full = ozd.broadcast_batch(tuple(a.shape[:-2]), tuple(b.shape[:-2]))
    BN = math.prod(full)
    stream = torch.cuda.current_stream()
    out = {}

    def step():
        out["c"] = ozd.ozaki_matmul_batches(a, b, S, sd)
    for _ in range(args.warmup):
        step()
    with bench.ClockSampler(local_index(dev)) as clk:
        launches0 = ozd._lib.load().oz_launch_count()
        ms = _timed(step, args.steps, stream)
        launches = ozd._lib.load().oz_launch_count() - launches0
    # self-check: each rank compares a sample of its first and last output
    # batches with the oracle (fp16 slices: fp32 tensor-core sums)
    c, start, stop = out["c"]
    torch.cuda.synchronize()
    rows, cols = _sample_lines(M, 12), _sample_lines(N, 12)
    worst, rel = 0.0, 0.0
    a3 = a_h.expand(*full, M, K).reshape(BN, M, K)
    b3 = b_h.expand(*full, K, N).reshape(BN, K, N)
    for bi in sorted({start, stop - 1}) if stop > start else []:
        a_s = a3[bi][rows].numpy()
        b_s = b3[bi][:, cols].numpy()
        want = oracle.ozaki_matmul(a_s, b_s, S, slice_kind, "fp64")
        got = c[bi - start][torch.as_tensor(rows, device=dev)][:, torch.as_tensor(
            cols, device=dev)].double().cpu().numpy()
        worst = max(worst, float(np.linalg.norm(got - want) / np.linalg.norm(want)))
        ex = a_s @ b_s
        rel = max(rel, float(np.linalg.norm(got - ex) / np.linalg.norm(ex)))
    tol = max(1e-6, 2.5e-7 * math.sqrt(K))
    flags = torch.tensor([worst, rel], dtype=torch.float64, device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    if rank != 0:
        return None
    return {
        "metric": f"emulated TFLOPS (2MNK/t), {cfg['desc']}",
        "value": 2.0 * BN * M * N * K / (ms * 1e-3) / 1e12, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": slice_kind, "data": "synthetic",
        "config": {"workload": cfg["desc"], "name": "C4", "batches": BN, "num_splits": S,
                   "parallelism": f"contiguous ranges of the {BN} output batches over {world} "
                                  "GPUs; each rank splits only the A and B members its range "
                                  "uses; no exchange",
                   "l2": "no flush: operands larger than the 126 MB L2"},
        "parity_checked": bool(flags[0].item() < tol),
        "vs_oracle": (f"rel diff < {tol:.2g} (the fp16 tensor cores sum each pair product "
                      "over K in fp32; the oracle rounds the exact product once: "
                      "max(1e-6, 2.5e-7 sqrt(K)), as in tests/test_configs_gpu.py) on 12x12 "
                      "samples of every rank's first and last batch"),
        "max_diff_vs_oracle": float(flags[0].item()),
        "rel_err_vs_fp64_sample": float(flags[1].item()),
        "clocks": clk.summary(), "gpu_launches": launches, "e2e": None,
    }


def emulate_rank(args):
    """One rank's GEMM phase of the N-GPU C3 p2p layout, on one GPU, with every
    column block already present (a diagnostic of the transport's GEMM
    scheduling; the transfer itself is not emulated).  Rank 0's rows of A
    (M / N of them) times all of B in N column blocks of the blocked layout
    the transport fills, three ways: one oz_cross_gemm_blocked launch per
    block (the own block on the current stream, the others alternating over
    two side streams, P2P_ONE_LAUNCH = False), the own block's launch plus one
    oz_cross_gemm_arrivals launch over the other blocks (the transport's
    default), and one arrivals launch over all blocks.  CUDA events, median of
    20 after 3 warm-up runs; every variant's C is compared bit for bit with
    the first's."""
    import bench
    import ozaki_triton_b200 as oz
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    world = args.emulate_rank
    M, N, K, S = bench.M, bench.N, bench.K, bench.NUM_SPLITS
    m = M // world
    w = ozd.block_width(N, world)
    blocks = -(-N // w)
    a_h, b_h = bench.make_inputs()
    A = a_h[:m].to(dev)
    B = b_h.to(dev)
    sd = torch.int8
    alpha = ozd.compute_split_bits(K, sd, ozd.select_dot_accum_dtype(sd))
    be = ozd.Backend()
    A3 = A.reshape(1, m, K)
    a_sl, a_sc = be.split(A3, A3.stride(1), A3.stride(2), m, K, S, alpha, sd, 0)
    ld = a_sl.shape[-1]
    sl = torch.zeros((1, blocks, S, w, ld), dtype=sd, device=dev)
    sc = torch.zeros((1, blocks, S, w), dtype=torch.float32, device=dev)
    for j in range(blocks):
        ozd._split_block(be, B[:, j * w:min(N, (j + 1) * w)], K, S, alpha, sd, 0, sl[0, j],
                         sc[0, j])
    ready = torch.ones(blocks, dtype=torch.int32, device=dev)
    c = torch.empty((1, m, N), dtype=torch.float64, device=dev)
    cur = torch.cuda.current_stream(dev)
    side = [torch.cuda.Stream(dev) for _ in range(2)]

    def own_block():
        be.gemm(a_sl, sl[:, 0:1], a_sc, sc[:, 0:1], 1, m, min(N, w), K, S, torch.float64, False,
                out=c, col0=0, b_block_cols=w, stream=cur)

    def per_block():
        own_block()
        ev = torch.cuda.Event()
        ev.record(cur)
        for st in side:
            st.wait_event(ev)
        for j in range(1, blocks):
            c0, c1 = j * w, min(N, (j + 1) * w)
            be.gemm(a_sl, sl[:, j:j + 1], a_sc, sc[:, j:j + 1], 1, m, c1 - c0, K, S,
                    torch.float64, False, out=c, col0=c0, b_block_cols=w,
                    stream=side[(j - 1) % 2])
        for st in side:
            cur.wait_stream(st)

    def own_plus_arrivals():
        own_block()
        ev = torch.cuda.Event()
        ev.record(cur)
        side[0].wait_event(ev)
        be.gemm(a_sl, sl, a_sc, sc, 1, m, N, K, S, torch.float64, False, out=c, b_block_cols=w,
                stream=side[0], ready=ready, first_block=1 % blocks, block_count=blocks - 1)
        cur.wait_stream(side[0])

    def one_launch():
        be.gemm(a_sl, sl, a_sc, sc, 1, m, N, K, S, torch.float64, False, out=c, b_block_cols=w,
                stream=cur, ready=ready, first_block=0)

    out, ref = {}, None
    for name, fn in (("per_block_launches", per_block),
                     ("own_block_plus_one_peer_launch", own_plus_arrivals),
                     ("one_launch_all_blocks", one_launch)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(20):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            fn()
            e1.record(cur)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        if ref is None:
            ref = c.clone()
        out[name] = {"median_ms": statistics.median(ts), "min_ms": min(ts),
                     "same_bits": bool(torch.equal(c, ref))}
        c.fill_(float("nan"))
    print(json.dumps({"emulated_rank_of": world, "rows": m, "block_cols": w, "blocks": blocks,
                      "config": "C3 rank 0: FP64->INT8 s=4, K = 8192, every block present",
                      "device_status": oz.device_status(), **out}))


def local_index(dev):
    return dev.index if dev.index is not None else torch.cuda.current_device()
