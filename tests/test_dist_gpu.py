"""Sharded paths on >= 2 GPUs with NCCL (one process per GPU): the
M-row-sharded GEMM with the B broadcast, rows x column panels with the
all-gather or copy-engine pulls (each GEMM scheduling of the pulls), the
gather of C to one rank, and batch sharding give the same bits as the
single-GPU call.
Skipped with fewer than two GPUs."""

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist

    import ozaki_triton_b200 as oz
    from ozaki_triton_b200 import dist as ozd
    try:
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        g = torch.Generator().manual_seed(3)
        A = (torch.rand(1000, 700, generator=g, dtype=torch.float64) - 0.5) * torch.exp(
            torch.randn(1000, 700, generator=g, dtype=torch.float64))
        B = (torch.rand(700, 300, generator=g, dtype=torch.float64) - 0.5) * torch.exp(
            torch.randn(700, 300, generator=g, dtype=torch.float64))
        lo, hi = ozd.block_range(1000, world, rank)
        c = ozd.ozaki_matmul_mrows(A[lo:hi].to(dev), B.to(dev) if rank == 0 else None, 4,
                                   torch.int8)
        want = oz.ozaki_matmul(A.to(dev), B.to(dev), 4, torch.int8)[lo:hi]
        ok1 = torch.equal(c, want)
        c3 = ozd.ozaki_matmul_mrows(A[lo:hi].to(dev), B.to(dev) if rank == 0 else None, 4,
                                    torch.int8, b_blocks=2)
        ok1 = ok1 and torch.equal(c3, want)
        # A by rows, B by column panels, slices all-gathered
        for n in (300, 1000):
            Bn = (torch.rand(700, n, generator=g, dtype=torch.float64) - 0.5) * 3.0
            p0, p1 = ozd.column_panel(n, world, rank)
            want_n = oz.ozaki_matmul(A.to(dev), Bn.to(dev), 4, torch.int8)[lo:hi]
            # collective all-gather, then copy-engine pulls (three calls: both
            # buffer sets of the alternation, and the reuse of the first) with
            # each GEMM scheduling of the p2p transport: the peer blocks in one
            # arrival-flag launch (default), every block in it, a launch per block
            for transport in ("collective", "p2p", "p2p", "p2p"):
                cs = ozd.ozaki_matmul_sharded(A[lo:hi].to(dev), Bn[:, p0:p1].to(dev), 4,
                                              torch.int8, transport=transport)
                ok1 = ok1 and torch.equal(cs, want_n)
            default_mode = ozd.P2P_ONE_LAUNCH
            for mode in ("all", None, "all"):
                ozd.P2P_ONE_LAUNCH = mode
                cs = ozd.ozaki_matmul_sharded(A[lo:hi].to(dev), Bn[:, p0:p1].to(dev), 4,
                                              torch.int8, transport="p2p")
                ok1 = ok1 and torch.equal(cs, want_n)
            ozd.P2P_ONE_LAUNCH = default_mode
            # C gathered to rank 1: the whole product there, own rows elsewhere
            full_n = oz.ozaki_matmul(A.to(dev), Bn.to(dev), 4, torch.int8)
            for transport in ("collective", "p2p"):
                cg = ozd.ozaki_matmul_sharded(A[lo:hi].to(dev), Bn[:, p0:p1].to(dev), 4,
                                              torch.int8, transport=transport, gather_to=1)
                ok1 = ok1 and torch.equal(cg, full_n if rank == 1 else want_n)
            cm = ozd.ozaki_matmul_mrows(A[lo:hi].to(dev), Bn.to(dev) if rank == 0 else None, 4,
                                        torch.int8, gather_to=1)
            ok1 = ok1 and torch.equal(cm, full_n if rank == 1 else want_n)
        ozd.release_peer_buffers()
        A4 = torch.randn(4, 1, 64, 96, generator=g, dtype=torch.float64)
        B4 = torch.randn(1, 3, 96, 40, generator=g, dtype=torch.float64)
        cb, s0, s1 = ozd.ozaki_matmul_batches(A4.to(dev), B4.to(dev), 3, torch.float16)
        wb = oz.ozaki_matmul(A4.to(dev), B4.to(dev), 3, torch.float16).reshape(12, 64, 40)[s0:s1]
        ok2 = torch.equal(cb, wb)
        np.save(os.path.join(out_dir, f"ok{rank}.npy"), np.array([ok1, ok2]))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as fh:
            fh.write(traceback.format_exc())
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_paths_match_single_gpu(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    errs = [f.read_text() for f in tmp_path.glob("err*.txt")]
    assert all(p.exitcode == 0 for p in procs), errs
    for r in range(world):
        assert np.load(tmp_path / f"ok{r}.npy").all()
