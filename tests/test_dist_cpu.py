"""Host-side multi-rank logic of ozaki_triton_b200.dist on CPU gloo ranks.

The device compute is replaced by the CPU oracle (a Backend with the same
interface), so these tests check the partitioning, the B broadcast protocol,
the batch-range bookkeeping and failure behaviour -- not the kernels (the
GPU tests do that).
"""

import os
import socket
import time
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from ozaki_triton_b200 import dist as ozd

KIND = {torch.float64: "fp64", torch.float32: "fp32", torch.float16: "fp16", torch.int8: "int8"}


class OracleBackend:
    """CPU stand-in for the CUDA library with the library's slice layout."""

    def __init__(self, residual="compat"):
        self.residual = residual

    def split(self, x3, stride_line, stride_k, lines, k, s, alpha, slice_dtype, mode, out=None):
        x = torch.as_strided(x3, (x3.shape[0], lines, k), (x3.stride(0), stride_line, stride_k))
        sl, sc = oracle.split_lines(x.numpy(), s, alpha, KIND[slice_dtype], KIND[x3.dtype],
                                    residual="compat" if mode == 0 else "exact")
        ld = ozd._lib_row(k, slice_dtype)
        if out is None:
            out = (torch.empty((x3.shape[0], s, lines, ld), dtype=slice_dtype),
                   torch.empty((x3.shape[0], s, lines), dtype=torch.float32))
        o_sl, o_sc = out
        o_sl.zero_()
        o_sl[..., :k] = torch.from_numpy(sl.astype(np.float32) if slice_dtype != torch.int8 else sl
                                         ).to(slice_dtype)
        o_sc.copy_(torch.from_numpy(sc))
        return o_sl, o_sc

    def gemm(self, a_sl, b_sl, a_sc, b_sc, batch, m, n, k, s, out_dtype, skip_tail,
             a_idx=None, b_idx=None, out=None, col0=0, b_block_cols=0):
        if b_block_cols:
            # column blocks (BB, blocks, s, w, ld) -> plain (BB, s, n, ld)
            bb, blocks, _, w, ld = b_sl.shape
            b_sl = b_sl.permute(0, 2, 1, 3, 4).reshape(bb, s, blocks * w, ld)[:, :, :n]
            b_sc = b_sc.permute(0, 2, 1, 3).reshape(bb, s, blocks * w)[:, :, :n]
        ai = a_idx.long() if a_idx is not None else torch.arange(batch)
        bi = b_idx.long() if b_idx is not None else torch.arange(batch)
        a = a_sl[ai, ..., :k].numpy()
        b = b_sl[bi, ..., :k].numpy()
        c = torch.from_numpy(np.ascontiguousarray(oracle.cross_gemm(
            a, b, a_sc[ai].numpy(), b_sc[bi].numpy(), KIND[a_sl.dtype], KIND[out_dtype],
            skip_tail)))
        if out is None:
            return c
        out[..., col0:col0 + n] = c
        return out


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, out_dir):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=20))
        case(rank, world, out_dir)
        dist.destroy_process_group()
    except BaseException:  # report to the parent
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as fh:
            fh.write(traceback.format_exc())
        raise


def run_ranks(case, world, tmp_path):
    port = free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    return [p.exitcode for p in procs]


def law(g, shape):
    return (torch.rand(shape, generator=g, dtype=torch.float64) - 0.5) * torch.exp(
        torch.randn(shape, generator=g, dtype=torch.float64))


def case_mrows(rank, world, out_dir):
    g = torch.Generator().manual_seed(5)
    A = law(g, (37, 64))
    B = law(g, (64, 23))
    lo, hi = ozd.block_range(37, world, rank)
    c = ozd.ozaki_matmul_mrows(A[lo:hi], B if rank == 0 else None, 4, torch.int8,
                               backend=OracleBackend())
    np.save(os.path.join(out_dir, f"c{rank}.npy"), c.numpy())
    # the same through three broadcast blocks of B's columns (256, 256, 88)
    B2 = law(g, (64, 600))
    c2 = ozd.ozaki_matmul_mrows(A[lo:hi], B2 if rank == 0 else None, 4, torch.int8,
                                b_blocks=3, backend=OracleBackend())
    np.save(os.path.join(out_dir, f"d{rank}.npy"), c2.numpy())


def case_sharded(rank, world, out_dir):
    g = torch.Generator().manual_seed(8)
    A = law(g, (37, 64))
    for name, n in (("a", 600), ("b", 100), ("c", 256)):
        B = law(g, (64, n))
        c0, c1 = ozd.column_panel(n, world, rank)
        lo, hi = ozd.block_range(37, world, rank)
        c = ozd.ozaki_matmul_sharded(A[lo:hi], B[:, c0:c1], 4, torch.int8,
                                     n=None if name == "a" else n, backend=OracleBackend())
        np.save(os.path.join(out_dir, f"{name}{rank}.npy"), c.numpy())


def case_batches(rank, world, out_dir):
    g = torch.Generator().manual_seed(6)
    A = law(g, (4, 1, 8, 16))
    B = law(g, (1, 3, 16, 5))
    c, lo, hi = ozd.ozaki_matmul_batches(A, B, 3, torch.float16, backend=OracleBackend())
    np.save(os.path.join(out_dir, f"c{rank}.npy"), c.numpy())
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([lo, hi]))


def case_root_fails(rank, world, out_dir):
    """The root dies before the broadcast: the other rank's collective must end
    with an error within the process-group timeout, not hang."""
    g = torch.Generator().manual_seed(7)
    A = law(g, (8, 16))
    B = law(g, (16, 4))
    if rank == 0:
        raise RuntimeError("injected failure on the root before the broadcast")
    t0 = time.time()
    try:
        ozd.ozaki_matmul_mrows(A, None, 2, torch.int8, backend=OracleBackend())
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(out_dir, "peer_error.txt"), "w") as fh:
            fh.write(f"{type(e).__name__} after {time.time() - t0:.1f}s: {e}")
        return
    with open(os.path.join(out_dir, "peer_error.txt"), "w") as fh:
        fh.write("NO ERROR")


def case_panel_rank_fails(rank, world, out_dir):
    """A non-root rank dies before the all-gather of the sharded path: the
    surviving rank's collective must end with an error, not hang."""
    g = torch.Generator().manual_seed(10)
    A = law(g, (8, 16))
    B = law(g, (16, 300))
    c0, c1 = ozd.column_panel(300, world, rank)
    if rank == 1:
        raise RuntimeError("injected failure before the all-gather")
    t0 = time.time()
    try:
        ozd.ozaki_matmul_sharded(A, B[:, c0:c1], 2, torch.int8, n=300, backend=OracleBackend())
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(out_dir, "peer_error.txt"), "w") as fh:
            fh.write(f"{type(e).__name__} after {time.time() - t0:.1f}s: {e}")
        return
    with open(os.path.join(out_dir, "peer_error.txt"), "w") as fh:
        fh.write("NO ERROR")


def test_panel_rank_failure_is_reported_not_hung(tmp_path):
    t0 = time.time()
    codes = run_ranks(case_panel_rank_fails, 2, tmp_path)
    assert codes[1] != 0                       # the injected failure
    msg = (tmp_path / "peer_error.txt").read_text()
    assert msg != "NO ERROR", msg              # the survivor saw an error ...
    assert time.time() - t0 < 110              # ... within the timeout, no hang


def test_block_range_covers_everything():
    for total in [0, 1, 7, 128, 8192, 8193]:
        for world in [1, 2, 3, 4, 8]:
            ranges = [ozd.block_range(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c and b >= a
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_mrows_two_ranks_bit_identical(tmp_path):
    codes = run_ranks(case_mrows, 2, tmp_path)
    assert codes == [0, 0], [open(p).read() for p in tmp_path.glob("err*.txt")]
    c = np.concatenate([np.load(tmp_path / f"c{r}.npy") for r in range(2)])
    g = torch.Generator().manual_seed(5)
    A = law(g, (37, 64))
    B = law(g, (64, 23))
    want = oracle.ozaki_matmul(A.numpy(), B.numpy(), 4, "int8", "fp64")
    assert np.array_equal(c, want)
    B2 = law(g, (64, 600))
    d = np.concatenate([np.load(tmp_path / f"d{r}.npy") for r in range(2)])
    assert np.array_equal(d, oracle.ozaki_matmul(A.numpy(), B2.numpy(), 4, "int8", "fp64"))


def test_sharded_two_ranks_bit_identical(tmp_path):
    """A by rows, B by column panels (ragged last panel, an empty panel, exact
    fit), slices all-gathered into the column-blocked buffer."""
    codes = run_ranks(case_sharded, 2, tmp_path)
    assert codes == [0, 0], [open(p).read() for p in tmp_path.glob("err*.txt")]
    g = torch.Generator().manual_seed(8)
    A = law(g, (37, 64))
    for name, n in (("a", 600), ("b", 100), ("c", 256)):
        B = law(g, (64, n))
        got = np.concatenate([np.load(tmp_path / f"{name}{r}.npy") for r in range(2)])
        assert np.array_equal(got, oracle.ozaki_matmul(A.numpy(), B.numpy(), 4, "int8", "fp64"))


def case_world3(rank, world, out_dir):
    """Three ranks: ragged panels (256, 256, 88 columns), uneven rows, and the
    root broadcast in two blocks."""
    g = torch.Generator().manual_seed(9)
    A = law(g, (37, 64))
    B = law(g, (64, 600))
    lo, hi = ozd.block_range(37, world, rank)
    c0, c1 = ozd.column_panel(600, world, rank)
    c = ozd.ozaki_matmul_sharded(A[lo:hi], B[:, c0:c1], 3, torch.int8, backend=OracleBackend())
    np.save(os.path.join(out_dir, f"s{rank}.npy"), c.numpy())
    d = ozd.ozaki_matmul_mrows(A[lo:hi], B if rank == 1 else None, 3, torch.int8, root=1,
                               b_blocks=2, backend=OracleBackend())
    np.save(os.path.join(out_dir, f"m{rank}.npy"), d.numpy())


def test_three_ranks_sharded_and_root_broadcast(tmp_path):
    codes = run_ranks(case_world3, 3, tmp_path)
    assert codes == [0, 0, 0], [open(p).read() for p in tmp_path.glob("err*.txt")]
    g = torch.Generator().manual_seed(9)
    A = law(g, (37, 64))
    B = law(g, (64, 600))
    want = oracle.ozaki_matmul(A.numpy(), B.numpy(), 3, "int8", "fp64")
    for tag in ("s", "m"):
        got = np.concatenate([np.load(tmp_path / f"{tag}{r}.npy") for r in range(3)])
        assert np.array_equal(got, want), tag


def test_column_panels_cover_n():
    for n in [0, 1, 100, 128, 129, 600, 8192, 8193]:
        for world in [1, 2, 3, 8]:
            panels = [ozd.column_panel(n, world, r) for r in range(world)]
            assert panels[0][0] == 0 and panels[-1][1] == n
            w = ozd.block_width(n, world)
            for r, (a, b) in enumerate(panels):
                assert a <= b and (b - a) <= w
                if b > a:
                    assert a == r * w                 # block r of the gather buffer
            assert w == n or w % 128 == 0


def test_batches_two_ranks_cover_the_broadcast(tmp_path):
    codes = run_ranks(case_batches, 2, tmp_path)
    assert codes == [0, 0], [open(p).read() for p in tmp_path.glob("err*.txt")]
    parts = [np.load(tmp_path / f"c{r}.npy") for r in range(2)]
    ranges = [tuple(np.load(tmp_path / f"r{r}.npy")) for r in range(2)]
    assert ranges[0][0] == 0 and ranges[0][1] == ranges[1][0] and ranges[1][1] == 12
    g = torch.Generator().manual_seed(6)
    A = law(g, (4, 1, 8, 16))
    B = law(g, (1, 3, 16, 5))
    want = oracle.ozaki_matmul(A.numpy(), B.numpy(), 3, "fp16", "fp64").reshape(12, 8, 5)
    got = np.concatenate(parts)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < 1e-12


def test_root_failure_is_reported_not_hung(tmp_path):
    t0 = time.time()
    codes = run_ranks(case_root_fails, 2, tmp_path)
    assert codes[0] != 0                       # the injected failure
    msg = (tmp_path / "peer_error.txt").read_text()
    assert msg != "NO ERROR", msg              # the peer saw an error ...
    assert time.time() - t0 < 110              # ... within the timeout, no hang


def test_weighted_rows_partition():
    for m in [1, 37, 128, 1000, 8192, 16384]:
        for world in [1, 2, 3, 8]:
            for disc in [0, 100, 768, 10 ** 6]:
                rows = ozd.weighted_rows(m, world, 0, disc)
                assert sum(rows) == m and min(rows) >= 0 and len(rows) == world
    assert ozd.weighted_rows(8192, 8, 0, 768)[0] < 8192 // 8


def case_gather(rank, world, out_dir):
    """C gathered to a root: ragged row blocks (an empty one on the last
    rank), both layouts, root 1; the other ranks keep their own rows."""
    g = torch.Generator().manual_seed(12)
    A = law(g, (41, 64))
    B = law(g, (64, 300))
    rows = [20, 21, 0][:world]
    lo = sum(rows[:rank])
    hi = lo + rows[rank]
    c0, c1 = ozd.column_panel(300, world, rank)
    c = ozd.ozaki_matmul_sharded(A[lo:hi], B[:, c0:c1], 4, torch.int8, gather_to=1,
                                 backend=OracleBackend())
    np.save(os.path.join(out_dir, f"s{rank}.npy"), c.numpy())
    d = ozd.ozaki_matmul_mrows(A[lo:hi], B if rank == 0 else None, 4, torch.int8, gather_to=1,
                               backend=OracleBackend())
    np.save(os.path.join(out_dir, f"m{rank}.npy"), d.numpy())
    # the helper alone, with the row counts given
    e = ozd.gather_rows(torch.full((rows[rank], 3), float(rank)), root=0, rows=rows)
    if rank == 0:
        np.save(os.path.join(out_dir, "e.npy"), e.numpy())
    else:
        assert e is None


def test_gather_to_root_three_ranks(tmp_path):
    codes = run_ranks(case_gather, 3, tmp_path)
    assert codes == [0, 0, 0], [open(p).read() for p in tmp_path.glob("err*.txt")]
    g = torch.Generator().manual_seed(12)
    A = law(g, (41, 64))
    B = law(g, (64, 300))
    want = oracle.ozaki_matmul(A.numpy(), B.numpy(), 4, "int8", "fp64")
    rows = [20, 21, 0]
    for tag in ("s", "m"):
        assert np.array_equal(np.load(tmp_path / f"{tag}1.npy"), want), tag
        for r in (0, 2):
            lo = sum(rows[:r])
            assert np.array_equal(np.load(tmp_path / f"{tag}{r}.npy"), want[lo:lo + rows[r]])
    e = np.load(tmp_path / "e.npy")
    assert e.shape == (41, 3) and (e[:20] == 0).all() and (e[20:] == 1).all()
