"""Multi-GPU Ozaki GEMM: one process per GPU over ``torch.distributed``.

The reference runs one GPU per independent problem only (its harness pools
processes, ``test.py:77-81``); it has no sharded path.  Two partitions are
provided here, both without a reduction collective because every A row and
every B column is split independently (per-row / per-column scales), so a
shard's slices are bit-identical to the corresponding rows of the global
split:

* ``ozaki_matmul_sharded``: A sharded by rows and B by column panels; each
  rank splits only its own rows and its own panel, and one all-gather moves
  the panels' slices (for int8 slices half the bytes of the fp64 panels) to
  every rank while the A rows are split; every rank computes its rows of C.
* ``ozaki_matmul_mrows``: A sharded by row blocks; B lives on one root rank,
  which splits it in column blocks and broadcasts each block's slices and
  scales while it splits the next; every rank computes its rows of C.
* ``ozaki_matmul_batches``: the broadcast batch of a batched matmul is cut in
  contiguous ranges of output batches; each rank computes its range from the
  operand members that range references (no exchange at all).

The device work goes through a ``Backend`` (the CUDA library by default); the
CPU tests plug in the oracle to check the partitioning and the collective
protocol on ``gloo`` ranks.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .api import (
    MAX_SPLITS,
    SLICE_DTYPE_INFO,
    _OZ_DTYPE,
    _batch_index,
    _residual_mode,
    _split_lines,
    compute_split_bits,
    select_dot_accum_dtype,
)


def block_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, stop) of ``total`` units for ``rank``."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class Backend:
    """Device compute used by the sharded drivers (the CUDA library)."""

    def split(self, x3: torch.Tensor, stride_line: int, stride_k: int, lines: int, k: int,
              num_splits: int, alpha: int, slice_dtype: torch.dtype, mode: int, out=None):
        return _split_lines(x3, stride_line, stride_k, lines, k, num_splits, alpha,
                            slice_dtype, mode, out=out)

    def gemm(self, a_sl, b_sl, a_sc, b_sc, batch: int, m: int, n: int, k: int, num_splits: int,
             out_dtype: torch.dtype, skip_tail: bool, a_idx=None, b_idx=None,
             out: Optional[torch.Tensor] = None, col0: int = 0,
             b_block_cols: int = 0) -> torch.Tensor:
        """C (batch, m, n); with ``out`` (batch, m, N_total) the result is written
        into its columns [col0, col0 + n) instead.  With ``b_block_cols`` the B
        slices are (BB, blocks, s, b_block_cols, ld) and their scales
        (BB, blocks, s, b_block_cols): column blocks as a gather produces them."""
        c = torch.empty((batch, m, n), dtype=out_dtype, device=a_sl.device) if out is None else out
        if batch == 0 or m == 0 or n == 0:
            return c
        ptr = c.data_ptr() + col0 * c.element_size()
        _lib.check(_lib.load().oz_cross_gemm_blocked(
            a_sl.data_ptr(), b_sl.data_ptr(), a_sc.data_ptr(), b_sc.data_ptr(), batch, m, n, k,
            a_sl.shape[-1], num_splits, _OZ_DTYPE[a_sl.dtype], _OZ_DTYPE[out_dtype],
            a_idx.data_ptr() if a_idx is not None else None,
            b_idx.data_ptr() if b_idx is not None else None, a_sl.shape[0], b_sl.shape[0],
            b_block_cols, ptr, c.stride(-2), _lib.OZ_GEMM_SKIP_TAIL if skip_tail else 0,
            torch.cuda.current_stream(a_sl.device).cuda_stream))
        return c


def _check_args(dtype, num_splits, slice_dtype):
    assert slice_dtype in SLICE_DTYPE_INFO, f"unsupported slice dtype: {slice_dtype}"
    assert 1 <= num_splits <= MAX_SPLITS, f"num_splits must be in [1, {MAX_SPLITS}]"
    assert dtype in (torch.float64, torch.float32, torch.float16, torch.bfloat16), \
        f"unsupported input dtype: {dtype}"


def weighted_rows(m: int, world: int, root: int = 0, root_discount: int = 0,
                  align: int = 128) -> list:
    """Row counts per rank: balanced in blocks of ``align`` rows, with about
    ``root_discount`` rows (times (world - 1) / world) moved off the root,
    which also splits and broadcasts B."""
    blocks = (m + align - 1) // align
    if world == 1:
        return [m]
    root_blocks = max(0, round((m / world - root_discount * (world - 1) / world) / align))
    root_blocks = min(root_blocks, blocks)
    rest = blocks - root_blocks
    counts = [0] * world
    others = [r for r in range(world) if r != root]
    for i, r in enumerate(others):
        counts[r] = rest // len(others) + (1 if i < rest % len(others) else 0)
    counts[root] = root_blocks
    rows = [c * align for c in counts]
    # the last rank that has rows absorbs the ragged end
    excess = sum(rows) - m
    for r in reversed(range(world)):
        if excess <= 0:
            break
        take = min(excess, rows[r])
        rows[r] -= take
        excess -= take
    return rows


def block_width(n: int, parts: int, align: int = 128) -> int:
    """Width of the column blocks B's slices travel in: n in ``parts`` blocks
    of a multiple of ``align`` columns (the GEMM's tile width), the last one
    possibly narrower.  One block (width n) for parts <= 1."""
    if parts <= 1 or n <= align:
        return n
    return -(-n // (parts * align)) * align


def column_panel(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of the B columns rank ``rank`` holds in ``ozaki_matmul_sharded``:
    blocks of ``block_width(n, world)`` columns, trailing ranks possibly empty."""
    w = block_width(n, world)
    return min(n, rank * w), min(n, (rank + 1) * w)


def _blocked_buffers(blocks: int, num_splits: int, w: int, ld: int, slice_dtype, dev):
    sl = torch.empty((1, blocks, num_splits, w, ld), dtype=slice_dtype, device=dev)
    sc = torch.empty((1, blocks, num_splits, w), dtype=torch.float32, device=dev)
    return sl, sc


def _split_block(backend, Bc: torch.Tensor, k: int, num_splits: int, alpha: int, slice_dtype,
                 mode: int, sl_block: torch.Tensor, sc_block: torch.Tensor):
    """Split the columns of Bc (k, nc) into one block (s, w, ld) / (s, w) of the
    gather buffers; nc <= w (a narrower block leaves its last rows unused)."""
    nc = Bc.shape[1]
    w = sl_block.shape[1]
    if nc == 0:
        return
    B3 = Bc.reshape(1, k, nc)
    if nc == w:
        backend.split(B3, B3.stride(2), B3.stride(1), nc, k, num_splits, alpha, slice_dtype,
                      mode, out=(sl_block.unsqueeze(0), sc_block.unsqueeze(0)))
    else:
        t_sl, t_sc = backend.split(B3, B3.stride(2), B3.stride(1), nc, k, num_splits, alpha,
                                   slice_dtype, mode)
        sl_block[:, :nc].copy_(t_sl[0])
        sc_block[:, :nc].copy_(t_sc[0])


def ozaki_matmul_mrows(A_local: torch.Tensor, B: Optional[torch.Tensor], num_splits: int = 3,
                       slice_dtype: torch.dtype = torch.float16, *, root: int = 0,
                       group=None, skip_tail: bool = False, residual: Optional[str] = "auto",
                       b_blocks: Optional[int] = None,
                       backend: Optional[Backend] = None) -> torch.Tensor:
    """C_local = A_local @ B, A sharded by rows, B on ``root`` only.

    Every rank passes its own rows of A (M_local, K) (M_local may differ per
    rank, including 0); the root passes B (K, N), the others may pass None.
    Returns this rank's rows of C (M_local, N) in the input dtype, equal bit
    for bit to the same rows of the single-GPU ``ozaki_matmul``.

    The root splits B in ``b_blocks`` column blocks and broadcasts each block's
    slices as soon as it is split, so the broadcast of block c overlaps the
    split of block c + 1.  The blocks land in place in a column-blocked slice
    buffer that the GEMM reads directly (one launch over all of N).
    """
    backend = backend or Backend()
    dev = A_local.device
    _check_args(A_local.dtype, num_splits, slice_dtype)
    m_loc, k = A_local.shape
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    # the root announces N (and checks K); every rank takes the same steps
    shape = torch.tensor([B.shape[0], B.shape[1]] if rank == root else [0, 0],
                         dtype=torch.int64, device=dev)
    dist.broadcast(shape, src=root, group=group)
    k_b, n = int(shape[0]), int(shape[1])
    assert k_b == k, f"contraction dim mismatch: A K={k}, B K={k_b}"
    alpha = compute_split_bits(k, slice_dtype=slice_dtype,
                               dot_accum_dtype=select_dot_accum_dtype(slice_dtype))
    mode = _residual_mode(residual, num_splits, A_local.dtype)
    ld = _lib_row(k, slice_dtype)
    if b_blocks is None:
        b_blocks = 4 if (world > 1 and n >= 4096) else 1
    w = block_width(n, b_blocks)
    blocks = -(-n // w) if n > 0 else 0
    b_sl, b_sc = _blocked_buffers(blocks, num_splits, w, ld, slice_dtype, dev)
    works = []
    for c in range(blocks):
        if rank == root:
            _split_block(backend, B[:, c * w:min(n, (c + 1) * w)], k, num_splits, alpha,
                         slice_dtype, mode, b_sl[0, c], b_sc[0, c])
        works.append(dist.broadcast(b_sl[0, c], src=root, group=group, async_op=True))
        works.append(dist.broadcast(b_sc[0, c], src=root, group=group, async_op=True))
    # this rank's rows of A are split while the blocks of B travel
    A3 = A_local.reshape(1, m_loc, k)
    a_sl, a_sc = backend.split(A3, A3.stride(1), A3.stride(2), m_loc, k, num_splits, alpha,
                               slice_dtype, mode)
    for wk in works:
        wk.wait()
    c = backend.gemm(a_sl, b_sl, a_sc, b_sc, 1, m_loc, n, k, num_splits, A_local.dtype,
                     skip_tail, b_block_cols=w)
    return c.reshape(m_loc, n)


def _all_gather_inplace(buf: torch.Tensor, rank: int, group, async_op: bool):
    """All-gather of buf[0, r] from every rank r into buf (1, world, ...)."""
    if dist.get_backend(group) == "nccl":
        return dist.all_gather_into_tensor(buf.view(-1), buf[0, rank].reshape(-1), group=group,
                                           async_op=async_op)
    parts = [buf[0, r] for r in range(buf.shape[1])]
    return dist.all_gather(parts, buf[0, rank].clone(), group=group, async_op=async_op)


def ozaki_matmul_sharded(A_local: torch.Tensor, B_local: torch.Tensor, num_splits: int = 3,
                         slice_dtype: torch.dtype = torch.float16, *, n: Optional[int] = None,
                         group=None, skip_tail: bool = False, residual: Optional[str] = "auto",
                         backend: Optional[Backend] = None) -> torch.Tensor:
    """C_local = A_local @ B with A sharded by rows and B by column panels.

    Rank r passes its rows of A (M_local, K) (any split of the rows) and its
    panel of B's columns (K, N_r), the columns ``column_panel(N, world, r)``;
    ``n`` (N) may be given to save one small collective.  Each rank splits
    only its own panel and its own rows; one all-gather then moves the int8
    (or float) slices of every panel to every rank -- for int8 slices half the
    bytes of the fp64 panels -- into a column-blocked buffer that the GEMM
    reads in place.  The split of A's rows overlaps the all-gather.  Returns
    this rank's rows of C (M_local, N), bit-identical to the same rows of the
    single-GPU ``ozaki_matmul``.
    """
    backend = backend or Backend()
    dev = A_local.device
    _check_args(A_local.dtype, num_splits, slice_dtype)
    assert A_local.dtype == B_local.dtype
    m_loc, k = A_local.shape
    assert B_local.shape[0] == k, f"contraction dim mismatch: {A_local.shape} @ {B_local.shape}"
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if n is None:
        t = torch.tensor([B_local.shape[1]], dtype=torch.int64, device=dev)
        dist.all_reduce(t, group=group)
        n = int(t.item())
    c0, c1 = column_panel(n, world, rank)
    assert B_local.shape[1] == c1 - c0, \
        f"rank {rank} holds {B_local.shape[1]} columns of B, expected {c1 - c0} ({c0}:{c1})"
    alpha = compute_split_bits(k, slice_dtype=slice_dtype,
                               dot_accum_dtype=select_dot_accum_dtype(slice_dtype))
    mode = _residual_mode(residual, num_splits, A_local.dtype)
    ld = _lib_row(k, slice_dtype)
    w = block_width(n, world)
    if world == 1 or n == 0:
        w = max(n, 1)
    # one block per rank (blocks past ceil(n / w) stay empty and are not read)
    b_sl, b_sc = _blocked_buffers(world, num_splits, w, ld, slice_dtype, dev)
    _split_block(backend, B_local, k, num_splits, alpha, slice_dtype, mode, b_sl[0, rank],
                 b_sc[0, rank])
    works = [_all_gather_inplace(b_sl, rank, group, True),
             _all_gather_inplace(b_sc, rank, group, True)]
    A3 = A_local.reshape(1, m_loc, k)
    a_sl, a_sc = backend.split(A3, A3.stride(1), A3.stride(2), m_loc, k, num_splits, alpha,
                               slice_dtype, mode)
    for wk in works:
        wk.wait()
    c = backend.gemm(a_sl, b_sl, a_sc, b_sc, 1, m_loc, n, k, num_splits, A_local.dtype,
                     skip_tail, b_block_cols=w)
    return c.reshape(m_loc, n)


def ozaki_matmul_batches(A: torch.Tensor, B: torch.Tensor, num_splits: int = 3,
                         slice_dtype: torch.dtype = torch.float16, *, group=None,
                         skip_tail: bool = False, residual: Optional[str] = "auto",
                         backend: Optional[Backend] = None) -> Tuple[torch.Tensor, int, int]:
    """This rank's contiguous range of the broadcast batch of A @ B.

    A: (..., M, K), B: (..., K, N) on every rank (torch.matmul broadcasting).
    Returns (C_range (n_b, M, N), start, stop): output batches [start, stop)
    of the flattened broadcast batch.  Only the A and B members the range
    references are split.
    """
    backend = backend or Backend()
    _check_args(A.dtype, num_splits, slice_dtype)
    assert A.dtype == B.dtype
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    M, K = A.shape[-2:]
    K2, N = B.shape[-2:]
    assert K == K2
    a_batch, b_batch = tuple(A.shape[:-2]), tuple(B.shape[:-2])
    full = tuple(torch.broadcast_shapes(a_batch, b_batch))
    bn = math.prod(full)
    start, stop = block_range(bn, world, rank)
    alpha = compute_split_bits(K, slice_dtype=slice_dtype,
                               dot_accum_dtype=select_dot_accum_dtype(slice_dtype))
    mode = _residual_mode(residual, num_splits, A.dtype)
    a_all = _batch_index(a_batch, full, "cpu")
    b_all = _batch_index(b_batch, full, "cpu")
    a_all = torch.arange(bn, dtype=torch.int32) if a_all is None else a_all
    b_all = torch.arange(bn, dtype=torch.int32) if b_all is None else b_all
    a_need = torch.unique(a_all[start:stop]) if stop > start else a_all[:0]
    b_need = torch.unique(b_all[start:stop]) if stop > start else b_all[:0]
    A3 = A.reshape(math.prod(a_batch), M, K)[a_need.long().to(A.device)]
    B3 = B.reshape(math.prod(b_batch), K, N)[b_need.long().to(B.device)]
    if stop == start:
        return torch.empty((0, M, N), dtype=A.dtype, device=A.device), start, stop
    # renumber the members this range uses
    a_map = {int(v): i for i, v in enumerate(a_need.tolist())}
    b_map = {int(v): i for i, v in enumerate(b_need.tolist())}
    a_idx = torch.tensor([a_map[int(v)] for v in a_all[start:stop].tolist()], dtype=torch.int32,
                         device=A.device)
    b_idx = torch.tensor([b_map[int(v)] for v in b_all[start:stop].tolist()], dtype=torch.int32,
                         device=A.device)
    b_sl, b_sc = backend.split(B3, B3.stride(2), B3.stride(1), N, K, num_splits, alpha,
                               slice_dtype, mode)
    a_sl, a_sc = backend.split(A3, A3.stride(1), A3.stride(2), M, K, num_splits, alpha,
                               slice_dtype, mode)
    c = backend.gemm(a_sl, b_sl, a_sc, b_sc, stop - start, M, N, K, num_splits, A.dtype,
                     skip_tail, a_idx, b_idx)
    return c, start, stop


def _lib_row(k: int, slice_dtype: torch.dtype) -> int:
    es = torch.empty((), dtype=slice_dtype).element_size()
    return ((k * es + 127) // 128 * 128) // es if k > 0 else 0
