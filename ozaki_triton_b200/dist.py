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

import ctypes
import math
from typing import Dict, Optional, Tuple

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
    broadcast_batch,
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
             b_block_cols: int = 0, stream: Optional[torch.cuda.Stream] = None,
             ready: Optional[torch.Tensor] = None, first_block: int = 0,
             block_count: int = 0) -> torch.Tensor:
        """C (batch, m, n); with ``out`` (batch, m, N_total) the result is written
        into its columns [col0, col0 + n) instead.  With ``b_block_cols`` the B
        slices are (BB, blocks, s, b_block_cols, ld) and their scales
        (BB, blocks, s, b_block_cols): column blocks as a gather produces them.
        ``stream``: launch there instead of on the current stream.  ``ready``
        (int32 per block, on the device; one batch): the blocks are still
        arriving and block c is read once ready[c] == 1; one launch computes
        the columns of ``block_count`` blocks (0: all) from ``first_block``
        on, in that order (oz_cross_gemm_arrivals)."""
        c = torch.empty((batch, m, n), dtype=out_dtype, device=a_sl.device) if out is None else out
        if batch == 0 or m == 0 or n == 0:
            return c
        ptr = c.data_ptr() + col0 * c.element_size()
        st = (stream or torch.cuda.current_stream(a_sl.device)).cuda_stream
        if ready is not None:
            _lib.check(_lib.load().oz_cross_gemm_arrivals(
                a_sl.data_ptr(), b_sl.data_ptr(), a_sc.data_ptr(), b_sc.data_ptr(), m, n, k,
                a_sl.shape[-1], num_splits, _OZ_DTYPE[a_sl.dtype], _OZ_DTYPE[out_dtype],
                b_block_cols, ready.data_ptr(), 1, first_block, block_count, ptr, c.stride(-2),
                _lib.OZ_GEMM_SKIP_TAIL if skip_tail else 0, st))
            return c
        _lib.check(_lib.load().oz_cross_gemm_blocked(
            a_sl.data_ptr(), b_sl.data_ptr(), a_sc.data_ptr(), b_sc.data_ptr(), batch, m, n, k,
            a_sl.shape[-1], num_splits, _OZ_DTYPE[a_sl.dtype], _OZ_DTYPE[out_dtype],
            a_idx.data_ptr() if a_idx is not None else None,
            b_idx.data_ptr() if b_idx is not None else None, a_sl.shape[0], b_sl.shape[0],
            b_block_cols, ptr, c.stride(-2), _lib.OZ_GEMM_SKIP_TAIL if skip_tail else 0, st))
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


def gather_rows(c_local: torch.Tensor, root: int = 0, group=None,
                rows: Optional[list] = None) -> Optional[torch.Tensor]:
    """Row blocks of C from every rank to ``root``, in rank order.

    ``c_local`` is this rank's (M_r, N) block (M_r may differ per rank,
    including 0).  Returns the whole (sum M_r, N) matrix on ``root`` and None
    elsewhere.  ``rows`` (every rank's M_r) saves one small all-gather when
    the caller knows it.  Point-to-point sends of contiguous row blocks (NCCL
    on GPUs, gloo on CPU), one per rank, all posted at once.  The reference
    returns the whole C on the caller's device (ozaki_triton.py:604-606);
    this is the multi-GPU counterpart.
    """
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    m_loc, n = c_local.shape
    if rows is None:
        t = torch.tensor([m_loc], dtype=torch.int64, device=c_local.device)
        allr = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allr, t, group=group)
        rows = [int(x.item()) for x in allr]
    assert rows[rank] == m_loc, f"rank {rank}: {m_loc} rows, expected {rows[rank]}"
    g_root = dist.get_global_rank(group, root) if group is not None else root
    c_local = c_local.contiguous()
    if rank != root:
        if m_loc > 0:
            for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, c_local, g_root, group)]):
                w.wait()
        return None
    out = torch.empty((sum(rows), n), dtype=c_local.dtype, device=c_local.device)
    offs = [sum(rows[:r]) for r in range(world)]
    ops = []
    for r in range(world):
        if r == root or rows[r] == 0:
            continue
        g_r = dist.get_global_rank(group, r) if group is not None else r
        ops.append(dist.P2POp(dist.irecv, out[offs[r]:offs[r] + rows[r]], g_r, group))
    works = dist.batch_isend_irecv(ops) if ops else []
    out[offs[root]:offs[root] + m_loc].copy_(c_local)
    for w in works:
        w.wait()
    return out


def ozaki_matmul_mrows(A_local: torch.Tensor, B: Optional[torch.Tensor], num_splits: int = 3,
                       slice_dtype: torch.dtype = torch.float16, *, root: int = 0,
                       group=None, skip_tail: bool = False, residual: Optional[str] = "auto",
                       b_blocks: Optional[int] = None, gather_to: Optional[int] = None,
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

    ``gather_to=r``: rank r returns the whole C (M, N) instead (the row
    blocks of every rank, in rank order, ``gather_rows``); the other ranks
    still return their own rows.
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
    return _maybe_gather(c.reshape(m_loc, n), gather_to, group)


def _maybe_gather(c_local: torch.Tensor, gather_to: Optional[int], group) -> torch.Tensor:
    if gather_to is None:
        return c_local
    full = gather_rows(c_local, gather_to, group)
    return full if full is not None else c_local


def _all_gather_inplace(buf: torch.Tensor, rank: int, group, async_op: bool):
    """All-gather of buf[0, r] from every rank r into buf (1, world, ...)."""
    if dist.get_backend(group) == "nccl":
        return dist.all_gather_into_tensor(buf.view(-1), buf[0, rank].reshape(-1), group=group,
                                           async_op=async_op)
    parts = [buf[0, r] for r in range(buf.shape[1])]
    return dist.all_gather(parts, buf[0, rank].clone(), group=group, async_op=async_op)


class PeerBlocks:
    """Column-blocked slice buffers of this rank, mapped into every peer.

    Two buffer sets alternate between calls, so a rank's split into one set
    never races a peer still copying from the other; each set is a slice
    tensor (1, world, s, w, ld) and a scale tensor (1, world, s, w) whose block
    r is rank r's panel.  The allocations are exported once as CUDA IPC
    handles, exchanged with ``all_gather_object`` and mapped by every peer;
    afterwards a block moves with one copy-engine copy over NVLink.
    """

    def __init__(self, group, shape_sl, shape_sc, slice_dtype, dev):
        lib = _lib.load()
        self.group = group
        self.dev = dev
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.sl = [torch.empty(shape_sl, dtype=slice_dtype, device=dev) for _ in range(2)]
        self.sc = [torch.empty(shape_sc, dtype=torch.float32, device=dev) for _ in range(2)]
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        # Every rank takes the same collective steps whatever fails locally:
        # a failed export sends None, a failed import is counted, and one
        # all-reduce decides for all ranks whether the mappings are usable.
        self.error = ""
        mine = []
        for t in self.sl + self.sc:
            h = ctypes.create_string_buffer(_lib.OZ_IPC_HANDLE_BYTES)
            off = ctypes.c_int64()
            if lib.oz_ipc_export(t.data_ptr(), h, ctypes.byref(off)) != _lib.OZ_OK:
                self.error = lib.oz_last_error().decode(errors="replace")
                mine = None
                break
            mine.append((h.raw, off.value))
        torch.cuda.synchronize(dev)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self.peer: Dict[Tuple[int, int], Tuple[int, int]] = {}
        ok = all(e is not None for e in everyone)
        if not ok and not self.error:
            self.error = "a peer could not export its buffers"
        for q in range(self.world):
            if q == self.rank or not ok:
                continue
            for i, (h, off) in enumerate(everyone[q]):
                ptr = ctypes.c_void_p()
                if lib.oz_ipc_import(h, off, ctypes.byref(ptr)) != _lib.OZ_OK:
                    self.error = lib.oz_last_error().decode(errors="replace")
                    ok = False
                    break
                self.peer[(q, i)] = (ptr.value, off)
        agree = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(agree, op=dist.ReduceOp.MIN, group=group)
        self.usable = bool(agree.item())
        if not self.usable:
            self.close()
            self.sl, self.sc = [], []
            return
        self.copy_streams = []
        self.gemm_streams = []
        self.calls = 0
        # per buffer set: block views, and (dst, src) byte addresses of every
        # peer block's slices and scales
        self.blocks = []
        for par in range(2):
            sl, sc = self.sl[par], self.sc[par]
            bsl = sl[0, 0].numel() * sl.element_size()
            bsc = sc[0, 0].numel() * 4
            views = [(sl[:, j:j + 1], sc[:, j:j + 1]) for j in range(self.world)]
            copies = {}
            for q in range(self.world):
                if q != self.rank:
                    copies[q] = (sl[0, q].data_ptr(), self.peer[(q, par)][0] + q * bsl, bsl,
                                 sc[0, q].data_ptr(), self.peer[(q, 2 + par)][0] + q * bsc, bsc)
            self.blocks.append((views, copies))
        self.ready = torch.cuda.Event()
        self.b_split = torch.cuda.Event()
        self.bar_stream = torch.cuda.Stream(dev)
        self.a_ready = torch.cuda.Event()
        self.arrived = [torch.cuda.Event() for _ in range(self.world)]
        # arrival flags of the one-launch GEMM (P2P_ONE_LAUNCH): block j of
        # the current call is in place once flags[j] == 1.  The flags are set
        # by 4-byte copies from pinned host memory ordered after the block's
        # copies, and reset per call, all on the copy stream: copy engines,
        # which the GEMM holding every SM cannot starve.
        self.flags = torch.zeros(self.world, dtype=torch.int32, device=dev)
        self.zeros_h = torch.zeros(self.world, dtype=torch.int32, pin_memory=True)
        self.own_h = torch.zeros(self.world, dtype=torch.int32, pin_memory=True)
        self.own_h[self.rank] = 1                 # the reset of "all": the own block is here
        self.one_h = torch.ones(1, dtype=torch.int32, pin_memory=True)
        self.reset_done = torch.cuda.Event()

    def streams(self, copies: int, gemms: int):
        while len(self.copy_streams) < copies:
            self.copy_streams.append(torch.cuda.Stream(self.dev))
        while len(self.gemm_streams) < gemms:
            self.gemm_streams.append(torch.cuda.Stream(self.dev))
        return self.copy_streams[:copies], self.gemm_streams[:gemms]

    def close(self):
        lib = _lib.load()
        for ptr, off in self.peer.values():
            lib.oz_ipc_close(ptr, off)
        self.peer = {}


_PEER_CACHE: Dict[tuple, PeerBlocks] = {}

# streams of the p2p transport: copy streams (blocks arrive one after another,
# so the first block GEMMs start early) and streams the block GEMMs run on
# (None = one per peer block, besides the current stream, which runs the GEMM
# of the rank's own block).  Measured on 8 B200s at 8192^3: 1 copy stream and
# 2 GEMM streams with the table's (1, 64) tiles for the 1024 x 1024 blocks:
# 1107 TFLOPS; CTA-pair tiles on one stream per block: 1043 TFLOPS (although
# a 1-GPU emulation with every block already present favoured them).
P2P_COPY_STREAMS = 1
P2P_GEMM_STREAMS: Optional[int] = 2
# One persistent GEMM launch (oz_cross_gemm_arrivals) that takes each block's
# tiles as its arrival flag is set, used when every rank owns a block:
#   "all"   : every block in the launch, the own block's tiles first; the
#             launch waits for the barrier (its copies' only kernel dependency)
#   "peers" : the own block's GEMM at once on the current stream, the peer
#             blocks in the launch
#   None    : one GEMM launch per peer block, on two side streams.
# `python bench.py --emulate-rank N` times a rank's GEMM phase the three ways
# on one GPU with every block present (C3: 0.746 / 0.853 / 0.872 ms at 8,
# 1.443 / 1.637 / 1.628 ms at 4 GPUs), but the transfer and the barrier turn
# that order around on the GPUs themselves: C3 on 4 B200s 685.5 / 688.0
# TFLOPS with "all" against 692.6 / 693.0 with "peers" (alternating runs), on
# 8 B200s 1196-1200 with "peers" against 1162 per block.
P2P_ONE_LAUNCH: Optional[str] = "peers"


def p2p_status(group=None) -> str:
    """"ok", "unused" or why the p2p transport fell back to the all-gather."""
    pbs = [pb for k, pb in _PEER_CACHE.items() if k[0] == id(group)]
    if not pbs:
        return "unused"
    bad = [pb.error or "unusable" for pb in pbs if not pb.usable]
    return bad[0] if bad else "ok"


def release_peer_buffers(group=None) -> None:
    """Unmap and free the cached peer buffers (collective: every rank calls it)."""
    for key in [k for k in _PEER_CACHE if k[0] == id(group)]:
        pb = _PEER_CACHE.pop(key)
        torch.cuda.synchronize(pb.dev)
        dist.barrier(group=group)          # no peer copies from our buffers any more
        pb.close()
        dist.barrier(group=group)          # every peer has unmapped them


def _peer_blocks(group, shape_sl, shape_sc, slice_dtype, dev) -> PeerBlocks:
    key = (id(group), tuple(shape_sl), slice_dtype, str(dev))
    pb = _PEER_CACHE.get(key)
    if pb is None:
        pb = _PEER_CACHE[key] = PeerBlocks(group, shape_sl, shape_sc, slice_dtype, dev)
    return pb


def _sharded_p2p(backend, A_local, B_local, num_splits, slice_dtype, alpha, mode, n, w, ld,
                 skip_tail, group):
    """Pipelined gather: every block GEMM starts as soon as its block is here.

    Host work per call is kept small (views, addresses and events are cached
    in the PeerBlocks), since at 8 GPUs a whole call takes about a millisecond
    of device time.  Returns None, on every rank alike, when the peer
    mappings could not be set up (the caller then uses the all-gather).
    """
    dev = A_local.device
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    m_loc, k = A_local.shape
    pb = _peer_blocks(group, (1, world, num_splits, w, ld), (1, world, num_splits, w),
                      slice_dtype, dev)
    if not pb.usable:
        return None
    par = pb.calls % 2
    pb.calls += 1
    sl, sc = pb.sl[par], pb.sc[par]
    views, copies = pb.blocks[par]
    cur = torch.cuda.current_stream(dev)
    _split_block(backend, B_local, k, num_splits, alpha, slice_dtype, mode, sl[0, rank],
                 sc[0, rank])
    # every rank's panel is split, and no peer still copies from the buffer
    # set this call reuses (its copies of two calls ago ended before it
    # entered this all-reduce).  The all-reduce runs on a stream of its own
    # that waits for the panel's split only, so the split of A's rows and the
    # GEMM of the own block go ahead on the current stream meanwhile.
    pb.b_split.record(cur)
    pb.bar_stream.wait_event(pb.b_split)
    with torch.cuda.stream(pb.bar_stream):
        dist.all_reduce(pb.flag, group=group)
        pb.ready.record(pb.bar_stream)
    A3 = A_local.reshape(1, m_loc, k)
    a_sl, a_sc = backend.split(A3, A3.stride(1), A3.stride(2), m_loc, k, num_splits, alpha,
                               slice_dtype, mode)
    pb.a_ready.record(cur)
    blocks = -(-n // w)
    order = [j for j in ((rank + d) % world for d in range(1, world)) if j < blocks]
    lib = _lib.load()
    if P2P_ONE_LAUNCH in ("all", "peers") and blocks == world and world > 1:
        every = P2P_ONE_LAUNCH == "all"
        # copies in ring order behind a reset of the arrival flags, each
        # block followed by its flag.  "peers": the own block's GEMM runs at
        # once on the current stream.  The arrival launch waits for the reset
        # (so no flag of the previous call is seen), which follows the
        # barrier: the NCCL kernel has finished before a kernel holding every
        # SM waits on flags
        copy_streams, gemm_streams = pb.streams(1, 1)
        cs, gs = copy_streams[0], gemm_streams[0]
        fl = pb.flags.data_ptr()
        cs.wait_event(pb.ready)
        _lib.check(lib.oz_copy_async(fl, (pb.own_h if every else pb.zeros_h).data_ptr(),
                                     4 * world, cs.cuda_stream))
        pb.reset_done.record(cs)
        for j in order:
            d_sl, s_sl, n_sl, d_sc, s_sc, n_sc = copies[j]
            _lib.check(lib.oz_copy_async(d_sl, s_sl, n_sl, cs.cuda_stream))
            _lib.check(lib.oz_copy_async(d_sc, s_sc, n_sc, cs.cuda_stream))
            _lib.check(lib.oz_copy_async(fl + 4 * j, pb.one_h.data_ptr(), 4, cs.cuda_stream))
        c = torch.empty((1, m_loc, n), dtype=A_local.dtype, device=dev)
        if not every:
            b_sl, b_sc = views[rank]
            backend.gemm(a_sl, b_sl, a_sc, b_sc, 1, m_loc, min(n, (rank + 1) * w) - rank * w,
                         k, num_splits, A_local.dtype, skip_tail, out=c, col0=rank * w,
                         b_block_cols=w, stream=cur)
        gs.wait_event(pb.a_ready)
        gs.wait_event(pb.reset_done)
        backend.gemm(a_sl, sl, a_sc, sc, 1, m_loc, n, k, num_splits, A_local.dtype, skip_tail,
                     out=c, b_block_cols=w, stream=gs, ready=pb.flags,
                     first_block=rank if every else (rank + 1) % world,
                     block_count=0 if every else world - 1)
        cur.wait_stream(gs)
        cur.wait_stream(cs)
        return c
    copy_streams, gemm_streams = pb.streams(
        max(1, P2P_COPY_STREAMS), max(1, P2P_GEMM_STREAMS or len(order)))
    for cs in copy_streams:
        cs.wait_event(pb.ready)
    for i, j in enumerate(order):
        cs = copy_streams[i % len(copy_streams)]
        d_sl, s_sl, n_sl, d_sc, s_sc, n_sc = copies[j]
        _lib.check(lib.oz_copy_async(d_sl, s_sl, n_sl, cs.cuda_stream))
        _lib.check(lib.oz_copy_async(d_sc, s_sc, n_sc, cs.cuda_stream))
        pb.arrived[j].record(cs)
    c = torch.empty((1, m_loc, n), dtype=A_local.dtype, device=dev)

    def block_gemm(j, stream):
        b_sl, b_sc = views[j]
        c0, c1 = j * w, min(n, (j + 1) * w)
        backend.gemm(a_sl, b_sl, a_sc, b_sc, 1, m_loc, c1 - c0, k, num_splits, A_local.dtype,
                     skip_tail, out=c, col0=c0, b_block_cols=w, stream=stream)

    if rank < blocks:
        block_gemm(rank, cur)
    for gs in gemm_streams:
        gs.wait_event(pb.a_ready)
    for i, j in enumerate(order):
        gs = gemm_streams[i % len(gemm_streams)]
        gs.wait_event(pb.arrived[j])
        block_gemm(j, gs)
    # the current stream joins every GEMM stream before anything else runs on
    # it, so c, a_sl and a_sc (allocated on it) are not reused while the side
    # streams still read or write them
    for gs in gemm_streams:
        cur.wait_stream(gs)
    cur.wait_event(pb.ready)             # the barrier is part of the call
    return c


def ozaki_matmul_sharded(A_local: torch.Tensor, B_local: torch.Tensor, num_splits: int = 3,
                         slice_dtype: torch.dtype = torch.float16, *, n: Optional[int] = None,
                         group=None, skip_tail: bool = False, residual: Optional[str] = "auto",
                         transport: str = "auto", gather_to: Optional[int] = None,
                         backend: Optional[Backend] = None) -> torch.Tensor:
    """C_local = A_local @ B with A sharded by rows and B by column panels.

    Rank r passes its rows of A (M_local, K) (any split of the rows) and its
    panel of B's columns (K, N_r), the columns ``column_panel(N, world, r)``;
    ``n`` (N) may be given to save one small collective.  Each rank splits
    only its own panel and its own rows; the int8 (or float) slices of every
    panel -- for int8 slices half the bytes of the fp64 panels -- then reach
    every rank in a column-blocked buffer that the GEMM reads in place.
    Returns this rank's rows of C (M_local, N), bit-identical to the same rows
    of the single-GPU ``ozaki_matmul``.

    ``transport``:
    * ``"auto"`` (default): ``"p2p"`` for CUDA tensors in an NCCL group, else
      ``"collective"``;
    * ``"collective"``: one all-gather (NCCL, or gloo on CPU) while the A rows
      are split, then one GEMM over all of N;
    * ``"p2p"`` (NCCL groups of one process per GPU): every rank maps its
      peers' slice buffers once (CUDA IPC) and pulls block after block with
      copy-engine copies; the GEMM of each block starts as soon as it has
      arrived (on one of two streams), so the transfer overlaps the GEMMs.
      If the mappings cannot be set up on some rank, every rank uses the
      collective transport instead (``p2p_status`` reports why).

    ``gather_to=r``: rank r returns the whole C (M, N) (``gather_rows``); the
    other ranks still return their own rows.
    """
    backend = backend or Backend()
    dev = A_local.device
    _check_args(A_local.dtype, num_splits, slice_dtype)
    assert A_local.dtype == B_local.dtype
    assert transport in ("auto", "collective", "p2p"), f"unknown transport {transport!r}"
    if transport == "auto":
        transport = ("p2p" if A_local.is_cuda and dist.get_backend(group) == "nccl"
                     else "collective")
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
    if transport == "p2p" and world > 1 and n > 0:
        c = _sharded_p2p(backend, A_local, B_local, num_splits, slice_dtype, alpha, mode, n, w,
                         ld, skip_tail, group)
        if c is not None:
            return _maybe_gather(c.reshape(m_loc, n), gather_to, group)
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
    return _maybe_gather(c.reshape(m_loc, n), gather_to, group)


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
    full = broadcast_batch(a_batch, b_batch)
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
