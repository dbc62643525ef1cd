"""Host side of the Ozaki-scheme GEMM: the reference's Python operator API.

Same names, argument meaning and error behaviour as ``ozaki_triton.py`` of
WhFanatic/Ozaki_triton (``compute_split_bits``, ``split_matrix``,
``cross_gemm``, ``ozaki_matmul``); the device work goes through the C ABI of
liboz_b200.so (hand-written sm_100a kernels).  Nothing here computes on the
CPU and there is no Triton and no autotuner.

Differences from the reference, all deliberate:
* ``num_splits`` may be 1..8 (the reference stops at 4, ozaki_triton.py:563);
* broadcast batch dimensions are not materialised: each distinct A and B
  batch member is split once and the GEMM indexes them per output batch
  (the reference copies the expanded operands, ozaki_triton.py:528-529);
* slices are stored with their rows padded to a multiple of 128 bytes (the
  tensor-memory-access tile width); ``split_matrix`` returns a view with the
  reference's shape (B, s, M, K);
* ``residual="exact"`` keeps the residual in fp64 between levels (the
  reference rounds it to fp32, ozaki_triton.py:233); the default ``"auto"``
  uses the reference's fp32 rounding for num_splits <= 4 (bit-exact slices)
  and fp64 for num_splits > 4, where FP64 inputs need it to reach FP64
  accuracy;
* ``skip_tail=True`` drops the slice pairs with i + j >= num_splits.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib

# ozaki_triton.py:36-41 -- slice dtype -> (mantissa bits, is integer)
SLICE_DTYPE_INFO = {
    torch.float32: (23, False),
    torch.float16: (10, False),
    torch.bfloat16: (7, False),
    torch.int8: (7, True),
}

# ozaki_triton.py:43-49 -- accepted input dtypes (int8 inputs are split like
# fp32 ones and give an int8 C, truncated toward zero and saturated)
INPUT_DTYPES = {torch.float64, torch.float32, torch.float16, torch.bfloat16, torch.int8}

MAX_SPLITS = 8

_OZ_DTYPE = {
    torch.float64: _lib.OZ_F64,
    torch.float32: _lib.OZ_F32,
    torch.float16: _lib.OZ_F16,
    torch.bfloat16: _lib.OZ_BF16,
    torch.int8: _lib.OZ_I8,
}


def select_dot_accum_dtype(slice_dtype: torch.dtype) -> torch.dtype:
    """Tensor-core accumulator: int32 for int8 slices, else fp32 (ozaki_triton.py:62-66)."""
    return torch.int32 if slice_dtype == torch.int8 else torch.float32


def select_out_accum_dtype(input_dtype: torch.dtype) -> torch.dtype:
    """Outer accumulator: fp64 for fp64 inputs, else fp32 (ozaki_triton.py:69-73)."""
    return torch.float64 if input_dtype == torch.float64 else torch.float32


def compute_split_bits(n: int, slice_dtype: torch.dtype = torch.float16,
                       dot_accum_dtype: torch.dtype = torch.float32) -> int:
    """alpha = int((acc_bits - log2 n) / 2), capped by the slice bits (ozaki_triton.py:76-98).

    Raises ValueError for an unknown accumulator or n <= 0 and AssertionError
    when alpha < 1, like the reference.
    """
    if dot_accum_dtype == torch.int32:
        acc_bits = 31
    elif dot_accum_dtype == torch.float32:
        acc_bits = 23
    else:
        raise ValueError(f"unsupported dot_accum_dtype: {dot_accum_dtype}")
    slice_bits, _ = SLICE_DTYPE_INFO[slice_dtype]
    alpha = int((acc_bits - math.log2(n)) / 2)
    alpha = min(alpha, slice_bits)
    assert alpha >= 1, f"n={n} too large to split safely (alpha={alpha})"
    return alpha


def slice_row_elems(k: int, slice_dtype: torch.dtype) -> int:
    """Row pitch (elements) of the library's slice layout: k padded to 128 bytes."""
    es = torch.empty((), dtype=slice_dtype).element_size()
    return ((k * es + 127) // 128 * 128) // es if k > 0 else 0


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(device: torch.device) -> int:
    """The current CUDA stream of ``device`` as an address (the raw accessor
    when torch has it: a tenth of the host time of building a Stream object)."""
    if _RAW_STREAM is not None and device.index is not None:
        return _RAW_STREAM(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _residual_mode(residual: Optional[str], num_splits: int, input_dtype: torch.dtype) -> int:
    if residual in (None, "auto"):
        residual = "compat" if num_splits <= 4 else "exact"
    if residual == "compat":
        return _lib.OZ_RESIDUAL_COMPAT
    if residual == "exact":
        return _lib.OZ_RESIDUAL_EXACT
    raise ValueError(f"unknown residual mode {residual!r}")


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("ozaki_triton_b200 computes on CUDA tensors only "
                             f"(got a tensor on {t.device})")


def _split_lines(x3: torch.Tensor, stride_line: int, stride_k: int, lines: int, k: int,
                 num_splits: int, alpha: int, slice_dtype: torch.dtype, mode: int,
                 out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Split the lines of a (batch, ., .) view; returns padded slices + scales
    (written into ``out`` = contiguous (slices, scales) of that shape if given)."""
    batch = x3.shape[0]
    ld = slice_row_elems(k, slice_dtype)
    if out is not None:
        slices, scales = out
        assert slices.shape == (batch, num_splits, lines, ld) and slices.is_contiguous()
        assert scales.shape == (batch, num_splits, lines) and scales.is_contiguous()
        assert slices.dtype == slice_dtype and scales.dtype == torch.float32
    else:
        slices = torch.empty((batch, num_splits, lines, ld), dtype=slice_dtype, device=x3.device)
        scales = torch.empty((batch, num_splits, lines), dtype=torch.float32, device=x3.device)
    if batch == 0 or lines == 0:
        return slices, scales
    lib = _lib.load()
    code = _OZ_DTYPE[x3.dtype]
    ws_bytes = lib.oz_split_workspace_bytes(code, batch, lines, k, stride_line, stride_k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x3.device) if ws_bytes > 0 else None
    _lib.check(lib.oz_split_ex(
        x3.data_ptr(), code, batch, lines, k,
        x3.stride(0), stride_line, stride_k, num_splits, alpha, _OZ_DTYPE[slice_dtype], mode,
        slices.data_ptr(), ld, scales.data_ptr(), ws.data_ptr() if ws is not None else None,
        ws_bytes, _stream_ptr(x3.device)))
    return slices, scales


def split_matrix(A: torch.Tensor, num_splits: int, alpha: int, slice_dtype: torch.dtype,
                 residual: Optional[str] = "compat") -> Tuple[torch.Tensor, torch.Tensor]:
    """Split each row of A (B, M, K) into num_splits slices (ozaki_triton.py:214-256).

    Any strides are accepted (e.g. the transposed view of B).  Returns
    ``slices`` (B, num_splits, M, K) of ``slice_dtype`` -- a view of a buffer
    whose rows are padded to 128 bytes -- and ``scales`` (B, num_splits, M)
    fp32 powers of two.
    """
    assert A.dim() == 3
    _check_cuda(A)
    if A.dtype not in INPUT_DTYPES:
        raise AssertionError(f"unsupported input dtype: {A.dtype}")
    if slice_dtype not in SLICE_DTYPE_INFO:
        raise AssertionError(f"unsupported slice dtype: {slice_dtype}")
    B, M, K = A.shape
    mode = _residual_mode(residual, num_splits, A.dtype)
    slices, scales = _split_lines(A, A.stride(1), A.stride(2), M, K, num_splits, alpha,
                                  slice_dtype, mode)
    return slices[..., :K], scales


def _as_library_slices(t: torch.Tensor, k: int) -> Tuple[torch.Tensor, int]:
    """(batch, s, rows, k) K-contiguous slices in the padded library layout.

    Returns the padded base tensor and its row pitch; copies only when the
    given tensor is not already laid out that way.
    """
    batch, s, rows, kk = t.shape
    assert kk == k
    es = t.element_size()
    ld = t.stride(2)
    ok = (t.stride(3) == 1 and (ld * es) % 128 == 0 and ld >= k and t.stride(1) == rows * ld
          and t.stride(0) == s * rows * ld and t.data_ptr() % 16 == 0)
    if ok:
        base = t.as_strided((batch, s, rows, ld), (s * rows * ld, rows * ld, ld, 1))
        if ld == k or _pad_is_zero(base, k):
            return base, ld
    ld = slice_row_elems(k, t.dtype)
    buf = torch.zeros((batch, s, rows, ld), dtype=t.dtype, device=t.device)
    buf[..., :k] = t
    return buf, ld


def _pad_is_zero(base: torch.Tensor, k: int) -> bool:
    # slices produced by split_matrix carry zero padding; anything else is
    # re-laid out (checking costs one reduction, only for foreign tensors)
    return bool((base[..., k:] == 0).all().item())


def cross_gemm(A_slices: torch.Tensor, B_slices: torch.Tensor, A_scales: torch.Tensor,
               B_scales: torch.Tensor, num_splits: int, output_dtype: torch.dtype,
               skip_tail: bool = False, a_index: Optional[torch.Tensor] = None,
               b_index: Optional[torch.Tensor] = None, batch: Optional[int] = None
               ) -> torch.Tensor:
    """Fused cross-GEMM over all slice pairs (ozaki_triton.py:455-498).

    A_slices (BA, s, M, K); B_slices (BB, s, K, N) -- like the reference, the
    transposed view of K-contiguous (BB, s, N, K) storage; scales fp32
    (BA, s, M) / (BB, s, N).  Returns C (batch, M, N) in ``output_dtype``.
    ``a_index`` / ``b_index`` (int32, CUDA) pick the A / B batch member of each
    output batch (torch.matmul broadcasting); by default batch b uses member b.
    """
    assert A_slices.dim() == 4 and B_slices.dim() == 4
    _check_cuda(A_slices, B_slices, A_scales, B_scales)
    BA, s, M, K = A_slices.shape
    BB, _, K2, N = B_slices.shape
    assert K == K2
    assert s == num_splits and B_slices.shape[1] == num_splits
    slice_dtype = A_slices.dtype
    assert B_slices.dtype == slice_dtype
    if batch is None:
        batch = BA if a_index is None else a_index.numel()
    C = torch.empty((batch, M, N), dtype=output_dtype, device=A_slices.device)
    if batch == 0 or M == 0 or N == 0:
        return C
    a_base, ld = _as_library_slices(A_slices, K)
    b_base, ldb = _as_library_slices(B_slices.transpose(-1, -2), K)
    assert ld == ldb
    sa = A_scales.contiguous().float()
    sb = B_scales.contiguous().float()
    lib = _lib.load()
    _lib.check(lib.oz_cross_gemm(
        a_base.data_ptr(), b_base.data_ptr(), sa.data_ptr(), sb.data_ptr(),
        batch, M, N, K, ld, num_splits, _OZ_DTYPE[slice_dtype], _OZ_DTYPE[output_dtype],
        a_index.data_ptr() if a_index is not None else None,
        b_index.data_ptr() if b_index is not None else None,
        BA, BB, C.data_ptr(), N, _lib.OZ_GEMM_SKIP_TAIL if skip_tail else 0,
        _stream_ptr(A_slices.device)))
    return C


def broadcast_batch(a: Tuple[int, ...], b: Tuple[int, ...]) -> Tuple[int, ...]:
    """torch.broadcast_shapes of two batch shapes (ozaki_triton.py:518), as plain
    tuple arithmetic: the torch call costs about 0.1 ms of host time, more
    than a whole small product on the GPU.  Raises RuntimeError like torch."""
    n = max(len(a), len(b))
    pa = (1,) * (n - len(a)) + tuple(a)
    pb = (1,) * (n - len(b)) + tuple(b)
    out = []
    for x, y in zip(pa, pb):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise RuntimeError(f"Shape mismatch: objects cannot be broadcast to a single shape. "
                               f"Mismatch is between {tuple(a)} and {tuple(b)}.")
    return tuple(out)


def _batch_index(own: Tuple[int, ...], full: Tuple[int, ...], device) -> Optional[torch.Tensor]:
    """Member of an operand with batch shape ``own`` used by each batch of ``full``."""
    if tuple(own) == tuple(full):
        return None
    n_own = math.prod(own)
    idx = torch.arange(n_own, dtype=torch.int32).reshape(own) if own else torch.zeros(
        (), dtype=torch.int32)
    idx = idx.expand(full).reshape(-1)
    return idx.to(device, non_blocking=True)


def ozaki_matmul(A: torch.Tensor, B: torch.Tensor, num_splits: int = 3,
                 slice_dtype: torch.dtype = torch.float16, verbose: bool = False, *,
                 skip_tail: bool = False, residual: Optional[str] = "auto") -> torch.Tensor:
    """C = A @ B emulated with low-precision tensor-core slices (ozaki_triton.py:534-606).

    A: (..., M, K), B: (..., K, N) of the same dtype (fp64/fp32/fp16/bf16),
    batch dims broadcast like torch.matmul.  Returns (broadcast(...), M, N)
    in the input dtype.
    """
    assert A.dtype == B.dtype, f"A/B dtype mismatch: {A.dtype} vs {B.dtype}"
    assert A.dtype in INPUT_DTYPES, f"unsupported input dtype: {A.dtype}"
    assert slice_dtype in SLICE_DTYPE_INFO, f"unsupported slice dtype: {slice_dtype}"
    assert 1 <= num_splits <= MAX_SPLITS, \
        f"num_splits must be in [1, {MAX_SPLITS}], got {num_splits}"
    assert A.dim() >= 2 and B.dim() >= 2
    M, K = A.shape[-2:]
    K2, N = B.shape[-2:]
    assert K == K2, f"contraction dim mismatch: A K={K}, B K={K2}"
    _check_cuda(A, B)

    key = (A.dtype, slice_dtype, num_splits, A.shape, A.stride(), B.shape, B.stride(),
           residual, bool(skip_tail), A.device)
    plan = _PLANS.get(key)
    if plan is None:
        plan = _matmul_plan(A, B, num_splits, slice_dtype, residual, skip_tail)
        if len(_PLANS) >= 256:
            _PLANS.clear()
        _PLANS[key] = plan
    if verbose and plan.log_line is not None:
        print(plan.log_line)
    if plan.empty:
        return torch.empty(plan.out_shape, dtype=A.dtype, device=A.device)
    # each distinct batch member is split once (no broadcast copies); one
    # library call splits B by columns and A by rows into the workspace and
    # runs the fused cross-GEMM
    if plan.flat:
        a_ptr, b_ptr = A.data_ptr(), B.data_ptr()
        a_st, b_st = plan.a_strides, plan.b_strides
    else:
        A3 = A.reshape(plan.a_batches, plan.m, plan.k)
        B3 = B.reshape(plan.b_batches, plan.k, plan.n)
        a_ptr, b_ptr = A3.data_ptr(), B3.data_ptr()
        a_st, b_st = A3.stride(), B3.stride()
    ws = torch.empty(plan.ws_alloc, dtype=torch.uint8, device=A.device)
    C = torch.empty(plan.c_shape, dtype=A.dtype, device=A.device)
    _lib.check(plan.lib.oz_matmul(
        a_ptr, b_ptr, plan.code, plan.bn, plan.a_batches, plan.b_batches, plan.a_idx, plan.b_idx,
        plan.m, plan.n, plan.k, a_st[0], a_st[1], a_st[2], b_st[0], b_st[1], b_st[2],
        num_splits, plan.scode, plan.mode, C.data_ptr(), plan.n, plan.flags,
        ws.data_ptr(), plan.ws_bytes, _stream_ptr(A.device)))
    return C.view(plan.out_shape)


class _MatmulPlan:
    """What ``ozaki_matmul`` derives from the operands' dtypes, shapes and
    strides alone (alpha, the batch index arrays, the workspace size, the
    output shape), kept per distinct call signature so that a repeated small
    product pays only for its allocations and one library call."""
    __slots__ = ("empty", "out_shape", "log_line", "flat", "a_strides", "b_strides", "a_batches",
                 "b_batches", "m", "n", "k", "bn", "code", "scode", "mode", "flags", "ws_bytes",
                 "ws_alloc", "c_shape", "a_idx", "b_idx", "a_idx_t", "b_idx_t", "lib")


_PLANS = {}


def _matmul_plan(A, B, num_splits, slice_dtype, residual, skip_tail) -> _MatmulPlan:
    p = _MatmulPlan()
    input_dtype = A.dtype
    M, K = A.shape[-2:]
    N = B.shape[-1]
    dot_accum_dtype = select_dot_accum_dtype(slice_dtype)
    a_batch, b_batch = tuple(A.shape[:-2]), tuple(B.shape[:-2])
    batch_shape = broadcast_batch(a_batch, b_batch)
    BN = math.prod(batch_shape)
    p.out_shape = (*batch_shape, M, N)
    p.log_line = None
    p.empty = BN == 0
    if p.empty:
        return p
    alpha = compute_split_bits(K, slice_dtype=slice_dtype, dot_accum_dtype=dot_accum_dtype)
    p.log_line = (f"[Ozaki] batch={batch_shape}, M={M}, K={K}, N={N}, "
                  f"input={input_dtype}, slice={slice_dtype}, "
                  f"dot_accum={dot_accum_dtype}, out_accum={select_out_accum_dtype(input_dtype)}, "
                  f"splits={num_splits}, alpha={alpha}")
    p.empty = M == 0 or N == 0
    if p.empty:
        return p
    p.m, p.n, p.k, p.bn = M, N, K, BN
    p.mode = _residual_mode(residual, num_splits, input_dtype)
    p.a_batches, p.b_batches = math.prod(a_batch), math.prod(b_batch)
    p.flat = A.dim() == 2 and B.dim() == 2
    A3 = A.reshape(p.a_batches, M, K)
    B3 = B.reshape(p.b_batches, K, N)
    p.a_strides, p.b_strides = A3.stride(), B3.stride()
    p.a_idx_t = _batch_index(a_batch, batch_shape, A.device)
    p.b_idx_t = _batch_index(b_batch, batch_shape, A.device)
    p.a_idx = p.a_idx_t.data_ptr() if p.a_idx_t is not None else None
    p.b_idx = p.b_idx_t.data_ptr() if p.b_idx_t is not None else None
    p.lib = _lib.load()
    p.code, p.scode = _OZ_DTYPE[input_dtype], _OZ_DTYPE[slice_dtype]
    p.flags = _lib.OZ_GEMM_SKIP_TAIL if skip_tail else 0
    p.ws_bytes = p.lib.oz_matmul_workspace_bytes(p.code, p.a_batches, p.b_batches, M, N, K,
                                                 p.a_strides[1], p.a_strides[2], p.b_strides[1],
                                                 p.b_strides[2], num_splits, p.scode)
    p.ws_alloc = max(p.ws_bytes, 1)
    p.c_shape = (BN, M, N)
    return p


_STREAMS = {}


def _side_streams(dev: torch.device):
    """Three side streams per device, created once (copy-in, compute, copy-out)."""
    key = dev.index
    if key not in _STREAMS:
        _STREAMS[key] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return _STREAMS[key]


def ozaki_matmul_from_host(A: torch.Tensor, B: torch.Tensor, num_splits: int = 3,
                           slice_dtype: torch.dtype = torch.float16, *,
                           device: Optional[torch.device] = None, row_blocks: int = 16,
                           skip_tail: bool = False, residual: Optional[str] = "auto",
                           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``ozaki_matmul`` for operands in (pinned) host memory; returns C on the host.

    The host<->device copies are pipelined with the device work: B is copied
    first and split as soon as it has arrived, A follows in ``row_blocks`` row
    blocks whose splits and GEMMs start as each block lands, and every block of
    C goes back while the next is computed (the link is full duplex).  All
    work is enqueued on side streams joined to the current stream: like a
    ``non_blocking`` copy, the returned tensor is ready once the current CUDA
    stream has been synchronised.  Operands that are not 2-D, not contiguous or
    not pinned take the plain path (copy, ``ozaki_matmul``, copy back).
    """
    assert A.dtype == B.dtype, f"A/B dtype mismatch: {A.dtype} vs {B.dtype}"
    assert A.dtype in INPUT_DTYPES, f"unsupported input dtype: {A.dtype}"
    assert slice_dtype in SLICE_DTYPE_INFO, f"unsupported slice dtype: {slice_dtype}"
    assert 1 <= num_splits <= MAX_SPLITS, \
        f"num_splits must be in [1, {MAX_SPLITS}], got {num_splits}"
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    main = torch.cuda.current_stream(dev)
    if (A.dim() != 2 or B.dim() != 2 or not A.is_contiguous() or not B.is_contiguous()
            or not A.is_pinned() or not B.is_pinned()):
        c = ozaki_matmul(A.to(dev, non_blocking=True), B.to(dev, non_blocking=True), num_splits,
                         slice_dtype, skip_tail=skip_tail, residual=residual)
        host = out if out is not None else torch.empty(c.shape, dtype=c.dtype, pin_memory=True)
        host.copy_(c, non_blocking=True)
        return host
    M, K = A.shape
    K2, N = B.shape
    assert K == K2, f"contraction dim mismatch: A K={K}, B K={K2}"
    dt = A.dtype
    C_host = out if out is not None else torch.empty((M, N), dtype=dt, pin_memory=True)
    if M == 0 or N == 0:
        return C_host
    alpha = compute_split_bits(K, slice_dtype=slice_dtype,
                               dot_accum_dtype=select_dot_accum_dtype(slice_dtype))
    mode = _residual_mode(residual, num_splits, dt)
    h2d, comp, d2h = _side_streams(dev)
    for st in (h2d, comp, d2h):
        st.wait_stream(main)
    lib = _lib.load()
    blocks = max(1, min(row_blocks, (M + 127) // 128))
    bounds = []
    for i in range(blocks):
        r0 = (M * i // blocks) // 128 * 128 if i else 0
        r1 = M if i == blocks - 1 else (M * (i + 1) // blocks) // 128 * 128
        if r1 > r0:
            bounds.append((r0, r1))
    with torch.cuda.stream(h2d):
        Bd = B.to(dev, non_blocking=True)
        ev_b = torch.cuda.Event()
        ev_b.record(h2d)
        Ad = torch.empty((M, K), dtype=dt, device=dev)
        ev_a = []
        for r0, r1 in bounds:
            Ad[r0:r1].copy_(A[r0:r1], non_blocking=True)
            e = torch.cuda.Event()
            e.record(h2d)
            ev_a.append(e)
    Cd = torch.empty((M, N), dtype=dt, device=dev)
    with torch.cuda.stream(comp):
        comp.wait_event(ev_b)
        B3 = Bd.reshape(1, K, N)
        b_sl, b_sc = _split_lines(B3, B3.stride(2), B3.stride(1), N, K, num_splits, alpha,
                                  slice_dtype, mode)
        ev_c = []
        for (r0, r1), e in zip(bounds, ev_a):
            comp.wait_event(e)
            A3 = Ad[r0:r1].reshape(1, r1 - r0, K)
            a_sl, a_sc = _split_lines(A3, A3.stride(1), A3.stride(2), r1 - r0, K, num_splits,
                                      alpha, slice_dtype, mode)
            _lib.check(lib.oz_cross_gemm(
                a_sl.data_ptr(), b_sl.data_ptr(), a_sc.data_ptr(), b_sc.data_ptr(), 1, r1 - r0,
                N, K, b_sl.shape[-1], num_splits, _OZ_DTYPE[slice_dtype], _OZ_DTYPE[dt], None,
                None, 1, 1, Cd[r0:r1].data_ptr(), N, _lib.OZ_GEMM_SKIP_TAIL if skip_tail else 0,
                comp.cuda_stream))
            ec = torch.cuda.Event()
            ec.record(comp)
            ev_c.append(ec)
    with torch.cuda.stream(d2h):
        for (r0, r1), e in zip(bounds, ev_c):
            d2h.wait_event(e)
            C_host[r0:r1].copy_(Cd[r0:r1], non_blocking=True)
    # the caller's stream sees everything; memory used on streams other than
    # the one it was allocated on is not reused before that work is done
    main.wait_stream(d2h)
    main.wait_stream(comp)
    main.wait_stream(h2d)
    Bd.record_stream(comp)
    Ad.record_stream(comp)
    Cd.record_stream(comp)
    Cd.record_stream(d2h)
    return C_host


def device_status() -> int:
    """Synchronise the current stream and return (and clear) the kernels'
    timeout code (0 = none).  Raises OzakiError if a bound was hit."""
    code = _lib.ctypes.c_int32(0)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.load().oz_device_status(st, _lib.ctypes.byref(code)))
    return code.value
