"""Plain-numpy restatement of the reference Ozaki split + cross-GEMM.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Every function cites
the line range of ``ozaki_triton.py`` (reference repository root) that it
restates.  Arrays are numpy; dtype "kinds" are the strings
``"fp64" "fp32" "fp16" "bf16" "int8"``.  BF16 values are carried in float32
arrays whose values are exactly representable in bfloat16.
"""

from __future__ import annotations

import math

import numpy as np

# ozaki_triton.py:36-41 -- slice dtype -> effective mantissa bits
SLICE_BITS = {"fp32": 23, "fp16": 10, "bf16": 7, "int8": 7}

# ozaki_triton.py:62-66 -- tl.dot accumulator: int32 for int8 slices, else fp32
def dot_accum_kind(slice_kind: str) -> str:
    return "int32" if slice_kind == "int8" else "fp32"


# ozaki_triton.py:69-73 -- outer accumulator / residual dtype
def out_accum_kind(input_kind: str) -> str:
    return "fp64" if input_kind == "fp64" else "fp32"


def compute_split_bits(n: int, slice_kind: str = "fp16", dot_accum: str = "fp32") -> int:
    """alpha = int((acc_bits - log2 n) / 2), capped by the slice bits.

    ozaki_triton.py:76-98.  Raises ValueError for n <= 0 (math.log2) and
    AssertionError when alpha < 1, exactly like the reference.
    """
    if dot_accum == "int32":
        acc_bits = 31
    elif dot_accum == "fp32":
        acc_bits = 23
    else:
        raise ValueError(f"unsupported dot_accum_dtype: {dot_accum}")
    alpha = int((acc_bits - math.log2(n)) / 2)
    alpha = min(alpha, SLICE_BITS[slice_kind])
    assert alpha >= 1, f"n={n} too large to split safely (alpha={alpha})"
    return alpha


def ceil_log2_f32(m: np.ndarray) -> np.ndarray:
    """ceil(float32(log2(m))) for positive float32 m (ozaki_triton.py:174).

    The reference evaluates ``tl.ceil(tl.log2(row_max))`` in float32.  The
    float32 log2 is formed here by rounding the float64 log2 to float32; the
    float64 value is ~1e-16 relative from the true log2 while the nearest
    float32 rounding boundary near the ceil decision is >= 2e-10 relative away
    (checked over every float32 binade by tests/test_oracle.py), so this equals
    the correctly rounded float32 log2 at every point where ceil can change.
    """
    m = np.asarray(m, dtype=np.float32)
    return np.ceil(np.log2(m.astype(np.float64)).astype(np.float32)).astype(np.int64)


def pow2_f32(e: np.ndarray) -> np.ndarray:
    """Exact float32 2**e for integer e in [-149, 127] (incl. subnormals)."""
    e = np.asarray(e, dtype=np.int64)
    return np.ldexp(np.ones(e.shape, dtype=np.float64), e).astype(np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float64/float32 values to bfloat16 (nearest, ties to even), once.

    Returned as float32 holding bfloat16-representable values.  This is the
    GPU semantics of Triton's ``.to(tl.bfloat16)`` (default rounding
    "rtne"); the Triton interpreter truncates instead, so BF16 slicing is not
    pinned by interpreter golden vectors.
    """
    x = np.asarray(x, dtype=np.float64)
    out = np.zeros_like(x)
    fin = np.isfinite(x) & (x != 0)
    m, e = np.frexp(x[fin])                # x = m * 2**e, 0.5 <= |m| < 1
    # quantum of bf16 at this magnitude: 2**(e-8), but never below the
    # smallest bf16 subnormal 2**-133
    q = np.maximum(e - 8, -133)
    r = np.rint(np.ldexp(x[fin], -q))       # rint = ties to even
    out[fin] = np.ldexp(r, q)
    out[~fin] = x[~fin]
    big = np.abs(out) > float(np.finfo(np.float32).max)
    # values beyond the largest bf16 (3.3895e38) round to inf in bf16
    bmax = float.fromhex("0x1.fep127")
    over = np.abs(out) > bmax
    out[over | big] = np.copysign(np.inf, out[over | big])
    return out.astype(np.float32)


def _rd(input_kind: str):
    return np.float64 if input_kind == "fp64" else np.float32


def _to_slice(x: np.ndarray, slice_kind: str, rd) -> np.ndarray:
    """One level's quantisation, ozaki_triton.py:196-202."""
    if slice_kind == "int8":
        half = rd(0.5)
        t = np.where(x >= 0, x + half, x - half).astype(rd)
        t = np.minimum(np.maximum(t, rd(-128)), rd(127))
        return np.trunc(t).astype(np.int8)
    if slice_kind == "fp16":
        return x.astype(np.float16)     # numpy rounds once, to nearest even
    if slice_kind == "bf16":
        return round_to_bf16(x)
    if slice_kind == "fp32":
        return x.astype(np.float32)
    raise ValueError(slice_kind)


def _slice_np_dtype(slice_kind: str):
    return {"int8": np.int8, "fp16": np.float16, "bf16": np.float32, "fp32": np.float32}[slice_kind]


def split_lines(x: np.ndarray, num_splits: int, alpha: int, slice_kind: str,
                input_kind: str, residual: str = "compat"):
    """Split every line of x (B, L, K) along K into num_splits slices.

    Restates ``split_matrix_kernel`` (ozaki_triton.py:136-211) and its
    wrapper (ozaki_triton.py:214-256):

    * residual dtype rd = float64 for fp64 input, else float32 (:227);
    * per level: row_max = max(float32(1e-38), float32(max|res|)) (:172,192),
      scale = float32(2**(ceil(log2 row_max) - alpha)) (:174);
    * x = res / scale in rd; int8: round half away from zero, clamp to
      [-128, 127], truncate (:196-200); float slices: one rounding (:202);
    * res -= q * scale in rd (:210), then the reference stores res in a
      *float32* buffer (:233) and reloads it (:188), i.e. res is rounded to
      float32 between levels.  ``residual="exact"`` keeps rd instead (the
      new FP64-accurate mode for num_splits > 4; identical for fp32 rd).

    Returns (slices (B, s, L, K), scales (B, s, L) float32).
    """
    x = np.asarray(x)
    assert x.ndim == 3
    B, L, K = x.shape
    rd = _rd(input_kind)
    res = x.astype(rd)
    slices = np.zeros((B, num_splits, L, K), dtype=_slice_np_dtype(slice_kind))
    scales = np.zeros((B, num_splits, L), dtype=np.float32)
    floor = np.float32(1e-38)
    for lvl in range(num_splits):
        if K > 0:
            mx = np.abs(res).max(axis=-1).astype(np.float32)
        else:
            mx = np.zeros((B, L), dtype=np.float32)
        row_max = np.maximum(floor, mx)
        scale = pow2_f32(ceil_log2_f32(row_max) - alpha)
        scales[:, lvl] = scale
        xs = (res / scale.astype(rd)[..., None]).astype(rd)
        q = _to_slice(xs, slice_kind, rd)
        slices[:, lvl] = q
        if lvl < num_splits - 1:
            prod = (q.astype(rd) * scale.astype(rd)[..., None]).astype(rd)
            res = (res - prod).astype(rd)
            if residual == "compat":
                res = res.astype(np.float32).astype(rd)
    return slices, scales


def cross_gemm(a_slices: np.ndarray, b_slices_t: np.ndarray, a_scales: np.ndarray,
               b_scales: np.ndarray, slice_kind: str, out_kind: str,
               skip_tail: bool = False) -> np.ndarray:
    """C = sum_i sum_j od(f32(f32(acc_ij) * sa_i) * sb_j), i-major, j-minor.

    Restates ``cross_gemm_kernel`` (ozaki_triton.py:305-452):
    acc_ij = A_i @ B_j exactly in int32 for int8 slices (:403-418), the
    epilogue multiplies in float32 in the order acc*sa*sb (:431) and adds
    into the outer accumulator od (float64 iff output fp64, :426,447),
    then casts to the output dtype (:452).

    a_slices (B, s, M, K); b_slices_t (B, s, N, K) -- the K-major storage the
    reference uses for B (``B_slices_T``, :594); scales (B, s, M) / (B, s, N).
    For float slices acc_ij is the float64 product rounded to float32 (the
    GPU's fp32 accumulation order is not reproducible; tolerance only).
    ``skip_tail`` drops pairs with i + j >= s (no reference counterpart).
    """
    Bn, s, M, K = a_slices.shape
    N = b_slices_t.shape[2]
    od = np.float64 if out_kind == "fp64" else np.float32
    out = np.zeros((Bn, M, N), dtype=od)
    af = a_slices.astype(np.float64)
    bf = b_slices_t.astype(np.float64)
    for i in range(s):
        sa = a_scales[:, i, :, None].astype(np.float32)
        for j in range(s):
            if skip_tail and i + j >= s:
                continue
            acc = np.matmul(af[:, i], np.swapaxes(bf[:, j], -1, -2))
            acc32 = acc.astype(np.float32)
            sb = b_scales[:, j, None, :].astype(np.float32)
            v = ((acc32 * sa).astype(np.float32) * sb).astype(np.float32)
            out = (out + v.astype(od)).astype(od)
    return _cast_out(out, out_kind)


def _cast_out(out: np.ndarray, out_kind: str) -> np.ndarray:
    if out_kind == "fp64":
        return out.astype(np.float64)
    if out_kind == "fp32":
        return out.astype(np.float32)
    if out_kind == "fp16":
        return out.astype(np.float16)
    if out_kind == "bf16":
        return round_to_bf16(out)
    if out_kind == "int8":
        # ozaki_triton.py:452 casts the fp32 accumulator to the int8 output.
        # Inside [-128, 127] that is truncation toward zero on every backend;
        # outside it the GPU conversion saturates (the interpreter's numpy
        # cast wraps), and this restatement follows the GPU: saturate, NaN -> 0.
        t = np.trunc(np.nan_to_num(out.astype(np.float64), nan=0.0))
        return np.clip(t, -128, 127).astype(np.int8)
    raise ValueError(out_kind)


def ozaki_matmul(a: np.ndarray, b: np.ndarray, num_splits: int, slice_kind: str,
                 input_kind: str, residual: str = "compat", skip_tail: bool = False):
    """End-to-end restatement of ``ozaki_matmul`` (ozaki_triton.py:534-606).

    Broadcasts the batch dims like ``_canonicalize_batch`` (:504-531),
    splits A by rows and B by columns (B is split through its transposed
    view, :593-594), and runs the cross-GEMM (:604).
    """
    M, K = a.shape[-2:]
    K2, N = b.shape[-2:]
    assert K == K2
    batch = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    BN = int(np.prod(batch)) if len(batch) else 1
    a3 = np.broadcast_to(a, (*batch, M, K)).reshape(BN, M, K)
    b3 = np.broadcast_to(b, (*batch, K, N)).reshape(BN, K, N)
    out_kind = input_kind
    if BN == 0:
        return np.zeros((*batch, M, N), dtype=a.dtype)
    alpha = compute_split_bits(K, slice_kind, dot_accum_kind(slice_kind))
    bs, bsc = split_lines(np.swapaxes(b3, -1, -2), num_splits, alpha, slice_kind,
                          input_kind, residual)
    as_, asc = split_lines(a3, num_splits, alpha, slice_kind, input_kind, residual)
    c = cross_gemm(as_, bs, asc, bsc, slice_kind, out_kind, skip_tail)
    return c.reshape(*batch, M, N)
