"""Loader for the committed golden vectors (made by tests/golden/make_golden.py)."""

from __future__ import annotations

import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _table():
    rows = []
    with open(os.path.join(GOLDEN, "cases.txt")) as fh:
        for line in fh:
            rows.append(line.split())
    return rows


def split_cases():
    """[(name, input_kind, slice_kind, s, layout, x, slices, scales, alpha)].

    For layout "rows" x is (B, L, K) and lines are rows; for "cols" x is the
    stored B matrix (B, K, L) and lines are its columns.
    """
    z = np.load(os.path.join(GOLDEN, "split_cases.npz"))
    out = []
    for r in _table():
        if r[0] != "split":
            continue
        name, ik, sk, s, layout = r[1], r[2], r[3], int(r[4]), r[8]
        meta = z[name + "/meta"]
        out.append(dict(name=name, input_kind=ik, slice_kind=sk, s=s, layout=layout,
                        x=z[name + "/x"], slices=z[name + "/slices"],
                        scales=z[name + "/scales"], alpha=int(meta[1])))
    return out


def c1_inputs():
    """The 256^3 fp32 config: U(-1, 1) from torch's CPU generator, seed 0."""
    import torch

    g = torch.Generator().manual_seed(0)
    a = torch.rand(256, 256, generator=g, dtype=torch.float32) * 2 - 1
    b = torch.rand(256, 256, generator=g, dtype=torch.float32) * 2 - 1
    return a, b


def matmul_cases():
    """[(name, input_kind, slice_kind, s, a, b, c)] (a/b/c numpy; fp16 as float32)."""
    z = np.load(os.path.join(GOLDEN, "matmul_cases.npz"))
    out = []
    for r in _table():
        if r[0] != "matmul":
            continue
        name, ik, sk, s = r[1], r[2], r[3], int(r[4])
        if name == "mm_c1":
            a, b = c1_inputs()
            chk = z["mm_c1/checksum"]
            assert abs(a.double().sum().item() - chk[0]) < 1e-9 and \
                abs(b.double().sum().item() - chk[1]) < 1e-9, "torch CPU generator drifted"
            out.append(dict(name=name, input_kind=ik, slice_kind=sk, s=s,
                            a=a.numpy(), b=b.numpy(), c=z["mm_c1/c"]))
            continue
        out.append(dict(name=name, input_kind=ik, slice_kind=sk, s=s,
                        a=z[name + "/a"], b=z[name + "/b"], c=z[name + "/c"]))
    return out


def np_input(x, kind):
    """Golden inputs are stored as float32 for fp16/bf16; return the right numpy dtype."""
    if kind == "fp16":
        return x.astype(np.float16)
    if kind == "fp64":
        return x.astype(np.float64)
    if kind == "int8":
        return x.astype(np.int8)
    return x.astype(np.float32)   # fp32, bf16 (bf16 values carried in float32)


def same_bits(a, b):
    """Bitwise equality that treats NaN == NaN (and distinguishes +0 / -0)."""
    a = np.asarray(a)
    b = np.asarray(b)
    if a.shape != b.shape:
        return False
    if a.dtype.kind == "f":
        a64 = a.astype(np.float64)
        b64 = b.astype(np.float64)
        both_nan = np.isnan(a64) & np.isnan(b64)
        eq = (a64 == b64) & (np.signbit(a64) == np.signbit(b64))
        return bool(np.all(eq | both_nan))
    return bool(np.array_equal(a, b))
