"""Generate the golden vectors in this folder from the reference implementation.

Runs the UNMODIFIED reference module ``ozaki_triton.py`` of
WhFanatic/Ozaki_triton on the CPU under ``TRITON_INTERPRET=1``.  Two shims
are needed because this machine has no GPU and no optuna:

* ``mytuner.optuna_autotune`` (imported at ozaki_triton.py:28) is replaced by
  a one-config ``triton.autotune``.  The split results do not depend on the
  tile config (the row max spans every K tile) and int8 cross-GEMM results
  are exact in int32, so the chosen config does not change those outputs;
* ``torch.cuda.Stream / current_stream / stream`` (ozaki_triton.py:588-601)
  become no-ops.

Usage (needs the reference checkout; not run by the tests)::

    python tests/golden/make_golden.py /path/to/Ozaki_triton

Writes ``split_cases.npz`` and ``matmul_cases.npz`` next to this file.
Inputs are stored as arrays; the two largest inputs (the 256^3 config) are
regenerated from their seeded torch CPU generator recipe instead and only a
checksum of them is stored.
"""

from __future__ import annotations

import contextlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference(ref_dir: str):
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    import triton

    shim = types.ModuleType("mytuner")
    cfg_keys = {"num_warps", "num_stages", "num_ctas", "maxnreg"}

    def optuna_autotune(param_space, key, prune_configs_by=None, n_trials=None, **kw):
        # one legal config: the smallest of every parameter
        first = {k: v[0] for k, v in param_space.items() if k not in cfg_keys}
        if "BLOCK_M" in first and "BLOCK_N" in first:
            first = {"BLOCK_M": 16, "BLOCK_N": 16, "BLOCK_K": 32}
        return triton.autotune([triton.Config(first)], key=key)

    shim.optuna_autotune = optuna_autotune
    sys.modules["mytuner"] = shim

    class _NoStream:
        def wait_stream(self, other):
            pass

    torch.cuda.Stream = lambda *a, **k: _NoStream()
    torch.cuda.current_stream = lambda *a, **k: _NoStream()
    torch.cuda.stream = lambda s: contextlib.nullcontext()
    sys.path.insert(0, ref_dir)
    import ozaki_triton  # noqa: E402

    return ozaki_triton


def special_rows(rng, K: int, input_kind: str) -> np.ndarray:
    """Edge-case rows shared by the split cases (all finite in the input dtype)."""
    rows = []
    rows.append(np.zeros(K))                                  # all zero: 1e-38 floor
    r = np.zeros(K); r[:4] = [1.0, 0.5, -1.0, 0.3]; rows.append(r)   # clamp at +128 -> 127
    lim = 20 if input_kind in ("fp64", "fp32") else 14
    r = np.ldexp(1.0, rng.integers(-lim, lim, K)) * rng.choice([-1, 1], K); rows.append(r)  # powers of two
    r = np.zeros(K); r[K // 2] = 3.0; rows.append(r)          # single nonzero
    k = np.arange(K)
    r = np.ldexp(1.0 + (k % 40) * 2.0 ** -23, (k % 31) - 15); rows.append(r)  # mantissas just above 1
    r = (rng.integers(-60, 60, K) + 0.5) * 2.0 ** -7; rows.append(r)  # exact .5 ties after scaling
    if input_kind in ("fp64", "fp32"):
        r = rng.standard_normal(K) * 1e-30; rows.append(r)    # tiny
        r = rng.standard_normal(K) * 1e20; rows.append(r)     # large
    else:
        r = rng.standard_normal(K) * 1e-6; rows.append(r)     # fp16 subnormal range
        r = rng.standard_normal(K) * 1e4; rows.append(r)      # large but finite
    if input_kind == "fp64":
        r = rng.standard_normal(K) * 1e-300; rows.append(r)   # below fp32 range
    return np.array(rows)


def spread(rng, shape):
    """randn with a per-line 10**U(-2, 2) factor (reference test.py:105-108)."""
    x = rng.standard_normal(shape)
    return x * 10.0 ** rng.uniform(-2, 2, shape[:-1] + (1,))


def c3_dist(rng, shape, sigma=1.0):
    """(U(0,1) - 0.5) * exp(sigma * N(0,1)) -- the headline input law."""
    return (rng.uniform(0, 1, shape) - 0.5) * np.exp(sigma * rng.standard_normal(shape))


def main(ref_dir: str):
    import torch

    oz = import_reference(ref_dir)
    tdt = {"fp64": torch.float64, "fp32": torch.float32, "fp16": torch.float16,
           "bf16": torch.bfloat16, "int8": torch.int8}
    rng = np.random.default_rng(20261201)
    split_out = {}
    # (name, input kind, slice kind, s, B, L, K, layout)
    split_cases = [
        ("rows_f64_i8_s4", "fp64", "int8", 4, 2, 24, 300, "rows"),
        ("rows_f64_i8_s1", "fp64", "int8", 1, 1, 16, 64, "rows"),
        ("rows_f32_i8_s3", "fp32", "int8", 3, 2, 20, 257, "rows"),
        ("rows_f64_f16_s3", "fp64", "fp16", 3, 2, 20, 190, "rows"),
        ("rows_f32_f16_s2", "fp32", "fp16", 2, 1, 24, 513, "rows"),
        ("rows_f64_f32_s2", "fp64", "fp32", 2, 1, 20, 96, "rows"),
        ("rows_f16_f32_s1", "fp16", "fp32", 1, 1, 12, 80, "rows"),
        ("rows_f16_i8_s2", "fp16", "int8", 2, 1, 12, 144, "rows"),
        ("rows_bf16_f32_s1", "bf16", "fp32", 1, 1, 12, 80, "rows"),
        ("rows_f32_f16_s4_k2048", "fp32", "fp16", 4, 1, 8, 2048, "rows"),
        ("cols_f64_i8_s4", "fp64", "int8", 4, 2, 70, 260, "cols"),
        ("cols_f32_f16_s2", "fp32", "fp16", 2, 1, 40, 129, "cols"),
        ("cols_f64_f16_s3", "fp64", "fp16", 3, 1, 33, 1040, "cols"),
        # int8 inputs (accepted by ozaki_triton.py:43-49); drawn from their own
        # generator so that the cases above keep their inputs
        ("rows_i8_i8_s2", "int8", "int8", 2, 1, 12, 96, "rows"),
        ("rows_i8_f32_s1", "int8", "fp32", 1, 1, 8, 64, "rows"),
        ("cols_i8_f16_s3", "int8", "fp16", 3, 1, 24, 80, "cols"),
        # more shapes and types, from their own generator as well
        ("rows_bf16_i8_s3", "bf16", "int8", 3, 1, 12, 200, "rows"),
        ("cols_f32_i8_s4", "fp32", "int8", 4, 1, 30, 300, "cols"),
        ("rows_f64_i8_s4_k8192", "fp64", "int8", 4, 1, 10, 8192, "rows"),
        ("cols_f64_i8_s2_k4100", "fp64", "int8", 2, 1, 12, 4100, "cols"),
        ("cols_f16_f16_s2", "fp16", "fp16", 2, 1, 16, 130, "cols"),
    ]
    extra_split = {"rows_bf16_i8_s3", "cols_f32_i8_s4", "rows_f64_i8_s4_k8192",
                   "cols_f64_i8_s2_k4100", "cols_f16_f16_s2"}
    rng_x = np.random.default_rng(9)
    rng_i8 = np.random.default_rng(8)
    for name, ik, sk, s, B, L, K, layout in split_cases:
        if ik == "int8":
            x = rng_i8.integers(-128, 128, (B, L, K)).astype(np.float64)
            x[0, 0] = 0; x[0, 1] = -128; x[0, 2] = 127          # zero, clamp-edge rows
            x[0, 3] = 0; x[0, 3, K // 2] = 5                     # single nonzero
            x[0, 4] = np.where(np.arange(K) % 2 == 0, 1, -1)     # alternating signs
        else:
            r = rng_x if name in extra_split else rng
            x = spread(r, (B, L, K))
            sp = special_rows(r, K, ik)
            assert np.all(np.isfinite(torch.from_numpy(sp).to(tdt[ik]).double().numpy()))
            n_sp = min(len(sp), L)
            x[0, :n_sp] = sp[:n_sp]
        t = torch.from_numpy(x).to(tdt[ik])
        if layout == "cols":
            # store B as (B, K, N) and split its transposed view, as
            # ozaki_triton.py:593-594 does
            b = t.transpose(-1, -2).contiguous()          # (B, K, L)
            view = b.transpose(-1, -2)
        else:
            b = t.contiguous()
            view = b
        alpha = oz.compute_split_bits(K, tdt[sk], oz._select_dot_accum_dtype(tdt[sk]))
        sl, sc = oz.split_matrix(view, s, alpha, tdt[sk])
        stored_in = b.float().numpy() if ik in ("fp16", "bf16") else b.numpy()
        split_out[name + "/x"] = stored_in
        split_out[name + "/slices"] = sl.float().numpy() if sk != "int8" else sl.numpy()
        split_out[name + "/scales"] = sc.numpy()
        split_out[name + "/meta"] = np.array([s, alpha], dtype=np.int64)
        print(name, "alpha", alpha)

    mm_out = {}
    # C1 of the benchmark configs: fp32 256^3 U(-1,1) from torch seed 0, fp16 slices, s=2
    g = torch.Generator().manual_seed(0)
    A = torch.rand(256, 256, generator=g, dtype=torch.float32) * 2 - 1
    Bm = torch.rand(256, 256, generator=g, dtype=torch.float32) * 2 - 1
    C = oz.ozaki_matmul(A, Bm, num_splits=2, slice_dtype=torch.float16)
    mm_out["mm_c1/checksum"] = np.array([A.double().sum().item(), Bm.double().sum().item()])
    mm_out["mm_c1/c"] = C.numpy()
    print("mm_c1", C.shape)

    mm_cases = [
        # name, input kind, slice kind, s, A shape, B shape, law
        ("mm_f64_i8_s4", "fp64", "int8", 4, (96, 200), (200, 72), "c3"),
        ("mm_f64_i8_s3_bcast", "fp64", "int8", 3, (3, 1, 20, 40), (1, 2, 40, 12), "spread"),
        ("mm_f64_f16_s3_bcast", "fp64", "fp16", 3, (2, 1, 24, 64), (1, 3, 64, 16), "normal"),
        ("mm_f32_i8_s2_odd", "fp32", "int8", 2, (65, 130), (130, 33), "spread"),
        ("mm_f32_i8_s4", "fp32", "int8", 4, (40, 160), (160, 48), "c3"),
        ("mm_f16_f32_s1", "fp16", "fp32", 1, (48, 64), (64, 40), "normal"),
        ("mm_f64_i8_s2_k1", "fp64", "int8", 2, (17, 1), (1, 9), "normal"),
        # int8 inputs and an int8 result: entries in [-3, 3] and K = 8 keep C
        # inside the int8 range (the reference's out-of-range conversion
        # depends on the backend)
        ("mm_i8_i8_s2", "int8", "int8", 2, (24, 8), (8, 16), "int_small"),
        ("mm_i8_f16_s1", "int8", "fp16", 1, (12, 6), (6, 10), "int_small"),
        # more shapes and types (own generator; no bf16 C: the interpreter's
        # float-to-bf16 conversion truncates, unlike the GPU's)
        ("mm_f64_i8_s4_k2048", "fp64", "int8", 4, (64, 2048), (2048, 32), "c3_x"),
        ("mm_f32_i8_s3_bcast", "fp32", "int8", 3, (2, 3, 16, 40), (3, 40, 8), "normal_x"),
    ]
    for name, ik, sk, s, ash, bsh, law in mm_cases:
        if law == "int_small":
            a = rng_i8.integers(-3, 4, ash).astype(np.float64)
            b = rng_i8.integers(-3, 4, bsh).astype(np.float64)
        elif law == "normal_x":
            a = rng_x.standard_normal(ash); b = rng_x.standard_normal(bsh)
        elif law == "c3_x":
            a = c3_dist(rng_x, ash); b = c3_dist(rng_x, bsh)
        elif law == "c3":
            a = c3_dist(rng, ash); b = c3_dist(rng, bsh)
        elif law == "spread":
            a = spread(rng, ash); b = np.swapaxes(spread(rng, bsh[:-2] + (bsh[-1], bsh[-2])), -1, -2)
        else:
            a = rng.standard_normal(ash); b = rng.standard_normal(bsh)
        ta = torch.from_numpy(np.ascontiguousarray(a)).to(tdt[ik])
        tb = torch.from_numpy(np.ascontiguousarray(b)).to(tdt[ik])
        C = oz.ozaki_matmul(ta, tb, num_splits=s, slice_dtype=tdt[sk])
        f = (lambda t: t.float().numpy()) if ik in ("fp16", "bf16") else (lambda t: t.numpy())
        mm_out[name + "/a"] = f(ta)
        mm_out[name + "/b"] = f(tb)
        mm_out[name + "/c"] = f(C)
        mm_out[name + "/meta"] = np.array([s], dtype=np.int64)
        print(name, C.shape)

    np.savez_compressed(os.path.join(HERE, "split_cases.npz"), **split_out)
    np.savez_compressed(os.path.join(HERE, "matmul_cases.npz"), **mm_out)
    # the case table, for the tests
    with open(os.path.join(HERE, "cases.txt"), "w") as fh:
        for name, ik, sk, s, B, L, K, layout in split_cases:
            fh.write(f"split {name} {ik} {sk} {s} {B} {L} {K} {layout}\n")
        fh.write("matmul mm_c1 fp32 fp16 2 256x256 256x256 seed0\n")
        for name, ik, sk, s, ash, bsh, law in mm_cases:
            fh.write(f"matmul {name} {ik} {sk} {s} {'x'.join(map(str, ash))} "
                     f"{'x'.join(map(str, bsh))} {law}\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
