"""The CPU oracle against the reference's own outputs (golden vectors)."""

import math

import numpy as np
import pytest

import oracle
from golden_cases import matmul_cases, np_input, same_bits, split_cases

SPLITS = split_cases()
MATMULS = matmul_cases()


@pytest.mark.parametrize("case", SPLITS, ids=[c["name"] for c in SPLITS])
def test_split_oracle_matches_reference(case):
    x = np_input(case["x"], case["input_kind"])
    lines = x if case["layout"] == "rows" else np.swapaxes(x, -1, -2)
    sl, sc = oracle.split_lines(lines, case["s"], case["alpha"], case["slice_kind"],
                                case["input_kind"])
    assert same_bits(sc, case["scales"])
    assert same_bits(sl.astype(np.float64) if sl.dtype != np.int8 else sl,
                     case["slices"].astype(np.float64) if case["slices"].dtype != np.int8
                     else case["slices"])


@pytest.mark.parametrize("case", MATMULS, ids=[c["name"] for c in MATMULS])
def test_matmul_oracle_matches_reference(case):
    a = np_input(case["a"], case["input_kind"])
    b = np_input(case["b"], case["input_kind"])
    c = oracle.ozaki_matmul(a, b, case["s"], case["slice_kind"], case["input_kind"])
    ref = case["c"]
    assert c.shape == ref.shape
    if case["slice_kind"] == "int8":
        # int8 pair products are exact in int32: the whole C is bit-exact
        assert same_bits(c.astype(np.float64), ref.astype(np.float64))
    else:
        # float slices: the fp32 accumulation order inside the dot differs;
        # fp16 outputs may then round one ulp apart
        err = np.linalg.norm(c.astype(np.float64) - ref) / np.linalg.norm(ref)
        assert err < (2e-3 if case["input_kind"] in ("fp16", "bf16") else 1e-6)


def test_alpha_rule_configs():
    # ozaki_triton.py:76-98 at the benchmark configs' K
    assert oracle.compute_split_bits(256, "fp16", "fp32") == 7
    assert oracle.compute_split_bits(8192, "fp16", "fp32") == 5
    assert oracle.compute_split_bits(8192, "int8", "int32") == 7
    assert oracle.compute_split_bits(4096, "fp16", "fp32") == 5
    assert oracle.compute_split_bits(16384, "int8", "int32") == 7
    with pytest.raises(ValueError):
        oracle.compute_split_bits(0, "fp16", "fp32")
    with pytest.raises(AssertionError):
        oracle.compute_split_bits(2 ** 22, "fp16", "fp32")


def test_ceil_log2_every_binade():
    """ceil(fl32(log2 m)) via float64 equals numpy's float32 log2 path near the
    ceil decision in every float32 binade, with a wide margin."""
    worst = 1.0
    for e in range(-126, 128):
        k = np.arange(0, 200, dtype=np.int64)
        m = np.ldexp(1.0 + k * 2.0 ** -23, e).astype(np.float32)
        c_ref = np.ceil(np.log2(m)).astype(np.int64)
        assert np.array_equal(oracle.ceil_log2_f32(m), c_ref), e
        if e != 0:
            l64 = np.log2(m.astype(np.float64))
            nxt = float(np.nextafter(np.float32(e), np.float32(np.inf)))
            mid = (e + nxt) / 2
            worst = min(worst, float(np.min(np.abs(l64 - mid) / abs(mid))))
    assert worst > 1e-12
    # the 1e-38 floor is a float32 subnormal and gives exponent -126
    assert oracle.ceil_log2_f32(np.float32(1e-38)) == -126


def test_bf16_rounding_is_single_rtne():
    x = np.array([1 + 2 ** -8 + 2 ** -30, 1 + 2 ** -8, 1 + 3 * 2 ** -8, -0.3, 3.4e38])
    r = oracle.round_to_bf16(x)
    assert r[0] == np.float32(1 + 2 ** -7)      # above the tie: up (double rounding would give 1)
    assert r[1] == np.float32(1.0)              # tie to even
    assert r[2] == np.float32(1 + 2 ** -6)      # tie to even (up)
    assert r[3] == np.float32(-0.30078125)
    assert np.isinf(r[4])


def test_ceil_log2_table_matches_oracle():
    """The device's per-binade threshold table (generated header) gives the
    oracle's ceil(fl32(log2 m)) for every normal binade."""
    import os
    import re

    hdr = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                       "ozaki_triton_b200", "csrc", "oz_log2_table.h")
    txt = open(hdr).read()
    thr = np.array([int(v) for v in re.findall(r"-?\d+", txt.split("{", 1)[1])][:256])
    rng = np.random.default_rng(1)
    bits = rng.integers(0x00800000, 0x7F7FFFFF, 200_000).astype(np.uint32)
    k = np.arange(0, 200, dtype=np.uint32)
    edge = ((np.arange(1, 255, dtype=np.uint32)[:, None] << 23) | k[None, :]).ravel()
    bits = np.concatenate([bits, edge])
    m = bits.view(np.float32)
    b = (bits >> 23).astype(np.int64)
    c = b - 127 + ((bits & 0x7FFFFF).astype(np.int64) >= thr[b])
    assert np.array_equal(c, oracle.ceil_log2_f32(m))
