"""The BASELINE.json configurations at their full sizes on one B200.

Each product runs at its real shape through ``ozaki_matmul``; its parity is
checked on a sample of C: the split is per line (per-row scales of A,
per-column scales of B), so the block of C at sampled rows and columns is
reproduced exactly by the CPU oracle from those rows of A and columns of B.
int8 slices: bit for bit.  Float slices: the tensor cores sum each pair
product over K in fp32, the oracle rounds the exact product once, so within
the tolerance of the smaller float-slice tests.  Accuracy against an fp64
product is reported per configuration (and per num_splits for C5).  One
configuration's buffers are freed before the next.
"""

import numpy as np
import pytest
import torch

import bench
import oracle
import ozaki_triton_b200 as oz
from golden_cases import same_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _sample(total, k):
    pick = {0, 1, 127, 128, total // 2, total - 1}
    pick.update(np.linspace(0, total - 1, k - len(pick)).astype(int).tolist())
    return np.array(sorted(pick)[:k])


def _free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def test_c2_fp32_fp16_8192():
    """C2: FP32 -> FP16, s = 2, 8192^3, N(0, 1) from seed 1."""
    a_h, b_h = bench.config_inputs(bench.CONFIGS["C2"])
    a, b = a_h.to(DEV), b_h.to(DEV)
    c = oz.ozaki_matmul(a, b, num_splits=2, slice_dtype=torch.float16)
    ref = torch.matmul(a.double(), b.double())
    rel = ((c.double() - ref).norm() / ref.norm()).item()
    del ref
    # two fp16 slices with alpha = 5 keep ~21 bits of every element
    assert rel < 3e-5, rel
    rows, cols = _sample(8192, 48), _sample(8192, 48)
    want = oracle.ozaki_matmul(a_h.numpy()[rows], b_h.numpy()[:, cols], 2, "fp16", "fp32")
    got = c.cpu().numpy()[np.ix_(rows, cols)].astype(np.float64)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < max(1e-6, 2.5e-7 * np.sqrt(8192)), err
    assert oz.device_status() == 0
    del a, b, c
    _free()


def test_c4_broadcast_batches_fp64_fp16():
    """C4: FP64 -> FP16, s = 3, (16,1,2048,4096) x (1,8,4096,2048) -> 128
    GEMMs from 16 + 8 distinct operands; three output batches checked."""
    a_h, b_h = bench.config_inputs(bench.CONFIGS["C4"])
    a, b = a_h.to(DEV), b_h.to(DEV)
    c = oz.ozaki_matmul(a, b, num_splits=3, slice_dtype=torch.float16)
    assert c.shape == (16, 8, 2048, 2048)
    rows, cols = _sample(2048, 24), _sample(2048, 24)
    for i, j in [(0, 0), (7, 3), (15, 7)]:
        a_s = a_h[i, 0].numpy()[rows]
        b_s = b_h[0, j].numpy()[:, cols]
        want = oracle.ozaki_matmul(a_s, b_s, 3, "fp16", "fp64")
        got = c[i, j].cpu().numpy()[np.ix_(rows, cols)]
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert err < max(1e-6, 2.5e-7 * np.sqrt(4096)), (i, j, err)
        exact = a_s @ b_s
        assert np.linalg.norm(got - exact) / np.linalg.norm(exact) < 3e-5
    assert oz.device_status() == 0
    del a, b, c
    _free()


@pytest.fixture(scope="module")
def c5_inputs():
    return bench.config_inputs(bench.CONFIGS["C5"])


@pytest.mark.parametrize("s", [4, 6, 8])
def test_c5_fp64_int8_16384(s, c5_inputs):
    """C5: FP64 -> INT8, 16384^3 with a wide exponent spread (exp(4 N(0,1))):
    s = 4 with the reference's fp32 residual, s = 6 and 8 with the fp64
    residual (``residual="auto"``), each bit for bit on a sample and against
    an fp64 product, whose error falls with s."""
    a_h, b_h = c5_inputs
    a, b = a_h.to(DEV), b_h.to(DEV)
    c = oz.ozaki_matmul(a, b, num_splits=s, slice_dtype=torch.int8)
    ref = torch.matmul(a, b)
    rel = ((c - ref).norm() / ref.norm()).item()
    del ref
    bound = {4: 3e-7, 6: 1e-11, 8: 5e-15}[s]
    assert rel < bound, (s, rel)
    rows, cols = _sample(16384, 12), _sample(16384, 12)
    residual = "compat" if s <= 4 else "exact"
    want = oracle.ozaki_matmul(a_h.numpy()[rows], b_h.numpy()[:, cols], s, "int8", "fp64",
                               residual=residual)
    assert same_bits(c.cpu().numpy()[np.ix_(rows, cols)], want)
    assert oz.device_status() == 0
    del a, b, c
    _free()
