"""Parity of the CUDA path (through the C ABI) with the reference's golden
vectors and with the CPU oracle.  Needs a B200."""

import numpy as np
import pytest
import torch

import oracle
import ozaki_triton_b200 as oz
from golden_cases import matmul_cases, np_input, same_bits, split_cases

pytestmark = pytest.mark.gpu

TDT = {"fp64": torch.float64, "fp32": torch.float32, "fp16": torch.float16,
       "bf16": torch.bfloat16, "int8": torch.int8}
KINDS = {v: k for k, v in TDT.items()}
DEV = "cuda"


def to_dev(x_np, kind):
    return torch.from_numpy(np.ascontiguousarray(x_np)).to(TDT[kind]).to(DEV)


def host(t):
    if t.dtype == torch.bfloat16 or t.dtype == torch.float16:
        return t.float().cpu().numpy()
    return t.cpu().numpy()


def check_split(x_dev, lines_np, s, alpha, sk, ik, residual="compat"):
    """Run split_matrix on x_dev (B, L, K) (any strides) and compare with the oracle."""
    sl, sc = oz.split_matrix(x_dev, s, alpha, TDT[sk], residual=residual)
    rsl, rsc = oracle.split_lines(lines_np, s, alpha, sk, ik, residual=residual)
    torch.cuda.synchronize()
    assert oz.device_status() == 0
    assert same_bits(host(sc), rsc)
    got = host(sl)
    want = rsl if sk == "int8" else rsl.astype(np.float32)
    assert same_bits(got, want)


# ------------------------------------------------------------------ golden
SPLITS = split_cases()


@pytest.mark.parametrize("case", SPLITS, ids=[c["name"] for c in SPLITS])
def test_split_matches_reference_golden(case):
    ik, sk = case["input_kind"], case["slice_kind"]
    x = to_dev(case["x"], ik)
    view = x if case["layout"] == "rows" else x.transpose(-1, -2)
    sl, sc = oz.split_matrix(view, case["s"], case["alpha"], TDT[sk])
    torch.cuda.synchronize()
    assert same_bits(host(sc), case["scales"])
    got = host(sl)
    want = case["slices"]
    assert same_bits(got if sk == "int8" else got.astype(np.float64),
                     want if sk == "int8" else want.astype(np.float64))


@pytest.mark.parametrize("cta", ["default", "256", "512"])
@pytest.mark.parametrize("name", ["rows_f64_i8_s4_k8192", "cols_f64_i8_s2_k4100"])
def test_split_fp64_row_kernel_both_cta_shapes(name, cta, monkeypatch):
    """fp64 rows of 4097..8192 elements with an fp32 residual run by default
    on three 256-thread CTAs per SM that take level 0 from shared memory
    (split_rows_f64s); OZ_SPLIT_ROWS_CTA (read on every call) selects the
    register-resident kernels instead: two 256-thread CTAs per SM (256) or
    one 512-thread CTA (512, also the fallback when fewer CTAs are
    resident).  All are bit-exact on the K = 8192 and K = 4100 goldens,
    presented as contiguous rows."""
    if cta == "default":
        monkeypatch.delenv("OZ_SPLIT_ROWS_CTA", raising=False)
    else:
        monkeypatch.setenv("OZ_SPLIT_ROWS_CTA", cta)
    case = next(c for c in SPLITS if c["name"] == name)
    x = case["x"] if case["layout"] == "rows" else np.swapaxes(case["x"], -1, -2)
    xd = to_dev(np.ascontiguousarray(x), "fp64")
    from ozaki_triton_b200 import _lib
    n0 = _lib.load().oz_launch_count()
    sl, sc = oz.split_matrix(xd, case["s"], case["alpha"], torch.int8)
    torch.cuda.synchronize()
    assert _lib.load().oz_launch_count() - n0 == 1      # the row kernel, no generic fallback
    assert same_bits(host(sc), case["scales"])
    assert same_bits(host(sl), case["slices"])


MATMULS = matmul_cases()


@pytest.mark.parametrize("case", MATMULS, ids=[c["name"] for c in MATMULS])
def test_matmul_matches_reference_golden(case):
    ik, sk = case["input_kind"], case["slice_kind"]
    a, b = to_dev(case["a"], ik), to_dev(case["b"], ik)
    c = oz.ozaki_matmul(a, b, num_splits=case["s"], slice_dtype=TDT[sk])
    got = host(c).astype(np.float64)
    ref = case["c"].astype(np.float64)
    assert got.shape == ref.shape
    if sk == "int8":
        # int8 slice products are exact in int32 and the epilogue follows the
        # reference's order: bit-exact
        assert same_bits(got, ref)
    else:
        err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert err < (2e-3 if ik in ("fp16", "bf16") else 1e-6), err


# ------------------------------------------------------------------ split vs oracle
def rand_lines(rng, shape, kind):
    x = rng.standard_normal(shape) * 10.0 ** rng.uniform(-2, 2, shape[:-1] + (1,))
    if kind in ("fp16", "bf16"):
        x = np.clip(x, -6e4, 6e4)
    return x


COMBOS = [(ik, sk) for ik in ("fp64", "fp32", "fp16", "bf16") for sk in ("int8", "fp16", "bf16", "fp32")]


@pytest.mark.parametrize("ik,sk", COMBOS)
@pytest.mark.parametrize("K", [1, 37, 256, 1000, 1002, 4096])
def test_split_rows_all_dtypes(ik, sk, K):
    rng = np.random.default_rng(K * 31 + len(ik) * 7 + len(sk))
    x = rand_lines(rng, (2, 19, K), ik)
    xd = to_dev(x, ik)
    lines = host(xd).astype(np.float64 if ik == "fp64" else np.float32)
    s = 3
    alpha = oz.compute_split_bits(max(K, 1), TDT[sk], oz.select_dot_accum_dtype(TDT[sk]))
    check_split(xd, lines, s, alpha, sk, ik)


@pytest.mark.parametrize("ik,sk", [("fp64", "int8"), ("fp32", "fp16"), ("fp16", "int8"),
                                   ("bf16", "bf16"), ("fp64", "fp16"), ("fp32", "int8")])
@pytest.mark.parametrize("K", [5, 128, 1000, 3000, 8192, 16384])
def test_split_cols_all_sizes(ik, sk, K):
    """Columns of a row-major (K, N) matrix: the cluster kernel."""
    rng = np.random.default_rng(K + 5)
    N = 45
    b = rand_lines(rng, (1, N, K), ik)              # lines first, then store transposed
    bd = to_dev(np.swapaxes(b, -1, -2), ik)         # (1, K, N) row-major
    lines = host(bd).astype(np.float64 if ik == "fp64" else np.float32)
    lines = np.swapaxes(lines, -1, -2)
    alpha = oz.compute_split_bits(K, TDT[sk], oz.select_dot_accum_dtype(TDT[sk]))
    check_split(bd.transpose(-1, -2), lines, 4, alpha, sk, ik)


@pytest.mark.parametrize("residual", ["compat", "exact"])
@pytest.mark.parametrize("s", [1, 2, 5, 8])
def test_split_levels_and_residual_modes(residual, s):
    rng = np.random.default_rng(s)
    x = (rng.uniform(0, 1, (1, 33, 700)) - 0.5) * np.exp(4 * rng.standard_normal((1, 33, 700)))
    xd = to_dev(x, "fp64")
    check_split(xd, x, s, 7, "int8", "fp64", residual=residual)
    check_split(xd.transpose(-1, -2).contiguous().transpose(-1, -2), x, s, 7, "int8", "fp64",
                residual=residual)


def test_split_generic_strides():
    """Neither the split axis nor the lines contiguous: the generic kernel."""
    rng = np.random.default_rng(3)
    big = rng.standard_normal((2, 40, 3, 90))
    xd = to_dev(big, "fp64")[:, :, 1, :]            # (2, 40, 90), strides (10800, 270, 1)
    check_split(xd, big[:, :, 1, :], 4, 7, "int8", "fp64")
    xt = to_dev(big, "fp64").permute(0, 3, 2, 1)[:, :, 1, :]   # (2, 90, 40), both strided
    check_split(xt, np.ascontiguousarray(big.transpose(0, 3, 2, 1)[:, :, 1, :]), 3, 7, "fp16",
                "fp64")


def test_split_unaligned_row_pitch():
    """K not a multiple of the 16-byte vector: vector path refused, generic path used."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, 10, 77))
    xd = to_dev(x, "fp32")
    check_split(xd, x.astype(np.float32), 2, 6, "fp16", "fp32")


def test_split_edge_rows():
    K = 512
    rows = np.zeros((6, K))
    rows[1, :4] = [1.0, 0.5, -1.0, 0.3]
    rows[2, :] = 1e-300
    rows[3, ::3] = -2.0 ** 40
    rows[4, :] = np.ldexp(1.0 + np.arange(K) % 7 * 2.0 ** -23, np.arange(K) % 50 - 25)
    rows[5, :] = (np.arange(K) - 256 + 0.5) / 2.0 ** 7
    xd = to_dev(rows[None], "fp64")
    check_split(xd, rows[None], 4, 7, "int8", "fp64")
    check_split(xd.transpose(-1, -2).contiguous().transpose(-1, -2), rows[None], 4, 7, "int8",
                "fp64")


# ------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("s", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("shape", [(128, 128, 128), (200, 72, 300), (1, 1, 1), (257, 383, 1000)])
def test_int8_pair_products_exact(s, shape):
    """Each int8 pair product is exact in int32: with unit scales C is the
    exact integer sum over all pairs."""
    M, N, K = shape
    g = torch.Generator().manual_seed(M + N + K + s)
    a = torch.randint(-128, 128, (1, s, M, K), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (1, s, N, K), generator=g, dtype=torch.int8)
    sa = torch.ones((1, s, M))
    sb = torch.ones((1, s, N))
    c = oz.cross_gemm(a.to(DEV), b.to(DEV).transpose(-1, -2), sa.to(DEV), sb.to(DEV), s,
                      torch.float64)
    want = (a.sum(1).long()[0] @ b.sum(1).long()[0].T).double()
    assert torch.equal(c[0].cpu(), want)


@pytest.mark.parametrize("sk", ["int8", "fp16", "bf16", "fp32"])
@pytest.mark.parametrize("out", ["fp64", "fp32", "fp16", "bf16"])
def test_cross_gemm_dtypes_vs_oracle(sk, out):
    rng = np.random.default_rng(11)
    s, M, N, K = 3, 150, 140, 333
    a = rng.standard_normal((2, M, K)); b = rng.standard_normal((2, N, K))
    alpha = oz.compute_split_bits(K, TDT[sk], oz.select_dot_accum_dtype(TDT[sk]))
    asl, asc = oracle.split_lines(a, s, alpha, sk, "fp64")
    bsl, bsc = oracle.split_lines(b, s, alpha, sk, "fp64")
    want = oracle.cross_gemm(asl, bsl, asc, bsc, sk, out).astype(np.float64)
    def dev_slices(x):
        t = torch.from_numpy(x.astype(np.float32) if sk != "int8" else x)
        return t.to(TDT[sk]).to(DEV)
    c = oz.cross_gemm(dev_slices(asl), dev_slices(bsl).transpose(-1, -2),
                      torch.from_numpy(asc).to(DEV), torch.from_numpy(bsc).to(DEV), s, TDT[out])
    got = host(c).astype(np.float64)
    if sk == "int8" and out in ("fp64", "fp32"):
        assert same_bits(got, want)
    else:
        tol = {"fp64": 1e-6, "fp32": 1e-6, "fp16": 2e-3, "bf16": 1e-2}[out]
        if sk == "fp32":
            tol = max(tol, 2e-3)   # TF32 tensor-core inputs keep 10 mantissa bits
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert err < tol, err


@pytest.mark.parametrize("ik,sk,s", [("fp64", "int8", 4), ("fp32", "int8", 3), ("fp64", "int8", 6),
                                     ("fp64", "fp16", 3), ("fp32", "fp16", 2), ("fp64", "bf16", 3),
                                     ("fp16", "fp32", 1), ("bf16", "fp16", 2)])
@pytest.mark.parametrize("shape", [(300, 200, 520), (129, 64, 8192), (1024, 1024, 1024)])
def test_matmul_vs_oracle(ik, sk, s, shape):
    M, N, K = shape
    rng = np.random.default_rng(M * 3 + N + s)
    a = (rng.uniform(0, 1, (M, K)) - 0.5) * np.exp(rng.standard_normal((M, K)))
    b = (rng.uniform(0, 1, (K, N)) - 0.5) * np.exp(rng.standard_normal((K, N)))
    ad, bd = to_dev(a, ik), to_dev(b, ik)
    a_np = host(ad).astype(np.float64 if ik == "fp64" else np.float32)
    b_np = host(bd).astype(np.float64 if ik == "fp64" else np.float32)
    c = oz.ozaki_matmul(ad, bd, num_splits=s, slice_dtype=TDT[sk])
    residual = "compat" if s <= 4 else "exact"
    want = oracle.ozaki_matmul(a_np, b_np, s, sk, ik, residual=residual).astype(np.float64)
    got = host(c).astype(np.float64)
    if sk == "int8":
        assert same_bits(got, want)
    else:
        # the tensor cores accumulate each pair product over K in fp32 (as the
        # reference's tl.dot does); the oracle rounds the exact product once
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        tol = 2e-3 if ik in ("fp16", "bf16") else max(1e-6, 2.5e-7 * np.sqrt(K))
        assert err < tol, err


def test_broadcast_batch_semantics():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((4, 1, 3, 40, 64))
    b = rng.standard_normal((2, 1, 64, 24))
    ad, bd = to_dev(a, "fp64"), to_dev(b, "fp64")
    c = oz.ozaki_matmul(ad, bd, num_splits=4, slice_dtype=torch.int8)
    assert c.shape == torch.matmul(ad, bd).shape
    want = oracle.ozaki_matmul(a, b, 4, "int8", "fp64")
    assert same_bits(host(c), want)


@pytest.mark.parametrize("s", [2, 4])
def test_skip_tail_matches_oracle(s):
    """skip_tail drops the pairs i + j >= s; with s = 2 both A slices share a
    pass (the second one with one B slice)."""
    rng = np.random.default_rng(6)
    a = rng.standard_normal((96, 256)); b = rng.standard_normal((256, 80))
    c = oz.ozaki_matmul(to_dev(a, "fp64"), to_dev(b, "fp64"), num_splits=s,
                        slice_dtype=torch.int8, skip_tail=True)
    want = oracle.ozaki_matmul(a, b, s, "int8", "fp64", skip_tail=True)
    assert same_bits(host(c), want)


@pytest.mark.parametrize("sk,tile,s,batch", [
    ("int8", "2,128", 2, 1), ("int8", "1,128", 2, 1), ("fp16", "2,128", 2, 1),
    ("fp16", "1,64", 2, 1), ("fp32", "2,128", 2, 1), ("int8", "2,64", 3, 1),
    ("int8", "1,64", 3, 3), ("fp16", "2,64", 3, 2), ("int8", "1,64", 4, 1),
    ("int8", "2,64", 4, 2)])
def test_two_a_slices_per_pass_bit_identical(sk, tile, s, batch, monkeypatch):
    """When two A slices' accumulators fit TMEM (s = 2 with 128-column tiles,
    s <= 4 with 64) a GEMM pass covers two A slices; OZ_GEMM_PA=1 runs one per
    pass.  Both give the same bits: the same MMAs per pair and the same
    epilogue order.  With s = 3 the last pass has one slice, and its A box
    reaches into the next batch member's slices (or past the last one)."""
    rng = np.random.default_rng(78 + s + batch)
    M, N, K = 333, 260, 1500
    a = rng.standard_normal((batch, M, K)); b = rng.standard_normal((K, N))
    ad, bd = to_dev(a, "fp64"), to_dev(b, "fp64")
    monkeypatch.setenv("OZ_GEMM_TILE", tile)
    c2 = oz.ozaki_matmul(ad, bd, num_splits=s, slice_dtype=TDT[sk])
    monkeypatch.setenv("OZ_GEMM_PA", "1")
    c1 = oz.ozaki_matmul(ad, bd, num_splits=s, slice_dtype=TDT[sk])
    assert torch.equal(c1.view(torch.int64), c2.view(torch.int64))
    if sk == "int8":
        for i in range(batch):
            assert same_bits(host(c2[i]), oracle.ozaki_matmul(a[i], b, s, "int8", "fp64"))
    assert oz.device_status() == 0


def test_error_paths():
    a = torch.randn(8, 16, device=DEV, dtype=torch.float64)
    b = torch.randn(16, 4, device=DEV, dtype=torch.float64)
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a, b.float())
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a.to(torch.int32), b.to(torch.int32))
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a, b, num_splits=9)
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a, b, num_splits=0)
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a, torch.randn(15, 4, device=DEV, dtype=torch.float64))
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a, b, slice_dtype=torch.float64)
    with pytest.raises(ValueError):   # K == 0: log2(0), like the reference
        oz.ozaki_matmul(torch.zeros(3, 0, device=DEV), torch.zeros(0, 2, device=DEV))
    with pytest.raises(AssertionError):   # alpha < 1
        oz.ozaki_matmul(torch.zeros(1, 2 ** 22, device=DEV), torch.zeros(2 ** 22, 1, device=DEV),
                        num_splits=1, slice_dtype=torch.float16)
    # empty batch and empty M / N
    assert oz.ozaki_matmul(torch.zeros(0, 3, 4, device=DEV), torch.zeros(4, 2, device=DEV)).shape == (0, 3, 2)
    assert oz.ozaki_matmul(torch.zeros(0, 4, device=DEV), torch.zeros(4, 2, device=DEV)).shape == (0, 2)
    assert oz.device_status() == 0


def test_headline_size_properties():
    """8192^3 fp64 -> int8, s=4 at full size: exact against the oracle on a
    sample of rows x columns (the split is per line, so a sub-block of C is
    reproduced exactly from its A rows and B columns), and accuracy against
    an fp64 matmul."""
    M = N = K = 8192
    g = torch.Generator().manual_seed(2)
    a = (torch.rand(M, K, generator=g, dtype=torch.float64) - 0.5) * torch.exp(
        torch.randn(M, K, generator=g, dtype=torch.float64))
    b = (torch.rand(K, N, generator=g, dtype=torch.float64) - 0.5) * torch.exp(
        torch.randn(K, N, generator=g, dtype=torch.float64))
    ad, bd = a.to(DEV), b.to(DEV)
    c = oz.ozaki_matmul(ad, bd, num_splits=4, slice_dtype=torch.int8)
    ref = ad @ bd
    rel = ((c - ref).norm() / ref.norm()).item()
    # 4 int8 levels with the reference's fp32 residual carry ~30 bits
    assert rel < 3e-8, rel
    rows = np.array([0, 1, 127, 128, 4095, 8191])
    cols = np.array([0, 63, 64, 1000, 8190, 8191])
    want = oracle.ozaki_matmul(a.numpy()[rows], b.numpy()[:, cols], 4, "int8", "fp64")
    assert same_bits(c.cpu().numpy()[np.ix_(rows, cols)], want)


@pytest.mark.parametrize("sk,K,lines,s", [("int8", 1000, 63, 4), ("int8", 8192, 64, 4),
                                          ("fp16", 2048, 33, 3), ("fp32", 4100, 10, 2),
                                          ("bf16", 7, 5, 1)])
@pytest.mark.parametrize("residual", ["compat", "exact"])
def test_split_fp64_column_pairs(sk, K, lines, s, residual):
    """fp64 columns of a row-major B through the column-pair kernel (no
    transposed copy): an odd number of columns (the last panel's second
    column lies past the view and is zero-filled), batch 2, K not a multiple
    of the 2048-row chunk, every slice type, both residual modes."""
    rng = np.random.default_rng(K + lines)
    N = 64                                            # row pitch: 512 bytes
    b = rand_lines(rng, (2, N, K), "fp64")
    bd = to_dev(np.ascontiguousarray(np.swapaxes(b, -1, -2)), "fp64")   # (2, K, N)
    view = bd[:, :, :lines].transpose(-1, -2)         # (2, lines, K), lines contiguous
    lines_np = np.swapaxes(host(bd), -1, -2)[:, :lines]
    alpha = oz.compute_split_bits(K, TDT[sk], oz.select_dot_accum_dtype(TDT[sk]))
    check_split(view, lines_np, s, alpha, sk, "fp64", residual=residual)


@pytest.mark.parametrize("kind", ["default", "pairs"])
@pytest.mark.parametrize("sk,K,lines,s", [("int8", 8192, 67, 4), ("int8", 8100, 64, 3),
                                          ("fp16", 8192, 5, 2), ("int8", 8192, 1, 1),
                                          ("int8", 8065, 33, 4), ("bf16", 8130, 6, 3),
                                          ("fp32", 8192, 3, 2), ("int8", 8192, 601, 8),
                                          ("int8", 8192, 66, 4), ("fp16", 8192, 7, 3)])
def test_split_fp64_columns_k_split_over_a_cta_pair(kind, sk, K, lines, s, monkeypatch):
    """fp64 columns of 4097..8192 rows with 8192-element slice rows go by
    default to split_colpairs_kx (two CTAs of a cluster hold the upper and
    lower half of a column pair and exchange each level's partial maxima);
    OZ_SPLIT_COLS=pairs (read on every call) selects split_colpairs_tma.
    Odd and even column counts, K short of 8192 (zero rows at the end), every
    slice type, up to 8 levels, more panels than clusters, batch 2: one
    launch, bit-exact against the oracle."""
    if kind == "pairs":
        monkeypatch.setenv("OZ_SPLIT_COLS", "pairs")
    else:
        monkeypatch.delenv("OZ_SPLIT_COLS", raising=False)
    rng = np.random.default_rng(K + lines + s)
    N = max(80, (lines + 16) // 2 * 2)                # row pitch: a multiple of 16 bytes
    b = rand_lines(rng, (2, N, K), "fp64")
    bd = to_dev(np.ascontiguousarray(np.swapaxes(b, -1, -2)), "fp64")   # (2, K, N)
    view = bd[:, :, :lines].transpose(-1, -2)         # (2, lines, K), lines contiguous
    lines_np = np.swapaxes(host(bd), -1, -2)[:, :lines]
    alpha = oz.compute_split_bits(K, TDT[sk], oz.select_dot_accum_dtype(TDT[sk]))
    from ozaki_triton_b200 import _lib
    n0 = _lib.load().oz_launch_count()
    check_split(view, lines_np, s, alpha, sk, "fp64")
    assert _lib.load().oz_launch_count() - n0 == 1
    assert oz.device_status() == 0


def test_bounded_wait_times_out_and_the_context_stays_usable():
    """Failure detection without a GPU fault: a kernel waits on a barrier that
    nothing arrives on, gives up after a short bound (~0.1 s of SM cycles),
    records its code and returns; the host reads the timeout, and the next
    computation on the same context is correct."""
    from ozaki_triton_b200 import _lib
    lib = _lib.load()
    assert oz.device_status() == 0
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.oz_wait_selftest(200_000_000, st))
    with pytest.raises(_lib.OzakiError) as ei:
        oz.device_status()
    assert ei.value.status == _lib.OZ_ERR_TIMEOUT and "code 9" in str(ei.value)
    assert oz.device_status() == 0                      # the code was cleared by the read
    rng = np.random.default_rng(12)
    a = rng.standard_normal((200, 96)); b = rng.standard_normal((96, 72))
    c = oz.ozaki_matmul(to_dev(a, "fp64"), to_dev(b, "fp64"), num_splits=3,
                        slice_dtype=torch.int8)
    assert same_bits(host(c), oracle.ozaki_matmul(a, b, 3, "int8", "fp64"))
    assert lib.oz_wait_selftest(0, st) == _lib.OZ_ERR_INVALID


def test_launch_count_of_a_matmul():
    """oz_launch_count: a small fp64 matmul is two library kernels (both
    operands split in one launch, then the cross-GEMM); one with long rows
    (K = 8192: 64 KB fp64 lines) is three (split of A's rows, column-pair
    split of B, cross-GEMM) -- the count bench.py reports."""
    from ozaki_triton_b200 import _lib
    rng = np.random.default_rng(3)
    lib = _lib.load()
    for (m, k, n), want in [((512, 512, 256), 2), ((256, 8192, 256), 3)]:
        a = to_dev(rng.standard_normal((m, k)), "fp64")
        b = to_dev(rng.standard_normal((k, n)), "fp64")
        n0 = lib.oz_launch_count()
        oz.ozaki_matmul(a, b, num_splits=2, slice_dtype=torch.int8)
        assert lib.oz_launch_count() - n0 == want, (m, k, n)


@pytest.mark.parametrize("ik,sk,s", [("fp64", "int8", 4), ("fp64", "fp16", 3), ("fp32", "fp16", 2),
                                     ("fp32", "int8", 3), ("bf16", "fp32", 2), ("fp16", "bf16", 2),
                                     ("int8", "int8", 2), ("fp64", "int8", 8)])
@pytest.mark.parametrize("shape", [(3, 100, 70, 300), (1, 1024, 768, 1024), (2, 33, 40, 5000)])
def test_one_launch_split_matches_streaming_kernels(ik, sk, s, shape):
    """ozaki_matmul splits small operand pairs in one launch (one CTA per
    line, the line held in shared memory).  Its C is the same bits as the
    product of the separately launched streaming split kernels (split_matrix
    of A's rows and of B's transposed view, then cross_gemm)."""
    bn, m, n, k = shape
    rng = np.random.default_rng(m + n + k)
    a = to_dev(rand_lines(rng, (bn, m, k), ik), ik)
    b = to_dev(rand_lines(rng, (bn, k, n), ik), ik)
    got = oz.ozaki_matmul(a, b, num_splits=s, slice_dtype=TDT[sk])
    alpha = oz.compute_split_bits(k, TDT[sk], oz.select_dot_accum_dtype(TDT[sk]))
    mode = "compat" if s <= 4 else "exact"
    a_sl, a_sc = oz.split_matrix(a, s, alpha, TDT[sk], residual=mode)
    b_sl, b_sc = oz.split_matrix(b.transpose(-1, -2), s, alpha, TDT[sk], residual=mode)
    want = oz.cross_gemm(a_sl, b_sl.transpose(-1, -2), a_sc, b_sc, s, a.dtype)
    torch.cuda.synchronize()
    assert oz.device_status() == 0
    assert torch.equal(got.view(torch.uint8) if got.dtype != torch.int8 else got,
                       want.view(torch.uint8) if want.dtype != torch.int8 else want)


def test_int8_inputs_saturate_out_of_range():
    """int8 inputs (accepted by the reference) give an int8 C; results outside
    [-128, 127] saturate like the GPU's float-to-int8 conversion."""
    rng = np.random.default_rng(9)
    a = rng.integers(-128, 128, (40, 64)).astype(np.int8)
    b = rng.integers(-128, 128, (64, 24)).astype(np.int8)
    for sk in ("int8", "fp16"):
        c = oz.ozaki_matmul(to_dev(a, "int8"), to_dev(b, "int8"), num_splits=3,
                            slice_dtype=TDT[sk])
        assert c.dtype == torch.int8
        want = oracle.ozaki_matmul(a, b, 3, sk, "int8")
        assert same_bits(host(c), want)
        assert (want == 127).any() and (want == -128).any()       # saturation exercised


@pytest.mark.parametrize("tile", ["1,128", "2,128", "1,64", "2,64"])
@pytest.mark.parametrize("s", [2, 4])
def test_gemm_tile_configs_bit_identical(tile, s, monkeypatch):
    """Every tile-table entry (single CTA or CTA pair, 64 or 128 columns)
    gives the same bits for int8 slices, including ragged M/N edges."""
    rng = np.random.default_rng(77)
    M, N, K = 397, 300, 1100
    a = rng.standard_normal((M, K)); b = rng.standard_normal((K, N))
    ad, bd = to_dev(a, "fp64"), to_dev(b, "fp64")
    monkeypatch.setenv("OZ_GEMM_TILE", tile)
    c = oz.ozaki_matmul(ad, bd, num_splits=s, slice_dtype=torch.int8)
    want = oracle.ozaki_matmul(a, b, s, "int8", "fp64")
    assert same_bits(host(c), want)
    assert oz.device_status() == 0


@pytest.mark.parametrize("n,w,sk,tile", [(1000, 256, "int8", "2,128"), (1000, 128, "int8", "1,64"),
                                         (700, 128, "fp16", "2,128"), (300, 512, "int8", "2,128"),
                                         (384, 384, "int8", "1,128"), (130, 128, "fp32", "2,64")])
def test_gemm_column_blocked_b_bit_identical(n, w, sk, tile, monkeypatch):
    """oz_cross_gemm_blocked (B's slices in column blocks, the layout of the
    multi-GPU gather) gives the same bits as oz_cross_gemm on the plain layout,
    with the unused rows of the last block (and their scales) holding garbage."""
    from ozaki_triton_b200 import api
    from ozaki_triton_b200 import dist as ozd
    monkeypatch.setenv("OZ_GEMM_TILE", tile)
    rng = np.random.default_rng(5)
    M, K, s = 300, 520, 3
    a = to_dev(rng.standard_normal((1, M, K)), "fp64")
    b = to_dev(rng.standard_normal((1, K, n)), "fp64")
    sd = TDT[sk]
    alpha = oz.compute_split_bits(K, sd, oz.select_dot_accum_dtype(sd))
    a_sl, a_sc = api._split_lines(a, a.stride(1), a.stride(2), M, K, s, alpha, sd, 0)
    b_sl, b_sc = api._split_lines(b, b.stride(2), b.stride(1), n, K, s, alpha, sd, 0)
    be = ozd.Backend()
    want = be.gemm(a_sl, b_sl, a_sc, b_sc, 1, M, n, K, s, torch.float64, False)
    blocks = -(-n // w)
    ld = b_sl.shape[-1]
    g_sl = torch.full((1, blocks, s, w, ld), 77, dtype=torch.int8, device=DEV).view(sd) \
        if sk != "fp32" else torch.full((1, blocks, s, w, ld), 3.0e30, device=DEV)
    if sk == "fp16":
        g_sl = torch.full((1, blocks, s, w, ld), 6.0e4, dtype=sd, device=DEV)
    g_sc = torch.full((1, blocks, s, w), 1.0e30, device=DEV)
    for c in range(blocks):
        c0, c1 = c * w, min(n, (c + 1) * w)
        g_sl[0, c, :, :c1 - c0] = b_sl[0, :, c0:c1]
        g_sc[0, c, :, :c1 - c0] = b_sc[0, :, c0:c1]
    got = be.gemm(a_sl, g_sl, a_sc, g_sc, 1, M, n, K, s, torch.float64, False, b_block_cols=w)
    assert torch.equal(got, want)
    assert oz.device_status() == 0


def _blocked_operands(n, w, sk, seed=5, M=300, K=520, s=3):
    """A's slices, B's slices in the plain and in the column-blocked layout
    (unused rows of the last block hold garbage), and the plain GEMM's C."""
    from ozaki_triton_b200 import api
    from ozaki_triton_b200 import dist as ozd
    rng = np.random.default_rng(seed)
    a = to_dev(rng.standard_normal((1, M, K)), "fp64")
    b = to_dev(rng.standard_normal((1, K, n)), "fp64")
    sd = TDT[sk]
    alpha = oz.compute_split_bits(K, sd, oz.select_dot_accum_dtype(sd))
    a_sl, a_sc = api._split_lines(a, a.stride(1), a.stride(2), M, K, s, alpha, sd, 0)
    b_sl, b_sc = api._split_lines(b, b.stride(2), b.stride(1), n, K, s, alpha, sd, 0)
    want = ozd.Backend().gemm(a_sl, b_sl, a_sc, b_sc, 1, M, n, K, s, torch.float64, False)
    blocks = -(-n // w)
    ld = b_sl.shape[-1]
    g_sl = torch.full((1, blocks, s, w, ld), 77, dtype=torch.int8, device=DEV).view(sd) \
        if sk != "fp32" else torch.full((1, blocks, s, w, ld), 3.0e30, device=DEV)
    if sk == "fp16":
        g_sl = torch.full((1, blocks, s, w, ld), 6.0e4, dtype=sd, device=DEV)
    g_sc = torch.full((1, blocks, s, w), 1.0e30, device=DEV)
    for c in range(blocks):
        c0, c1 = c * w, min(n, (c + 1) * w)
        g_sl[0, c, :, :c1 - c0] = b_sl[0, :, c0:c1]
        g_sc[0, c, :, :c1 - c0] = b_sc[0, :, c0:c1]
    return dict(a_sl=a_sl, a_sc=a_sc, g_sl=g_sl, g_sc=g_sc, want=want, M=M, K=K, s=s,
                blocks=blocks)


@pytest.mark.parametrize("n,w,sk,tile,first,count", [(600, 256, "int8", "2,128", 1, 0),
                                                     (1000, 128, "int8", "1,64", 7, 0),
                                                     (700, 128, "fp16", "2,128", 0, 0),
                                                     (1024, 256, "int8", "1,64", 3, 3),
                                                     (1000, 128, "int8", "1,64", 5, 7),
                                                     (130, 128, "fp32", "2,64", 1, 1)])
def test_gemm_arriving_blocks_bit_identical(n, w, sk, tile, first, count, monkeypatch):
    """oz_cross_gemm_arrivals (one launch over column blocks that are still
    arriving, tiles in arrival order from first_block on) gives the bits of
    oz_cross_gemm on the columns of its block_count blocks and leaves the
    others alone: with every flag set before the launch, and with the flags
    set by copies on another stream that are held back behind a large
    host-to-device copy, so that the kernel waits for them.  A short last
    block (n = 600 with 256-column blocks: a tile past n that is skipped),
    garbage in the unused rows, every slice kind, all blocks or all but
    one (the multi-GPU use: every block except the rank's own)."""
    from ozaki_triton_b200 import dist as ozd
    from ozaki_triton_b200 import _lib
    monkeypatch.setenv("OZ_GEMM_TILE", tile)
    o = _blocked_operands(n, w, sk)
    be = ozd.Backend()
    lib = _lib.load()
    blocks = o["blocks"]
    run = [(first + i) % blocks for i in range(count or blocks)]
    cols = torch.zeros(n, dtype=torch.bool)
    for c in run:
        cols[c * w:(c + 1) * w] = True
    want = torch.where(cols.to(DEV), o["want"], torch.full_like(o["want"], -7.0))
    flags = torch.ones(blocks, dtype=torch.int32, device=DEV)
    got = torch.full_like(o["want"], -7.0)
    be.gemm(o["a_sl"], o["g_sl"], o["a_sc"], o["g_sc"], 1, o["M"], n, o["K"], o["s"],
            torch.float64, False, out=got, b_block_cols=w, ready=flags, first_block=first,
            block_count=count)
    torch.cuda.synchronize()
    assert oz.device_status() == 0
    assert torch.equal(got, want)
    # late flags: a copy stream sets them after ~200 MB of host-to-device copy
    flags.zero_()
    big_h = torch.empty(200 << 20, dtype=torch.uint8, pin_memory=True)
    big_d = torch.empty(200 << 20, dtype=torch.uint8, device=DEV)
    one_h = torch.ones(1, dtype=torch.int32, pin_memory=True)
    side = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        big_d.copy_(big_h, non_blocking=True)
        for c in range(o["blocks"]):
            _lib.check(lib.oz_copy_async(flags.data_ptr() + 4 * c, one_h.data_ptr(), 4,
                                         side.cuda_stream))
    got2 = torch.full_like(o["want"], -7.0)
    be.gemm(o["a_sl"], o["g_sl"], o["a_sc"], o["g_sc"], 1, o["M"], n, o["K"], o["s"],
            torch.float64, False, out=got2, b_block_cols=w, ready=flags, first_block=first,
            block_count=count)
    torch.cuda.synchronize()
    assert oz.device_status() == 0
    assert torch.equal(got2, want)


def test_gemm_arriving_block_that_never_arrives_times_out():
    """Failure detection without a GPU fault: a column block whose flag is
    never set makes the one-launch GEMM give up after its bounded wait (about
    2 s of SM clock), record code 5 and return; the host reads the timeout,
    and the next computation on the same context is correct."""
    from ozaki_triton_b200 import dist as ozd
    from ozaki_triton_b200 import _lib
    o = _blocked_operands(512, 256, "int8")
    be = ozd.Backend()
    flags = torch.tensor([1, 0], dtype=torch.int32, device=DEV)   # block 1 never arrives
    assert oz.device_status() == 0
    be.gemm(o["a_sl"], o["g_sl"], o["a_sc"], o["g_sc"], 1, o["M"], 512, o["K"], o["s"],
            torch.float64, False, b_block_cols=256, ready=flags, first_block=0)
    torch.cuda.synchronize()
    with pytest.raises(_lib.OzakiError) as ei:
        oz.device_status()
    assert ei.value.status == _lib.OZ_ERR_TIMEOUT and "code 5" in str(ei.value)
    assert oz.device_status() == 0
    flags[1] = 1
    got = be.gemm(o["a_sl"], o["g_sl"], o["a_sc"], o["g_sc"], 1, o["M"], 512, o["K"], o["s"],
                  torch.float64, False, b_block_cols=256, ready=flags, first_block=0)
    torch.cuda.synchronize()
    assert oz.device_status() == 0
    assert torch.equal(got, o["want"])


def test_gemm_arrivals_argument_errors():
    from ozaki_triton_b200 import _lib
    lib = _lib.load()
    o = _blocked_operands(512, 256, "int8")
    flags = torch.ones(2, dtype=torch.int32, device=DEV)
    c = torch.empty((1, o["M"], 512), dtype=torch.float64, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    args = lambda ready, first, width, count=0: (o["a_sl"].data_ptr(), o["g_sl"].data_ptr(),
                                        o["a_sc"].data_ptr(), o["g_sc"].data_ptr(), o["M"], 512,
                                        o["K"], o["a_sl"].shape[-1], o["s"], _lib.OZ_I8,
                                        _lib.OZ_F64, width, ready, 1, first, count,
                                        c.data_ptr(), 512, 0, st)
    assert lib.oz_cross_gemm_arrivals(*args(None, 0, 256)) == _lib.OZ_ERR_INVALID
    assert lib.oz_cross_gemm_arrivals(*args(flags.data_ptr(), 2, 256)) == _lib.OZ_ERR_INVALID
    assert lib.oz_cross_gemm_arrivals(*args(flags.data_ptr(), 0, 0)) == _lib.OZ_ERR_INVALID
    assert lib.oz_cross_gemm_arrivals(*args(flags.data_ptr(), 0, 256, 3)) == _lib.OZ_ERR_INVALID


@pytest.mark.parametrize("use_ws", [False, True])
@pytest.mark.parametrize("ik,sk,K,N", [("fp64", "int8", 8192, 70), ("fp64", "int8", 300, 70),
                                       ("fp32", "fp16", 1000, 70), ("bf16", "int8", 2048, 70),
                                       ("fp64", "fp32", 77, 70), ("fp32", "fp16", 1000, 64),
                                       ("fp32", "int8", 16384, 64), ("bf16", "fp16", 512, 64)])
def test_split_columns_c_abi_workspace_and_cluster(use_ws, ik, sk, K, N):
    """Columns of a row-major matrix through the C ABI: oz_split (cluster
    kernel where the layout allows it, no scratch) and oz_split_ex (fp32/fp16/
    bf16: the cluster kernel where it applies, else the transpose workspace;
    fp64: the workspace) give the same bits as the oracle.  N = 70 rows are
    not 16-byte aligned for fp32 (no cluster kernel); K = 16384 fp32 exceeds
    the cluster's reach (transpose path)."""
    from ozaki_triton_b200 import _lib
    from ozaki_triton_b200.api import _OZ_DTYPE
    rng = np.random.default_rng(K + len(ik))
    b = rand_lines(rng, (2, N, K), ik)
    bd = to_dev(np.ascontiguousarray(np.swapaxes(b, -1, -2)), ik)     # (2, K, N) row-major
    lines_np = np.swapaxes(host(bd).astype(np.float64 if ik == "fp64" else np.float32), -1, -2)
    s = 3
    alpha = oz.compute_split_bits(K, TDT[sk], oz.select_dot_accum_dtype(TDT[sk]))
    ld = oz.slice_row_elems(K, TDT[sk])
    sl = torch.empty((2, s, N, ld), dtype=TDT[sk], device=DEV)
    sc = torch.empty((2, s, N), dtype=torch.float32, device=DEV)
    lib = _lib.load()
    code = _OZ_DTYPE[TDT[ik]]
    st = torch.cuda.current_stream().cuda_stream
    if use_ws:
        nbytes = lib.oz_split_workspace_bytes(code, 2, N, K, 1, N)
        assert nbytes > 0
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        rc = lib.oz_split_ex(bd.data_ptr(), code, 2, N, K, K * N, 1, N, s, alpha,
                             _OZ_DTYPE[TDT[sk]], 0, sl.data_ptr(), ld, sc.data_ptr(),
                             ws.data_ptr(), nbytes, st)
    else:
        rc = lib.oz_split(bd.data_ptr(), code, 2, N, K, K * N, 1, N, s, alpha,
                          _OZ_DTYPE[TDT[sk]], 0, sl.data_ptr(), ld, sc.data_ptr(), st)
    _lib.check(rc)
    rsl, rsc = oracle.split_lines(lines_np, s, alpha, sk, ik)
    torch.cuda.synchronize()
    assert same_bits(host(sc), rsc)
    got = host(sl[..., :K])
    assert same_bits(got, rsl if sk == "int8" else rsl.astype(np.float32))
    # padding beyond K is zero
    assert not host(sl[..., K:]).any()


@pytest.mark.parametrize("ik,sk,s,shape", [("fp64", "int8", 4, (1000, 900, 700)),
                                           ("fp32", "fp16", 2, (520, 256, 384)),
                                           ("fp64", "int8", 3, (100, 50, 64))])
def test_from_host_pipeline_matches_device_call(ik, sk, s, shape):
    """The pipelined host-operand call gives the device call's bits."""
    M, N, K = shape
    g = torch.Generator().manual_seed(M + N)
    a = (torch.rand(M, K, generator=g, dtype=torch.float64) - 0.5).to(TDT[ik])
    b = (torch.rand(K, N, generator=g, dtype=torch.float64) - 0.5).to(TDT[ik])
    want = oz.ozaki_matmul(a.to(DEV), b.to(DEV), num_splits=s, slice_dtype=TDT[sk]).cpu()
    for _ in range(2):
        got = oz.ozaki_matmul_from_host(a.pin_memory(), b.pin_memory(), num_splits=s,
                                        slice_dtype=TDT[sk], row_blocks=3)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    # unpinned / batched operands take the plain path
    got = oz.ozaki_matmul_from_host(a, b, num_splits=s, slice_dtype=TDT[sk])
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_cuda_graph_capture_and_replay():
    """ozaki_matmul enqueues only stream-ordered work (no host sync, no
    allocation outside torch's allocator), so a step can be captured once
    and replayed -- the launch-bound small shapes gain the most."""
    g = torch.Generator().manual_seed(9)
    a = torch.rand(256, 256, generator=g).to(DEV) * 2 - 1
    b = torch.rand(256, 256, generator=g).to(DEV) * 2 - 1
    want = oz.ozaki_matmul(a, b, num_splits=2, slice_dtype=torch.float16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):                       # warm up outside the capture
            oz.ozaki_matmul(a, b, num_splits=2, slice_dtype=torch.float16)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = oz.ozaki_matmul(a, b, num_splits=2, slice_dtype=torch.float16)
    for scale in (1.0, 3.0):
        a.mul_(scale)
        graph.replay()
        torch.cuda.synchronize()
        ref = oz.ozaki_matmul(a, b, num_splits=2, slice_dtype=torch.float16)
        assert torch.equal(out, ref)
    assert oz.device_status() == 0
    del graph
