"""The allocation-free split entry point (oz_split_noalloc).

It exists for callers that cannot call cudaMalloc -- a foreign-function
binding that only holds the device pointers it was given, or a latency-
critical loop that cannot afford cudaMalloc's implicit device-wide
synchronisation -- and takes its transpose scratch from a fixed 32 MiB array
the library keeps in device memory.  This file is collected last so that a
run stopping at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _run(lib, fn, x, K, N, s, alpha, ws=None):
    from ozaki_triton_b200 import _lib
    ld = ((K + 127) // 128) * 128                          # int8 slice rows
    sl = torch.full((x.shape[0], s, N, ld), 77, dtype=torch.int8, device=DEV)
    sc = torch.full((x.shape[0], s, N), -1.0, dtype=torch.float32, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    # columns of the row-major (batch, K, N) input: lines are contiguous
    args = [x.data_ptr(), _lib.OZ_F64, x.shape[0], N, K, K * N, 1, N, s, alpha, _lib.OZ_I8,
            _lib.OZ_RESIDUAL_COMPAT, sl.data_ptr(), ld, sc.data_ptr()]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    rc = fn(*args, st)
    _lib.check(rc)
    torch.cuda.synchronize()
    return sl, sc


def test_noalloc_split_matches_workspace_split_twice():
    from ozaki_triton_b200 import _lib
    lib = _lib.load()
    assert lib.oz_split_noalloc_max_bytes() == 32 << 20
    g = torch.Generator().manual_seed(11)
    K, N, s, alpha = 1000, 300, 4, 7
    for call in range(2):      # the second call sees the first call's leftovers
        x = (torch.randn(2, K, N, generator=g, dtype=torch.float64) *
             10.0 ** (call * 3 - 1)).to(DEV)
        need = lib.oz_split_workspace_bytes(_lib.OZ_F64, 2, N, K, 1, N)
        assert 0 < need <= lib.oz_split_noalloc_max_bytes()
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        want_sl, want_sc = _run(lib, lib.oz_split_ex, x, K, N, s, alpha, ws)
        got_sl, got_sc = _run(lib, lib.oz_split_noalloc, x, K, N, s, alpha)
        assert torch.equal(got_sl, want_sl)
        assert torch.equal(got_sc, want_sc)


@pytest.mark.parametrize("K,N,batch", [(9000, 300, 1), (1000, 301, 2)])
def test_noalloc_transposes_into_the_fixed_array(K, N, batch):
    """Inputs that no column kernel takes go through the fixed array: fp64
    columns with K > 8192 (beyond the column-pair kernel's four 2048-row
    chunks), or an odd column count (a row pitch that is not a multiple of 16
    bytes, which TMA cannot address).  They are transposed into the array and
    split as rows: two launches.  Two calls in a row with different data (the
    second finds the first call's values in the array) give the same bits as
    oz_split_ex with a caller workspace, and as the CPU oracle."""
    import oracle
    from ozaki_triton_b200 import _lib
    lib = _lib.load()
    s = 4
    alpha = int(oracle.compute_split_bits(K, "int8", "int32"))
    need = lib.oz_split_workspace_bytes(_lib.OZ_F64, batch, N, K, 1, N)
    assert 0 < need <= lib.oz_split_noalloc_max_bytes()
    g = torch.Generator().manual_seed(K + N)
    for call, scale in enumerate((1e-3, 1e4)):
        x_h = (torch.rand(batch, K, N, generator=g, dtype=torch.float64) - 0.5) * torch.exp(
            2.0 * torch.randn(batch, K, N, generator=g, dtype=torch.float64)) * scale
        x = x_h.to(DEV)
        # the workspace starts as a sentinel: oz_split_ex must overwrite it
        # (the transpose ran), like oz_split_noalloc overwrites the array
        ws = torch.full((need,), 0xFF, dtype=torch.uint8, device=DEV)
        want_sl, want_sc = _run(lib, lib.oz_split_ex, x, K, N, s, alpha, ws)
        assert not bool((ws == 0xFF).all())
        n0 = lib.oz_launch_count()
        got_sl, got_sc = _run(lib, lib.oz_split_noalloc, x, K, N, s, alpha)
        assert lib.oz_launch_count() - n0 == 2, "transpose + row split expected"
        assert torch.equal(got_sl, want_sl), f"call {call}: slices differ"
        assert torch.equal(got_sc, want_sc), f"call {call}: scales differ"
        lines = np.swapaxes(x_h.numpy(), -1, -2)
        rsl, rsc = oracle.split_lines(lines, s, alpha, "int8", "fp64")
        got = got_sl.cpu().numpy()
        assert np.array_equal(got[..., :K], rsl), f"call {call}: slices differ from the oracle"
        assert not got[..., K:].any(), "slice row padding must be zero"
        assert np.array_equal(got_sc.cpu().numpy().view(np.uint32), rsc.view(np.uint32))


def test_noalloc_rejects_inputs_beyond_the_scratch():
    from ozaki_triton_b200 import _lib
    lib = _lib.load()
    # (1, K=4096, N=1025) fp64 columns need 4096*1025*8 bytes > 32 MiB
    K, N = 4096, 1025
    assert lib.oz_split_workspace_bytes(_lib.OZ_F64, 1, N, K, 1, N) > lib.oz_split_noalloc_max_bytes()
    p = ctypes.c_void_p(256)   # never touched: the size check comes first
    rc = lib.oz_split_noalloc(p, _lib.OZ_F64, 1, N, K, K * N, 1, N, 4, 7, _lib.OZ_I8, 0, p, 4096,
                              p, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OZ_ERR_INVALID
    assert "scratch" in lib.oz_last_error().decode()


def test_noalloc_takes_large_fp64_columns_without_scratch():
    """fp64 columns whose transposed copy would exceed the array, but which the
    column-pair kernel splits without scratch, are accepted; same bits as
    oz_split_ex."""
    from ozaki_triton_b200 import _lib
    lib = _lib.load()
    K, N, s = 4096, 2048, 4
    assert lib.oz_split_workspace_bytes(_lib.OZ_F64, 1, N, K, 1, N) > lib.oz_split_noalloc_max_bytes()
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(1, K, N, generator=g, dtype=torch.float64, device=DEV)
    alpha = 7
    ld = K
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for noalloc in (True, False):
        sl = torch.full((1, s, N, ld), 77, dtype=torch.int8, device=DEV)
        sc = torch.full((1, s, N), -1.0, dtype=torch.float32, device=DEV)
        args = [x.data_ptr(), _lib.OZ_F64, 1, N, K, K * N, 1, N, s, alpha, _lib.OZ_I8, 0,
                sl.data_ptr(), ld, sc.data_ptr()]
        if noalloc:
            _lib.check(lib.oz_split_noalloc(*args, st))
        else:
            need = lib.oz_split_workspace_bytes(_lib.OZ_F64, 1, N, K, 1, N)
            ws = torch.empty(need, dtype=torch.uint8, device=DEV)
            _lib.check(lib.oz_split_ex(*args, ws.data_ptr(), need, st))
        torch.cuda.synchronize()
        outs.append((sl, sc))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])

