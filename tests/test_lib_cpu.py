"""Host-side checks that need no GPU: the C ABI library loads, exports every
symbol the header declares, and validates arguments before any launch; the
Python policy layer mirrors the reference."""

import ctypes
import os
import re

import pytest
import torch

import oracle
import ozaki_triton_b200 as oz
from ozaki_triton_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = []
    for hdr in os.listdir(os.path.join(ROOT, "include")):
        if hdr.endswith(".h"):
            with open(os.path.join(ROOT, "include", hdr)) as fh:
                text = fh.read()
            names += re.findall(r"^[A-Za-z_][\w \*]*?\b(oz_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    names = header_functions()
    assert "oz_split" in names and "oz_cross_gemm" in names
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert _lib.version().startswith("ozaki_b200")


def test_alpha_rule_c_python_oracle_agree():
    lib = _lib.load()
    for sd, kind, code in [(torch.int8, "int8", _lib.OZ_I8), (torch.float16, "fp16", _lib.OZ_F16),
                           (torch.bfloat16, "bf16", _lib.OZ_BF16), (torch.float32, "fp32", _lib.OZ_F32)]:
        acc = oz.select_dot_accum_dtype(sd)
        for n in [1, 2, 3, 100, 256, 1000, 4096, 8192, 16384, 65536, 2 ** 17, 2 ** 20]:
            out = ctypes.c_int32(0)
            rc = lib.oz_compute_split_bits(n, code, ctypes.byref(out))
            try:
                py = oz.compute_split_bits(n, sd, acc)
            except AssertionError:
                assert rc == _lib.OZ_ERR_INVALID
                continue
            assert rc == 0 and out.value == py == oracle.compute_split_bits(
                n, kind, "int32" if kind == "int8" else "fp32"), (kind, n)
    out = ctypes.c_int32(0)
    assert lib.oz_compute_split_bits(0, _lib.OZ_I8, ctypes.byref(out)) == _lib.OZ_ERR_INVALID
    with pytest.raises(ValueError):
        oz.compute_split_bits(0, torch.int8, torch.int32)
    with pytest.raises(ValueError):
        oz.compute_split_bits(8, torch.int8, torch.float64)


def test_slice_row_pitch():
    lib = _lib.load()
    for k in [1, 15, 16, 127, 128, 129, 8192, 8193]:
        for code, es, sd in [(_lib.OZ_I8, 1, torch.int8), (_lib.OZ_F16, 2, torch.float16),
                             (_lib.OZ_F32, 4, torch.float32)]:
            b = lib.oz_slice_row_bytes(k, code)
            assert b % 128 == 0 and b >= k * es and b - k * es < 128
            assert oz.slice_row_elems(k, sd) * es == b


def test_argument_validation_without_launch():
    lib = _lib.load()
    p = ctypes.c_void_p(16)       # never dereferenced: validation fails first
    sc = ctypes.c_void_p(16)
    # num_splits out of range
    assert lib.oz_split(p, _lib.OZ_F64, 1, 4, 8, 32, 8, 1, 0, 7, _lib.OZ_I8, 0, p, 128, sc, None) \
        == _lib.OZ_ERR_INVALID
    assert lib.oz_split(p, _lib.OZ_F64, 1, 4, 8, 32, 8, 1, 9, 7, _lib.OZ_I8, 0, p, 128, sc, None) \
        == _lib.OZ_ERR_INVALID
    assert "num_splits" in _lib.load().oz_last_error().decode()
    # unsupported dtypes / modes
    assert lib.oz_split(p, 7, 1, 4, 8, 32, 8, 1, 2, 7, _lib.OZ_I8, 0, p, 128, sc, None) \
        == _lib.OZ_ERR_UNSUPPORTED
    assert lib.oz_split(p, _lib.OZ_F64, 1, 4, 8, 32, 8, 1, 2, 7, _lib.OZ_F64, 0, p, 128, sc, None) \
        == _lib.OZ_ERR_UNSUPPORTED
    assert lib.oz_split(p, _lib.OZ_F64, 1, 4, 8, 32, 8, 1, 2, 7, _lib.OZ_I8, 5, p, 128, sc, None) \
        == _lib.OZ_ERR_INVALID
    # pitch shorter than k, alpha out of range
    assert lib.oz_split(p, _lib.OZ_F64, 1, 4, 200, 800, 200, 1, 2, 7, _lib.OZ_I8, 0, p, 128, sc,
                        None) == _lib.OZ_ERR_INVALID
    assert lib.oz_split(p, _lib.OZ_F64, 1, 4, 8, 32, 8, 1, 2, 0, _lib.OZ_I8, 0, p, 128, sc, None) \
        == _lib.OZ_ERR_INVALID
    # empty problems are a no-op
    assert lib.oz_split(None, _lib.OZ_F64, 0, 4, 8, 32, 8, 1, 2, 7, _lib.OZ_I8, 0, None, 128, None,
                        None) == _lib.OZ_OK
    # cross-GEMM: bad pitch, bad flags, bad dtypes, bad batches
    args = dict(a=p, b=p, sa=sc, sb=sc, batch=1, m=4, n=4, k=8, ld=128, s=2, sd=_lib.OZ_I8,
                od=_lib.OZ_F64, ai=None, bi=None, ba=1, bb=1, c=p, ldc=4, flags=0, st=None)

    def gemm(**kw):
        a = dict(args, **kw)
        return lib.oz_cross_gemm(a["a"], a["b"], a["sa"], a["sb"], a["batch"], a["m"], a["n"],
                                 a["k"], a["ld"], a["s"], a["sd"], a["od"], a["ai"], a["bi"],
                                 a["ba"], a["bb"], a["c"], a["ldc"], a["flags"], a["st"])
    assert gemm(ld=100) == _lib.OZ_ERR_INVALID
    assert gemm(ld=4) == _lib.OZ_ERR_INVALID
    assert gemm(flags=4) == _lib.OZ_ERR_INVALID
    assert gemm(s=0) == _lib.OZ_ERR_INVALID
    assert gemm(s=9) == _lib.OZ_ERR_INVALID
    assert gemm(sd=_lib.OZ_F64) == _lib.OZ_ERR_UNSUPPORTED
    assert gemm(od=7) == _lib.OZ_ERR_UNSUPPORTED
    assert gemm(batch=3) == _lib.OZ_ERR_INVALID          # 1 A batch for 3 outputs, no index
    assert gemm(ldc=2) == _lib.OZ_ERR_INVALID
    assert gemm(a=ctypes.c_void_p(17)) == _lib.OZ_ERR_INVALID   # misaligned slices
    assert gemm(m=0) == _lib.OZ_OK


def test_blocked_gemm_and_peer_entries_validate_without_a_gpu():
    lib = _lib.load()
    p = ctypes.c_void_p(256)      # never dereferenced: validation fails first
    # B column block width: 0, >= n or a multiple of 128
    rc = lib.oz_cross_gemm_blocked(p, p, p, p, 1, 256, 1000, 64, 128, 2, _lib.OZ_I8, _lib.OZ_F64,
                                   None, None, 1, 1, 200, p, 1000, 0, None)
    assert rc == _lib.OZ_ERR_INVALID and "block width" in lib.oz_last_error().decode()
    rc = lib.oz_cross_gemm_blocked(p, p, p, p, 1, 256, 1000, 64, 128, 2, _lib.OZ_I8, _lib.OZ_F64,
                                   None, None, 1, 1, -128, p, 1000, 0, None)
    assert rc == _lib.OZ_ERR_INVALID
    # empty problems return before any device work, whatever the block width
    assert lib.oz_cross_gemm_blocked(p, p, p, p, 1, 0, 1000, 64, 128, 2, _lib.OZ_I8, _lib.OZ_F64,
                                     None, None, 1, 1, 256, p, 1000, 0, None) == _lib.OZ_OK
    # peer mappings and copies
    off = ctypes.c_int64()
    h = ctypes.create_string_buffer(_lib.OZ_IPC_HANDLE_BYTES)
    assert lib.oz_ipc_export(None, h, ctypes.byref(off)) == _lib.OZ_ERR_INVALID
    assert lib.oz_ipc_import(None, 0, None) == _lib.OZ_ERR_INVALID
    assert lib.oz_ipc_import(h, -1, ctypes.byref(ctypes.c_void_p())) == _lib.OZ_ERR_INVALID
    assert lib.oz_ipc_close(None, 0) == _lib.OZ_ERR_INVALID
    assert lib.oz_copy_async(p, p, -1, None) == _lib.OZ_ERR_INVALID
    assert lib.oz_copy_async(None, p, 16, None) == _lib.OZ_ERR_INVALID
    assert lib.oz_copy_async(p, p, 0, None) == _lib.OZ_OK


def test_wait_selftest_validates_its_bound_without_a_gpu():
    lib = _lib.load()
    assert lib.oz_wait_selftest(0, None) == _lib.OZ_ERR_INVALID
    assert lib.oz_wait_selftest(10 ** 12, None) == _lib.OZ_ERR_INVALID


def test_launch_count_is_not_moved_by_rejected_calls():
    lib = _lib.load()
    n0 = lib.oz_launch_count()
    p = ctypes.c_void_p(256)
    assert lib.oz_split(p, _lib.OZ_F64, 1, 4, 8, 32, 8, 1, 0, 7, _lib.OZ_I8, 0, p, 128, p,
                        None) == _lib.OZ_ERR_INVALID
    assert lib.oz_launch_count() == n0 >= 0


def test_policy_tables_match_reference():
    # ozaki_triton.py:36-41, 62-73
    assert oz.SLICE_DTYPE_INFO[torch.float32] == (23, False)
    assert oz.SLICE_DTYPE_INFO[torch.float16] == (10, False)
    assert oz.SLICE_DTYPE_INFO[torch.bfloat16] == (7, False)
    assert oz.SLICE_DTYPE_INFO[torch.int8] == (7, True)
    assert oz.select_dot_accum_dtype(torch.int8) == torch.int32
    assert oz.select_dot_accum_dtype(torch.float16) == torch.float32
    assert oz.select_out_accum_dtype(torch.float64) == torch.float64
    assert oz.select_out_accum_dtype(torch.float32) == torch.float32
    assert oz.select_out_accum_dtype(torch.bfloat16) == torch.float32


def test_host_api_rejects_cpu_tensors():
    a = torch.randn(4, 4, dtype=torch.float64)
    with pytest.raises(ValueError):
        oz.ozaki_matmul(a, a)
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a, a.float())
    with pytest.raises(AssertionError):
        oz.ozaki_matmul(a, a, num_splits=9)


def test_batch_index_matches_broadcast():
    from ozaki_triton_b200.api import _batch_index
    for own, full in [((16, 1), (16, 8)), ((1, 8), (16, 8)), ((), (3, 2)), ((3, 2), (3, 2)),
                      ((2, 1, 3), (4, 2, 5, 3))]:
        idx = _batch_index(own, full, "cpu")
        n_own = 1
        for d in own:
            n_own *= d
        members = torch.arange(n_own).reshape(own) if own else torch.tensor(0)
        want = members.expand(full).reshape(-1)
        if idx is None:
            assert tuple(own) == tuple(full)
        else:
            assert torch.equal(idx.long(), want)
