"""ctypes binding of liboz_b200.so (the C ABI declared in include/ozaki_b200.h).

The library is built in-tree by ``ozaki_triton_b200/csrc/build.py``.  There is
no fallback: if the shared library is missing or does not load, every call
that needs it raises ``OzakiLibraryError``.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboz_b200.so")

# element type codes (enum oz_dtype)
OZ_F64, OZ_F32, OZ_F16, OZ_BF16, OZ_I8 = 0, 1, 2, 3, 4
# status codes (enum oz_status)
OZ_OK, OZ_ERR_INVALID, OZ_ERR_UNSUPPORTED, OZ_ERR_CUDA, OZ_ERR_TIMEOUT = 0, -1, -2, -3, -4
# residual modes (enum oz_residual_mode)
OZ_RESIDUAL_COMPAT, OZ_RESIDUAL_EXACT = 0, 1
# oz_cross_gemm flags
OZ_GEMM_SKIP_TAIL = 1
OZ_IPC_HANDLE_BYTES = 64

# every function the header declares: name -> (restype, argtypes)
_i64, _i32, _u32, _vp, _int = ctypes.c_int64, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int
SIGNATURES = {
    "oz_compute_split_bits": (_int, [_i64, _int, ctypes.POINTER(_i32)]),
    "oz_slice_row_bytes": (_i64, [_i64, _int]),
    "oz_split": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _int, _int,
                        _vp, _i64, _vp, _vp]),
    "oz_split_workspace_bytes": (_i64, [_int, _i64, _i64, _i64, _i64, _i64]),
    "oz_split_ex": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _int, _int,
                           _vp, _i64, _vp, _vp, _i64, _vp]),
    "oz_split_noalloc": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _int,
                                _int, _vp, _i64, _vp, _vp]),
    "oz_split_noalloc_max_bytes": (_i64, []),
    "oz_cross_gemm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _int, _int,
                             _vp, _vp, _i64, _i64, _vp, _i64, _u32, _vp]),
    "oz_cross_gemm_blocked": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _int,
                                     _int, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _u32, _vp]),
    "oz_cross_gemm_arrivals": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _int,
                                      _int, _i64, _vp, _i32, _i32, _i32, _vp, _i64, _u32, _vp]),
    "oz_matmul_workspace_bytes": (_i64, [_int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                         _i64, _i32, _int]),
    "oz_matmul": (_int, [_vp, _vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64,
                         _i64, _i64, _i64, _i64, _i64, _i32, _int, _int, _vp, _i64, _u32, _vp,
                         _i64, _vp]),
    "oz_ipc_export": (_int, [_vp, _vp, ctypes.POINTER(_i64)]),
    "oz_ipc_import": (_int, [_vp, _i64, ctypes.POINTER(_vp)]),
    "oz_ipc_close": (_int, [_vp, _i64]),
    "oz_copy_async": (_int, [_vp, _vp, _i64, _vp]),
    "oz_device_status": (_int, [_vp, ctypes.POINTER(_i32)]),
    "oz_launch_count": (_i64, []),
    "oz_profile_next_gemm": (_int, [_vp, _vp]),
    "oz_wait_selftest": (_int, [_i64, _vp]),
    "oz_last_error": (ctypes.c_char_p, []),
    "oz_version": (ctypes.c_char_p, []),
}


class OzakiLibraryError(RuntimeError):
    """The CUDA library could not be loaded (it is never silently replaced)."""


class OzakiError(RuntimeError):
    """A library call returned an error status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[oz status {status}] {message}")
        self.status = status


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load liboz_b200.so once and bind its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise OzakiLibraryError(
                f"{LIB_PATH} is missing: build it with `python -m ozaki_triton_b200.csrc.build`")
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as e:  # pragma: no cover - depends on the machine
            raise OzakiLibraryError(f"cannot load {LIB_PATH}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != OZ_OK:
        msg = load().oz_last_error().decode(errors="replace")
        raise OzakiError(status, msg)


def version() -> str:
    return load().oz_version().decode()
