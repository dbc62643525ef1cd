"""B200-native (sm_100a) Ozaki-scheme GEMM.

Drop-in for the ``ozaki_matmul`` path of WhFanatic/Ozaki_triton: the same
Python operator API (``ozaki_matmul``, ``split_matrix``, ``cross_gemm``,
``compute_split_bits``) backed by hand-written CUDA kernels in
``liboz_b200.so`` (C ABI: ``include/ozaki_b200.h``).
"""

from .api import (  # noqa: F401
    INPUT_DTYPES,
    MAX_SPLITS,
    SLICE_DTYPE_INFO,
    compute_split_bits,
    cross_gemm,
    device_status,
    ozaki_matmul,
    ozaki_matmul_from_host,
    select_dot_accum_dtype,
    select_out_accum_dtype,
    slice_row_elems,
    split_matrix,
)
from ._lib import OzakiError, OzakiLibraryError, load as load_library, version  # noqa: F401

__all__ = [
    "ozaki_matmul", "ozaki_matmul_from_host", "split_matrix", "cross_gemm", "compute_split_bits",
    "select_dot_accum_dtype", "select_out_accum_dtype", "slice_row_elems",
    "device_status", "OzakiError", "OzakiLibraryError", "load_library", "version",
]
