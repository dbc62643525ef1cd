"""CPU oracle for the Ozaki-scheme hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the arithmetic of the reference
implementation (WhFanatic/Ozaki_triton, ``ozaki_triton.py``) for the split
and cross-GEMM path.  It is the checker for the CUDA product, never part of
it: only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product package
``ozaki_triton_b200`` never imports anything from here and fails loudly when
its CUDA library is missing.

Parity pin: the restatement is checked against golden vectors produced by the
reference itself (imported under ``TRITON_INTERPRET=1``), committed under
``tests/golden/`` together with the script that made them.  Two parts are
not pinned by those vectors:
* BF16 slicing and BF16 outputs, which the Triton interpreter mis-converts.
  They follow Triton's documented GPU rounding (round to nearest even) and
  are marked "parity unpinned" in the tests.
* int8 results outside [-128, 127] (int8 inputs).  The reference's cast is
  backend-dependent there: the interpreter wraps and the GPU saturates. The
  restatement saturates, like the GPU; in-range int8 results are pinned.
"""

from .ozaki_oracle import (  # noqa: F401
    SLICE_BITS,
    compute_split_bits,
    ceil_log2_f32,
    split_lines,
    cross_gemm,
    ozaki_matmul,
    round_to_bf16,
)
