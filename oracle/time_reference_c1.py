"""Time the reference's own ``ozaki_matmul`` on the CPU at config C1.

TEST INFRASTRUCTURE (a measurement, not part of the product): runs the
UNMODIFIED reference module ``ozaki_triton.py`` of WhFanatic/Ozaki_triton
under ``TRITON_INTERPRET=1`` with the two shims of
``tests/golden/make_golden.py`` (a one-config autotuner in place of Optuna,
no-op CUDA streams), on the C1 inputs of ``bench.py`` (FP32 -> FP16,
num_splits = 2, 256^3, U(-1, 1) from seed 0), and prints one JSON line: the
emulated TFLOPS over the host cores used, and the result's relative error
against an fp64 product.  The reference is not installable (no setup.py or
pyproject.toml) and its sources are not copied into this repository, so this
runs only where a reference checkout exists, never on the GPU box.

    python oracle/time_reference_c1.py /path/to/Ozaki_triton [repeats]
"""

from __future__ import annotations

import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def main():
    ref_dir = sys.argv[1]
    repeats = int(sys.argv[2]) if len(sys.argv) > 2 else 3
    from make_golden import import_reference

    ozt = import_reference(ref_dir)
    import torch

    import bench

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    a, b = bench.config_inputs(bench.CONFIGS["C1"])
    ozt.ozaki_matmul(a, b, 2, torch.float16)          # first call compiles / tunes
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        c = ozt.ozaki_matmul(a, b, 2, torch.float16)
        times.append(time.perf_counter() - t0)
    t = sorted(times)[len(times) // 2]
    ref = a.double() @ b.double()
    rel = float((c.double() - ref).norm() / ref.norm())
    print(json.dumps({"config": "C1", "impl": "reference ozaki_matmul, TRITON_INTERPRET=1",
                      "seconds": t, "tflops": 2.0 * 256 ** 3 / t / 1e12, "cores": threads,
                      "repeats": repeats, "rel_err_vs_fp64": rel}))


if __name__ == "__main__":
    main()
