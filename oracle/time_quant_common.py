"""Times the reference's own Python quantizer on config 1, for the CPU
baseline record of `quantize` (test infrastructure; nothing in the library
imports this file).

    python oracle/time_quant_common.py <path to the web-xpu-ops checkout>

`llm/tools/quant_common.py#quantize_per_row` (quant_common.py:40-57) is the
numpy routine the reference's weight converter runs.  Its input here is
config 1: a 4096 x 4096 f32 matrix of the seeded N(0, 0.02^2) recipe
(xpuops/synth.py; the device fill and the oracle follow the same recipe).
The script checks that its codes and scales equal the oracle's
(or_quantize, ops/quantize/reference.ts:13-38), then reports the best of
five timed calls in GB/s of algorithmic bytes: 4NK read + NK (int8 codes) +
4N (scales) written, the bytes of quantize without the pack.
"""
import importlib.util
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
# The repository root first: run from this folder, `oracle` would otherwise
# name oracle.py instead of the package.
sys.path[:] = [str(ROOT), str(ROOT / "web-xpu-ops_b200")] + [
    q for q in sys.path if Path(q or ".").resolve() != ROOT / "oracle"]


def main():
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    ref = Path(sys.argv[1]).resolve()
    spec = importlib.util.spec_from_file_location("quant_common", ref / "llm" / "tools" / "quant_common.py")
    qc = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(qc)

    import oracle.oracle as orc
    from xpuops.synth import fill_normal

    N = K = 4096
    w = fill_normal(N * K, 0, 0.0, 0.02)
    m = w.reshape(N, K)
    codes, scales = qc.quantize_per_row(m)
    want_codes, want_scales = orc.quantize(w, N, K)
    assert np.array_equal(np.asarray(codes, np.int64).ravel(), np.asarray(want_codes, np.int64)), "codes differ"
    assert np.array_equal(np.asarray(scales, np.float32).ravel(), want_scales), "scales differ"
    best = 1e30
    for _ in range(5):
        t0 = time.perf_counter()
        qc.quantize_per_row(m)
        best = min(best, time.perf_counter() - t0)
    nbytes = 4 * N * K + N * K + 4 * N
    print(f"quant_common.quantize_per_row, {N} x {K} f32 (config 1): best of 5 {best * 1e3:.1f} ms = "
          f"{nbytes / best / 1e9:.3f} GB/s; codes and scales equal the oracle's; numpy {np.__version__}, "
          f"{os.cpu_count()} host threads visible")


if __name__ == "__main__":
    main()
