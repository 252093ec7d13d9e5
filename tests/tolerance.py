"""Output tolerance of the GEMV against the fp64-accumulated oracle.

The split-K and tensor-core accumulation order differs from the reference's
sequential f32 order, so outputs are compared normwise, not bitwise:
  * per element: |y - y64| <= NORMWISE * sum_k |W[n,k] x[k]|
  * rel-L2:      ||y - y64|| / ||y64|| <= REL_L2      (the reference bench's own
                 bound, source/q4rdna_gemv_bench.hip:259)
  * max rel err: <= MAX_REL over rows with |y64| >= 1e-2 * rms(y64)
The reference's own f32 order measures ~3e-7 normwise and ~1e-6 rel-L2 at
12288 x 4096, so these bounds leave 10-30x headroom over f32 reordering.
"""
import numpy as np

NORMWISE = 1e-5
REL_L2 = 1e-5
MAX_REL = 1e-3


def check(y, y64, mag, what=""):
    y = np.asarray(y, np.float64)
    y64 = np.asarray(y64, np.float64)
    mag = np.asarray(mag, np.float64)
    assert np.all(np.isfinite(y)), f"{what}: non-finite output"
    err = np.abs(y - y64)
    nw = float(np.max(err / np.maximum(mag, 1e-30)))
    rl2 = float(np.linalg.norm(y - y64) / max(np.linalg.norm(y64), 1e-30))
    rms = float(np.sqrt(np.mean(y64 ** 2)))
    big = np.abs(y64) >= 1e-2 * rms
    mre = float(np.max(err[big] / np.abs(y64[big]))) if big.any() else 0.0
    assert nw <= NORMWISE, f"{what}: normwise {nw:.3e} > {NORMWISE}"
    assert rl2 <= REL_L2, f"{what}: rel-L2 {rl2:.3e} > {REL_L2}"
    assert mre <= MAX_REL, f"{what}: max rel {mre:.3e} > {MAX_REL}"
    return nw, rl2, mre
