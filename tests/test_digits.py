"""Host-side check of the activation digit arithmetic the int8 kernels use
(act_digits / act_scale / act_unscale in q4rdna_gemv_i8.cuh), restated in numpy:
the digit word (X + 0x808080) ^ 0x808080, read as four s8 bytes, recombines to
X for every |X| <= 2^30, and the power-of-two scaling puts a group's largest
magnitude in [2^29, 2^30)."""
import numpy as np


def digits(X):
    w = ((X.astype(np.int64) + 0x808080) & 0xFFFFFFFF) ^ 0x808080
    b = w.astype(np.uint32).view(np.uint8).reshape(-1, 4).view(np.int8).astype(np.int64)
    return b


def test_balanced_digits_recombine():
    rng = np.random.default_rng(1)
    X = np.concatenate([rng.integers(-(1 << 30), (1 << 30) + 1, 200000),
                        np.array([0, 1, -1, 127, 128, -128, -129, 255, 256, 32767, 32768, -32768, -32769,
                                  (1 << 23) - 1, 1 << 23, -(1 << 23), (1 << 30), -(1 << 30)])])
    d = digits(X)
    assert d.min() >= -128 and d.max() <= 127
    back = d[:, 0] + 256 * d[:, 1] + 65536 * d[:, 2] + (1 << 24) * d[:, 3]
    assert np.array_equal(back, X)
    # the top digit stays far from the s8 limits: |d3| <= 64
    assert np.abs(d[:, 3]).max() <= 64


def test_group_scaling_range():
    rng = np.random.default_rng(2)
    m = np.abs(rng.standard_normal(100000)).astype(np.float32) * np.float32(10.0) ** rng.integers(-20, 20, 100000)
    m = m[m > 0].astype(np.float32)
    E = np.maximum((m.view(np.uint32) >> 23) & 0xFF, 30).astype(np.int64)
    f = ((283 - E) << 23).astype(np.uint32).view(np.float32)
    u = ((E - 29) << 23).astype(np.uint32).view(np.float32)
    s = m.astype(np.float64) * f.astype(np.float64)
    normal = ((m.view(np.uint32) >> 23) & 0xFF) >= 30
    assert np.all(s[normal] >= 2.0 ** 29) and np.all(s < 2.0 ** 30)
    assert np.all(np.rint(s) <= 2.0 ** 30)
    assert np.all(f.astype(np.float64) * u.astype(np.float64) == 1.0)
