"""The oracle's calibrators against numpy restatements of the reference's
calibrator formulas (CPU): MinMax range, the percentile order statistics at
the reference's fp32 indices (src/core/quantization/calibrator.cu:136-141),
the MSE clipping search, and the static per-tensor INT8 quantizer."""
import numpy as np
import pytest


def _data(seed=0):
    rng = np.random.default_rng(seed)
    return np.concatenate([rng.standard_normal(20_001).astype(np.float32),
                           rng.standard_t(2, size=3_000).astype(np.float32)])


def test_minmax(orc):
    x = _data(1)
    assert orc.calibrate(x, "minmax") == (float(x.min()), float(x.max()))
    assert orc.calibrate(x[:0], "minmax") == (0.0, 0.0)


@pytest.mark.parametrize("p", [99.9, 99.0, 75.0, 50.0, 100.0])
def test_percentile_indices(orc, p):
    x = _data(2)
    n = x.size
    v = np.sort(x)
    lo = int(np.float32(np.float32(100.0) - np.float32(p)) * np.float32(n) / np.float32(100.0))
    hi = min(int(np.float32(p) * np.float32(n) / np.float32(100.0)), n - 1)
    assert orc.calibrate(x, "percentile", p) == (float(v[lo]), float(v[hi]))


def test_mse_search(orc):
    x = _data(3)
    a = np.float32(np.abs(x).max())
    errs = []
    for t in range(100):
        clip = np.float32(a * np.float32(t + 1)) / np.float32(100.0)
        s = np.float32(clip / np.float32(127.0))
        q = np.clip(np.sign(x / s) * np.floor(np.abs(x / s) + np.float32(0.5)), -127, 127)
        d = (x - (q * s).astype(np.float32)).astype(np.float64)
        errs.append(float(np.sum(d * d)))
        assert abs(orc.calib_mse_error(x, float(clip)) - errs[-1]) <= 1e-9 * errs[-1] + 1e-12
    best = int(np.argmin(errs))
    lo, hi = orc.calibrate(x, "mse")
    clip = float(np.float32(a * np.float32(best + 1)) / np.float32(100.0))
    assert (lo, hi) == (-clip, clip)
    assert best < 99  # heavy tails: clipping below the max wins


def test_static_quantizer(orc):
    s = np.float32(2.0 ** -5)
    x = np.array([(j + 0.5) * s for j in range(-140, 140)] + [0.0, -0.0, 1e-9], np.float32)
    q = orc.quant_int8_static(x, float(s))
    t = x / s
    want = np.clip(np.sign(t) * np.floor(np.abs(t) + 0.5), -127, 127).astype(np.int8)
    assert np.array_equal(q, want)
    assert np.array_equal(orc.quant_int8_static(x, 0.0), np.zeros_like(q))
