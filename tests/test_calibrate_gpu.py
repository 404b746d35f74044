"""Activation-range calibrators (MinMax, Percentile, MSE) and the static
per-tensor INT8 quantizer on the GPU against the oracle: MinMax and
Percentile ranges exactly (they are order statistics of the collected
values), the MSE range at the oracle's least error (the device sums the
trials' errors in another order, so a trial within 1e-9 of the best may win
instead), static INT8 codes bit-exact, ties included."""
import numpy as np
import pytest

from _util import to_device

pytestmark = pytest.mark.gpu


def _batches(seed, dt):
    rng = np.random.default_rng(seed)
    parts = [rng.standard_normal(100_003).astype(np.float32) * 1.5 - 0.25,
             rng.standard_t(3, size=65_536).astype(np.float32),  # heavy tails
             -np.abs(rng.standard_normal(4097).astype(np.float32)) * 3]
    dev = [to_device(p, dt) for p in parts]
    return dev, np.concatenate([d.float().cpu().numpy() for d in dev])


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_minmax_calibrator(ltm, orc, dt):
    dev, allv = _batches(1, dt)
    cal = ltm.Calibrator(ltm.CALIB_MINMAX)
    assert cal.compute_range() == (0.0, 0.0)
    for d in dev:
        cal.collect(d)
    assert cal.compute_range() == orc.calibrate(allv, "minmax")
    cal.reset()
    cal.collect(dev[2])
    assert cal.compute_range() == orc.calibrate(dev[2].float().cpu().numpy(), "minmax")
    cal.close()


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("p", [99.9, 99.0, 50.0, 100.0])
def test_percentile_calibrator(ltm, orc, dt, p):
    dev, allv = _batches(2, dt)
    cal = ltm.Calibrator(ltm.CALIB_PERCENTILE, p)
    for d in dev:
        cal.collect(d)
    assert cal.compute_range() == orc.calibrate(allv, "percentile", p)
    cal.close()


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_mse_calibrator(ltm, orc, dt):
    dev, allv = _batches(3, dt)
    cal = ltm.Calibrator(ltm.CALIB_MSE)
    for d in dev:
        cal.collect(d)
    lo, hi = cal.compute_range()
    olo, ohi = orc.calibrate(allv, "mse")
    assert lo == -hi and 0 < hi <= np.abs(allv).max()
    best = orc.calib_mse_error(allv, ohi)
    assert orc.calib_mse_error(allv, hi) <= best * (1 + 1e-9)
    assert ohi < np.abs(allv).max(), "heavy tails: the best clip is below the max"
    cal.close()


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_static_int8_quantizer(ltm, orc, dt):
    import torch
    dev, allv = _batches(4, dt)
    cal = ltm.Calibrator(ltm.CALIB_PERCENTILE, 99.9)
    cal.collect(dev[0])
    scale = cal.static_scale()
    x = dev[1]
    q = ltm.quantize_int8_static(x, scale)
    want = orc.quant_int8_static(x.float().cpu().numpy(), scale)
    assert np.array_equal(q.cpu().numpy(), want)
    # exact ties x / s = j + 0.5 round away from zero; beyond the range clamps
    s = 2.0 ** -6
    ties = torch.tensor([(j + 0.5) * s for j in range(-130, 130)], dtype=torch.float32,
                        device="cuda")
    qt = ltm.quantize_int8_static(ties, s).cpu().numpy()
    assert np.array_equal(qt, orc.quant_int8_static(ties.cpu().numpy(), s))
    assert qt.max() == 127 and qt.min() == -127
    assert np.array_equal(ltm.quantize_int8_static(ties, 0.0).cpu().numpy(), np.zeros(260, np.int8))
    cal.close()
