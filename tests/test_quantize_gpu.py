"""INT8 / INT4 quantize, pack and dequantize on the GPU (through the C ABI)
against the CPU oracle: codes, packed nibbles, scales and zero-points must be
bit-exact."""
import numpy as np
import pytest

from _util import DT_NAMES, as_f32, orc_dtype, to_device

pytestmark = pytest.mark.gpu

# widths cover the warp-per-row (<= 128 vectors), 4-warp (<= 1024 vectors) and
# streaming row quantizers
INT8_SHAPES = [(1, 16), (3, 8), (37, 100), (64, 768), (300, 3072), (64, 4096), (33, 8192),
               (5, 28672), (2, 1)]


def _weights(shape, seed, special=True):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    if special and shape[0] >= 3:
        w[1] = 0.0                          # all-zero channel -> s = 0, q = 0
        w[2, :] = 0.0
        w[2, 0] = 0.5                       # single non-zero
    return w


@pytest.mark.parametrize("dt", DT_NAMES)
@pytest.mark.parametrize("shape", INT8_SHAPES)
def test_int8_per_channel_bit_exact(ltm, orc, dt, shape):
    w = _weights(shape, 1)
    wd = to_device(w, dt)
    q, s = ltm.quantize_int8_per_channel(wd)
    qo, so = orc.quant_int8_rows(as_f32(wd))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))


def test_int8_rounding_ties_and_clamp(ltm, orc):
    """Values at exact .5 code boundaries round half away from zero."""
    s = np.float32(0.25) / np.float32(127.0)
    k = np.arange(-127, 128, dtype=np.float32)
    row = np.concatenate([(k + 0.5) * s, (k - 0.5) * s, [0.25, -0.25]]).astype(np.float32)
    row = row[np.abs(row) <= 0.25]
    w = np.stack([row, -row, row * 0.5]).astype(np.float32)
    q, sc = ltm.quantize_int8_per_channel(to_device(w, "f32"))
    qo, so = orc.quant_int8_rows(w)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(sc.cpu().numpy(), so)
    assert qo.max() == 127 and qo.min() == -127


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
# 4096-8192 (16-bit) / 2048-4096 (fp32): eight warps per row; from 12288
# (16-bit): the two-pass kernel
@pytest.mark.parametrize("K", [768, 3072, 4096, 6144, 8192, 12288, 28672, 49152])
def test_act_per_token_rounding_ties(ltm, orc, dt, K):
    """Per-token activation codes at exact .5 boundaries (row absmax 127, so
    s = 1 and every k + 0.5 is a tie) and just off them: the warp quantizer's
    fast path must hand every near-tie to the exact IEEE quotient and round
    half away from zero.  Rows mix ties, near-ties, zeros and plain values."""
    rng = np.random.default_rng(K)
    k = rng.integers(-126, 126, size=(64, K)).astype(np.float32)
    a = k + 0.5
    a[:, 0] = 127.0                                  # absmax 127 -> s = 1
    a[1::4] = k[1::4] + 0.5 + np.float32(2e-3)      # just above a tie in f32 (f16 / bf16 storage rounds it onto the tie)
    a[2::4] = rng.standard_normal((16, K)).astype(np.float32) * 40.0
    a[2::4, 0] = 127.0
    a[3, :] = 0.0                                    # all-zero row: s = 0, codes 0
    ad = to_device(a, dt)
    q, s = ltm.quantize_act_int8_per_token(ad)
    qo, so = orc.quant_int8_rows(as_f32(ad))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_act_per_token_long_rows_many_per_cta(ltm, orc, dt):
    """The FFN-hidden width of the hidden-8192 block (28672 values, 56 KiB per
    row) over many rows: the long-row kernel (a warp per row, max pass then
    quantize pass)."""
    a = np.random.default_rng(29).standard_normal((611, 28672)).astype(np.float32)
    a[::7] *= 30.0
    a[5] = 0.0
    ad = to_device(a, dt)
    q, s = ltm.quantize_act_int8_per_token(ad)
    qo, so = orc.quant_int8_rows(as_f32(ad))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    assert ltm.device_error() == 0


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_act_per_token_bit_exact(ltm, orc, dt):
    a = np.random.default_rng(3).standard_normal((2048, 768)).astype(np.float32)
    ad = to_device(a, dt)
    q, s = ltm.quantize_act_int8_per_token(ad)
    qo, so = orc.quant_int8_rows(as_f32(ad))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


@pytest.mark.parametrize("dt", DT_NAMES)
@pytest.mark.parametrize("shape", [(1, 128), (7, 256), (64, 4096), (3, 11008)])
def test_int4_group128_bit_exact(ltm, orc, dt, shape):
    w = _weights(shape, 2)
    if shape[0] >= 7:
        w[4, :128] = np.abs(w[4, :128])    # all-positive group (zero-point clamps at 0)
        w[5, 128:256] = -np.abs(w[5, 128:256])
    wd = to_device(w, dt)
    packed, s, zp = ltm.quantize_int4_grouped(wd, 128)
    po, so, zo = orc.quant_int4_g128(as_f32(wd))
    np.testing.assert_array_equal(packed.cpu().numpy(), po)
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    np.testing.assert_array_equal(zp.cpu().numpy(), zo)


@pytest.mark.parametrize("dt", DT_NAMES)
def test_dequant_int8_and_int4(ltm, orc, dt):
    import torch
    from _util import torch_dtype
    w = _weights((96, 512), 4)
    wd = to_device(w, "f32")
    q, s = ltm.quantize_int8_per_channel(wd)
    out = ltm.dequantize_int8_per_channel(q, s, torch_dtype(dt))
    ref = orc.dequant_int8_rows(q.cpu().numpy(), s.cpu().numpy(), orc_dtype(dt))
    np.testing.assert_array_equal(as_f32(out), ref)
    packed, s4, zp = ltm.quantize_int4_grouped(wd, 128)
    out4 = ltm.dequantize_int4_grouped(packed, s4, zp, 128, torch_dtype(dt))
    ref4 = orc.dequant_int4_g128(packed.cpu().numpy(), s4.cpu().numpy(), zp.cpu().numpy(),
                                 orc_dtype(dt))
    np.testing.assert_array_equal(as_f32(out4), ref4)
    # round trip error bound of the asymmetric int4 code: |w - deq| <= s/2 (+ dtype rounding)
    err = np.abs(orc.dequant_int4_g128(packed.cpu().numpy(), s4.cpu().numpy(), zp.cpu().numpy(), 0) - w)
    bound = np.repeat(s4.cpu().numpy(), 128, axis=1) * 0.5 + 1e-7
    assert (err <= bound).all()
    del torch


def test_invalid_arguments_are_reported(ltm):
    import torch
    w = torch.zeros((4, 100), device="cuda")
    with pytest.raises(ltm.LtmError) as e:
        ltm.quantize_int4_grouped(w, 128)
    assert e.value.status == ltm.ERR_INVALID_ARG
    with pytest.raises(ltm.LtmError) as e:
        ltm.quantize_int4_grouped(torch.zeros((4, 256), device="cuda"), 64)
    assert e.value.status == ltm.ERR_UNSUPPORTED


def test_empty_inputs(ltm):
    import torch
    q, s = ltm.quantize_int8_per_channel(torch.zeros((0, 64), device="cuda"))
    assert q.shape == (0, 64) and s.shape == (0,)
    torch.cuda.synchronize()
