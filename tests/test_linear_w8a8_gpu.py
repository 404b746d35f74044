"""W8A8 tcgen05 GEMM: int32 accumulators bit-exact against the oracle, fused
epilogue (dequant, bias, GELU / sigmoid) within the dtype tolerance."""
import numpy as np
import pytest

from _util import as_f32, assert_close, torch_dtype

pytestmark = pytest.mark.gpu

# N % 256 == 0 with M >= 256 runs the CTA-pair kernel (256 x 256 tiles): ragged
# M, a single pair tile, several tiles per pair, the minimum K
ACC_SHAPES = [(128, 128, 128), (1, 32, 16), (200, 96, 48), (256, 384, 768), (513, 2304, 768),
              (64, 768, 3072), (130, 160, 1040), (256, 256, 16), (2048, 3072, 768),
              (4100, 512, 1024), (300, 768, 3072)]


def _rand_i8(shape, seed):
    return np.random.default_rng(seed).integers(-127, 128, size=shape, dtype=np.int8)


@pytest.mark.parametrize("M,N,K", ACC_SHAPES)
def test_acc_i32_bit_exact(ltm, orc, M, N, K):
    import torch
    qa, qw = _rand_i8((M, K), 1), _rand_i8((N, K), 2)
    acc = ltm.linear_w8a8_acc_i32(torch.from_numpy(qa).cuda(), torch.from_numpy(qw).cuda())
    np.testing.assert_array_equal(acc.cpu().numpy(), orc.gemm_i8(qa, qw))
    assert ltm.device_error() == 0


def test_acc_extremes(ltm, orc):
    """All +-127 operands: largest accumulators (K * 127^2) stay exact."""
    import torch
    M, N, K = 128, 128, 3072
    qa = np.full((M, K), 127, np.int8)
    qa[::2] = -127
    qw = np.full((N, K), 127, np.int8)
    acc = ltm.linear_w8a8_acc_i32(torch.from_numpy(qa).cuda(), torch.from_numpy(qw).cuda())
    np.testing.assert_array_equal(acc.cpu().numpy(), orc.gemm_i8(qa, qw))


@pytest.mark.parametrize("out", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("act", [0, 1, 2])
def test_epilogue(ltm, orc, out, act):
    import torch
    M, N, K = 300, 768, 768
    rng = np.random.default_rng(7)
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    qa, sa = orc.quant_int8_rows(a)
    qw, sw = orc.quant_int8_rows(w)
    dev = lambda x: torch.from_numpy(x).cuda()  # noqa: E731
    y = ltm.linear_w8a8(dev(qa), dev(sa), dev(qw), dev(sw), dev(b), act, torch_dtype(out))
    ref = orc.linear_w8a8(qa, sa, qw, sw, b, act)
    if out == "f32":
        assert_close(as_f32(y), ref, 1e-5, 1e-5, "w8a8 f32")
    else:
        assert_close(as_f32(y), ref, 2e-2, 1e-2, f"w8a8 {out}")


def test_rejects_bad_shapes(ltm):
    import torch
    qa = torch.zeros((4, 24), dtype=torch.int8, device="cuda")
    qw = torch.zeros((32, 24), dtype=torch.int8, device="cuda")
    with pytest.raises(ltm.LtmError):
        ltm.linear_w8a8_acc_i32(qa, qw)   # K % 16 != 0
    qw = torch.zeros((40, 32), dtype=torch.int8, device="cuda")
    with pytest.raises(ltm.LtmError):
        ltm.linear_w8a8_acc_i32(torch.zeros((4, 32), dtype=torch.int8, device="cuda"), qw)


@pytest.mark.parametrize("M,N,K", [(300, 768, 768), (4100, 768, 768), (600, 512, 2048),
                                   (1024, 3072, 768)])
@pytest.mark.parametrize("out", ["f16", "bf16"])
@pytest.mark.parametrize("act", [0, 1, 2])
def test_short_k_16bit_epilogue_equals_rounded_f32(ltm, orc, M, N, K, out, act):
    """At K <= 2048 the CTA-pair kernel's plain 16-bit epilogue runs on
    sixteen warps (four column quarters per tile); its outputs must be the
    fp32 epilogue's values (eight warps) rounded to 16 bits, bit for bit."""
    import torch
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    qa, sa = orc.quant_int8_rows(a)
    qw, sw = orc.quant_int8_rows(w)
    dev = lambda x: torch.from_numpy(x).cuda()  # noqa: E731
    y32 = ltm.linear_w8a8(dev(qa), dev(sa), dev(qw), dev(sw), dev(b), act, torch.float32)
    y16 = ltm.linear_w8a8(dev(qa), dev(sa), dev(qw), dev(sw), dev(b), act, torch_dtype(out))
    assert torch.equal(y16, y32.to(torch_dtype(out))), "16-bit epilogue differs from rounded fp32"
