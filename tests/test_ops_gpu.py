"""LayerNorm, attention (causal self-attention and memory attention), W8A32
and W4A16 linears on the GPU (through the C ABI) against the CPU oracle."""
import numpy as np
import pytest

from _util import as_f32, assert_close, orc_dtype, to_device

pytestmark = pytest.mark.gpu

TOL = {"f32": (1e-4, 1e-4), "f16": (2e-2, 1e-2), "bf16": (2e-2, 1e-2)}


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("H", [64, 768, 4096, 8192])  # 4096 / 8192: a CTA per row
def test_layernorm_x2(ltm, orc, dt, H):
    import torch
    rng = np.random.default_rng(H)
    x = rng.standard_normal((37, H)).astype(np.float32) * 2 + 0.5
    g = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    b = (0.1 * rng.standard_normal(H)).astype(np.float32)
    xd = to_device(x, dt)
    y = ltm.layernorm_residual(xd, xd, torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda())
    ref = orc.round_to(orc.layernorm_x2(as_f32(xd), g, b), orc_dtype(dt))
    assert_close(as_f32(y), ref, *(TOL[dt] if dt != "f32" else (2e-5, 2e-5)), what=f"ln {dt}")


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,S", [(2, 200), (1, 64), (1, 1), (3, 129)])
def test_causal_self_attention(ltm, orc, dt, D, B, S):
    nh = 2
    rng = np.random.default_rng(S * D)
    qkv = rng.standard_normal((B * S, 3 * nh * D)).astype(np.float32)
    qd = to_device(qkv, dt)
    H = nh * D
    o = ltm.attention(qd[:, :H], qd[:, H:2 * H], qd[:, 2 * H:], B, S, S, nh, D, True)
    qf = as_f32(qd)
    ref = orc.attention(qf[:, :H], qf[:, H:2 * H], qf[:, 2 * H:], B, S, S, nh, D, True, orc_dtype(dt))
    assert_close(as_f32(o), ref, *TOL[dt], what=f"self-attn {dt} D{D}")


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Ms", [64, 96, 512])
def test_memory_attention_shared_bank(ltm, orc, dt, D, Ms):
    B, S, nh = 3, 70, 2
    H = nh * D
    rng = np.random.default_rng(Ms + D)
    q = rng.standard_normal((B * S, H)).astype(np.float32)
    kv = rng.standard_normal((Ms, 2 * H)).astype(np.float32)
    qd, kvd = to_device(q, dt), to_device(kv, dt)
    o = ltm.attention(qd, kvd[:, :H], kvd[:, H:], B, S, Ms, nh, D, False, kv_shared=True)
    kf = as_f32(kvd)
    ref = orc.attention(as_f32(qd), kf[:, :H], kf[:, H:], B, S, Ms, nh, D, False, orc_dtype(dt),
                        kv_shared=True)
    assert_close(as_f32(o), ref, *TOL[dt], what=f"mem-attn {dt} D{D}")


@pytest.mark.parametrize("act", [0, 1, 2])
@pytest.mark.parametrize("M,N,K", [(512, 768, 768), (37, 96, 100), (300, 3072, 768)])
def test_linear_w8a32(ltm, orc, act, M, N, K):
    import torch
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    qw, sw = orc.quant_int8_rows(w)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    y = ltm.linear_w8a32(dev(a), dev(qw), dev(sw), dev(b), act)
    ref = orc.linear_w8a32(a, qw, sw, b, act)
    assert_close(as_f32(y), ref, 1e-4, 1e-4, "w8a32")


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (300, 384, 1024), (64, 4096, 4096),
                                   (130, 11008 // 32 * 32, 512),
                                   # small grids: K split over CTAs, partials summed by the epilogue
                                   (1, 8192, 4096), (3, 256, 11008), (64, 11008, 4096),
                                   (129, 512, 2048)])
def test_linear_w4a16(ltm, orc, dt, act, M, N, K):
    import torch
    rng = np.random.default_rng(M + N + K + act)
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    packed, s, zp = orc.quant_int4_g128(w)
    ad = to_device(a, dt)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    y = ltm.linear_w4a16(ad, dev(packed), dev(s), dev(zp), dev(b), act)
    ref = orc.round_to(orc.linear_w4a16(as_f32(ad), packed, s, zp, b, act, orc_dtype(dt)),
                       orc_dtype(dt))
    assert_close(as_f32(y), ref, 2e-2, 1e-2, f"w4a16 {dt}")


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("scores", [True, False])
@pytest.mark.parametrize("Ms,H,nh,T", [(64, 256, 4, 96), (512, 768, 12, 2048), (2048, 4096, 32, 64)])
def test_memory_store(ltm, orc, dt, scores, Ms, H, nh, T):
    """MemoryBank::store: slot weights from the mean memory query, EMA of the bank."""
    import torch
    rng = np.random.default_rng(Ms + H + T)
    mem = (rng.standard_normal((Ms, H)) / np.sqrt(H)).astype(np.float32)
    kv = rng.standard_normal((Ms, 2 * H)).astype(np.float32)
    qkvm = rng.standard_normal((T, 4 * H)).astype(np.float32)
    qkvm[:, 3 * H:] += 2.0 * rng.standard_normal(H).astype(np.float32)  # a shared query direction
    state = (0.3 * rng.standard_normal(H)).astype(np.float32)
    memd, kvd, qd = to_device(mem, dt), to_device(kv, dt), to_device(qkvm, dt)
    mem0 = as_f32(memd)
    rate = 0.5
    ltm.memory_store(memd, kvd[:, :H], qd[:, 3 * H:], torch.from_numpy(state).cuda(), nh, rate,
                     scores)
    ref = orc.memory_store(mem0, as_f32(kvd)[:, :H], as_f32(qd)[:, 3 * H:], state, nh, rate,
                           scores, orc_dtype(dt))
    atol, rtol = (1e-5, 1e-4) if dt == "f32" else (2e-3, 1e-2)
    assert_close(as_f32(memd), ref, atol, rtol, what=f"memory store {dt}")
    assert np.abs(ref - mem0).max() > (1e-4 if scores else 1e-2)  # the bank moved
    assert ltm.device_error() == 0


def test_memory_store_rejects_bad_arguments(ltm):
    import torch
    mem = torch.zeros((8, 64), device="cuda")
    state = torch.zeros(64, device="cuda")
    with pytest.raises(ltm.LtmError):
        ltm.memory_store(mem, mem, mem[:0], state, 4, 0.9, True)  # no query rows
    with pytest.raises(ltm.LtmError):
        ltm.memory_store(mem, mem, mem, state, 3, 0.9, True)  # 64 % 3 != 0
