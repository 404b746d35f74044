"""TitanBlock / TitanModel forward on the GPU (through the C ABI) against the
TB-v1 CPU oracle, for every quantization scheme, with and without the memory
write, including the fp32 parity workload (hidden 768, seq 512) at 1e-4."""
import numpy as np
import pytest

from _util import as_f32, assert_close, orc_dtype, to_device

pytestmark = pytest.mark.gpu

SCHEMES = [("w8a32", "f32"), ("w8a8", "f16"), ("w8a8", "bf16"), ("w4a16", "bf16"), ("w4a16", "f16")]
TOL = {"f32": (1e-4, 1e-4), "f16": (2e-2, 1e-2), "bf16": (2e-2, 1e-2)}


def make(ltm, scheme, dt, H, nh, F, Ms, memory_write=False, scores=True, **cfg_kw):
    sch = {"w8a32": ltm.SCHEME_W8A32, "w8a8": ltm.SCHEME_W8A8, "w4a16": ltm.SCHEME_W4A16}[scheme]
    dtc = {"f32": ltm.DTYPE_F32, "f16": ltm.DTYPE_F16, "bf16": ltm.DTYPE_BF16}[dt]
    cfg = ltm.TitanBlockConfig(hidden_dim=H, ffn_dim=F, num_heads=nh, head_dim=H // nh,
                               memory_slots=Ms, **cfg_kw)
    q = ltm.QuantConfig(scheme=sch, act_dtype=dtc, memory_write=memory_write,
                        use_attention_scores=scores)
    ocfg = dict(H=H, F=F, nh=nh, dh=H // nh, Ms=Ms, scheme=sch, dtype=orc_dtype(dt),
                memory_write=int(memory_write), use_attention_scores=int(scores),
                update_rate=cfg.memory_update_rate, use_rotary=int(cfg.use_rotary),
                use_bias=int(cfg.use_bias), use_layer_norm=int(cfg.use_layer_norm),
                use_memory_gating=int(cfg.use_memory_gating))
    return cfg, q, ocfg


def run_block(ltm, orc, scheme, dt, H=256, nh=4, F=512, Ms=64, B=2, S=96, seed=0, **kw):
    from ltm_b200 import synthetic
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms, **kw)
    w = synthetic.block_weights(H, F, Ms, seed)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    x = synthetic.activations(B * S, H, seed + 1)
    xd = to_device(x, dt).reshape(B, S, H)
    y = blk(xd)
    ref, mem_ref = orc.block_forward(ocfg, w, as_f32(xd).reshape(B * S, H), B, S)
    return blk, w, xd, y, ref, mem_ref, ocfg


@pytest.mark.parametrize("scheme,dt", SCHEMES)
@pytest.mark.parametrize("nh", [4, 2])   # head_dim 64 and 128
def test_block_forward_matches_oracle(ltm, orc, scheme, dt, nh):
    blk, *_, y, ref, _, _ = run_block(ltm, orc, scheme, dt, nh=nh)
    assert_close(as_f32(y).reshape(ref.shape), ref, *TOL[dt], what=f"block {scheme} {dt}")
    assert ltm.device_error() == 0
    blk.close()


@pytest.mark.parametrize("scheme,dt", SCHEMES)
@pytest.mark.parametrize("scores", [True, False])
def test_block_memory_write(ltm, orc, scheme, dt, scores):
    """The bank after the write, and a second forward that reads it."""
    blk, w, xd, y, ref, mem_ref, ocfg = run_block(ltm, orc, scheme, dt, memory_write=True,
                                                  scores=scores, S=64)
    assert_close(as_f32(y).reshape(ref.shape), ref, *TOL[dt], what="first forward")
    mem = as_f32(blk.memory())
    atol = 1e-5 if dt == "f32" else 2e-3
    assert_close(mem, mem_ref, atol, 1e-2 if dt != "f32" else 1e-4, what="bank after write")
    assert not np.allclose(mem_ref, orc.round_to(w["memory"], ocfg["dtype"]))  # bank moved
    y2 = blk(xd)
    B, S, H = xd.shape
    ref2, _ = orc.block_forward(ocfg, w, as_f32(xd).reshape(B * S, H), B, S, memory=mem_ref)
    assert_close(as_f32(y2).reshape(ref2.shape), ref2, *TOL[dt], what="second forward")
    blk.close()


def test_block_fp32_parity_workload(ltm, orc):
    """hidden 768, 12 heads, FFN 3072, 512 slots, batch 1, seq 512, fp32 at 1e-4."""
    blk, *_, y, ref, _, _ = run_block(ltm, orc, "w8a32", "f32", H=768, nh=12, F=3072, Ms=512,
                                      B=1, S=512, seed=0)
    assert_close(as_f32(y).reshape(ref.shape), ref, 1e-4, 1e-4, what="c1 fp32 block")
    blk.close()


def _nudge_bf16_ulp(x: np.ndarray, frac: float, seed: int) -> np.ndarray:
    """x (bf16-representable fp32) with `frac` of its entries moved by one bf16 ulp."""
    import torch
    bits = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16)
    bits = bits.view(torch.int16).numpy().copy()
    rng = np.random.default_rng(seed)
    m = rng.random(bits.shape) < frac
    bits[m] += rng.choice([-1, 1], size=int(m.sum())).astype(np.int16)
    return torch.from_numpy(bits).view(torch.bfloat16).float().numpy()


def _outside(got, want, atol, rtol):
    err = np.abs(np.asarray(got, np.float64) - want)
    return float((err > atol + rtol * np.abs(want)).mean()), float(err.max())


@pytest.mark.parametrize("scheme,dt", [("w8a8", "bf16"), ("w4a16", "bf16")])
def test_block_large_hidden(ltm, orc, scheme, dt):
    """hidden 4096, 32 heads of 128: the CTA-per-row LayerNorm + quantizer, the
    4-warp row quantizer, GEMMs at K = 4096, head_dim 128 attention.

    At this width the block output is sensitive to one-ulp changes of its
    input at the level of the bf16 tolerance: the oracle run on inputs with
    one-ulp nudges on 10% of the entries leaves ~30% (W8A8: per-token int8
    codes of bf16 intermediates flip at rounding boundaries and the flips add
    up over K = 4096) or ~0.2% (W4A16) of the outputs outside 2e-2 / 1e-2.  The
    parity check is therefore relative: the GPU's deviation from the oracle
    must not exceed the oracle's own one-ulp sensitivity on the same inputs
    (integer stages stay bit-exact in the quantizer and GEMM tests)."""
    B, S, H = 1, 128, 4096
    blk, w, xd, y, ref, _, ocfg = run_block(ltm, orc, scheme, dt, H=H, nh=32, F=4096, Ms=256,
                                            B=B, S=S, seed=5)
    got = as_f32(y).reshape(ref.shape)
    x = as_f32(xd).reshape(B * S, H)
    ref_nudged, _ = orc.block_forward(ocfg, w, _nudge_bf16_ulp(x, 0.1, 9), B, S)
    sens_frac, sens_max = _outside(ref_nudged, ref, *TOL[dt])
    gpu_frac, gpu_max = _outside(got, ref, *TOL[dt])
    if scheme == "w8a8":
        assert sens_frac > 0.05, "the sensitivity premise no longer holds: tighten this test"
    assert gpu_frac <= max(sens_frac, 1e-5) and gpu_max <= 1.25 * sens_max, (
        f"GPU outside {gpu_frac:.4f} (max {gpu_max:.3e}) vs oracle one-ulp sensitivity "
        f"{sens_frac:.4f} (max {sens_max:.3e})")
    blk.close()


@pytest.mark.parametrize("flags", [dict(use_rotary=False), dict(use_bias=False),
                                   dict(use_layer_norm=False), dict(use_memory_gating=False)])
def test_block_config_flags(ltm, orc, flags):
    blk, *_, y, ref, _, _ = run_block(ltm, orc, "w8a8", "f16", **flags)
    assert_close(as_f32(y).reshape(ref.shape), ref, 2e-2, 1e-2, what=str(flags))
    blk.close()


def test_block_rejects_mask_and_aliasing(ltm):
    import torch
    cfg, q, _ = make(ltm, "w8a8", "f16", 256, 4, 512, 64)
    from ltm_b200 import synthetic
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(synthetic.block_weights(256, 512, 64, 0))
    x = torch.zeros((1, 16, 256), dtype=torch.float16, device="cuda")
    with pytest.raises(ltm.LtmError) as e:
        blk.forward(x, attention_mask=x)
    assert e.value.status == ltm.ERR_UNSUPPORTED
    with pytest.raises(ltm.LtmError):
        ltm._check(ltm.lib().ltm_block_forward(blk._h, ltm._ptr(x), ltm._ptr(x), None, 1, 16,
                                               ltm._stream()))
    blk.close()


@pytest.mark.parametrize("scheme,dt", [("w8a8", "f16"), ("w4a16", "bf16")])
def test_model_embedding_and_layers(ltm, orc, scheme, dt):
    import torch
    from ltm_b200 import synthetic
    H, nh, F, Ms, V, L, B, S = 256, 4, 512, 64, 1000, 2, 2, 64
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms)
    model = ltm.TitanModel(cfg, q, L, V)
    emb = synthetic.embedding(V, H, 11)
    model.load_embedding(emb)
    layers = [synthetic.block_weights(H, F, Ms, 100 + i) for i in range(L)]
    for i, w in enumerate(layers):
        model.load_layer(i, w)
    tok = synthetic.tokens(B, S, V, 5)
    y = model(torch.from_numpy(tok).cuda())
    ref = orc.model_forward(ocfg, layers, emb, tok, B, S)
    assert_close(as_f32(y).reshape(ref.shape), ref, *TOL[dt], what=f"model {scheme}")
    model.close()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("H,nh,F", [(256, 4, 512), (384, 3, 768)])
def test_block_w4a16_large_m(ltm, orc, dt, H, nh, F):
    """W4A16 at M >= 1024 tokens: every linear dequantises its INT4 weight
    once and runs the persistent 16-bit tcgen05 GEMM (CTA-pair tiles when N is
    a multiple of 256, 128-wide tiles otherwise) with each fused epilogue;
    1024 memory slots take the same path for K_M / V_M; the memory write and
    a second forward over the written bank."""
    blk, w, xd, y, ref, mem_ref, ocfg = run_block(ltm, orc, "w4a16", dt, H=H, nh=nh, F=F,
                                                  Ms=1024, B=2, S=640, seed=4,
                                                  memory_write=True)
    assert_close(as_f32(y).reshape(ref.shape), ref, *TOL[dt], what=f"w4a16 large-M {dt} H{H}")
    assert_close(as_f32(blk.memory()), mem_ref, 2e-3, 1e-2, what="bank after the write")
    B, S = 2, 640
    y2 = blk(xd)
    ref2, _ = orc.block_forward(ocfg, w, as_f32(xd).reshape(B * S, H), B, S, memory=mem_ref)
    assert_close(as_f32(y2).reshape(ref2.shape), ref2, *TOL[dt], what="second forward")
    assert ltm.device_error() == 0
    blk.close()


def test_empty_batches_are_no_ops(ltm):
    """B = 0 or S = 0 forwards, a B = 0 decode step and M = 0 linears return
    OK without touching their outputs."""
    import torch
    from ltm_b200 import synthetic
    H, nh, F, Ms = 256, 4, 512, 64
    cfg, q, _ = make(ltm, "w4a16", "bf16", H, nh, F, Ms)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(synthetic.block_weights(H, F, Ms, 23))
    for shape in ((0, 16, H), (2, 0, H)):
        x = torch.zeros(shape, dtype=torch.bfloat16, device="cuda")
        y = torch.full(shape, 7.0, dtype=torch.bfloat16, device="cuda")
        blk.forward(x, out=y)
        assert torch.all(y == 7.0)
    x = torch.zeros((0, H), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((0, nh, 8, H // nh), dtype=torch.bfloat16, device="cuda")
    assert blk.decode_step(x, kc, torch.zeros_like(kc), 0).shape == (0, H)
    packed, s, zp = ltm.quantize_int4_grouped(torch.zeros((64, 256), device="cuda"))
    y = ltm.linear_w4a16(torch.zeros((0, 256), dtype=torch.bfloat16, device="cuda"), packed, s, zp)
    assert y.shape == (0, 64)
    assert ltm.device_error() == 0
    blk.close()
