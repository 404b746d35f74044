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
