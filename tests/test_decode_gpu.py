"""Batched decode step (ltm_block_decode_step) and the block memory write
(ltm_block_memory_write) on the GPU against the TB-v1 oracle:

* a decode step over a cache that holds the oracle's post-RoPE keys / values of
  a prefix equals the last row of the oracle's full causal forward over the
  prefix plus the new token (the decode step is the prefill's last row);
* several decode steps with the memory write (bank and resident K_M | V_M
  following the EMA) match the oracle's decode steps, step by step;
* caches long enough for many split-cache chunks, with a ragged last chunk,
  and the empty-prefix edge case (cache_len = 0);
* argument errors come back as LTM_ERR_INVALID_ARG."""
import numpy as np
import pytest

from _util import as_f32, assert_close, orc_dtype, to_device
from test_block_gpu import make

pytestmark = pytest.mark.gpu

TOL = {"f16": (2e-2, 1e-2), "bf16": (2e-2, 1e-2)}
SCHEMES = [("w8a8", "f16"), ("w8a8", "bf16"), ("w4a16", "bf16"), ("w4a16", "f16")]


def _round(a, dt):
    import torch
    from _util import torch_dtype
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch_dtype(dt)).float().numpy()


def _heads(a, nh):
    """[B, L, H] rows -> head-major [B, nh, L, dh]."""
    B, L, H = a.shape
    return np.ascontiguousarray(a.reshape(B, L, nh, H // nh).transpose(0, 2, 1, 3))


def _caches(B, P, H, nh, L, dt, seed, fill=None):
    """Head-major device caches [B, nh, P, dh] whose first L positions hold
    `fill` ([B, L, H] rows of K and of V) or seeded N(0,1) values, and the
    rest a sentinel that must not be read."""
    import torch
    from _util import torch_dtype
    rng = np.random.default_rng(seed)
    dh = H // nh
    k = np.full((B, nh, P, dh), 1e4, np.float32)  # a read past the cache would blow up the result
    v = np.full((B, nh, P, dh), -1e4, np.float32)
    if L:
        kf, vf = fill if fill is not None else (rng.standard_normal((B, L, H)),
                                                rng.standard_normal((B, L, H)))
        k[:, :, :L] = _heads(_round(kf, dt), nh)
        v[:, :, :L] = _heads(_round(vf, dt), nh)
    td = torch_dtype(dt)
    return (torch.from_numpy(k).to(td).cuda(), torch.from_numpy(v).to(td).cuda(),
            k.copy(), v.copy())


@pytest.mark.parametrize("scheme,dt", SCHEMES)
@pytest.mark.parametrize("nh", [4, 2])  # head_dim 64 and 128
def test_decode_is_last_row_of_prefill(ltm, orc, scheme, dt, nh):
    from ltm_b200 import synthetic
    H, F, Ms, B, L, P = 256, 512, 64, 3, 37, 48
    S = L + 1
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms)
    w = synthetic.block_weights(H, F, Ms, 5)
    x = _round(synthetic.activations(B * S, H, 6), dt)
    y_full, _, kv = orc.block_forward(ocfg, w, x, B, S, return_kv=True)
    kv = kv.reshape(B, S, 2 * H)
    kd, vd, _, _ = _caches(B, P, H, nh, L, dt, 0, fill=(kv[:, :L, :H], kv[:, :L, H:]))
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    xt = to_device(x.reshape(B, S, H)[:, L], dt)
    y = blk.decode_step(xt, kd, vd, L)
    want = y_full.reshape(B, S, H)[:, L]
    assert_close(as_f32(y), want, *TOL[dt], what=f"decode {scheme} {dt} vs prefill row")
    # the step appended the new token's key / value at position L
    assert_close(as_f32(kd[:, :, L]), _heads(kv[:, L:L + 1, :H], nh)[:, :, 0], *TOL[dt],
                 what="appended K")
    assert_close(as_f32(vd[:, :, L]), _heads(kv[:, L:L + 1, H:], nh)[:, :, 0], *TOL[dt],
                 what="appended V")
    sentinel = _round(np.float32(1e4), dt)
    assert np.all(as_f32(kd[:, :, L + 1:]) == sentinel), "positions past the new token were written"
    assert ltm.device_error() == 0
    blk.close()


@pytest.mark.parametrize("scheme,dt", SCHEMES)
@pytest.mark.parametrize("scores", [True, False])
def test_decode_steps_with_memory_write(ltm, orc, scheme, dt, scores):
    from ltm_b200 import synthetic
    H, nh, F, Ms, B, L0, P, steps = 256, 4, 512, 64, 4, 20, 40, 4
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms, memory_write=True, scores=scores)
    w = synthetic.block_weights(H, F, Ms, 7)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    kd, vd, kh, vh = _caches(B, P, H, nh, L0, dt, 8)
    mem = orc.round_to(w["memory"], ocfg["dtype"])
    kvm = orc.block_kvm(ocfg, w, mem)
    for i in range(steps):
        x = _round(synthetic.activations(B, H, 100 + i), dt)
        y = blk.decode_step(to_device(x, dt), kd, vd, L0 + i)
        ref = orc.block_decode_step(ocfg, w, x, kh, vh, L0 + i, mem, kvm)
        assert_close(as_f32(y), ref, *TOL[dt], what=f"step {i} {scheme} {dt}")
        # keep the oracle's cache on the device's values so the steps stay comparable
        kh[:, :, L0 + i] = as_f32(kd[:, :, L0 + i])
        vh[:, :, L0 + i] = as_f32(vd[:, :, L0 + i])
    assert_close(as_f32(blk.memory()), mem, 2e-3, 1e-2, what="bank after the decode writes")
    assert ltm.device_error() == 0
    blk.close()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("nh,L", [(2, 1537), (4, 2048), (2, 4095), (4, 0), (2, 1)])
def test_decode_long_and_edge_caches(ltm, orc, dt, nh, L):
    """Caches spanning many 512-position chunks (ragged last chunk), and the
    first token of a sequence (cache_len 0: the step attends to itself)."""
    from ltm_b200 import synthetic
    H, F, Ms, B = 256, 512, 64, 2
    P = L + 3
    cfg, q, ocfg = make(ltm, "w4a16", dt, H, nh, F, Ms)
    w = synthetic.block_weights(H, F, Ms, 9)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    kd, vd, kh, vh = _caches(B, P, H, nh, L, dt, 10)
    mem = orc.round_to(w["memory"], ocfg["dtype"])
    kvm = orc.block_kvm(ocfg, w, mem)
    x = _round(synthetic.activations(B, H, 11), dt)
    y = blk.decode_step(to_device(x, dt), kd, vd, L)
    ref = orc.block_decode_step(ocfg, w, x, kh, vh, L, mem, kvm)
    assert_close(as_f32(y), ref, *TOL[dt], what=f"decode L={L}")
    assert ltm.device_error() == 0
    blk.close()


def test_decode_after_forward_recomputes_memory_keys(ltm, orc):
    """A forward that writes the bank invalidates the resident K_M | V_M: the
    next decode step reads the keys / values of the new bank."""
    from ltm_b200 import synthetic
    H, nh, F, Ms, B, S, P, dt = 256, 4, 512, 64, 2, 16, 32, "bf16"
    cfg, q, ocfg = make(ltm, "w4a16", dt, H, nh, F, Ms, memory_write=True)
    w = synthetic.block_weights(H, F, Ms, 12)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    kd, vd, kh, vh = _caches(B, P, H, nh, 5, dt, 13)
    x0 = _round(synthetic.activations(B, H, 14), dt)
    blk.decode_step(to_device(x0, dt), kd, vd, 5)  # makes K_M | V_M resident
    xs = _round(synthetic.activations(B * S, H, 15), dt)
    blk(to_device(xs, dt).reshape(B, S, H))  # writes the bank
    mem = as_f32(blk.memory())
    kvm = orc.block_kvm(ocfg, w, mem)
    kh[:, :, 5] = as_f32(kd[:, :, 5])
    vh[:, :, 5] = as_f32(vd[:, :, 5])
    x1 = _round(synthetic.activations(B, H, 16), dt)
    y = blk.decode_step(to_device(x1, dt), kd, vd, 6)
    ref = orc.block_decode_step(ocfg, w, x1, kh, vh, 6, mem, kvm)
    assert_close(as_f32(y), ref, *TOL[dt], what="decode after a writing forward")
    blk.close()


@pytest.mark.parametrize("scores", [True, False])
def test_block_memory_write_api(ltm, orc, scores):
    import torch
    from ltm_b200 import synthetic
    H, nh, F, Ms, T, dt = 256, 4, 512, 64, 5, "bf16"
    cfg, q, ocfg = make(ltm, "w4a16", dt, H, nh, F, Ms, scores=scores)
    w = synthetic.block_weights(H, F, Ms, 17)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    rng = np.random.default_rng(18)
    state = rng.standard_normal(H).astype(np.float32) * 0.1
    qm = _round(rng.standard_normal((T, H)), dt)
    blk.memory_write(torch.from_numpy(state).cuda(), to_device(qm, dt))
    mem = orc.round_to(w["memory"], ocfg["dtype"])
    kvm = orc.block_kvm(ocfg, w, mem)
    mem = orc.memory_store(mem, kvm, qm, state, nh, cfg.memory_update_rate, scores, ocfg["dtype"])
    assert_close(as_f32(blk.memory()), mem, 2e-3, 1e-2, what="bank after ltm_block_memory_write")
    blk.close()


def test_decode_argument_errors(ltm):
    import torch
    from ltm_b200 import synthetic
    H, nh, F, Ms, B, P = 256, 4, 512, 64, 2, 8
    cfg, q, _ = make(ltm, "w4a16", "bf16", H, nh, F, Ms)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(synthetic.block_weights(H, F, Ms, 19))
    x = torch.zeros((B, H), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((B, nh, P, H // nh), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    for bad_len in (P, -1):
        with pytest.raises(ltm.LtmError) as e:
            blk.decode_step(x, kc, vc, bad_len)
        assert e.value.status == ltm.ERR_INVALID_ARG
    with pytest.raises(ltm.LtmError):
        blk.decode_step(x, kc, kc, 0)  # aliased caches
    cfg32, q32, _ = make(ltm, "w8a32", "f32", H, nh, F, Ms)
    b32 = ltm.TitanBlock(cfg32, q32)
    b32.load_weights(synthetic.block_weights(H, F, Ms, 19))
    x32 = torch.zeros((B, H), dtype=torch.float32, device="cuda")
    k32 = torch.zeros((B, nh, P, H // nh), dtype=torch.float32, device="cuda")
    with pytest.raises(ltm.LtmError):
        b32.decode_step(x32, k32, torch.zeros_like(k32), 0)
    assert ltm.device_error() == 0
    blk.close()
    b32.close()


def test_cache_manager_decode_loop(ltm, orc):
    """Two layers through CacheManager + decode_step for a few steps match
    the oracle's decode steps layer by layer."""
    from ltm_b200 import synthetic
    H, nh, F, Ms, B, P, dt = 256, 4, 512, 64, 2, 16, "bf16"
    cfg, q, ocfg = make(ltm, "w4a16", dt, H, nh, F, Ms)
    ws = [synthetic.block_weights(H, F, Ms, 20 + i) for i in range(2)]
    blocks = []
    for w in ws:
        b = ltm.TitanBlock(cfg, q)
        b.load_weights(w)
        blocks.append(b)
    cache = ltm.CacheManager(2, nh, H // nh, __import__("torch").bfloat16)
    cache.allocate(B, P)
    hk = [np.zeros((B, nh, P, H // nh), np.float32) for _ in ws]
    hv = [np.zeros((B, nh, P, H // nh), np.float32) for _ in ws]
    mems = [orc.round_to(w["memory"], ocfg["dtype"]) for w in ws]
    kvms = [orc.block_kvm(ocfg, w, m) for w, m in zip(ws, mems)]
    for step in range(3):
        x = _round(synthetic.activations(B, H, 30 + step), dt)
        pos = cache.length
        y = ltm.decode_step(blocks, to_device(x, dt), cache)
        cur = x
        for i, w in enumerate(ws):
            cur = orc.block_decode_step(ocfg, w, cur, hk[i], hv[i], pos, mems[i], kvms[i])
            k, v, _ = cache.get(i)
            hk[i][:, :, pos] = as_f32(k[:, :, pos])
            hv[i][:, :, pos] = as_f32(v[:, :, pos])
            cur = _round(cur, dt)
        assert_close(as_f32(y), cur, *TOL[dt], what=f"2-layer decode step {step}")
    assert cache.length == 3
    for b in blocks:
        b.close()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_decode_wide_block_split_k(ltm, orc, dt):
    """A block wide enough that the decode GEMMs split K over CTAs (every
    fused epilogue: RoPE, gate-mix with the write's column sums, GELU,
    residual) for a few steps with the memory write."""
    from ltm_b200 import synthetic
    H, nh, F, Ms, B, L0, P = 1024, 8, 2048, 64, 4, 30, 40
    cfg, q, ocfg = make(ltm, "w4a16", dt, H, nh, F, Ms, memory_write=True)
    w = synthetic.block_weights(H, F, Ms, 21)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    kd, vd, kh, vh = _caches(B, P, H, nh, L0, dt, 22)
    mem = orc.round_to(w["memory"], ocfg["dtype"])
    kvm = orc.block_kvm(ocfg, w, mem)
    for i in range(3):
        x = _round(synthetic.activations(B, H, 200 + i), dt)
        y = blk.decode_step(to_device(x, dt), kd, vd, L0 + i)
        ref = orc.block_decode_step(ocfg, w, x, kh, vh, L0 + i, mem, kvm)
        assert_close(as_f32(y), ref, *TOL[dt], what=f"wide step {i} {dt}")
        kh[:, :, L0 + i] = as_f32(kd[:, :, L0 + i])
        vh[:, :, L0 + i] = as_f32(vd[:, :, L0 + i])
    assert_close(as_f32(blk.memory()), mem, 2e-3, 1e-2, what="wide bank after the decode writes")
    assert ltm.device_error() == 0
    blk.close()
