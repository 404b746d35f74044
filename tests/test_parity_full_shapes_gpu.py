"""Parity against the oracle at the workloads' own sizes, where the smaller
op and block tests stop short of them:

* the 12-layer prefill's block exactly (W8A8, fp16, hidden 768, 12 heads,
  FFN 3072, 512 slots) over one 2048-token sequence, at the absolute bar;
* tcgen05 causal attention at 2048 (head_dim 64) and 8192 (head_dim 128)
  positions, including scores that climb along the keys so the running
  maximum is raised again and again (the lazy rescale of O in TMEM fires
  many times) and scores that fall (it never fires);
* memory attention over 4096- and 8192-slot banks;
* the decode step against a 32768-position cache, random and climbing keys;
* the hidden-4096 and hidden-8192 blocks stage by stage: every stage of the
  device's forward is recomputed by the oracle from the device's own input
  to that stage (its rounded activations, its int8 codes and scales), so
  each op is held to the absolute bar on its own -- int8 codes of a stage's
  input bit-exact, 16-bit outputs within max-abs 2e-2 / rel 1e-2.
"""
import numpy as np
import pytest

from _util import as_f32, assert_close, orc_dtype, to_device
from test_block_gpu import make, run_block

pytestmark = pytest.mark.gpu

TOL = {"f16": (2e-2, 1e-2), "bf16": (2e-2, 1e-2)}


def test_prefill_workload_block_w8a8_f16(ltm, orc):
    """One block of the 12-layer W8A8 prefill at its shape over a full
    2048-token sequence (batch 1 keeps the oracle within seconds)."""
    blk, *_, y, ref, _, _ = run_block(ltm, orc, "w8a8", "f16", H=768, nh=12, F=3072, Ms=512,
                                      B=1, S=2048, seed=21)
    assert_close(as_f32(y).reshape(ref.shape), ref, *TOL["f16"], what="prefill block S=2048")
    assert ltm.device_error() == 0
    blk.close()


def _scores_ramp(S, nh, D, slope, seed, dt):
    """q, k, v rows [S, nh*D]: a shared unit direction in q, keys whose
    component along it grows (slope > 0) or shrinks linearly with the key
    position, so the scaled score of key j is about slope * j / S plus noise."""
    rng = np.random.default_rng(seed)
    H = nh * D
    q = rng.standard_normal((S, H)).astype(np.float32) * 0.3
    k = rng.standard_normal((S, H)).astype(np.float32) * 0.3
    v = rng.standard_normal((S, H)).astype(np.float32)
    pos = np.arange(S, dtype=np.float32) / S
    for h in range(nh):
        q[:, h * D] += 4.0
        k[:, h * D] += slope * np.sqrt(D) / 4.0 * pos
    return to_device(q, dt), to_device(k, dt), to_device(v, dt)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("S,D,nh", [(2048, 64, 2), (8192, 128, 1)])
@pytest.mark.parametrize("slope", [0.0, 600.0, -300.0])
def test_causal_attention_long_sequences(ltm, orc, dt, S, D, nh, slope):
    """slope 600: the row maximum climbs by ~600 (natural log units) over the
    keys, i.e. by ~865 in the kernel's log2 units, raising the reference
    maximum past its 2^8 threshold on the order of a hundred times per row."""
    qd, kd, vd = _scores_ramp(S, nh, D, slope, S + D + int(slope), dt)
    o = ltm.attention(qd, kd, vd, 1, S, S, nh, D, True)
    ref = orc.attention(as_f32(qd), as_f32(kd), as_f32(vd), 1, S, S, nh, D, True, orc_dtype(dt))
    assert_close(as_f32(o), ref, *TOL[dt], what=f"causal S={S} D={D} slope={slope}")
    assert ltm.device_error() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("Ms", [4096, 8192])
@pytest.mark.parametrize("slope", [0.0, 400.0])
def test_memory_attention_large_banks(ltm, orc, dt, Ms, slope):
    B, S, nh, D = 2, 128, 2, 128
    H = nh * D
    rng = np.random.default_rng(Ms + int(slope))
    q = rng.standard_normal((B * S, H)).astype(np.float32) * 0.3
    kv = rng.standard_normal((Ms, 2 * H)).astype(np.float32) * 0.3
    pos = np.arange(Ms, dtype=np.float32) / Ms
    for h in range(nh):
        q[:, h * D] += 4.0
        kv[:, h * D] += slope * np.sqrt(D) / 4.0 * pos
    qd, kvd = to_device(q, dt), to_device(kv, dt)
    o = ltm.attention(qd, kvd[:, :H], kvd[:, H:], B, S, Ms, nh, D, False, kv_shared=True)
    kf = as_f32(kvd)
    ref = orc.attention(as_f32(qd), kf[:, :H], kf[:, H:], B, S, Ms, nh, D, False, orc_dtype(dt),
                        kv_shared=True)
    assert_close(as_f32(o), ref, *TOL[dt], what=f"memory attention Ms={Ms} slope={slope}")
    assert ltm.device_error() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("climb", [False, True])
def test_decode_32768_position_cache(ltm, orc, dt, climb):
    """The decode workload's cache length (32768 positions, the new token at
    position 32767) for one sequence of 2 heads of 128; with climb the cached
    keys' scores rise along the positions, so the split-cache chunks' maxima
    differ by hundreds and the combine step must rescale them."""
    from ltm_b200 import synthetic
    from test_decode_gpu import _caches, _round
    H, nh, F, Ms, B, P = 256, 2, 512, 64, 1, 32768
    L = P - 1
    cfg, q, ocfg = make(ltm, "w4a16", dt, H, nh, F, Ms)
    w = synthetic.block_weights(H, F, Ms, 31)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    fill = None
    if climb:
        rng = np.random.default_rng(32)
        kf = rng.standard_normal((B, L, H)).astype(np.float32)
        vf = rng.standard_normal((B, L, H)).astype(np.float32)
        ramp = np.linspace(0.0, 120.0, L, dtype=np.float32)
        kf += ramp[None, :, None]  # every dimension: scores follow the query's sum
        fill = (kf, vf)
    kd, vd, kh, vh = _caches(B, P, H, nh, L, dt, 33, fill=fill)
    mem = orc.round_to(w["memory"], ocfg["dtype"])
    kvm = orc.block_kvm(ocfg, w, mem)
    x = _round(synthetic.activations(B, H, 34), dt)
    y = blk.decode_step(to_device(x, dt), kd, vd, L)
    ref = orc.block_decode_step(ocfg, w, x, kh, vh, L, mem, kvm)
    assert_close(as_f32(y), ref, *TOL[dt], what=f"decode P=32768 climb={climb}")
    assert ltm.device_error() == 0
    blk.close()


# ------------------------------------------------------------ stage by stage --
def _rope(orc, rows, S, dh, width):
    """The oracle's interleaved RoPE on the first `width` columns of fp32 rows
    (row t at position t % S), in fp32 without contraction."""
    tab = orc.rope_table(S, dh)
    out = rows.copy()
    T = rows.shape[0]
    pos = np.arange(T) % S
    cols = np.arange(0, width, 2)
    i = (cols % dh) // 2
    cs = tab[pos[:, None], i[None, :], 0]
    sn = tab[pos[:, None], i[None, :], 1]
    a = rows[:, cols]
    b = rows[:, cols + 1]
    out[:, cols] = (a * cs).astype(np.float32) - (b * sn).astype(np.float32)
    out[:, cols + 1] = (a * sn).astype(np.float32) + (b * cs).astype(np.float32)
    return out


def _check_ln_codes(orc, q_dev, s_dev, x_in, g, b, what):
    """LN(x + x) of the device's stage input recomputed by the oracle: the
    per-token scales agree to fp32 rounding, and the int8 codes agree except
    where the oracle's value lies on a rounding boundary (the device's LN
    sums in another order, which moves values by a few fp32 ulps)."""
    ln = orc.layernorm_x2(x_in, g, b)
    q_ref, s_ref = orc.quant_int8_rows(ln)
    s_dev = np.asarray(s_dev, np.float32)
    assert_close(s_dev, s_ref, 0.0, 2e-6, what=f"{what} scales")
    diff = q_dev.astype(np.int32) - q_ref.astype(np.int32)
    assert np.abs(diff).max() <= 1, f"{what}: codes differ by more than one step"
    if diff.any():
        r, c = np.nonzero(diff)
        t = ln[r, c] / s_ref[r]
        frac = np.abs(np.abs(t - np.trunc(t)) - 0.5)
        assert frac.max() < 1e-3, f"{what}: a code differs away from a rounding boundary"
        assert diff.astype(bool).mean() < 1e-3, f"{what}: too many boundary flips"


def _cat(*a):
    return np.concatenate(a, axis=0)


@pytest.mark.parametrize("scheme,H,nh,F,S", [("w8a8", 4096, 32, 11008, 256),
                                             ("w4a16", 4096, 32, 11008, 256),
                                             ("w8a8", 8192, 64, 28672, 128),
                                             # the tensor-parallel tests' FFN-8192 block
                                             ("w8a8", 512, 8, 8192, 96)])
def test_wide_block_stage_by_stage(ltm, orc, scheme, H, nh, F, S):
    import torch
    from ltm_b200 import synthetic
    dt, B, Ms = "bf16", 1, 256
    T, dh, odt = B * S, H // nh, orc_dtype("bf16")
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms)
    w = synthetic.block_weights(H, F, Ms, 41)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    x = synthetic.activations(T, H, 42)
    xd = to_device(x, dt)
    out = as_f32(blk(xd.reshape(B, S, H))).reshape(T, H)
    xf = as_f32(xd)
    st = {n: blk.intermediate(n) for n in ("qkvm", "kvm", "attn_self", "attn_mem", "s", "m", "y",
                                           "ffn_hidden")}
    w8 = scheme == "w8a8"
    if w8:
        for n in ("ln1_q", "ln1_s", "x_q", "x_s", "attn_self_q", "attn_self_s", "attn_mem_q",
                  "attn_mem_s", "ln2_q", "ln2_s", "ffn_hidden_q", "ffn_hidden_s"):
            st[n] = blk.intermediate(n)
    else:
        st["ln1"] = blk.intermediate("ln1")
        st["ln2"] = blk.intermediate("ln2")
    st = {k: (v.cpu().numpy() if v.dtype in (torch.int8, torch.float32) else as_f32(v))
          for k, v in st.items()}
    mem_dev = as_f32(blk.memory())

    def lin(name, wmat, bias, a=None, qa=None, sa=None, act=0):
        """The oracle's linear of the block's quantized weight on the
        device's stage input (fp32 result, before the dtype rounding)."""
        if w8:
            qw, sw = orc.quant_int8_rows(wmat)
            return orc.linear_w8a8(qa, sa, qw, sw, bias, act)
        packed, s4, zp = orc.quant_int4_g128(wmat)
        return orc.linear_w4a16(a, packed, s4, zp, bias, act, odt)

    def rnd(a):
        return orc.round_to(a, odt)

    def close(got, want, what):
        assert_close(got, want, *TOL[dt], what=f"H{H} {scheme}: {what}")

    # 1. LN1 (+ per-token int8 of LN1(x) and of x)
    if w8:
        _check_ln_codes(orc, st["ln1_q"], st["ln1_s"], xf, w["ln1_g"], w["ln1_b"], "LN1 codes")
        xq, xs = orc.quant_int8_rows(xf)
        assert np.array_equal(st["x_q"], xq) and np.array_equal(st["x_s"], xs), "x codes"
    else:
        close(st["ln1"], rnd(orc.layernorm_x2(xf, w["ln1_g"], w["ln1_b"])), "LN1")
    # 2. Q | K | V | Qm with RoPE on Q, K
    wq = _cat(w["w_qkv"], w["w_qm"])
    bq = _cat(w["b_qkv"], w["b_qm"])
    qkvm = lin("qkvm", wq, bq, a=None if w8 else st["ln1"], qa=st.get("ln1_q"),
               sa=st.get("ln1_s"))
    close(st["qkvm"], rnd(_rope(orc, qkvm, S, dh, 2 * H)), "Q|K|V|Qm with RoPE")
    # 3. K_M | V_M of the device's bank
    if w8:
        mq, ms = orc.quant_int8_rows(mem_dev)
        kvm = lin("kvm", _cat(w["w_km"], w["w_vm"]), _cat(w["b_km"], w["b_vm"]), qa=mq, sa=ms)
    else:
        kvm = lin("kvm", _cat(w["w_km"], w["w_vm"]), _cat(w["b_km"], w["b_vm"]), a=mem_dev)
    close(st["kvm"], rnd(kvm), "K_M|V_M")
    # 4. attentions on the device's projections
    qd = st["qkvm"]
    os_ref = orc.attention(qd[:, :H], qd[:, H:2 * H], qd[:, 2 * H:3 * H], B, S, S, nh, dh, True,
                           odt)
    close(st["attn_self"], os_ref, "causal self-attention")
    om_ref = orc.attention(qd[:, 3 * H:], st["kvm"][:, :H], st["kvm"][:, H:], B, S, Ms, nh, dh,
                           False, odt, kv_shared=True)
    close(st["attn_mem"], om_ref, "memory attention")
    # 5. output projections (int8 codes of the attention outputs bit-exact)
    if w8:
        for n in ("attn_self", "attn_mem"):
            qr, sr = orc.quant_int8_rows(st[n])
            assert np.array_equal(st[n + "_q"], qr) and np.array_equal(st[n + "_s"], sr), n
    s_ref = lin("o", w["w_o"], w["b_o"], a=None if w8 else st["attn_self"],
                qa=st.get("attn_self_q"), sa=st.get("attn_self_s"))
    close(st["s"], rnd(s_ref), "output projection s")
    m_ref = lin("om", w["w_om"], w["b_om"], a=None if w8 else st["attn_mem"],
                qa=st.get("attn_mem_q"), sa=st.get("attn_mem_s"))
    close(st["m"], rnd(m_ref), "memory output projection m")
    # 6. gate and gated integration on the device's s, m and x
    g = lin("g", w["w_g"], w["b_g"], a=xf, qa=st.get("x_q"), sa=st.get("x_s"), act=orc.ACT_SIGMOID)
    y_ref = rnd(st["s"] + g * st["m"] + (np.float32(1) - g) * xf)
    close(st["y"], y_ref, "gated integration y")
    # 7. LN2, FFN up with GELU, FFN down with the residual
    if w8:
        _check_ln_codes(orc, st["ln2_q"], st["ln2_s"], st["y"], w["ln2_g"], w["ln2_b"],
                        "LN2 codes")
    else:
        close(st["ln2"], rnd(orc.layernorm_x2(st["y"], w["ln2_g"], w["ln2_b"])), "LN2")
    u = lin("w1", w["w_1"], w["b_1"], a=None if w8 else st["ln2"], qa=st.get("ln2_q"),
            sa=st.get("ln2_s"), act=orc.ACT_GELU)
    close(st["ffn_hidden"], rnd(u), "FFN hidden (GELU)")
    if w8:
        qr, sr = orc.quant_int8_rows(st["ffn_hidden"])
        assert np.array_equal(st["ffn_hidden_q"], qr) and np.array_equal(st["ffn_hidden_s"], sr)
    f = lin("w2", w["w_2"], w["b_2"], a=None if w8 else st["ffn_hidden"],
            qa=st.get("ffn_hidden_q"), sa=st.get("ffn_hidden_s"))
    close(out, rnd(f + st["y"]), "block output (FFN down + residual)")
    assert ltm.device_error() == 0
    blk.close()
