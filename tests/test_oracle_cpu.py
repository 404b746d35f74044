"""CPU suite for the oracle: independent numpy restatements of the integer
and floating formulas (known answers, ties, zeros, clamps) and the committed
golden fixtures (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from conftest import ROOT

GOLDEN = ROOT / "tests" / "golden" / "oracle_golden.npz"


def np_round_half_away(t):
    t = np.asarray(t, np.float64)  # exact widening of float32 quotients
    return np.sign(t) * np.floor(np.abs(t) + 0.5)


def np_quant_int8_rows(x):
    x = np.asarray(x, np.float32)
    amax = np.max(np.abs(x), axis=1).astype(np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = (x / s[:, None]).astype(np.float32)
    q = np.clip(np_round_half_away(t), -127, 127)
    q[s == 0] = 0
    return q.astype(np.int8), s


def np_quant_int4(w):
    w = np.asarray(w, np.float32)
    N, K = w.shape
    g = w.reshape(N, K // 128, 128)
    mn = np.minimum(g.min(axis=2), np.float32(0))
    mx = np.maximum(g.max(axis=2), np.float32(0))
    s = ((mx - mn) / np.float32(15)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        zp = np.clip(np_round_half_away((-mn / s).astype(np.float32)), 0, 15)
        t = ((g / s[..., None]).astype(np.float32) + zp[..., None].astype(np.float32)).astype(np.float32)
    q = np.clip(np_round_half_away(t), 0, 15)
    q[s == 0] = 0
    zp[s == 0] = 0
    q = q.reshape(N, K).astype(np.uint8)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return packed, s, zp.astype(np.uint8)


@pytest.mark.parametrize("shape", [(1, 1), (7, 100), (64, 768), (3, 3072)])
def test_int8_quant_matches_numpy_restatement(orc, shape):
    rng = np.random.default_rng(shape[1])
    x = (rng.standard_normal(shape) * 0.05).astype(np.float32)
    if shape[0] > 2:
        x[1] = 0
    q, s = orc.quant_int8_rows(x)
    qn, sn = np_quant_int8_rows(x)
    np.testing.assert_array_equal(s, sn)
    np.testing.assert_array_equal(q, qn)


def test_int8_quant_ties_round_half_away(orc):
    s = np.float32(0.25) / np.float32(127)
    k = np.arange(-126, 127, dtype=np.float32)
    row = np.concatenate([[0.25, -0.25], (k + 0.5) * s]).astype(np.float32)
    q, sc = orc.quant_int8_rows(row[None, :])
    qn, _ = np_quant_int8_rows(row[None, :])
    np.testing.assert_array_equal(q, qn)
    assert q[0, 0] == 127 and q[0, 1] == -127
    assert sc[0] == s


def test_int8_dequant_round_trip_bound(orc):
    x = np.random.default_rng(1).standard_normal((16, 512)).astype(np.float32)
    q, s = orc.quant_int8_rows(x)
    back = orc.dequant_int8_rows(q, s)
    assert (np.abs(back - x) <= s[:, None] * 0.5000001).all()


@pytest.mark.parametrize("N,K", [(1, 128), (5, 256), (16, 1024)])
def test_int4_quant_matches_numpy_restatement(orc, N, K):
    rng = np.random.default_rng(N * K)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    if N > 2:
        w[1, :128] = np.abs(w[1, :128])
        w[2, :128] = 0
    p, s, z = orc.quant_int4_g128(w)
    pn, sn, zn = np_quant_int4(w)
    np.testing.assert_array_equal(s, sn)
    np.testing.assert_array_equal(z, zn)
    np.testing.assert_array_equal(p, pn)
    back = orc.dequant_int4_g128(p, s, z)
    assert (np.abs(back - w) <= np.repeat(s, 128, axis=1) * 0.5 + 1e-7).all()


def test_gemm_and_linears_match_numpy(orc):
    rng = np.random.default_rng(3)
    qa = rng.integers(-127, 128, (40, 160), dtype=np.int8)
    qw = rng.integers(-127, 128, (48, 160), dtype=np.int8)
    acc = orc.gemm_i8(qa, qw)
    np.testing.assert_array_equal(acc, qa.astype(np.int64) @ qw.astype(np.int64).T)
    sa = rng.random(40).astype(np.float32)
    sw = rng.random(48).astype(np.float32)
    b = rng.standard_normal(48).astype(np.float32)
    y = orc.linear_w8a8(qa, sa, qw, sw, b, orc.ACT_NONE)
    want = acc.astype(np.float64) * sa[:, None] * sw[None, :] + b
    np.testing.assert_allclose(y, want, rtol=1e-6, atol=1e-6)
    g = orc.linear_w8a8(qa, sa * 1e-4, qw, sw, b, orc.ACT_GELU)
    z = acc.astype(np.float64) * (sa * 1e-4)[:, None] * sw[None, :] + b
    ref = z * 0.5 * (1 + np.tanh(0.797885 * (z + 0.044715 * z ** 3)))
    np.testing.assert_allclose(g, ref, rtol=1e-5, atol=1e-6)
    a = rng.standard_normal((40, 160)).astype(np.float32)
    y32 = orc.linear_w8a32(a, qw, sw * 1e-3, None, orc.ACT_SIGMOID)
    z32 = (a.astype(np.float64) @ qw.astype(np.float64).T) * (sw * 1e-3)
    np.testing.assert_allclose(y32, 1 / (1 + np.exp(-z32)), rtol=1e-5, atol=1e-6)


def test_layernorm_and_attention_match_numpy(orc):
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((9, 96)) * 2 + 1).astype(np.float32)
    g = rng.standard_normal(96).astype(np.float32)
    b = rng.standard_normal(96).astype(np.float32)
    v = 2.0 * x.astype(np.float64)
    ref = (v - v.mean(1, keepdims=True)) / np.sqrt(v.var(1, keepdims=True) + 1e-5) * g + b
    np.testing.assert_allclose(orc.layernorm_x2(x, g, b), ref, rtol=1e-5, atol=1e-5)
    B, S, nh, dh = 2, 11, 2, 64
    q = rng.standard_normal((B * S, nh * dh)).astype(np.float32)
    k = rng.standard_normal((B * S, nh * dh)).astype(np.float32)
    vv = rng.standard_normal((B * S, nh * dh)).astype(np.float32)
    o = orc.attention(q, k, vv, B, S, S, nh, dh, True, orc.F32)
    for bi in range(B):
        for h in range(nh):
            sl = slice(h * dh, (h + 1) * dh)
            qs, ks, vs = (t[bi * S:(bi + 1) * S, sl].astype(np.float64) for t in (q, k, vv))
            sc = qs @ ks.T / np.sqrt(dh)
            sc[np.triu_indices(S, 1)] = -np.inf
            p = np.exp(sc - sc.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            np.testing.assert_allclose(o[bi * S:(bi + 1) * S, sl], p @ vs, rtol=1e-5, atol=1e-6)


def test_rope_table_is_a_rotation(orc):
    tab = orc.rope_table(64, 64)
    np.testing.assert_allclose(tab[..., 0] ** 2 + tab[..., 1] ** 2, 1.0, atol=1e-6)
    assert np.allclose(tab[0, :, 0], 1.0) and np.allclose(tab[0, :, 1], 0.0)


def test_block_forward_properties(orc):
    from ltm_b200 import synthetic
    H, F, Ms, B, S = 128, 256, 32, 1, 16
    w = synthetic.block_weights(H, F, Ms, 1)
    x = synthetic.activations(B * S, H, 2)
    cfg = dict(H=H, F=F, nh=2, dh=64, Ms=Ms, scheme=orc.W8A32, dtype=orc.F32)
    y1, m1 = orc.block_forward(cfg, w, x, B, S)
    assert np.isfinite(y1).all() and np.array_equal(m1, w["memory"])  # no write by default
    # causality: appending tokens does not change earlier outputs (memory read only)
    x2 = np.concatenate([x, synthetic.activations(8, H, 3)])
    y2, _ = orc.block_forward(cfg, w, x2, 1, S + 8)
    np.testing.assert_allclose(y2[:S], y1, rtol=1e-5, atol=1e-5)


def test_golden_fixtures(orc):
    import importlib.util
    assert GOLDEN.exists(), "run tests/golden/make_golden.py"
    spec = importlib.util.spec_from_file_location("make_golden", ROOT / "tests" / "golden" / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    want = np.load(GOLDEN)
    got = mg.cases()
    assert set(got) == set(want.files)
    for k in want.files:
        if np.issubdtype(want[k].dtype, np.integer):
            np.testing.assert_array_equal(got[k], want[k], err_msg=k)
        else:
            np.testing.assert_allclose(got[k], want[k], rtol=1e-6, atol=1e-6, err_msg=k)


def test_oracle_decode_step_is_last_row_of_forward(orc):
    """The oracle's decode step over a cache holding its own prefix keys /
    values reproduces the last row of its causal forward (and appends that
    row's K | V)."""
    from ltm_b200 import synthetic
    for scheme, dt in ((1, 1), (2, 2)):
        H, nh, F, Ms, B, L, P = 128, 2, 256, 32, 2, 9, 12
        S = L + 1
        ocfg = dict(H=H, F=F, nh=nh, dh=H // nh, Ms=Ms, scheme=scheme, dtype=dt, memory_write=0,
                    use_attention_scores=1, update_rate=0.9)
        w = synthetic.block_weights(H, F, Ms, 3)
        x = orc.round_to(synthetic.activations(B * S, H, 4), dt)
        y, _, kv = orc.block_forward(ocfg, w, x, B, S, return_kv=True)
        kv = kv.reshape(B, S, 2 * H)
        dh = H // nh
        heads = kv.reshape(B, S, 2, nh, dh).transpose(2, 0, 3, 1, 4)  # K|V, b, head, pos, dim
        kc = np.zeros((B, nh, P, dh), np.float32)
        vc = np.zeros((B, nh, P, dh), np.float32)
        kc[:, :, :L], vc[:, :, :L] = heads[0][:, :, :L], heads[1][:, :, :L]
        mem = orc.round_to(w["memory"], dt)
        kvm = orc.block_kvm(ocfg, w, mem)
        yd = orc.block_decode_step(ocfg, w, x.reshape(B, S, H)[:, L], kc, vc, L, mem, kvm)
        np.testing.assert_array_equal(yd, y.reshape(B, S, H)[:, L])
        np.testing.assert_array_equal(kc[:, :, L], heads[0][:, :, L])
        np.testing.assert_array_equal(vc[:, :, L], heads[1][:, :, L])
