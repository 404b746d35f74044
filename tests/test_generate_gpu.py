"""Prefill that fills the KV caches, decode steps after it (one length for
the batch, and a length per sequence), the LM head and greedy generation
with the decode step replayed from a CUDA graph, against the oracle.

The chained checks rest on one identity of the causal block: the decode step
of the token at position p over a cache that holds the keys / values of
positions [0, p) equals row p of the forward over the whole sequence, so a
device prefill followed by device decode steps must equal the oracle's
forward over prompt + generated tokens, row by row (no memory write here:
the bank stays fixed)."""
import numpy as np
import pytest

from _util import as_f32, assert_close, orc_dtype, to_device
from test_block_gpu import make

pytestmark = pytest.mark.gpu

TOL = {"f32": (1e-4, 1e-4), "f16": (2e-2, 1e-2), "bf16": (2e-2, 1e-2)}
SCHEMES = [("w8a8", "f16"), ("w8a8", "bf16"), ("w4a16", "bf16")]


def _oracle_lm_head(orc, scheme, dt, w, hidden):
    """The oracle's LM head (no bias) on hidden rows (fp32 numpy)."""
    if scheme == "w8a8":
        qa, sa = orc.quant_int8_rows(hidden)
        qw, sw = orc.quant_int8_rows(w)
        y = orc.linear_w8a8(qa, sa, qw, sw, None)
    elif scheme == "w4a16":
        packed, s, zp = orc.quant_int4_g128(w)
        y = orc.linear_w4a16(hidden, packed, s, zp, None, 0, orc_dtype(dt))
    else:
        qw, sw = orc.quant_int8_rows(w)
        y = orc.linear_w8a32(hidden, qw, sw, None)
    return orc.round_to(y, orc_dtype(dt))


def _model(ltm, scheme, dt, H=256, nh=4, F=512, Ms=64, V=1000, L=2, seed=0):
    from ltm_b200 import synthetic
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms)
    model = ltm.TitanModel(cfg, q, L, V)
    emb = synthetic.embedding(V, H, seed + 1)
    model.load_embedding(emb)
    layers = [synthetic.block_weights(H, F, Ms, seed + 10 + i) for i in range(L)]
    for i, w in enumerate(layers):
        model.load_layer(i, w)
    head = (np.random.default_rng(seed + 2).standard_normal((V, H)) * 0.02).astype(np.float32)
    model.load_lm_head(head)
    return model, ocfg, emb, layers, head


@pytest.mark.parametrize("scheme,dt", SCHEMES + [("w8a32", "f32")])
@pytest.mark.parametrize("V", [1000, 1024])  # 1000: rows padded to a multiple of 32 inside
def test_lm_head_matches_oracle(ltm, orc, scheme, dt, V):
    import torch
    from _util import torch_dtype
    model, ocfg, emb, layers, head = _model(ltm, scheme, dt, V=V)
    rng = np.random.default_rng(V)
    hid = to_device(rng.standard_normal((3, 7, 256)).astype(np.float32), dt)
    got = model.lm_head(hid)
    want = _oracle_lm_head(orc, scheme, dt, head, as_f32(hid).reshape(-1, 256))
    assert_close(as_f32(got).reshape(want.shape), want, *TOL[dt], what=f"lm head {scheme} V={V}")
    # strided rows: the last position of each sequence
    got_last = model.lm_head(hid[:, -1, :])
    assert_close(as_f32(got_last), want.reshape(3, 7, V)[:, -1], *TOL[dt], what="strided rows")
    assert got.dtype == torch_dtype(dt) and ltm.device_error() == 0
    model.close()


@pytest.mark.parametrize("scheme,dt", SCHEMES)
@pytest.mark.parametrize("nh", [4, 2])
def test_block_prefill_fills_cache_then_decode(ltm, orc, scheme, dt, nh):
    """forward_with_cache writes the oracle's post-RoPE K / V; decode steps at
    cache_len = S, S+1, ... then reproduce rows S.. of the full forward."""
    import torch
    from _util import torch_dtype
    from ltm_b200 import synthetic
    H, F, Ms, B, S, N, P = 256, 512, 64, 2, 40, 5, 64
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms)
    w = synthetic.block_weights(H, F, Ms, 3)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    x = orc.round_to(synthetic.activations(B * (S + N), H, 4), orc_dtype(dt)).reshape(B, S + N, H)
    ref, _, kv = orc.block_forward(ocfg, w, x.reshape(-1, H), B, S + N, return_kv=True)
    ref = ref.reshape(B, S + N, H)
    kv = kv.reshape(B, S + N, 2 * H)
    td = torch_dtype(dt)
    kc = torch.full((B, nh, P, H // nh), 7.0, dtype=td, device="cuda")
    vc = torch.full_like(kc, 7.0)
    xd = to_device(x[:, :S].reshape(-1, H), dt).reshape(B, S, H)
    y = blk.forward(xd, k_cache=kc, v_cache=vc)
    assert_close(as_f32(y), ref[:, :S], *TOL[dt], what="prefill output")
    heads = lambda a: a.reshape(B, -1, nh, H // nh).transpose(0, 2, 1, 3)  # noqa: E731
    assert_close(as_f32(kc[:, :, :S]), heads(kv[:, :S, :H]), *TOL[dt], what="cached K")
    assert_close(as_f32(vc[:, :, :S]), heads(kv[:, :S, H:]), *TOL[dt], what="cached V")
    assert np.all(as_f32(kc[:, :, S:]) == 7.0), "the prefill wrote past its positions"
    for i in range(N):
        yt = blk.decode_step(to_device(x[:, S + i], dt), kc, vc, S + i)
        assert_close(as_f32(yt), ref[:, S + i], *TOL[dt], what=f"decode step {i} after prefill")
    assert ltm.device_error() == 0
    blk.close()


@pytest.mark.parametrize("scheme,dt", [("w8a8", "bf16"), ("w4a16", "bf16")])
def test_ragged_decode_lengths_per_sequence(ltm, orc, scheme, dt):
    """Three sequences with prompts of 5, 17 and 33 tokens, each prefilled into
    its own row of one batched cache, then one decode step of the batch with
    cache_lens = [5, 17, 33]: row b equals the last row of sequence b's own
    forward over its prompt plus the new token."""
    import torch
    from _util import torch_dtype
    from ltm_b200 import synthetic
    H, nh, F, Ms, P = 256, 2, 512, 64, 48
    lens = [5, 17, 33]
    B = len(lens)
    cfg, q, ocfg = make(ltm, scheme, dt, H, nh, F, Ms)
    w = synthetic.block_weights(H, F, Ms, 5)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(w)
    td = torch_dtype(dt)
    kc = torch.zeros((B, nh, P, H // nh), dtype=td, device="cuda")
    vc = torch.zeros_like(kc)
    seqs, wants = [], []
    for b, Lb in enumerate(lens):
        x = orc.round_to(synthetic.activations(Lb + 1, H, 50 + b), orc_dtype(dt))
        ref, _ = orc.block_forward(ocfg, w, x, 1, Lb + 1)
        wants.append(ref[-1])
        seqs.append(x)
        blk.forward(to_device(x[:Lb], dt).reshape(1, Lb, H), k_cache=kc[b:b + 1],
                    v_cache=vc[b:b + 1])
    xt = to_device(np.stack([s[-1] for s in seqs]), dt)
    cl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    y = blk.decode_step_ragged(xt, kc, vc, cl)
    assert_close(as_f32(y), np.stack(wants), *TOL[dt], what="ragged decode step")
    assert ltm.device_error() == 0
    # a length outside [0, max_positions): that sequence is skipped and flagged
    bad = torch.tensor([5, P, 33], dtype=torch.int32, device="cuda")
    k_before = kc.clone()
    y2 = blk.decode_step_ragged(xt, kc, vc, bad)
    torch.cuda.synchronize()
    assert ltm.device_error() == 5
    assert torch.equal(kc[1], k_before[1]), "the skipped sequence's cache was written"
    assert np.isfinite(as_f32(y2)).all()
    blk.close()


@pytest.mark.parametrize("scheme,dt", SCHEMES)
def test_greedy_generation_with_graph_matches_oracle(ltm, orc, scheme, dt):
    """Prefill + 8 greedy steps (the decode step replayed from a CUDA graph):
    each step's hidden state equals the oracle model's forward over prompt +
    generated tokens at that position, every generated token is the argmax
    of the device's own logits, and graph replay gives the same tokens as
    plain launches."""
    import torch
    from ltm_b200 import synthetic
    V, B, S, N = 1000, 2, 24, 8
    model, ocfg, emb, layers, head = _model(ltm, scheme, dt, V=V, seed=7)
    prompt = torch.from_numpy(synthetic.tokens(B, S, V, 9)).cuda()
    toks, trace = model.generate_greedy(prompt, N, use_graph=True, hidden_trace=True)
    toks_plain, _ = model.generate_greedy(prompt, N, use_graph=False)
    assert torch.equal(toks, toks_plain), "graph replay and plain launches generated differently"
    allt = np.concatenate([prompt.cpu().numpy(), toks.cpu().numpy()], axis=1)
    ref = orc.model_forward(ocfg, layers, emb, allt, B, S + N).reshape(B, S + N, -1)
    for j in range(N):
        assert_close(as_f32(trace[j]), ref[:, S + j], *TOL[dt], what=f"hidden of step {j}")
        if j + 1 < N:  # the next token is the argmax of this step's device logits
            lg = as_f32(model.lm_head(trace[j]))
            assert np.array_equal(lg.argmax(axis=1), toks[:, j + 1].cpu().numpy())
    assert ltm.device_error() == 0
    model.close()
