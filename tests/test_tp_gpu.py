"""Tensor-parallel Titan block on 2, 4 and 8 GPUs (one process per GPU, NCCL
through the library's communicator) against the TB-v1 oracle and the
single-GPU block: every rank returns the same full output, the memory bank
after the write is the same on every rank, and both match the oracle within
the dtype tolerance.  The sequence-parallel forward (each rank holds its
rows of the activations) is checked the same way on its gathered rows.
Each case is skipped on a machine with fewer GPUs than it needs."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

from _util import as_f32, assert_close, orc_dtype, to_device

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
TOL = {"f16": (2e-2, 1e-2), "bf16": (2e-2, 1e-2)}


def _case(scheme, dt, memory_write, n=2, F=1024):
    # per-rank widths stay multiples of 32 (W8A8) / 128 (W4A16) up to 8 ranks
    H = 1024 if (scheme == "w4a16" and n > 4) else 512
    nh, Ms, B, S = 8, 128, 2, 96
    return dict(H=H, nh=nh, F=F, Ms=Ms, B=B, S=S, scheme=scheme, dt=dt,
                memory_write=memory_write, seed=11)


def _build(ltm, c, comm=None):
    sch = {"w8a8": ltm.SCHEME_W8A8, "w4a16": ltm.SCHEME_W4A16}[c["scheme"]]
    dtc = {"f16": ltm.DTYPE_F16, "bf16": ltm.DTYPE_BF16}[c["dt"]]
    cfg = ltm.TitanBlockConfig(hidden_dim=c["H"], ffn_dim=c["F"], num_heads=c["nh"],
                               head_dim=c["H"] // c["nh"], memory_slots=c["Ms"])
    q = ltm.QuantConfig(scheme=sch, act_dtype=dtc, memory_write=c["memory_write"])
    return cfg, q, sch


def _worker(rank, n, uid, c, out, sp=False):
    sys.path[:0] = [str(ROOT), str(ROOT / "obsidian-memory-transformer_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import ltm_b200 as ltm
    from ltm_b200 import synthetic
    try:
        torch.cuda.set_device(rank)
        comm = ltm.Comm(uid, n, rank, rank)
        cfg, q, _ = _build(ltm, c, comm)
        blk = ltm.TitanBlock(cfg, q, comm=comm)
        blk.load_weights(synthetic.block_weights(c["H"], c["F"], c["Ms"], c["seed"]))
        B, S, H = c["B"], c["S"], c["H"]
        x = synthetic.activations(B * S, H, c["seed"] + 1)
        xd = to_device(x, c["dt"])
        if sp:  # this rank's rows only; the parent gathers the slices
            blk.set_overlap(sp.endswith("overlap"))
            blk.set_tp_reduction(sp.startswith("exact"))
            Tr = B * S // n
            xl = xd[rank * Tr:(rank + 1) * Tr].contiguous()
            y1 = blk.forward_sp(xl, B, S)
            y2 = blk.forward_sp(xl, B, S)
        else:
            y1 = blk(xd.reshape(B, S, H))
            y2 = blk(xd.reshape(B, S, H))  # reads the bank the first forward wrote (when enabled)
        torch.cuda.synchronize()
        out.put((rank, as_f32(y1), as_f32(y2), as_f32(blk.memory()), ltm.device_error()))
        blk.close()
        comm.close()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out.put((rank, repr(e), None, None, -1))


def _run_tp(c, n=2, sp=False):
    import torch.multiprocessing as mp
    import ltm_b200 as ltm
    uid = ltm.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, n, uid, c, q, sp)) for r in range(n)]
    for p in procs:
        p.start()
    try:
        res = {}
        for _ in procs:
            r, y1, y2, mem, derr = q.get(timeout=600)
            assert not isinstance(y1, str), f"rank {r}: {y1}"
            assert derr == 0
            res[r] = (y1, y2, mem)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    return res


# sp: False = allreduce form (every rank holds all rows); "serial" /
# "overlap" = sequence parallel with the partial sums reduced in the
# activation type; "exact" / "exact-overlap" = sequence parallel with the
# int32 accumulators reduced exactly (W8A8), which must equal the single-GPU
# block bit for bit.
_SP_ACT = [False, "overlap", "serial"]
_SP_W8 = _SP_ACT + ["exact", "exact-overlap"]
_TP_CASES = ([("w8a8", "f16", True, 1024, sp) for sp in _SP_W8] +
             [("w8a8", "bf16", False, 1024, sp) for sp in _SP_W8] +
             [("w4a16", "bf16", True, 1024, sp) for sp in _SP_ACT] +
             # 1024 FFN columns per rank at 8 ranks: the split row quantizers'
             # four-loads-per-lane loop, checked bit for bit against one GPU
             [("w8a8", "bf16", False, 8192, sp) for sp in ("exact", "exact-overlap")])


@pytest.mark.parametrize("n", [2, 4, 8])
@pytest.mark.parametrize("scheme,dt,memory_write,F,sp", _TP_CASES)
def test_tp_block_matches_single_gpu_and_oracle(ltm, orc, scheme, dt, memory_write, F, sp, n):
    import torch
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    from ltm_b200 import synthetic
    c = _case(scheme, dt, memory_write, n, F)
    res = _run_tp(c, n, sp)
    if sp:  # gather the row slices into the full outputs
        y1 = np.concatenate([res[r][0] for r in range(n)]).reshape(c["B"], c["S"], c["H"])
        y2 = np.concatenate([res[r][1] for r in range(n)]).reshape(c["B"], c["S"], c["H"])
        mem = res[0][2]
        for r in res:  # the bank update is identical on every rank
            assert np.array_equal(res[r][2], mem)
    else:
        y1, y2, mem = res[0]
        for r in res:  # the allreduce gives every rank the same result
            assert np.array_equal(res[r][0], y1) and np.array_equal(res[r][1], y2)
            assert np.array_equal(res[r][2], mem)
    # single-GPU block and the oracle on the same inputs
    cfg, qc, sch = _build(ltm, c)
    w = synthetic.block_weights(c["H"], c["F"], c["Ms"], c["seed"])
    blk = ltm.TitanBlock(cfg, qc)
    blk.load_weights(w)
    B, S, H = c["B"], c["S"], c["H"]
    xd = to_device(synthetic.activations(B * S, H, c["seed"] + 1), dt).reshape(B, S, H)
    s1 = as_f32(blk(xd))
    ocfg = dict(H=H, F=c["F"], nh=c["nh"], dh=H // c["nh"], Ms=c["Ms"], scheme=sch,
                dtype=orc_dtype(dt), memory_write=int(memory_write), use_attention_scores=1,
                update_rate=cfg.memory_update_rate, use_rotary=1, use_bias=1, use_layer_norm=1,
                use_memory_gating=1)
    ref, mem_ref = orc.block_forward(ocfg, w, as_f32(xd).reshape(B * S, H), B, S)
    what = f"tp{n}{' sp ' + sp if sp else ''} {scheme} {dt} F{F}"
    if sp and sp.startswith("exact"):
        assert np.array_equal(y1, s1), f"{what}: differs from the single-GPU block"
    assert_close(y1, s1, *TOL[dt], what=f"{what} vs single GPU")
    # End to end against the oracle at FFN width 1024.  At 8192 the block's
    # own end-to-end deviation (single GPU, no sharding) exceeds the bf16 bar
    # at a few elements: 1-ulp stage differences are amplified by the two
    # int8 re-quantizations (test_parity_full_shapes_gpu checks that shape
    # stage by stage); there the sharded forward must equal one GPU exactly.
    if F <= 1024:
        assert_close(y1.reshape(ref.shape), ref, *TOL[dt], what=f"{what} vs oracle")
    if memory_write:
        assert_close(mem, mem_ref, 2e-3, 1e-2, what=f"{what} bank after write")
        ref2, _ = orc.block_forward(ocfg, w, as_f32(xd).reshape(B * S, H), B, S, memory=mem_ref)
        assert_close(y2.reshape(ref2.shape), ref2, *TOL[dt], what=f"{what} second forward")
    blk.close()


def _decode_worker(rank, n, uid, c, caches, xs, L0, out):
    sys.path[:0] = [str(ROOT), str(ROOT / "obsidian-memory-transformer_b200")]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import ltm_b200 as ltm
    from ltm_b200 import synthetic
    try:
        torch.cuda.set_device(rank)
        comm = ltm.Comm(uid, n, rank, rank)
        cfg, q, _ = _build(ltm, c, comm)
        blk = ltm.TitanBlock(cfg, q, comm=comm)
        blk.load_weights(synthetic.block_weights(c["H"], c["F"], c["Ms"], c["seed"]))
        nhl = c["nh"] // n
        k, v = (torch.from_numpy(a[:, rank * nhl:(rank + 1) * nhl].copy()).to(
            torch.bfloat16 if c["dt"] == "bf16" else torch.float16).cuda() for a in caches)
        ys = []
        for i, x in enumerate(xs):
            ys.append(as_f32(blk.decode_step(to_device(x, c["dt"]), k, v, L0 + i)))
        torch.cuda.synchronize()
        out.put((rank, ys, as_f32(blk.memory()), ltm.device_error()))
        blk.close()
        comm.close()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out.put((rank, repr(e), None, -1))


@pytest.mark.parametrize("n", [2, 8])
@pytest.mark.parametrize("scheme,dt", [("w4a16", "bf16"), ("w8a8", "f16")])
def test_tp_decode_matches_oracle(ltm, orc, scheme, dt, n):
    """Tensor-parallel decode steps with the memory write: each rank holds its
    heads of the KV cache; every rank returns the same output, equal to the
    oracle's decode steps within the dtype tolerance."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    from ltm_b200 import synthetic
    c = _case(scheme, dt, True, n)
    H, nh, B, L0, P, steps = c["H"], c["nh"], 3, 40, 48, 3
    dh = H // nh
    rng = np.random.default_rng(5)
    caches = [orc.round_to(rng.standard_normal((B, nh, P, dh)), orc_dtype(dt)) for _ in range(2)]
    xs = [orc.round_to(synthetic.activations(B, H, 60 + i), orc_dtype(dt)) for i in range(steps)]
    uid = ltm.comm_unique_id()
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    procs = [ctx.Process(target=_decode_worker, args=(r, n, uid, c, caches, xs, L0, qu))
             for r in range(n)]
    for p in procs:
        p.start()
    try:
        res = {}
        for _ in procs:
            r, ys, mem, derr = qu.get(timeout=600)
            assert not isinstance(ys, str), f"rank {r}: {ys}"
            assert derr == 0
            res[r] = (ys, mem)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for i in range(steps):
        for r in range(1, n):
            assert np.array_equal(res[0][0][i], res[r][0][i])
    cfg, _, sch = _build(ltm, c)
    ocfg = dict(H=H, F=c["F"], nh=nh, dh=dh, Ms=c["Ms"], scheme=sch, dtype=orc_dtype(dt),
                memory_write=1, use_attention_scores=1, update_rate=cfg.memory_update_rate,
                use_rotary=1, use_bias=1, use_layer_norm=1, use_memory_gating=1)
    w = synthetic.block_weights(H, c["F"], c["Ms"], c["seed"])
    mem = orc.round_to(w["memory"], orc_dtype(dt))
    kvm = orc.block_kvm(ocfg, w, mem)
    kh, vh = caches[0].copy(), caches[1].copy()
    for i, x in enumerate(xs):
        ref = orc.block_decode_step(ocfg, w, x, kh, vh, L0 + i, mem, kvm)
        assert_close(res[0][0][i], ref, *TOL[dt], what=f"tp{n} decode step {i}")
    assert_close(res[0][1], mem, 2e-3, 1e-2, what=f"tp{n} bank after the decode writes")
