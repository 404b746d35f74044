"""Host side of the tensor-parallel block, on CPU.

* The communicator id travels from group rank 0 to every rank over a
  torch.distributed group (gloo, world size 2 here; the library's NCCL id
  generation needs no GPU).
* The sharding identities the library relies on, checked on the oracle's
  integer arithmetic: a row-parallel W8A8 layer whose weight codes come from
  the unsplit rows and whose activation scales come from the global row
  maxima sums, over the ranks, to exactly the unsplit int32 accumulators; the
  column-parallel layers' row shards carry the unsplit codes and scales; the
  per-rank head sums of the slot-weight softmax add up to the head mean.
* The exact sequence-parallel reduction's data flow on two gloo ranks: local
  row maxima allreduced to the unsplit per-token scales, int32 partials of
  every row sent to the rows' owners (all-to-all), the owner's slot sums equal
  to the unsplit accumulators and its epilogue to the unsplit layer's."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _id_worker(rank, world, port, out):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "obsidian-memory-transformer_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import ltm_b200
        uid = ltm_b200.broadcast_comm_id()
        out.put((rank, uid))
    finally:
        dist.destroy_process_group()


def test_comm_id_broadcast_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_id_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(got[0]) == 128 and got[0] == got[1]
    assert any(got[0])  # a real id, not zeros


@pytest.mark.parametrize("n", [2, 4])
def test_row_parallel_w8a8_shards_sum_exactly(orc, n):
    rng = np.random.default_rng(3)
    M, N, K = 37, 64, 256
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    a = rng.normal(0, 1.0, (M, K)).astype(np.float32)
    qw, sw = orc.quant_int8_rows(w)          # unsplit rows: one scale per output channel
    qa, sa = orc.quant_int8_rows(a)          # unsplit rows: one scale per token
    full = orc.gemm_i8(qa, qw)
    kl = K // n
    part_sum = np.zeros_like(full)
    for r in range(n):
        cols = slice(r * kl, (r + 1) * kl)
        # global row maximum = max over the ranks' local maxima
        amax = np.max([np.abs(a[:, slice(j * kl, (j + 1) * kl)]).max(1) for j in range(n)], 0)
        assert np.array_equal(np.float32(amax) / np.float32(127), sa)
        part_sum += orc.gemm_i8(qa[:, cols], qw[:, cols])
    assert np.array_equal(part_sum, full)


@pytest.mark.parametrize("n", [2, 3])
def test_column_parallel_shards_keep_unsplit_codes(orc, n):
    rng = np.random.default_rng(4)
    N, K = 96, 128
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    qw, sw = orc.quant_int8_rows(w)
    nl = N // n
    for r in range(n):
        rows = slice(r * nl, (r + 1) * nl)
        q_r, s_r = orc.quant_int8_rows(w[rows])
        assert np.array_equal(q_r, qw[rows]) and np.array_equal(s_r, sw[rows])


def test_slot_weight_head_sums_add_up_to_the_mean():
    rng = np.random.default_rng(5)
    nh, Ms, dh, n = 8, 64, 16, 4
    scores = rng.normal(size=(nh, Ms)).astype(np.float64)
    soft = np.exp(scores - scores.max(1, keepdims=True))
    soft /= soft.sum(1, keepdims=True)
    mean = soft.mean(0)
    per_rank = [soft[r * (nh // n):(r + 1) * (nh // n)].sum(0) / nh for r in range(n)]
    np.testing.assert_allclose(np.sum(per_rank, 0), mean, rtol=1e-12)


def _exact_reduce_worker(rank, world, port, out):
    """One rank of the exact sequence-parallel reduction: the int32 partial
    of its K columns for all T rows, rows sent to their owners (rank r owns
    rows [r T/n, (r+1) T/n)) with an all-to-all, the slots summed at the
    owner, then the W8A8 epilogue fma(acc * row_scale, col_scale, bias)."""
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch
    import torch.distributed as dist
    from oracle import oracle as orc
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(11)
        T, N, K = 64, 96, 256
        a = rng.normal(0, 1.0, (T, K)).astype(np.float32)
        w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
        b = rng.normal(0, 0.02, N).astype(np.float32)
        kl, tr = K // world, T // world
        cols = slice(rank * kl, (rank + 1) * kl)
        # global per-token scale: allreduce-max of the local row maxima
        amax = torch.from_numpy(np.abs(a[:, cols]).max(1).astype(np.float32))
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
        sa = (amax.numpy() / np.float32(127)).astype(np.float32)
        qa_full, sa_full = orc.quant_int8_rows(a)
        qw_full, sw_full = orc.quant_int8_rows(w)
        part = orc.gemm_i8(qa_full[:, cols], qw_full[:, cols]).astype(np.int32)  # [T, N]
        recv = torch.empty((T, N), dtype=torch.int32)
        dist.all_to_all_single(recv, torch.from_numpy(np.ascontiguousarray(part)))
        acc = recv.numpy().reshape(world, tr, N).sum(0, dtype=np.int64)
        rows = slice(rank * tr, (rank + 1) * tr)
        v = acc.astype(np.float32) * sa[rows, None]
        y = (v.astype(np.float64) * sw_full[None, :] + b[None, :]).astype(np.float32)  # fma
        out.put((rank, acc, np.array_equal(sa, sa_full), y))
    finally:
        dist.destroy_process_group()


def test_exact_sequence_parallel_reduction_gloo(orc):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exact_reduce_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (acc, same, y)) for r, acc, same, y in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(11)
    T, N, K = 64, 96, 256
    a = rng.normal(0, 1.0, (T, K)).astype(np.float32)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    b = rng.normal(0, 0.02, N).astype(np.float32)
    qa, sa = orc.quant_int8_rows(a)
    qw, sw = orc.quant_int8_rows(w)
    full = orc.gemm_i8(qa, qw)
    y_full = ((full.astype(np.float32) * sa[:, None]).astype(np.float64) * sw[None, :]
              + b[None, :]).astype(np.float32)
    for r in range(2):
        acc, same, y = got[r]
        assert same, "global row maxima differ from the unsplit scales"
        rows = slice(r * T // 2, (r + 1) * T // 2)
        assert np.array_equal(acc, full[rows]), "slot sums differ from the unsplit accumulators"
        assert np.array_equal(y, y_full[rows]), "epilogue of the owner's rows differs"
