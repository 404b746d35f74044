"""The allocation-free memory-bank store, called through the C ABI.

ltm_memory_store_noalloc exists for callers that cannot let the library
allocate device memory while they run (they plan every device byte
themselves, or must keep a fixed footprint).  It keeps its scratch in one
fixed device array that every call reuses, so this file checks it against the
allocating entry point ltm_memory_store on two calls in a row (the second
call must not see the first call's leftovers) and checks the size limit.
It is collected last so a stop-at-first-failure run has covered everything
else first, and it passes alone in a fresh process as well.  One case runs in
a child process of its own, where the allocation-free store is the first
library call that touches device memory: the library's allocation counter
must stay at zero over two calls, and the device's free memory must not move
over the second one.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from _util import as_f32, assert_close, to_device

pytestmark = pytest.mark.gpu


def _inputs(seed, Ms, H, T, dt):
    rng = np.random.default_rng(seed)
    mem = (rng.standard_normal((Ms, H)) / np.sqrt(H)).astype(np.float32)
    kv = rng.standard_normal((Ms, 2 * H)).astype(np.float32)
    q = rng.standard_normal((T, 4 * H)).astype(np.float32)
    q[:, 3 * H:] += 2.0 * rng.standard_normal(H).astype(np.float32)
    state = (0.3 * rng.standard_normal(H)).astype(np.float32)
    return to_device(mem, dt), to_device(kv, dt), to_device(q, dt), state


def _call_c_abi(ltm, fn, mem, keys, queries, state, nh, rate, scores):
    import torch
    st = torch.from_numpy(state).cuda()
    Ms, H = mem.shape
    status = fn(ltm._ptr(mem), ltm._ptr(keys), keys.stride(0), ltm._ptr(queries), queries.stride(0),
                queries.shape[0], ltm._ptr(st), Ms, H, nh, rate, int(scores),
                ltm.dtype_code(mem.dtype), ltm._stream())
    ltm._check(status)
    torch.cuda.synchronize()
    return as_f32(mem)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_noalloc_store_matches_allocating_store_twice(ltm, dt):
    lib = ltm.lib()
    H, nh = 768, 12
    atol, rtol = (1e-5, 1e-4) if dt == "f32" else (2e-3, 1e-2)
    # two calls in a row with different inputs and sizes: the shared scratch
    # must be cleared by each call
    for call, (Ms, T, scores, rate, seed) in enumerate([(512, 256, True, 0.5, 1),
                                                        (384, 64, True, 0.9, 2)]):
        mem, kv, q, state = _inputs(seed, Ms, H, T, dt)
        mem_ref = mem.clone()
        want = _call_c_abi(ltm, lib.ltm_memory_store, mem_ref, kv[:, :H], q[:, 3 * H:], state, nh,
                           rate, scores)
        got = _call_c_abi(ltm, lib.ltm_memory_store_noalloc, mem, kv[:, :H], q[:, 3 * H:], state,
                          nh, rate, scores)
        assert_close(got, want, atol, rtol, what=f"no-alloc store, call {call + 1}")
        assert ltm.device_error() == 0


def test_noalloc_store_rejects_sizes_beyond_its_scratch(ltm):
    """With attention-score slot weights the scratch holds round_up(H, 64) +
    Ms floats: 15360 + 51200 = 66560 > 65536 is refused (51200 slots is the
    slot-weight kernel's own limit, so the scratch is what refuses)."""
    import torch
    H, Ms = 15360, 51200
    mem = torch.zeros((Ms, H), dtype=torch.bfloat16, device="cuda")
    keys = torch.zeros((Ms, H), dtype=torch.bfloat16, device="cuda")
    q = torch.zeros((4, H), dtype=torch.bfloat16, device="cuda")
    state = torch.zeros(H, dtype=torch.float32, device="cuda")
    with pytest.raises(ltm.LtmError) as e:
        ltm.memory_store_noalloc(mem, keys, q, state, 32, 0.9, True)
    assert e.value.status == ltm.ERR_INVALID_ARG
    assert "scratch" in str(e.value)


_FRESH_PROCESS = r"""
import sys
sys.path[:0] = sys.argv[1:4]
import numpy as np
import torch
import ltm_b200 as ltm
from _util import assert_close
from test_zz_no_alloc import _inputs, _call_c_abi

lib = ltm.lib()
H, nh = 512, 8
cases = [(256, 128, 0.7, 11), (192, 32, 0.4, 12)]
inputs = [_inputs(seed, Ms, H, T, "bf16") for Ms, T, rate, seed in cases]
refs = [m.clone() for m, _, _, _ in inputs]
torch.cuda.synchronize()
assert ltm.device_alloc_count() == 0, "the library allocated before the test began"
torch_bytes = torch.cuda.memory_allocated()
outs, free = [], []
for (mem, kv, q, state), (Ms, T, rate, seed) in zip(inputs, cases):
    free.append(torch.cuda.mem_get_info()[0])
    outs.append(_call_c_abi(ltm, lib.ltm_memory_store_noalloc, mem, kv[:, :H], q[:, 3 * H:],
                            state, nh, rate, True))
    assert ltm.device_alloc_count() == 0, "the allocation-free store allocated device memory"
free.append(torch.cuda.mem_get_info()[0])
assert free[2] == free[1], f"device free memory moved over the second call: {free}"
assert torch.cuda.memory_allocated() == torch_bytes
# the allocating store on the same inputs, after: same results, and the
# counter sees its scratch allocation
for (mem, kv, q, state), ref, got, (Ms, T, rate, seed) in zip(inputs, refs, outs, cases):
    want = _call_c_abi(ltm, lib.ltm_memory_store, ref, kv[:, :H], q[:, 3 * H:], state, nh, rate,
                       True)
    assert_close(got, want, 2e-3, 1e-2, what="no-alloc store in a fresh process")
assert ltm.device_alloc_count() > 0
assert ltm.device_error() == 0
print("fresh-process no-alloc store ok")
"""


def test_noalloc_store_first_in_fresh_process_allocates_nothing(ltm):
    tests = Path(__file__).resolve().parent
    root = tests.parent
    env = dict(os.environ)
    r = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, str(root),
                        str(root / "obsidian-memory-transformer_b200"), str(tests)],
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, f"child failed:\n{r.stdout}\n{r.stderr}"
    assert "fresh-process no-alloc store ok" in r.stdout


def test_noalloc_rate_only_store_needs_no_scratch(ltm):
    """Rate-only updates read no scratch, so the scratch limit does not apply:
    a bank larger than the scratch still updates, equal to ltm_memory_store."""
    lib = ltm.lib()
    H, nh, Ms, T = 64, 2, 65536, 8
    mem, kv, q, state = _inputs(21, Ms, H, T, "bf16")
    ref = mem.clone()
    want = _call_c_abi(ltm, lib.ltm_memory_store, ref, kv[:, :H], q[:, 3 * H:], state, nh, 0.3,
                       False)
    got = _call_c_abi(ltm, lib.ltm_memory_store_noalloc, mem, kv[:, :H], q[:, 3 * H:], state, nh,
                      0.3, False)
    assert_close(got, want, 0.0, 0.0, what="rate-only no-alloc store")
