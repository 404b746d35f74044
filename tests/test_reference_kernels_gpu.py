"""The reference's own kernels (oracle/_ref, compiled from the reference's
sources by oracle/ref_kernels.py) run live on the GPU:

* they reproduce tests/golden/reference_kernels.npz bit for bit, so the CPU
  suite's pinning of the oracle rests on these kernels;
* on larger seeded inputs (natural near-ties, no constructed ones) the IEEE
  build's INT8 codes equal the oracle's and its LayerNorm / GELU / EMA stay
  within a few fp32 ulps, as in the CPU suite.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import ref_cases  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def libs():
    return {v: ref_cases.load(v) for v in ref_cases.VARIANTS}


@pytest.mark.parametrize("name", list(ref_cases.CASES))
def test_reference_kernels_reproduce_fixture(ltm, orc, libs, name):
    fix = np.load(ref_cases.FIXTURE)
    inp = ref_cases.inputs(name)
    for variant, lib in libs.items():
        out = ref_cases.run(lib, name, inp, orc)
        want = fix[f"{name}/{variant}"]
        assert np.array_equal(out.astype(want.dtype), want), f"{name} ({variant}) changed"


def test_ieee_build_matches_oracle_on_larger_inputs(ltm, orc, libs):
    import torch
    lib = libs["ieee"]
    rng = np.random.default_rng(123)
    R, K = 512, 4096
    w = (rng.standard_normal((R, K)) * 0.02).astype(np.float32)
    q_or, s_or = orc.quant_int8_rows(w)
    wd = torch.from_numpy(w).cuda()
    sd = torch.from_numpy(s_or).cuda()
    zd = torch.zeros(R, device="cuda")
    q = torch.empty((R, K), dtype=torch.int8, device="cuda")
    assert lib.ref_per_channel_quantize(wd.data_ptr(), 0, q.data_ptr(), sd.data_ptr(),
                                        zd.data_ptr(), R * K, R, K, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_or)
    # LayerNorm(x + x) over hidden 8192 rows
    x = (rng.standard_normal((64, 8192)) * 2 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(8192)).astype(np.float32)
    b = (0.1 * rng.standard_normal(8192)).astype(np.float32)
    xd, gd, bd = (torch.from_numpy(a).cuda() for a in (x, g, b))
    out = torch.empty_like(xd)
    assert lib.ref_layernorm_residual(xd.data_ptr(), xd.data_ptr(), gd.data_ptr(), bd.data_ptr(),
                                      out.data_ptr(), 0, 64, 8192, None) == 0
    torch.cuda.synchronize()
    want = orc.layernorm_x2(x, g, b)
    assert np.abs(out.cpu().numpy() - want).max() <= 64 * np.spacing(np.float32(np.abs(want).max()))
    # bank EMA with attention-score weights, hidden 1024 slots of 4096
    mem = (rng.standard_normal((4096, 1024)) / 32).astype(np.float32)
    st = (0.3 * rng.standard_normal(1024)).astype(np.float32)
    sc = rng.random(4096).astype(np.float32)
    md, std, scd = (torch.from_numpy(a).cuda() for a in (mem, st, sc))
    assert lib.ref_store_state(md.data_ptr(), std.data_ptr(), scd.data_ptr(), 0.9, 4096, 1024, 0,
                               None) == 0
    torch.cuda.synchronize()
    want = orc.ema_rows(mem, st, (np.float32(0.9) * sc).astype(np.float32), orc.F32)
    assert np.abs(md.cpu().numpy() - want).max() <= 4 * np.spacing(np.float32(np.abs(want).max()))
