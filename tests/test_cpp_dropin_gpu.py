"""The C++ drop-in on the GPU: tests/cpp/titan_block_test.cpp runs
TitanBlock<float> (W8A32), TitanBlock<half> and TitanBlock<__nv_bfloat16>
(W8A8) through include/ltm/titan_block.hpp on weights and inputs written
here, round-trips each block through a checkpoint (bit-exact, checked inside
the program), quantizes with Quantizer<half> (INT8) and
Quantizer<__nv_bfloat16> (INT4), and checks that a bad config throws
std::runtime_error.  Its outputs are compared with the oracle here."""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from _util import assert_close

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "cpp"))


def test_cpp_dropin_block_and_quantizer(ltm, orc, tmp_path):
    import cpp_build
    from ltm_b200 import synthetic
    H, F, nh, Ms, B, S = 256, 512, 4, 64, 2, 48
    w = synthetic.block_weights(H, F, Ms, 17)
    x = synthetic.activations(B * S, H, 18)
    (tmp_path / "meta.txt").write_text(f"{H} {F} {nh} {Ms} {B} {S}\n")
    for k, v in w.items():
        np.ascontiguousarray(v, np.float32).tofile(tmp_path / f"{k}.f32")
    x.astype(np.float32).tofile(tmp_path / "x.f32")
    exe = cpp_build.build_test()
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, f"titan_block_test failed ({r.returncode}):\n{r.stdout}\n{r.stderr}"
    assert "titan_block_test ok" in r.stdout
    for tag, scheme, dt, tol in (("f32", orc.W8A32, orc.F32, (1e-4, 1e-4)),
                                 ("f16", orc.W8A8, orc.F16, (2e-2, 1e-2)),
                                 ("bf16", orc.W8A8, orc.BF16, (2e-2, 1e-2))):
        ocfg = dict(H=H, F=F, nh=nh, dh=H // nh, Ms=Ms, scheme=scheme, dtype=dt)
        ref, _ = orc.block_forward(ocfg, w, orc.round_to(x, dt), B, S)
        got = np.fromfile(tmp_path / f"y_{tag}.f32", np.float32).reshape(ref.shape)
        assert_close(got, ref, *tol, what=f"C++ TitanBlock<{tag}>")
    w1h = orc.round_to(w["w_1"], orc.F16)
    q, s = orc.quant_int8_rows(w1h)
    assert np.array_equal(np.fromfile(tmp_path / "q8_codes.i8", np.int8).reshape(q.shape), q)
    assert np.array_equal(np.fromfile(tmp_path / "q8_scales.f32", np.float32), s)
    deq = np.fromfile(tmp_path / "q8_deq.f32", np.float32).reshape(q.shape)
    assert np.array_equal(deq, orc.dequant_int8_rows(q, s, orc.F16))
    packed, s4, zp = orc.quant_int4_g128(orc.round_to(w["w_1"], orc.BF16))
    assert np.array_equal(np.fromfile(tmp_path / "q4_packed.u8", np.uint8).reshape(packed.shape),
                          packed)
    assert np.array_equal(np.fromfile(tmp_path / "q4_scales.f32", np.float32).reshape(s4.shape), s4)
    assert np.array_equal(np.fromfile(tmp_path / "q4_zp.u8", np.uint8).reshape(zp.shape), zp)
