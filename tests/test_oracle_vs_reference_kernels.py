"""The oracle against the reference's own kernels (CPU; the kernels' outputs
come from tests/golden/reference_kernels.npz, made by make_ref_golden.py on a
GPU from the kernels that oracle/ref_kernels.py compiles out of the
reference's sources).

Two builds of each kernel are held to two bars:

* IEEE build (the kernel bodies with IEEE division and square root, the
  arithmetic the oracle specifies): INT8 codes, INT4 codes and dequantised
  values bit-exact; LayerNorm, GELU and the bank EMA within a few fp32 ulps
  (the kernels sum in another order, contract multiply-adds and use rsqrtf);
  16-bit outputs within one 16-bit ulp.
* the reference's own build (-O3 --use_fast_math, CMakeLists.txt:41-46):
  the same, except that its approximate division moves x / s off exact
  rounding ties, so INT8 / INT4 codes may differ by one step exactly where
  x / s lies within a few ulps of a tie, and nowhere else (the oracle keeps
  IEEE division: rounding ties away from zero is then well defined); and its
  fast tanhf moves GELU(x) by up to ~4e-6 |x| (most where 1 + tanh cancels),
  so GELU is held to 1e-5 |x| there (plus two 16-bit ulps for f16).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import ref_cases  # noqa: E402

FIX = np.load(ref_cases.FIXTURE) if ref_cases.FIXTURE.exists() else None


def _fixture(name, variant):
    assert FIX is not None, f"{ref_cases.FIXTURE} missing: run tests/golden/make_ref_golden.py"
    return FIX[f"{name}/{variant}"]


def _oracle_out(orc, name, inp):
    kind, dt, (R, Cn), _ = ref_cases.CASES[name]
    odt = orc.F16 if dt == "f16" else orc.F32
    if kind == "sym_quant":
        q, s = orc.quant_int8_rows(inp["x"].reshape(1, -1))
        assert s[0] == np.float32(np.abs(inp["x"]).max() / np.float32(127.0))
        return q.reshape(R, Cn), inp["x"] / s[0]
    if kind == "per_channel_quant":
        q, s = orc.quant_int8_rows(inp["x"])
        return q, inp["x"] / s[:, None]
    if kind == "per_channel_dequant":
        return orc.dequant_int8_rows(inp["q"], inp["s"], odt), None
    if kind == "int4_codes":
        packed, s, zp = orc.quant_int4_g128(inp["x"])
        q = np.empty((R, Cn), np.int8)
        q[:, 0::2] = packed & 15
        q[:, 1::2] = packed >> 4
        t = inp["x"] / np.repeat(s, 128, axis=1) + np.repeat(zp, 128, axis=1)
        return q, t
    if kind == "layernorm":
        return orc.round_to(orc.layernorm_x2(inp["x"], inp["g"], inp["b"]), odt), None
    if kind == "gelu":
        return orc.round_to(orc.activation(inp["x"] + inp["b"], orc.ACT_GELU), odt), None
    if kind == "store_state":
        w = (np.float32(ref_cases.RATE) * inp["scores"] if inp["scores"] is not None else
             np.full(R, ref_cases.RATE, np.float32)).astype(np.float32)
        return orc.ema_rows(inp["memory"], inp["state"], w, odt), None
    raise KeyError(kind)


def _ulps16(a):
    """One f16 ulp at each value of a (fp32 array of f16 values)."""
    a = np.abs(np.asarray(a, np.float32)).astype(np.float16)
    nxt = np.nextafter(a, np.float16(np.inf))
    return (nxt.astype(np.float32) - a.astype(np.float32))


def _assert_codes(got, want, t, fast, what):
    got = got.astype(np.int32)
    want = want.astype(np.int32)
    if not fast:
        assert np.array_equal(got, want), f"{what}: {np.sum(got != want)} codes differ"
        return 0
    diff = got - want
    assert np.abs(diff).max() <= 1, f"{what}: a code differs by more than one step"
    bad = diff != 0
    if bad.any():
        tt = np.asarray(t, np.float64)[bad]
        dist = np.abs(np.abs(tt - np.trunc(tt)) - 0.5)
        assert dist.max() <= 4 * np.spacing(np.float32(np.abs(tt).max())), (
            f"{what}: a code differs away from a rounding tie")
    return int(bad.sum())


@pytest.mark.parametrize("variant", ["ieee", "reference"])
@pytest.mark.parametrize("name", list(ref_cases.CASES))
def test_oracle_matches_reference_kernel(orc, name, variant):
    kind, dt, _, _ = ref_cases.CASES[name]
    inp = ref_cases.inputs(name)
    ref = _fixture(name, variant)
    want, t = _oracle_out(orc, name, inp)
    fast = variant == "reference"
    what = f"{name} ({variant} build)"
    if kind in ("sym_quant", "per_channel_quant", "int4_codes"):
        ref = ref.astype(np.int32)
        if kind == "int4_codes":
            ref = np.clip(ref, 0, 15)
        _assert_codes(ref, want, t, fast, what)
        return
    ref = ref.astype(np.float32)
    if kind == "per_channel_dequant":
        assert np.array_equal(ref, want), f"{what}: dequantised values differ"
        return
    if kind == "gelu" and fast:
        x = np.abs(inp["x"] + inp["b"])
        bound = 1e-5 * x + (2 * _ulps16(want) if dt == "f16" else 1e-7)
        err = np.abs(ref - want)
        assert np.all(err <= bound), f"{what}: max abs difference {err.max():.3e}"
        return
    if dt == "f16":
        err = np.abs(ref - want)
        assert np.all(err <= _ulps16(want) * 1.0001), f"{what}: beyond one f16 ulp"
        return
    # fp32: a few ulps of the output scale (LayerNorm: also the rsqrtf / sum order)
    scale = np.abs(want).max()
    ulp = np.spacing(np.float32(scale))
    bound = {"layernorm": 64, "gelu": 8, "store_state": 4}[kind] * ulp
    err = np.abs(ref - want).max()
    assert err <= bound, f"{what}: max abs difference {err:.3e} > {bound:.3e}"


def test_quantizer_cases_hold_exact_ties(orc):
    """The quantizer cases put thousands of entries exactly on rounding ties
    of x / s, which the IEEE build and the oracle both round away from zero."""
    for name in ("sym_quant_f32", "sym_quant_f16", "per_channel_quant_f32",
                 "per_channel_quant_f16"):
        _, t = _oracle_out(orc, name, ref_cases.inputs(name))
        ties = np.abs(np.abs(t - np.trunc(t)) - 0.5) == 0
        assert ties.sum() > 1000, f"{name} lost its exact ties"


def test_reference_kernel_recipe_extracts_and_builds():
    """Where the reference tree is present, every cited line range still
    holds its kernel and both builds exist and export the launchers."""
    import ctypes
    from oracle import ref_kernels
    if not (ref_kernels.reference_root() / "src").is_dir():
        pytest.skip("the reference tree is not on this machine")
    ref_kernels.extract(ref_kernels.reference_root())
    for path in ref_kernels.build().values():
        lib = ctypes.CDLL(str(path))
        for sym in ("ref_symmetric_quantize", "ref_linear_quantize", "ref_per_channel_quantize",
                    "ref_per_channel_dequantize", "ref_layernorm_residual", "ref_bias_gelu",
                    "ref_store_state"):
            assert hasattr(lib, sym), f"{path.name} lacks {sym}"
