"""Cases that pin the oracle to the reference's own kernels (test
infrastructure).

Each case is a seeded input of one reference kernel that
oracle/ref_kernels.py compiles from the reference's sources, plus the oracle
function it is checked against.  make_ref_golden.py runs the cases on a GPU
through oracle/_ref/libref_kernels.so (the reference's own flags, -O3
--use_fast_math) and libref_kernels_ieee.so (the same kernel bodies with IEEE
division / square root) and writes reference_kernels.npz; the CPU suite
recomputes the inputs from the seeds and compares the oracle with the stored
outputs, and the GPU suite re-runs the kernels and checks they reproduce the
stored outputs bit for bit.

Quantizer inputs contain exact rounding ties: a row whose largest magnitude
is 127 * 2^-e has the scale 2^-e exactly, and entries (j + 0.5) * 2^-e then
sit exactly on a tie of x / s.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
FIXTURE = Path(__file__).resolve().parent / "reference_kernels.npz"
REF_DIR = ROOT / "oracle" / "_ref"
VARIANTS = {"reference": REF_DIR / "libref_kernels.so", "ieee": REF_DIR / "libref_kernels_ieee.so"}

# name -> (kind, dtype, shape, seed)
CASES = {
    "sym_quant_f32": ("sym_quant", "f32", (64, 256), 1),
    "sym_quant_f16": ("sym_quant", "f16", (64, 256), 2),
    "per_channel_quant_f32": ("per_channel_quant", "f32", (96, 512), 3),
    "per_channel_quant_f16": ("per_channel_quant", "f16", (96, 512), 4),
    "per_channel_dequant_f32": ("per_channel_dequant", "f32", (64, 384), 5),
    "per_channel_dequant_f16": ("per_channel_dequant", "f16", (64, 384), 6),
    "int4_codes_f32": ("int4_codes", "f32", (48, 512), 7),
    "layernorm_f32_h768": ("layernorm", "f32", (32, 768), 8),
    "layernorm_f32_h4096": ("layernorm", "f32", (8, 4096), 9),
    "layernorm_f16_h768": ("layernorm", "f16", (32, 768), 10),
    "gelu_f32": ("gelu", "f32", (16, 1024), 11),
    "gelu_f16": ("gelu", "f16", (16, 1024), 12),
    "store_state_scores_f32": ("store_state", "f32", (64, 512), 13),
    "store_state_rate_f32": ("store_state", "f32", (64, 512), 14),
    "store_state_scores_f16": ("store_state", "f16", (48, 768), 15),
}
RATE = 0.9


def _as_dtype(a, dt):
    a = np.asarray(a, np.float32)
    return a.astype(np.float16).astype(np.float32) if dt == "f16" else a


def _tie_rows(rng, rows, cols, dt, e_fixed=None):
    """Rows N(0, 0.02) of which every second one has scale 2^-e exactly and
    about a quarter of its entries on exact (j + 0.5) * 2^-e ties."""
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    for r in range(0, rows, 2):
        e = e_fixed if e_fixed is not None else 7 + (r // 2) % 4
        s = np.float32(2.0 ** -e)
        w[r] = np.clip(w[r], -126 * s, 126 * s)
        w[r, rng.integers(cols)] = 127 * s * (1 if r % 4 == 0 else -1)
        idx = rng.choice(cols, cols // 4, replace=False)
        j = rng.integers(-126, 126, size=idx.size)
        w[r, idx] = ((j + 0.5) * s).astype(np.float32)
    return _as_dtype(w, dt)


def inputs(name: str) -> dict:
    """The case's inputs as fp32 numpy arrays (values representable in the
    case's dtype)."""
    kind, dt, (R, Cn), seed = CASES[name]
    rng = np.random.default_rng(seed)
    if kind == "sym_quant":
        x = _tie_rows(rng, R, Cn, dt, e_fixed=6)
        x[0, 0] = np.float32(127.0 / 64.0)  # per-tensor scale 2^-6
        x[1:] = np.clip(x[1:], -1.98, 1.98)
        return {"x": x}
    if kind == "per_channel_quant":
        return {"x": _tie_rows(rng, R, Cn, dt)}
    if kind == "per_channel_dequant":
        q = rng.integers(-127, 128, size=(R, Cn)).astype(np.int8)
        s = (rng.random(R) * 1e-3 + 1e-5).astype(np.float32)
        return {"q": q, "s": s}
    if kind == "int4_codes":
        return {"x": (rng.standard_normal((R, Cn)) * 0.02).astype(np.float32)}
    if kind == "layernorm":
        x = _as_dtype(rng.standard_normal((R, Cn)) * 2 + 0.5, dt)
        g = _as_dtype(1 + 0.1 * rng.standard_normal(Cn), dt)
        b = _as_dtype(0.1 * rng.standard_normal(Cn), dt)
        return {"x": x, "g": g, "b": b}
    if kind == "gelu":
        x = _as_dtype(rng.uniform(-6, 6, size=(R, Cn)), dt)
        b = _as_dtype(0.1 * rng.standard_normal(Cn), dt)
        return {"x": x, "b": b}
    if kind == "store_state":
        mem = _as_dtype(rng.standard_normal((R, Cn)) / np.sqrt(Cn), dt)
        state = _as_dtype(0.3 * rng.standard_normal(Cn), dt)
        sc = rng.random(R).astype(np.float32)
        scores = None if "rate" in name else _as_dtype(sc / sc.sum() * R * 0.5, dt)
        return {"memory": mem, "state": state, "scores": scores}
    raise KeyError(kind)


# ------------------------------------------------------------------ running --
def load(variant: str):
    path = VARIANTS[variant]
    if not path.exists():
        raise FileNotFoundError(
            f"{path} is missing: build it with `python oracle/ref_kernels.py` on a machine that "
            "holds the reference tree (the library then travels with the repository)")
    lib = C.CDLL(str(path))
    vp, ci, cf = C.c_void_p, C.c_int, C.c_float
    lib.ref_symmetric_quantize.argtypes = [vp, ci, vp, cf, ci, vp]
    lib.ref_linear_quantize.argtypes = [vp, ci, vp, cf, cf, ci, vp]
    lib.ref_per_channel_quantize.argtypes = [vp, ci, vp, vp, vp, ci, ci, ci, vp]
    lib.ref_per_channel_dequantize.argtypes = [vp, vp, ci, vp, vp, ci, ci, ci, vp]
    lib.ref_layernorm_residual.argtypes = [vp, vp, vp, vp, vp, ci, ci, ci, vp]
    lib.ref_bias_gelu.argtypes = [vp, vp, vp, ci, ci, ci, vp]
    lib.ref_store_state.argtypes = [vp, vp, vp, cf, ci, ci, ci, vp]
    for f in ("ref_symmetric_quantize", "ref_linear_quantize", "ref_per_channel_quantize",
              "ref_per_channel_dequantize", "ref_layernorm_residual", "ref_bias_gelu",
              "ref_store_state"):
        getattr(lib, f).restype = ci
    return lib


def run(lib, name: str, inp: dict | None = None, oracle=None) -> np.ndarray:
    """Runs the case's reference kernel on cuda:0; returns its output (int8
    codes, or floats as fp32).  The INT4 case needs the oracle's group scales
    and zero-points (oracle module)."""
    import torch
    kind, dt, (R, Cn), _ = CASES[name]
    inp = inp if inp is not None else inputs(name)
    tdt = torch.float32 if dt == "f32" else torch.float16
    code = 0 if dt == "f32" else 1
    dev = torch.device("cuda", 0)

    def d(a, t=None):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev, t if t is not None else tdt)

    def ok(rc):
        if rc != 0:
            raise RuntimeError(f"{name}: reference kernel launch failed (cudaError {rc})")

    if kind == "sym_quant":
        x = d(inp["x"])
        s = np.float32(np.abs(inp["x"]).max() / np.float32(127.0))
        q = torch.empty(x.shape, dtype=torch.int8, device=dev)
        ok(lib.ref_symmetric_quantize(x.data_ptr(), code, q.data_ptr(), float(s), x.numel(), None))
        torch.cuda.synchronize()
        return q.cpu().numpy()
    if kind == "per_channel_quant":
        x = d(inp["x"])
        s = (np.abs(inp["x"]).max(axis=1) / np.float32(127.0)).astype(np.float32)
        sd, zd = d(s, torch.float32), torch.zeros(R, dtype=torch.float32, device=dev)
        q = torch.empty(x.shape, dtype=torch.int8, device=dev)
        ok(lib.ref_per_channel_quantize(x.data_ptr(), code, q.data_ptr(), sd.data_ptr(),
                                        zd.data_ptr(), R * Cn, R, Cn, None))
        torch.cuda.synchronize()
        return q.cpu().numpy()
    if kind == "per_channel_dequant":
        q = d(inp["q"], torch.int8)
        sd, zd = d(inp["s"], torch.float32), torch.zeros(R, dtype=torch.float32, device=dev)
        out = torch.empty((R, Cn), dtype=tdt, device=dev)
        ok(lib.ref_per_channel_dequantize(q.data_ptr(), out.data_ptr(), code, sd.data_ptr(),
                                          zd.data_ptr(), R * Cn, R, Cn, None))
        torch.cuda.synchronize()
        return out.float().cpu().numpy()
    if kind == "int4_codes":
        # round(w / s + zp) of every 128-wide group with the oracle's group
        # scale and zero-point (the reference's asymmetric form)
        _, s, zp = oracle.quant_int4_g128(inp["x"])
        out = np.empty((R, Cn), np.int8)
        x = d(inp["x"])
        q = torch.empty((R, Cn), dtype=torch.int8, device=dev)
        for r in range(R):
            for g in range(Cn // 128):
                xs = x[r, g * 128:(g + 1) * 128]
                qs = q[r, g * 128:(g + 1) * 128]
                ok(lib.ref_linear_quantize(xs.data_ptr(), code, qs.data_ptr(), float(s[r, g]),
                                           float(zp[r, g]), 128, None))
        torch.cuda.synchronize()
        out[:] = q.cpu().numpy()
        return out
    if kind == "layernorm":
        x, g, b = d(inp["x"]), d(inp["g"]), d(inp["b"])
        out = torch.empty_like(x)
        ok(lib.ref_layernorm_residual(x.data_ptr(), x.data_ptr(), g.data_ptr(), b.data_ptr(),
                                      out.data_ptr(), code, R, Cn, None))
        torch.cuda.synchronize()
        return out.float().cpu().numpy()
    if kind == "gelu":
        x, b = d(inp["x"]), d(inp["b"])
        out = torch.empty_like(x)
        ok(lib.ref_bias_gelu(x.data_ptr(), b.data_ptr(), out.data_ptr(), code, R, Cn, None))
        torch.cuda.synchronize()
        return out.float().cpu().numpy()
    if kind == "store_state":
        mem, st = d(inp["memory"]), d(inp["state"])
        sc = d(inp["scores"]) if inp["scores"] is not None else None
        ok(lib.ref_store_state(mem.data_ptr(), st.data_ptr(),
                               sc.data_ptr() if sc is not None else None, RATE, R, Cn, code,
                               None))
        torch.cuda.synchronize()
        return mem.float().cpu().numpy()
    raise KeyError(kind)
