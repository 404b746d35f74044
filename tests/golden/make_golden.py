"""Generates the golden fixtures of the CPU oracle (regression pins).

    python tests/golden/make_golden.py

Writes tests/golden/oracle_golden.npz: small seeded cases of every oracle
function (INT8 / INT4 quantization, int32 GEMM, W8A8 / W8A32 / W4A16
linears, LayerNorm, attention, memory store, block forward per scheme).  The
reference itself ships no fixtures and cannot be built, so these pin the
oracle's own outputs: tests/test_oracle_cpu.py recomputes each case and
compares (integers bit-exact, floats to 1e-6).
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT), str(ROOT / "obsidian-memory-transformer_b200")]

from oracle import oracle as orc  # noqa: E402
from ltm_b200 import synthetic  # noqa: E402

OUT = Path(__file__).resolve().parent / "oracle_golden.npz"

BLOCK_CASES = [  # (name, scheme, dtype, memory_write)
    ("w8a32_f32", orc.W8A32, orc.F32, 0),
    ("w8a8_f16", orc.W8A8, orc.F16, 1),
    ("w8a8_bf16", orc.W8A8, orc.BF16, 0),
    ("w4a16_bf16", orc.W4A16, orc.BF16, 1),
]
BH, BNH, BF, BMS, BB, BS = 128, 2, 256, 32, 2, 24


def cases():
    rng = np.random.default_rng(20261201)
    d = {}
    w = (rng.standard_normal((24, 200)) * 0.02).astype(np.float32)
    w[3] = 0.0
    d["q8_in"] = w
    d["q8_q"], d["q8_s"] = orc.quant_int8_rows(w)
    w4 = (rng.standard_normal((6, 384)) * 0.02).astype(np.float32)
    w4[1, :128] = np.abs(w4[1, :128])
    w4[2, 128:256] = 0.0
    d["q4_in"] = w4
    d["q4_packed"], d["q4_s"], d["q4_zp"] = orc.quant_int4_g128(w4)
    qa = rng.integers(-127, 128, (33, 96), dtype=np.int8)
    qw = rng.integers(-127, 128, (64, 96), dtype=np.int8)
    d["gemm_qa"], d["gemm_qw"] = qa, qw
    d["gemm_acc"] = orc.gemm_i8(qa, qw)
    sa = rng.random(33).astype(np.float32) * 0.01
    sw = rng.random(64).astype(np.float32) * 0.01
    b = (rng.standard_normal(64) * 0.02).astype(np.float32)
    d["lin_sa"], d["lin_sw"], d["lin_b"] = sa, sw, b
    d["lin_w8a8_gelu"] = orc.linear_w8a8(qa, sa, qw, sw, b, orc.ACT_GELU)
    a = rng.standard_normal((33, 256)).astype(np.float32)
    wl = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    q8, s8 = orc.quant_int8_rows(wl)
    p4, s4, z4 = orc.quant_int4_g128(wl)
    d["lin_a"], d["lin_wl"] = a, wl
    d["lin_w8a32_sig"] = orc.linear_w8a32(a, q8, s8, b, orc.ACT_SIGMOID)
    d["lin_w4a16"] = orc.linear_w4a16(orc.round_to(a, orc.BF16), p4, s4, z4, b, orc.ACT_NONE, orc.BF16)
    x = rng.standard_normal((17, 64)).astype(np.float32) * 3
    g = (1 + 0.1 * rng.standard_normal(64)).astype(np.float32)
    bb = (0.1 * rng.standard_normal(64)).astype(np.float32)
    d["ln_x"], d["ln_g"], d["ln_b"] = x, g, bb
    d["ln_y"] = orc.layernorm_x2(x, g, bb)
    qkv = rng.standard_normal((2 * 20, 3 * 128)).astype(np.float32)
    d["attn_qkv"] = qkv
    d["attn_causal"] = orc.attention(qkv[:, :128], qkv[:, 128:256], qkv[:, 256:], 2, 20, 20, 2, 64,
                                     True, orc.F32)
    kvm = rng.standard_normal((16, 256)).astype(np.float32)
    d["attn_kvm"] = kvm
    d["attn_memory"] = orc.attention(qkv[:, :128], kvm[:, :128], kvm[:, 128:], 2, 20, 16, 2, 64,
                                     False, orc.F32, kv_shared=True)
    mem = (rng.standard_normal((16, 128)) / np.sqrt(128)).astype(np.float32)
    st = (0.3 * rng.standard_normal(128)).astype(np.float32)
    d["store_mem"], d["store_state"] = mem, st
    d["store_out"] = orc.memory_store(mem, kvm[:, :128], qkv[:, :128], st, 2, 0.5, True, orc.F32)
    wts = synthetic.block_weights(BH, BF, BMS, 7)
    xb = synthetic.activations(BB * BS, BH, 8)
    for name, scheme, dt, mw in BLOCK_CASES:
        cfg = dict(H=BH, F=BF, nh=BNH, dh=BH // BNH, Ms=BMS, scheme=scheme, dtype=dt,
                   memory_write=mw)
        y, m = orc.block_forward(cfg, wts, orc.round_to(xb, dt), BB, BS)
        d[f"block_{name}_y"] = y
        d[f"block_{name}_mem"] = m
    return d


def main():
    d = cases()
    np.savez_compressed(OUT, **d)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(d)} arrays)")


if __name__ == "__main__":
    main()
