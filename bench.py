#!/usr/bin/env python
"""Headline benchmark: Titan-block tokens/s of the quantized prefill, tensor
parallel over the N GPUs.

Workload (one step, the default): an 8-layer Titan prefill with W8A8 linears
and bf16 activations -- hidden 8192, 64 heads (head_dim 128), FFN 28672, 8192
memory slots, batch 16, seq 4096, per-token dynamic INT8 activations --
sharded by heads, memory slots' K_M / V_M and FFN columns over the N GPUs
with an NCCL allreduce after the output and FFN-down projections.  The job is
fixed as N grows (strong scaling), so `python bench.py --gpus N` for N = 1, 2,
4, 8 measures the tensor-parallel scaling of one workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config tp|prefill|w4a16|decode]

At N = 1 the line also carries `side_workloads`: the 12-layer hidden-768
W8A8 prefill (batch 8 x 2048), the 4-layer hidden-4096 W4A16 long-context
prefill (batch 4 x 8192) and the 32-layer W4A16 batched decode step (batch
64 against 32768 cached positions), each measured the same way with fewer
steps.  `--config` runs one of them as the headline instead (prefill and
decode: N independent replicas, weak scaling).  Rank 0 prints one JSON line.
`--impl reference` times the CPU restatement of the reference's algorithm
(the oracle; the reference itself does not compile) on all host cores with
the same metric and workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (str(ROOT), str(ROOT / "obsidian-memory-transformer_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

WL = dict(layers=12, B=8, S=2048, H=768, nh=12, F=3072, Ms=512, vocab=32000)
WORKLOAD_NAME = ("12-layer Titan prefill, W8A8 INT8 linears + fp16 activations, hidden 768, "
                 "12 heads, FFN 3072, 512 memory slots, vocab 32000, batch 8, seq 2048")
# the headline metric (value = whole-job tokens/s; tokens/s per GPU and the
# roofline fraction are reported beside it)
METRIC = "Titan-block tokens/s per GPU (prefill & decode) and % of tensor/HBM roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-probe", action="store_true", help="skip the per-kernel roofline probe")
    ap.add_argument("--no-side", action="store_true",
                    help="skip the side workloads measured after the headline at N = 1")
    ap.add_argument("--overlap", choices=["auto", "on", "off"], default="auto",
                    help="chunked collectives overlapping the GEMMs in the sequence-parallel "
                         "forward (auto: the library's default, off)")
    ap.add_argument("--comm-sms", type=int, default=16, help=argparse.SUPPRESS)
    ap.add_argument("--tp-reduce", choices=["act", "exact"], default="act",
                    help="row-parallel reductions of the sequence-parallel forward: partial sums "
                         "in the activation type (NCCL reduce-scatter) or exact int32 "
                         "accumulators (output equal to one GPU's)")
    ap.add_argument("--no-sp", action="store_true",
                    help="tensor parallel without sequence parallelism (every rank holds the "
                         "full activations; allreduce after the row-parallel projections)")
    ap.add_argument("--layers", type=int, default=None, help=argparse.SUPPRESS)
    ap.add_argument("--config", choices=["prefill", "tp", "w4a16", "decode"], default="tp",
                    help="tp: the 8-layer hidden-8192 W8A8 prefill, tensor-parallel over the N "
                         "GPUs (default); prefill: the 12-layer W8A8 prefill (N>1 = data-parallel "
                         "replicas); w4a16: the 4-layer hidden-4096 W4A16 long-context "
                         "prefill (tensor-parallel when N > 1); decode: the 32-layer hidden-4096 "
                         "W4A16 batched decode step against a 32768-position KV cache (N > 1 = "
                         "replicas)")
    ap.add_argument("--ncu-case", nargs="?", const="prefill", default=None,
                    choices=["prefill", "tp", "tplayer", "w4a16", "decode"],
                    help="launch each kernel of one block once at the workload's shapes (for ncu); "
                         "tp: the tensor-parallel layer's attention and K = 8192 GEMM at batch 2; "
                         "w4a16: one long-context block forward at 1 x 8192 tokens; decode: "
                         "one decode step of one block at batch 64, 2048 cached positions")
    return ap.parse_args()


# ----------------------------------------------------------------- plumbing --
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return d, "measured (MEASURED_PEAKS.json)"
    return dict(FALLBACK_PEAKS), "fallback (profiling recipe)"


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        rows = []
        with open(self.out.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.out.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- our path --
def build_model(torch, ltm, n_layers: int, device: int):
    from ltm_b200 import synthetic
    cfg = ltm.TitanBlockConfig(hidden_dim=WL["H"], ffn_dim=WL["F"], num_heads=WL["nh"],
                               head_dim=WL["H"] // WL["nh"], memory_slots=WL["Ms"])
    q = ltm.QuantConfig(scheme=ltm.SCHEME_W8A8, act_dtype=ltm.DTYPE_F16)
    model = ltm.TitanModel(cfg, q, n_layers, WL["vocab"], device=device)
    model.load_embedding(synthetic.embedding(WL["vocab"], WL["H"], 7))
    for i in range(n_layers):
        model.load_layer(i, synthetic.block_weights(WL["H"], WL["F"], WL["Ms"], 1000 + i))
    return model


def per_layer_ops():
    """(name, kind, shape, launches per layer) of the kernels of one block."""
    B, S, H, F, Ms = WL["B"], WL["S"], WL["H"], WL["F"], WL["Ms"]
    T = B * S
    return [
        ("gemm_qkvm", "w8a8", (T, 4 * H, H), 1),
        ("gemm_kvm", "w8a8", (Ms, 2 * H, H), 1),
        ("gemm_o_om_gate", "w8a8", (T, H, H), 3),
        ("gemm_ffn_up", "w8a8", (T, F, H), 1),
        ("gemm_ffn_down", "w8a8", (T, H, F), 1),
        ("attn_self_causal", "attn", (B, S, S, True), 1),
        ("attn_memory", "attn", (B, S, Ms, False), 1),
        ("ln_quant", "ln", (T, H), 2),
        ("quant_rows_h", "quant", (T, H), 2),
        ("quant_rows_f", "quant", (T, F), 1),
        ("quant_bank", "quant", (Ms, H), 1),
    ]


def step_work(layers: int) -> dict:
    """Algorithmic work of one step per kernel class: int8/bf16 ops of the
    GEMMs and attention (2 per multiply-add), bytes of the bandwidth kernels."""
    B, S, H, F, Ms, nh = WL["B"], WL["S"], WL["H"], WL["F"], WL["Ms"], WL["nh"]
    T, dh = B * S, WL["H"] // WL["nh"]
    gemm = 2.0 * (T * 4 * H * H + Ms * 2 * H * H + 3 * T * H * H + T * F * H + T * H * F)
    attn = 4.0 * B * nh * dh * (S * (S + 1) / 2 + S * Ms)
    # LN: f16 row in, int8 of LN(x) and of x out (LN1) / int8 out (LN2) + scales
    ln = (2 * T * H + 2 * T * H + 8 * T) + (2 * T * H + T * H + 4 * T)
    quant = 2 * (3 * T * H + 4 * T) + (3 * T * F + 4 * T) + (3 * Ms * H + 4 * Ms)
    return {"w8a8_tc_kernel": {"amount": gemm * layers, "unit": "flop"},
            "attn_tc_kernel": {"amount": attn * layers, "unit": "flop"},
            "ln_x2_kernel": {"amount": ln * layers, "unit": "byte"},
            "rowwise_int8_kernel": {"amount": quant * layers, "unit": "byte"}}


# Tensor-parallel prefill: hidden 8192, 64 heads (head_dim 128), FFN 28672,
# 8192 memory slots, batch 16 x seq 4096, 8 layers, W8A8 + bf16 activations.
TP_WL = dict(layers=8, B=16, S=4096, H=8192, nh=64, F=28672, Ms=8192)
TP_WORKLOAD_NAME = ("8-layer Titan prefill, tensor-parallel, W8A8 INT8 linears + bf16 activations, "
                    "hidden 8192, 64 heads (head_dim 128), FFN 28672, 8192 memory slots, "
                    "batch 16, seq 4096")


# W4A16 long-context prefill: hidden 4096, 32 heads (head_dim 128), FFN 11008,
# 4096 memory slots, batch 4 x seq 8192, 4 layers, INT4 group-128 weights,
# bf16 activations.
W4_WL = dict(layers=4, B=4, S=8192, H=4096, nh=32, F=11008, Ms=4096)
W4_WORKLOAD_NAME = ("4-layer Titan long-context prefill, W4A16 INT4 group-128 weights + bf16 "
                    "activations, hidden 4096, 32 heads (head_dim 128), FFN 11008, 4096 memory "
                    "slots, batch 4, seq 8192")


# Batched decode: hidden 4096, 32 heads (head_dim 128), FFN 11008, 2048 memory
# slots, 32 layers, INT4 group-128 weights, bf16 activations; batch 64, one new
# token per sequence against a bf16 KV cache of 32768 positions per sequence
# (N(0,1)); memory read and write (attention-score slot weights) every step.
DEC_WL = dict(layers=32, B=64, P=32768, H=4096, nh=32, F=11008, Ms=2048)
DEC_WORKLOAD_NAME = ("32-layer Titan batched decode, W4A16 INT4 group-128 weights + bf16 "
                     "activations, hidden 4096, 32 heads (head_dim 128), FFN 11008, 2048 memory "
                     "slots, batch 64 x 1 new token against a 32768-position bf16 KV cache per "
                     "sequence, memory read + write every step")


def decode_layer_bytes(wl: dict = DEC_WL) -> dict:
    """Algorithmic HBM bytes of one decode layer: the K and V rows of the
    cache's positions (the new one included), the packed INT4 weights with
    their fp32 scales and uint8 zero-points, and the bank / K_M | V_M traffic
    (bank read + write, K_M | V_M read + write by the EMA, K_M | V_M read by
    the memory attention, K_M read by the slot weights)."""
    B, P, H, F, Ms = (wl[k] for k in ("B", "P", "H", "F", "Ms"))
    kv = 2 * B * P * H * 2
    params = 4 * H * H + 2 * H * H + 3 * H * H + 2 * H * F
    weights = params // 2 + (params // 128) * 5
    bank = 2 * Ms * H * 2 + 2 * Ms * 2 * H * 2 + Ms * 2 * H * 2 + Ms * H * 2
    return {"kv": kv, "weights": weights, "bank": bank, "total": kv + weights + bank}


def step_work_tp(layers: int, tp: int, wl: dict = TP_WL, gemm_class: str = "w8a8_tc_kernel") -> dict:
    """Algorithmic ops of one tensor-parallel step on one rank (its head /
    FFN shards; the gate projection is replicated)."""
    B, S, H, F, Ms, nh = (wl[k] for k in ("B", "S", "H", "F", "Ms", "nh"))
    T, dh, Hl, Fl, nhl = B * S, H // nh, H // tp, F // tp, nh // tp
    gemm = 2.0 * (T * 4 * Hl * H + Ms * 2 * Hl * H + 2 * T * H * Hl + T * H * H + T * Fl * H
                  + T * H * Fl)
    attn = 4.0 * B * nhl * dh * (S * (S + 1) / 2 + S * Ms)
    return {gemm_class: {"amount": gemm * layers, "unit": "flop"},
            "attn_tc_kernel": {"amount": attn * layers, "unit": "flop"}}


def roofline_of(result: dict, work: dict, torch, workload: str = "B8 S2048 H768") -> tuple:
    """Roofline entry of the dominant kernel class of one timed step (kernel
    timer result) and the measured int8 peak; `workload` selects the ncu
    traffic row of profiles/traffic.md."""
    pk, pk_src = peaks()
    i8 = int8_peak(torch)
    by_kind = {}
    for name, (n, ms) in result.items():
        kind = name.split("/")[0]
        k = by_kind.setdefault(kind, dict(ms=0.0, launches=0))
        k["ms"] += ms
        k["launches"] += n
    dom = max((k for k in by_kind if k in work), key=lambda k: by_kind[k]["ms"])
    d = by_kind[dom]
    avg_ms = d["ms"] / d["launches"]
    per_launch = work[dom]["amount"] / d["launches"]
    if work[dom]["unit"] == "flop":
        achieved = per_launch / (avg_ms * 1e-3) / 1e12
        if dom.startswith("w8a8"):  # int8 tensor peak; the 16-bit classes use bf16
            peak = i8 if i8 else 2.0 * pk["bf16_tflops"]
            peak_src = ("int8 cuBLASLt (torch._int_mm 8192^3) measured in this run" if i8 else
                        "2 x bf16_tflops " + pk_src + " (derived int8)")
        else:
            peak = pk["bf16_tflops"]
            peak_src = "bf16_tflops " + pk_src
        unit, bound = "TFLOP/s", "tensor"
    else:
        achieved = per_launch / (avg_ms * 1e-3) / 1e9
        peak = pk["hbm_gbs"]
        peak_src = "hbm_gbs " + pk_src
        unit, bound = "GB/s", "hbm"
    roof = {"bound": bound, "kernel": dom, "achieved": round(achieved, 2),
            "peak": round(peak, 2), "unit": unit, "frac": round(achieved / peak, 4),
            "traffic": traffic_from_profiles(dom, workload), "peak_source": peak_src,
            "launches_per_step": d["launches"], "avg_launch_ms": round(avg_ms, 5),
            "algorithmic_per_launch": per_launch, "algorithmic_unit": work[dom]["unit"]}
    return roof, i8


def probe_kernels(torch, ltm, reps: int = 10, timed: bool = True):
    """Times each kernel of one block standalone at the workload's shapes with
    CUDA events on the launching stream (L2 flushed and cleaned before every
    launch)."""
    dev = torch.device("cuda")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    clean = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    H, nh = WL["H"], WL["nh"]
    dh = H // nh
    res = []
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    for name, kind, shape, per_layer in per_layer_ops():
        if kind == "w8a8":
            M, N, K = shape
            qa = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=gen)
            qw = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=gen)
            sa = torch.rand(M, device=dev) * 0.01
            sw = torch.rand(N, device=dev) * 0.01
            bias = torch.zeros(N, device=dev)
            y = torch.empty((M, N), dtype=torch.float16, device=dev)

            def call():
                ltm._check(ltm.lib().ltm_linear_w8a8(ltm._ptr(qa), ltm._ptr(sa), ltm._ptr(qw),
                                                     ltm._ptr(sw), ltm._ptr(bias), 0, ltm._ptr(y),
                                                     ltm.DTYPE_F16, M, N, K, ltm._stream()))
            flops = 2.0 * M * N * K
            nbytes = M * K + N * K + 2 * M * N + 4 * (M + 2 * N)
        elif kind == "attn":
            B, Sq, Skv, causal = shape
            q = torch.randn((B * Sq, 4 * H), dtype=torch.float16, device=dev, generator=gen)
            kv = q if causal else torch.randn((Skv, 2 * H), dtype=torch.float16, device=dev,
                                              generator=gen)
            o = torch.empty((B * Sq, H), dtype=torch.float16, device=dev)
            if causal:
                qq, kk, vv = q[:, :H], q[:, H:2 * H], q[:, 2 * H:3 * H]
            else:
                qq, kk, vv = q[:, 3 * H:], kv[:, :H], kv[:, H:]

            def call():
                ltm.attention(qq, kk, vv, B, Sq, Skv, nh, dh, causal, kv_shared=not causal, out=o)
            pairs = B * nh * (Sq * (Sq + 1) / 2 if causal else Sq * Skv)
            flops = 4.0 * pairs * dh
            nbytes = 2 * (B * Sq * H * 2 + (B if causal else 1) * Skv * H * 2)
        elif kind == "ln":
            T, Hh = shape
            x = torch.randn((T, Hh), dtype=torch.float16, device=dev, generator=gen)
            g = torch.ones(Hh, device=dev)
            b = torch.zeros(Hh, device=dev)

            def call():
                ltm.layernorm_residual(x, x, g, b)
            flops = 0.0
            nbytes = 2 * T * Hh + T * Hh  # f16 in, int8 out (fused-quant variant writes int8)
        else:
            T, K = shape
            x = torch.randn((T, K), dtype=torch.float16, device=dev, generator=gen)

            def call():
                ltm.quantize_act_int8_per_token(x)
            flops = 0.0
            nbytes = 2 * T * K + T * K + 4 * T
        call()
        torch.cuda.synchronize()
        if not timed:  # profiling case: one launch per kernel, no timing
            continue
        times = []
        for _ in range(reps):
            # write-flush L2, then read a second L2-sized buffer so the probed
            # kernel starts on a cold but clean L2 (no dirty-line writebacks)
            flush.fill_(1)
            clean.sum()
            torch.cuda._sleep(200_000)  # keeps the GPU busy while the host enqueues the launch
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            call()
            e.record()
            e.synchronize()
            times.append(s.elapsed_time(e))
        ms = statistics.median(times)
        res.append(dict(name=name, kind=kind, shape=list(shape), ms=ms, launches_per_layer=per_layer,
                        flops=flops, bytes=nbytes))
    del flush, clean
    return res


def probe_tp_case(torch, ltm):
    """One launch each of the tensor-parallel layer's kernels at a reduced
    batch (2 x 4096 tokens, 8 heads of 128, 8192 memory slots; a W8A8 GEMM
    with M = 8192, N = 8192, K = 8192): inputs larger than L2, a few GB on the
    device."""
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    B, S, nh, D, Ms = 2, 4096, 8, 128, 8192
    H = nh * D
    qkv = torch.randn((B * S, 4 * H), generator=gen, device=dev).to(torch.bfloat16)
    kv = torch.randn((Ms, 2 * H), generator=gen, device=dev).to(torch.bfloat16)
    o = torch.empty((B * S, H), dtype=torch.bfloat16, device=dev)
    ltm.attention(qkv[:, :H], qkv[:, H:2 * H], qkv[:, 2 * H:3 * H], B, S, S, nh, D, True, out=o)
    ltm.attention(qkv[:, 3 * H:], kv[:, :H], kv[:, H:], B, S, Ms, nh, D, False, kv_shared=True,
                  out=o)
    M = N = K = 8192
    qa = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=gen)
    qw = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=gen)
    sa = torch.rand(M, device=dev) * 1e-4
    sw = torch.rand(N, device=dev) * 1e-4
    bias = torch.zeros(N, device=dev)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    ltm._check(ltm.lib().ltm_linear_w8a8(ltm._ptr(qa), ltm._ptr(sa), ltm._ptr(qw), ltm._ptr(sw),
                                         ltm._ptr(bias), 0, ltm._ptr(y), ltm.DTYPE_BF16, M, N, K,
                                         ltm._stream()))
    torch.cuda.synchronize()


def probe_tp_layer_case(torch, ltm):
    """Two forwards of one hidden-8192 W8A8 block (the headline workload's
    layer at tensor-parallel size 1) at batch 2 x seq 4096 (8192 tokens, an
    eighth of the workload's rows): every kernel of the layer at its real
    widths, a few GB on the device (for ncu DRAM counts, scaled by 8)."""
    from ltm_b200 import synthetic
    wl = TP_WL
    H, F, Ms, nh, S = wl["H"], wl["F"], wl["Ms"], wl["nh"], wl["S"]
    cfg = ltm.TitanBlockConfig(hidden_dim=H, ffn_dim=F, num_heads=nh, head_dim=H // nh,
                               memory_slots=Ms)
    q = ltm.QuantConfig(scheme=ltm.SCHEME_W8A8, act_dtype=ltm.DTYPE_BF16)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(synthetic.block_weights(H, F, Ms, 1000))
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn((2, S, H), generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    blk(x)
    blk(x)
    torch.cuda.synchronize()
    blk.close()


def probe_w4a16_case(torch, ltm):
    """One forward of one long-context block (hidden 4096, 32 heads, FFN 11008,
    4096 slots, W4A16, bf16) at 1 x 8192 tokens, after a warm-up forward: the
    weight dequantisation pre-pass and the 16-bit GEMMs at the workload's
    per-sequence shapes (for ncu)."""
    from ltm_b200 import synthetic
    wl = W4_WL
    H, F, Ms, nh, S = wl["H"], wl["F"], wl["Ms"], wl["nh"], wl["S"]
    cfg = ltm.TitanBlockConfig(hidden_dim=H, ffn_dim=F, num_heads=nh, head_dim=H // nh,
                               memory_slots=Ms)
    q = ltm.QuantConfig(scheme=ltm.SCHEME_W4A16, act_dtype=ltm.DTYPE_BF16)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(synthetic.block_weights(H, F, Ms, 1000))
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn((1, S, H), generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    blk(x)
    blk(x)
    torch.cuda.synchronize()
    blk.close()


def int8_peak(torch):
    """cuBLASLt int8 GEMM (torch._int_mm) throughput at 8192^3, TOP/s."""
    try:
        n = 8192
        a = torch.randint(-64, 64, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-64, 64, (n, n), dtype=torch.int8, device="cuda")
        torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = 1e9
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch._int_mm(a, b)
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except Exception:  # noqa: BLE001 - report the derived figure instead
        return None


def traffic_from_profiles(kernel: str, workload: str = "B8 S2048 H768"):
    """DRAM bytes per launch of `kernel` on the workload whose description
    contains `workload`, recorded from an ncu capture in profiles/traffic.md
    (table rows: | kernel | workload | bytes/launch | ...)."""
    f = ROOT / "profiles" / "traffic.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        cells = [c.strip() for c in line.strip().strip("|").split("|")]
        if len(cells) >= 3 and cells[0] == kernel and workload in cells[1]:
            try:
                return float(cells[2])
            except ValueError:
                return None
    return None


def cpu_baseline(threads_hint=None):
    """The oracle's TB-v1 model on the host cores, bounded sample: 1 of the 12
    layers at the full batch (tokens/s scaled by 1/12)."""
    from ltm_b200 import synthetic
    from oracle import oracle as orc
    orc.set_threads(threads_hint or host_threads())
    H, nh, F, Ms, V = WL["H"], WL["nh"], WL["F"], WL["Ms"], WL["vocab"]
    cfg = dict(H=H, F=F, nh=nh, dh=H // nh, Ms=Ms, scheme=orc.W8A8, dtype=orc.F16)
    w = synthetic.block_weights(H, F, Ms, 1000)
    emb = synthetic.embedding(V, H, 7)
    B, S = WL["B"], WL["S"]
    tok = synthetic.tokens(B, S, V, 3)
    t0 = time.perf_counter()
    orc.model_forward(cfg, [w], emb, tok, B, S)
    dt = time.perf_counter() - t0
    tps = B * S / dt / WL["layers"]
    return {"value": tps, "unit": "tokens/s", "cores": orc.num_threads(), "kind": "port",
            "sample": f"oracle TB-v1, 1 of {WL['layers']} layers, batch {B} x seq {S}, "
                      f"{dt:.1f} s; tokens/s scaled to {WL['layers']} layers"}


def run_tp(args, wl: dict = TP_WL, w4a16: bool = False, side: bool = False):
    """The tensor-parallel prefill: one block per rank (its head / FFN shard of
    one random-init block, built from the same seeded full weights on every
    rank) applied at each of the layers; the input hidden states are the full
    [B,S,H] on every rank.  Strong scaling: the job is fixed, N GPUs share it.
    With w4a16 the same driver runs the W4A16 long-context prefill.  Returns
    the result line on rank 0 (None elsewhere); side: no CPU baseline."""
    import datetime
    import torch
    import torch.distributed as dist
    import ltm_b200 as ltm
    from ltm_b200 import synthetic
    ws, rank, local = dist_env()
    assert ws == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {ws}"
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local)
    L = args.layers or wl["layers"]
    B, S, H, F, Ms, nh = (wl[k] for k in ("B", "S", "H", "F", "Ms", "nh"))
    comm = (ltm.Comm.from_process_group(local) if ws > 1 else
            ltm.Comm(ltm.comm_unique_id(), 1, 0, local))
    cfg = ltm.TitanBlockConfig(hidden_dim=H, ffn_dim=F, num_heads=nh, head_dim=H // nh,
                               memory_slots=Ms)
    q = ltm.QuantConfig(scheme=ltm.SCHEME_W4A16 if w4a16 else ltm.SCHEME_W8A8,
                        act_dtype=ltm.DTYPE_BF16)
    blk = ltm.TitanBlock(cfg, q, comm=comm)
    ovl_mode = {"auto": None, "on": True, "off": False}[args.overlap]
    blk.set_overlap(ovl_mode, args.comm_sms)
    if not w4a16:
        blk.set_tp_reduction(args.tp_reduce == "exact")
    overlapped = bool(ovl_mode) and not w4a16
    w = synthetic.block_weights(H, F, Ms, 1000)
    blk.load_weights(w)
    want_cpu = rank == 0 and ws == 1 and not args.no_cpu_baseline and not side
    if not want_cpu:
        del w
    gen = torch.Generator(device=dev).manual_seed(7)
    x = (torch.randn((B, S, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    # sequence parallelism: each rank holds its B*S/N consecutive rows of the
    # activations between layers (the rows of whole sequences when N divides B)
    sp = ws > 1 and not args.no_sp
    Tr = B * S // ws
    if sp:
        x = x.reshape(B * S, H)[rank * Tr:(rank + 1) * Tr].contiguous()
    bufs = (torch.empty_like(x), torch.empty_like(x))
    stream = torch.cuda.current_stream()

    def forward_all(inp):
        a = inp
        for i in range(L):
            o = bufs[i % 2]
            if sp:
                blk.forward_sp(a, B, S, out=o)
            else:
                blk.forward(a, out=o)
            a = o
        return a

    def barrier():
        if ws > 1:
            dist.barrier()

    args.warmup = max(args.warmup, 3)
    for _ in range(args.warmup):
        forward_all(x)
    torch.cuda.synchronize()
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(cvd.split(",")[local] if cvd else local)
    launches0 = ltm.launch_count()
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    evs = []
    for _ in range(args.steps):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record(stream)
        forward_all(x)
        e_.record(stream)
        evs.append((s_, e_))
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    launches = ltm.launch_count() - launches0
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs)], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    value = B * S * args.steps / (total_ms * 1e-3)

    # end to end: pinned H2D of the input hidden states (this rank's rows
    # under sequence parallelism), the layers, D2H of the last hidden state
    # of each sequence (that this rank holds)
    x_host = x.cpu().pin_memory()
    if sp:
        rows = torch.arange(rank * Tr, (rank + 1) * Tr, device=dev)
        last_idx = (rows[(rows + 1) % S == 0] - rank * Tr).contiguous()
    else:
        last_idx = torch.arange(S - 1, B * S, S, device=dev)
    last_host = torch.empty((last_idx.numel(), H), dtype=torch.bfloat16).pin_memory()
    barrier()
    e2e_evs = []
    for _ in range(args.steps):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record(stream)
        x.copy_(x_host, non_blocking=True)
        y = forward_all(x)
        last_host.copy_(y.reshape(-1, H).index_select(0, last_idx), non_blocking=True)
        e_.record(stream)
        e2e_evs.append((s_, e_))
    torch.cuda.synchronize()
    barrier()
    e2e_t = torch.tensor([sum(a.elapsed_time(b) for a, b in e2e_evs)], dtype=torch.float64,
                         device=dev)
    if ws > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = B * S * args.steps / (float(e2e_t.item()) * 1e-3)

    torch.cuda.synchronize()
    # per-kernel times of one more forward with the collectives on the
    # caller's stream (not overlapped), so they have times of their own
    blk.set_overlap(False, args.comm_sms)
    with ltm.KernelTimer() as kt:
        forward_all(x)
    blk.set_overlap(ovl_mode, args.comm_sms)
    kernels = {name: {"launches": n, "ms": round(ms, 4), "ms_per_launch": round(ms / n, 5)}
               for name, (n, ms) in kt.result.items()}
    comm_ms = sum(ms for name, (n, ms) in kt.result.items() if name.startswith("nccl"))
    all_ms = sum(ms for name, (n, ms) in kt.result.items())
    roofline = None
    if rank == 0 and not args.no_probe:
        work = step_work_tp(L, ws, wl, "gemm_f16_tc_kernel" if w4a16 else "w8a8_tc_kernel")
        roofline, i8 = roofline_of(kt.result, work, torch,
                                   "B4 S8192 H4096" if w4a16 else f"hidden-8192 tp{ws}")
        if i8:
            kernels["int8_peak_tops_measured"] = round(i8, 1)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4xbf16" if w4a16 else "int8",
            "data": "synthetic (hidden states N(0,0.02^2), weights N(0,0.02), random init)",
            "config": {"workload": W4_WORKLOAD_NAME if w4a16 else TP_WORKLOAD_NAME, "layers": L,
                       "global_batch": B,
                       "seq_len": S, "act_dtype": "bf16",
                       "parallelism": f"tp{ws}" + ("-sp" if sp else ""),
                       "tokens_per_s_per_gpu": round(value / ws, 1),
                       "comm_fraction_of_rank0_step": round(comm_ms / all_ms, 4) if all_ms else None,
                       "comm_fraction_note": "collectives' share of rank 0's step in a forward "
                                             "with them serialised on the compute stream (the "
                                             "timed steps overlap them with the GEMMs)"
                                             if (sp and overlapped) else None,
                       "comm_overlap": bool(sp and overlapped),
                       "tp_reduction": args.tp_reduce if sp else None,
                       "weights": "one random-init block's shard applied at every layer",
                       "l2": "inputs (1 GiB per activation tensor) larger than L2"},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(x_host.numel() * 2),
                    "d2h_bytes_per_step": int(last_host.numel() * 2),
                    "copies": "H2D of the input hidden states from pinned memory (per rank: "
                              "its rows under sequence parallelism, else all [B,S,H]); D2H of "
                              "each sequence's last output hidden state (what the next step "
                              "of a prefill needs); the rest of the output stays on the device"},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "roofline": roofline,
            "cpu_baseline": None,
            "kernels": kernels,
        }
    blk.close()
    comm.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and want_cpu:
        line["cpu_baseline"] = cpu_sample_block(wl, w4a16, w, L, samples=2)
    return line if rank == 0 else None


def cpu_sample_block(wl: dict, w4a16: bool, w: dict, layers: int, samples: int,
                     warmup: int = 0, tokens: int = 64):
    """The oracle's block forward on the host cores, bounded sample of a
    prefill workload: K_M | V_M of the bank made once (the per-forward cost of
    one layer, timed), then `samples` forwards of one sequence's first
    `tokens` tokens with those K_M | V_M (per-token cost, timed); the job's
    time is layers x (K_M|V_M time + B*S x per-token time).  The sample's
    causal self-attention spans `tokens` positions, fewer than the workload's
    sequence, so it under-counts the attention share of the per-token work.
    Returns the cpu_baseline entry plus the per-sample times."""
    import numpy as np
    from oracle import oracle as orc
    threads = host_threads()
    orc.set_threads(threads)
    B, S, H, F, Ms, nh = (wl[k] for k in ("B", "S", "H", "F", "Ms", "nh"))
    dt = orc.BF16
    ocfg = dict(H=H, F=F, nh=nh, dh=H // nh, Ms=Ms, scheme=orc.W4A16 if w4a16 else orc.W8A8,
                dtype=dt)
    pb = orc.PreparedBlock(ocfg, w)
    mem = orc.round_to(w["memory"], dt)
    t0 = time.perf_counter()
    kvm = pb.kvm(mem)
    t_kvm = time.perf_counter() - t0
    rng = np.random.default_rng(7)
    x = orc.round_to(rng.standard_normal((tokens, H), dtype=np.float32) * 0.02, dt)
    for _ in range(warmup):
        pb.forward(x, 1, tokens, mem, kvm)
    times = []
    for _ in range(max(samples, 1)):
        t0 = time.perf_counter()
        pb.forward(x, 1, tokens, mem, kvm)
        times.append(time.perf_counter() - t0)
    pb.close()
    per_tok = statistics.median(times) / tokens
    job_s = layers * (t_kvm + B * S * per_tok)
    return {"value": B * S / job_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"oracle TB-v1 block on {threads} host threads: K_M|V_M of the "
                      f"{Ms}-slot bank once ({t_kvm:.1f} s), then {len(times)} forwards of one "
                      f"sequence's first {tokens} tokens ({statistics.median(times):.2f} s "
                      f"each); job time = {layers} layers x (K_M|V_M + {B}x{S} tokens x "
                      f"per-token time); the sample's causal attention spans {tokens} positions",
            "per_sample_s": times, "kvm_s": t_kvm}


def host_threads() -> int:
    """Host cores this process may run on (torchrun sets OMP_NUM_THREADS=1
    for its workers; the CPU baselines use every core they are given)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # not Linux
        return os.cpu_count() or 1


def cpu_baseline_decode(wl: dict = DEC_WL, budget_s: float = 12.0):
    """The oracle's decode step on the host cores, bounded sample: 1 of the
    layers, 1 of the batch's sequences against the full cache; tokens/s scaled
    to the whole stack (quantized weights made once, outside the timing)."""
    import numpy as np
    from ltm_b200 import synthetic
    from oracle import oracle as orc
    H, nh, F, Ms, P = (wl[k] for k in ("H", "nh", "F", "Ms", "P"))
    ocfg = dict(H=H, F=F, nh=nh, dh=H // nh, Ms=Ms, scheme=orc.W4A16, dtype=orc.BF16,
                memory_write=1, use_attention_scores=1, update_rate=0.9)
    w = synthetic.block_weights(H, F, Ms, 1000)
    orc.set_threads(host_threads())
    pb = orc.PreparedBlock(ocfg, w)
    rng = np.random.default_rng(5)
    kc = orc.round_to(rng.standard_normal((1, nh, P, H // nh), dtype=np.float32), orc.BF16)
    vc = orc.round_to(rng.standard_normal((1, nh, P, H // nh), dtype=np.float32), orc.BF16)
    mem = orc.round_to(w["memory"], orc.BF16)
    kvm = orc.round_to(rng.standard_normal((Ms, 2 * H), dtype=np.float32) * 0.1, orc.BF16)
    x = orc.round_to(rng.standard_normal((1, H), dtype=np.float32) * 0.02, orc.BF16)
    n, t0 = 0, time.perf_counter()
    while n < 5 and (n == 0 or time.perf_counter() - t0 < budget_s):
        pb.decode_step(x, kc, vc, P - 1, mem, kvm)
        n += 1
    dt = (time.perf_counter() - t0) / n
    pb.close()
    return {"value": 1.0 / (dt * wl["layers"]), "unit": "tokens/s", "cores": orc.num_threads(),
            "kind": "port",
            "sample": f"oracle decode step, 1 of {wl['layers']} layers, 1 of {wl['B']} sequences "
                      f"against the full {P}-position cache, {n} steps of {dt:.2f} s; tokens/s "
                      f"scaled to {wl['layers']} layers"}


def run_decode(args, wl: dict = DEC_WL, side: bool = False):
    """The batched decode step: one block per layer (each its own copy of the
    same seeded weights, bank and resident K_M | V_M), one shared KV-cache
    buffer for all layers (per-layer caches would need 1.1 TB), every step at
    the cache's last position (the step rewrites it).  N > 1: independent
    replicas, one batch per GPU."""
    import datetime
    import torch
    import torch.distributed as dist
    import ltm_b200 as ltm
    from ltm_b200 import synthetic
    ws, rank, local = dist_env()
    assert ws == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {ws}"
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local)
    L = args.layers or wl["layers"]
    B, P, H, F, Ms, nh = (wl[k] for k in ("B", "P", "H", "F", "Ms", "nh"))
    cfg = ltm.TitanBlockConfig(hidden_dim=H, ffn_dim=F, num_heads=nh, head_dim=H // nh,
                               memory_slots=Ms)
    q = ltm.QuantConfig(scheme=ltm.SCHEME_W4A16, act_dtype=ltm.DTYPE_BF16, memory_write=True,
                        use_attention_scores=True)
    w = synthetic.block_weights(H, F, Ms, 1000)
    blocks = []
    for _ in range(L):
        b = ltm.TitanBlock(cfg, q, device=local)
        b.load_weights(w)
        blocks.append(b)
    del w
    cache = ltm.CacheManager(L, nh, H // nh, torch.bfloat16, device=local, shared_layers=True)
    cache.allocate(B, P)
    gen = torch.Generator(device=dev).manual_seed(11 + rank)
    for t in cache.get(0)[:2]:
        flat = t.view(-1)
        chunk = 1 << 28
        for i in range(0, flat.numel(), chunk):
            n = min(chunk, flat.numel() - i)
            flat[i:i + n] = torch.randn(n, generator=gen, device=dev).to(torch.bfloat16)
    pos = P - 1
    x = (torch.randn((B, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    bufs = (torch.empty_like(x), torch.empty_like(x))
    stream = torch.cuda.current_stream()

    def step(inp):
        a = inp
        for i, b in enumerate(blocks):
            kc, vc, _ = cache.get(i)
            o = bufs[i % 2]
            b.decode_step(a, kc, vc, pos, out=o)
            a = o
        return a

    def barrier():
        if ws > 1:
            dist.barrier()

    args.warmup = max(args.warmup, 3)
    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(cvd.split(",")[local] if cvd else local)
    launches0 = ltm.launch_count()
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    evs = []
    for _ in range(args.steps):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record(stream)
        step(x)
        e_.record(stream)
        evs.append((s_, e_))
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    launches = ltm.launch_count() - launches0
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs)], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    value = ws * B * args.steps / (total_ms * 1e-3)

    # end to end: pinned H2D of the step's input hidden states, the layers,
    # D2H of the step's output hidden states
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((B, H), dtype=torch.bfloat16).pin_memory()
    barrier()
    e2e_evs = []
    for _ in range(args.steps):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record(stream)
        x.copy_(x_host, non_blocking=True)
        y = step(x)
        y_host.copy_(y, non_blocking=True)
        e_.record(stream)
        e2e_evs.append((s_, e_))
    torch.cuda.synchronize()
    barrier()
    e2e_t = torch.tensor([sum(a.elapsed_time(b) for a, b in e2e_evs)], dtype=torch.float64,
                         device=dev)
    if ws > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = ws * B * args.steps / (float(e2e_t.item()) * 1e-3)

    torch.cuda.synchronize()
    with ltm.KernelTimer() as kt:
        step(x)
    kernels = {name: {"launches": n, "ms": round(ms, 4), "ms_per_launch": round(ms / n, 5)}
               for name, (n, ms) in kt.result.items()}
    lb = decode_layer_bytes(wl)
    pk, pk_src = peaks()
    step_ms = total_ms / args.steps
    roofline = None
    if rank == 0 and not args.no_probe:
        work = {"decode_attn_kernel": {"amount": lb["kv"] * L, "unit": "byte"}}
        roofline, _ = roofline_of(kt.result, work, torch, "decode B64 H4096")
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and not side:
        cpu = cpu_baseline_decode(wl)
    if rank == 0:
        step_gbs = lb["total"] * L / (step_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4xbf16",
            "data": "synthetic (KV cache N(0,1), hidden states N(0,0.02^2), weights N(0,0.02), "
                    "random init)",
            "config": {"workload": DEC_WORKLOAD_NAME, "layers": L, "global_batch": B * ws,
                       "kv_positions": P, "act_dtype": "bf16", "parallelism": f"replicas{ws}",
                       "tokens_per_s_per_gpu": round(value / ws, 2),
                       "step_bytes": lb["total"] * L,
                       "step_hbm_gbs": round(step_gbs, 1),
                       "step_hbm_frac": round(step_gbs / pk["hbm_gbs"], 4),
                       "kv_cache": "head-major [64, 32, 32768, 128] bf16 K and V, one pair shared "
                                   "by the layers (34.4 GB)",
                       "l2": "inputs (34 GB KV cache per layer) larger than L2"},
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(x_host.numel() * 2),
                    "d2h_bytes_per_step": int(y_host.numel() * 2)},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "kernels": kernels,
        }
        result = line
    for b in blocks:
        b.close()
    cache.clear()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result if rank == 0 else None


def probe_decode_case(torch, ltm):
    """One decode step of one hidden-4096 block at batch 64 against a
    2048-position cache (2.1 GB), after a warm-up step: every decode kernel
    launched once more at the workload's batch (GEMMs at M = 64; the cache
    kernel with the same tiles, 1/16 of the positions) for ncu."""
    from ltm_b200 import synthetic
    wl = dict(DEC_WL, P=2048)
    B, P, H, F, Ms, nh = (wl[k] for k in ("B", "P", "H", "F", "Ms", "nh"))
    cfg = ltm.TitanBlockConfig(hidden_dim=H, ffn_dim=F, num_heads=nh, head_dim=H // nh,
                               memory_slots=Ms)
    q = ltm.QuantConfig(scheme=ltm.SCHEME_W4A16, act_dtype=ltm.DTYPE_BF16, memory_write=True,
                        use_attention_scores=True)
    blk = ltm.TitanBlock(cfg, q)
    blk.load_weights(synthetic.block_weights(H, F, Ms, 1000))
    gen = torch.Generator(device="cuda").manual_seed(3)
    kc = torch.randn((B, nh, P, H // nh), generator=gen, device="cuda").to(torch.bfloat16)
    vc = torch.randn((B, nh, P, H // nh), generator=gen, device="cuda").to(torch.bfloat16)
    x = (torch.randn((B, H), generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    blk.decode_step(x, kc, vc, P - 1)
    blk.decode_step(x, kc, vc, P - 1)
    torch.cuda.synchronize()
    blk.close()


def run_ours(args, side: bool = False):
    import torch
    import torch.distributed as dist
    import ltm_b200 as ltm
    ws, rank, local = dist_env()
    assert ws == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {ws}"
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local)
    model = build_model(torch, ltm, args.layers, local)
    from ltm_b200 import synthetic
    B, S, H = WL["B"], WL["S"], WL["H"]
    tok_host = torch.from_numpy(synthetic.tokens(B, S, WL["vocab"], 100 + rank)).pin_memory()
    tok = tok_host.to(dev)
    out = torch.empty((B, S, H), dtype=torch.float16, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    args.warmup = max(args.warmup, 3)
    for _ in range(args.warmup):
        model.forward(tok, out)
    torch.cuda.synchronize()

    def barrier():
        if ws > 1:
            dist.barrier()

    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(cvd.split(",")[local] if cvd else local)
    launches0 = ltm.launch_count()
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    evs = []
    for _ in range(args.steps):
        flush.fill_(0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        model.forward(tok, out)
        e.record(stream)
        evs.append((s, e))
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    launches = ltm.launch_count() - launches0
    my_ms = sum(s.elapsed_time(e) for s, e in evs)
    t = torch.tensor([my_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    tokens = ws * B * S * args.steps
    value = tokens / (total_ms * 1e-3)

    # end to end through the public API: pinned H2D of the tokens, forward,
    # D2H of each sequence's last hidden state (the prefill result)
    last_host = torch.empty((B, H), dtype=torch.float16).pin_memory()
    model.forward(tok, out)
    torch.cuda.synchronize()
    barrier()
    e2e_evs = []
    for _ in range(args.steps):
        flush.fill_(0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        tok.copy_(tok_host, non_blocking=True)
        model.forward(tok, out)
        last_host.copy_(out[:, -1, :], non_blocking=True)
        e.record(stream)
        e2e_evs.append((s, e))
    torch.cuda.synchronize()
    barrier()
    e2e_ms = torch.tensor([sum(s.elapsed_time(e) for s, e in e2e_evs)], dtype=torch.float64,
                          device=dev)
    if ws > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = tokens / (float(e2e_ms.item()) * 1e-3)

    # per-kernel device time of one more (untimed) forward, measured inside the
    # library with CUDA events on the launching stream
    flush.fill_(0)
    torch.cuda.synchronize()
    with ltm.KernelTimer() as kt:
        model.forward(tok, out)
    kernels = {name: {"launches": n, "ms": round(ms, 4), "ms_per_launch": round(ms / n, 5)}
               for name, (n, ms) in kt.result.items()}
    roofline = None
    if rank == 0 and not args.no_probe:
        roofline, i8 = roofline_of(kt.result, step_work(args.layers), torch)
        if i8:
            kernels["int8_peak_tops_measured"] = round(i8, 1)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and not side:
        cpu = cpu_baseline()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded tokens U[0,32000), weights N(0,0.02), random init)",
            "config": {"workload": WORKLOAD_NAME, "layers": args.layers, "global_batch": B * ws,
                       "seq_len": S, "act_dtype": "f16", "parallelism": f"replicas{ws}",
                       "tokens_per_s_per_gpu": round(value / ws, 1),
                       "l2": "flushed between timed steps (256 MiB write), per-step CUDA events"},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(tok_host.numel() * 4),
                    "d2h_bytes_per_step": int(last_host.numel() * 2)},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "kernels": kernels,
        }
        result = line
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    model.close()
    return result if rank == 0 else None


# ---------------------------------------------------------- reference path --
def run_reference(args):
    """The reference arm: the CPU restatement of the reference's algorithm
    (the oracle; the reference's own CUDA sources do not compile) timed on all
    host cores the process may use, for the same workload, metric and unit as
    our arm.  Each timed step is one bounded sample of the workload; the line's
    value is the whole job's tokens/s extrapolated from the samples.  Under
    torchrun only rank 0 runs."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    from ltm_b200 import synthetic
    from oracle import oracle as orc
    threads = host_threads()
    orc.set_threads(threads)
    base = {"metric": METRIC, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
            "impl": "reference",
            "note": "the reference's CUDA sources do not compile; this arm times the CPU "
                    "restatement of its algorithm (oracle/) on all host cores"}
    if args.config in ("tp", "w4a16"):
        w4 = args.config == "w4a16"
        wl = W4_WL if w4 else TP_WL
        L = args.layers or wl["layers"]
        w = synthetic.block_weights(wl["H"], wl["F"], wl["Ms"], 1000)
        cpu = cpu_sample_block(wl, w4, w, L, samples=args.steps, warmup=args.warmup)
        step_s = statistics.median(cpu.pop("per_sample_s"))
        cpu.pop("kvm_s")
        line = dict(base, value=round(cpu["value"], 3), ms_per_step=round(step_s * 1e3, 2),
                    scaling="strong", dtype="int4xbf16" if w4 else "int8",
                    data="synthetic (hidden states N(0,0.02^2), weights N(0,0.02), random init)",
                    config={"workload": W4_WORKLOAD_NAME if w4 else TP_WORKLOAD_NAME,
                            "layers": L, "global_batch": wl["B"], "seq_len": wl["S"],
                            "act_dtype": "bf16", "parallelism": "host cores",
                            "same_config": False,
                            "sampling": "each timed step: 1 layer, one sequence's first 64 "
                                        "tokens with K_M|V_M made once; the job's tokens/s "
                                        "extrapolated (see cpu_baseline.sample)"})
    elif args.config == "decode":
        cpu = cpu_baseline_decode(DEC_WL)
        line = dict(base, value=round(cpu["value"], 4), ms_per_step=None, scaling="weak",
                    dtype="int4xbf16",
                    data="synthetic (KV cache N(0,1), hidden states N(0,0.02^2), weights "
                         "N(0,0.02), random init)",
                    config={"workload": DEC_WORKLOAD_NAME, "layers": DEC_WL["layers"],
                            "global_batch": DEC_WL["B"], "kv_positions": DEC_WL["P"],
                            "act_dtype": "bf16", "parallelism": "host cores",
                            "same_config": False,
                            "sampling": "1 layer, 1 sequence per sample (see "
                                        "cpu_baseline.sample)"})
    else:
        H, nh, F, Ms, V = WL["H"], WL["nh"], WL["F"], WL["Ms"], WL["vocab"]
        cfg = dict(H=H, F=F, nh=nh, dh=H // nh, Ms=Ms, scheme=orc.W8A8, dtype=orc.F16)
        w = synthetic.block_weights(H, F, Ms, 1000)
        emb = synthetic.embedding(V, H, 7)
        Bs, S = 1, WL["S"]  # each step: 1 layer of 12, one sequence of the batch
        tok = synthetic.tokens(Bs, S, V, 3)
        for _ in range(args.warmup):
            orc.model_forward(cfg, [w], emb, tok, Bs, S)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            orc.model_forward(cfg, [w], emb, tok, Bs, S)
        dt = time.perf_counter() - t0
        value = args.steps * Bs * S / dt / WL["layers"]
        cpu = {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"each step: 1 of {WL['layers']} layers, 1 sequence of {S} tokens; "
                         f"tokens/s scaled to {WL['layers']} layers"}
        line = dict(base, value=round(value, 2), ms_per_step=round(dt / args.steps * 1e3, 2),
                    scaling="weak", dtype="int8",
                    data="synthetic (seeded tokens U[0,32000), weights N(0,0.02), random init)",
                    config={"workload": WORKLOAD_NAME, "layers": WL["layers"],
                            "global_batch": WL["B"], "seq_len": S, "act_dtype": "f16",
                            "parallelism": "host cores", "same_config": False,
                            "sampling": "each step: 1 of 12 layers, 1 of 8 sequences"})
    cpu["value"] = line["value"]
    line["cpu_baseline"] = cpu
    line["e2e"] = {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}
    emit(line)


def run_side_workloads(args) -> dict:
    """At N = 1, after the headline: the other single-GPU workloads, each
    measured like the headline (device-timed value, e2e, roofline of its
    dominant kernel class, clocks) with fewer steps and no CPU baseline."""
    import gc
    import torch
    side = {}
    steps = max(3, min(args.steps, 10))
    plans = [("prefill_12layer_w8a8", lambda a: run_ours(a, side=True)),
             ("prefill_4layer_w4a16_long_context", lambda a: run_tp(a, W4_WL, True, side=True)),
             ("decode_32layer_w4a16", lambda a: run_decode(a, side=True))]
    for name, fn in plans:
        a = argparse.Namespace(**vars(args))
        a.steps, a.warmup = steps, 3
        a.layers = WL["layers"] if name.startswith("prefill_12") else None
        try:
            line = fn(a)
            keep = ("value", "unit", "ms_per_step", "steps", "warmup", "dtype", "config", "e2e",
                    "roofline", "clocks", "gpu_launches", "scaling")
            side[name] = {k: line.get(k) for k in keep}
        except Exception as e:  # noqa: BLE001 - a side workload must not lose the headline
            side[name] = {"error": f"{type(e).__name__}: {e}"}
        gc.collect()
        torch.cuda.empty_cache()
    return side


_JSON_FD = 1


def emit(line: dict) -> None:
    """Writes the result line to the process's original stdout."""
    os.write(_JSON_FD, (json.dumps(line) + "\n").encode())


def main():
    global _JSON_FD
    args = parse()
    # stdout carries exactly one JSON line: everything else written to file
    # descriptor 1 (libraries' banners, e.g. NCCL's version line) goes to stderr
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    if args.ncu_case:
        import torch
        import ltm_b200 as ltm
        if args.ncu_case == "tp":
            probe_tp_case(torch, ltm)
        elif args.ncu_case == "tplayer":
            probe_tp_layer_case(torch, ltm)
        elif args.ncu_case == "w4a16":
            probe_w4a16_case(torch, ltm)
        elif args.ncu_case == "decode":
            probe_decode_case(torch, ltm)
        else:
            probe_kernels(torch, ltm, timed=False)
        emit({"ncu_case": "done", "device_error": ltm.device_error()})
        return
    if args.impl == "reference":
        run_reference(args)
        return
    if args.config == "tp":
        line = run_tp(args)
    elif args.config == "w4a16":
        line = run_tp(args, W4_WL, w4a16=True)
    elif args.config == "decode":
        line = run_decode(args)
    else:
        if args.layers is None:
            args.layers = WL["layers"]
        line = run_ours(args)
    if line is None:
        return
    if args.config == "tp" and args.gpus == 1 and not args.no_side:
        line["side_workloads"] = run_side_workloads(args)
    emit(line)


if __name__ == "__main__":
    main()
