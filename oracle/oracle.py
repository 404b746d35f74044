"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates the reference's per-op formulas on the CPU
(tb_oracle.cpp cites the reference file:line of each).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module,
and only to check or time against it; the product never calls it.
Parity is unpinned by the reference (it ships no tests/fixtures and does not
compile); the committed golden fixtures pin this oracle instead.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
F32, F16, BF16 = 0, 1, 2
ACT_NONE, ACT_GELU, ACT_SIGMOID = 0, 1, 2
W8A32, W8A8, W4A16 = 0, 1, 2

_lib = None


def lib():
    global _lib
    if _lib is None:
        from oracle.build import build  # noqa: WPS433
        _lib = C.CDLL(str(build()))
        _declare(_lib)
    return _lib


def _p(t):
    return C.POINTER(t)


class OrcBlockCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("H", "F", "nh", "dh", "Ms", "scheme", "dtype", "use_rotary",
                                       "use_bias", "use_layer_norm", "use_memory_gating",
                                       "memory_write", "use_attention_scores")] + [
        ("update_rate", C.c_float)]


WEIGHT_FIELDS = ("w_qkv", "b_qkv", "w_o", "b_o", "w_qm", "b_qm", "w_km", "b_km", "w_vm", "b_vm",
                 "w_om", "b_om", "w_g", "b_g", "w_1", "b_1", "w_2", "b_2", "ln1_g", "ln1_b",
                 "ln2_g", "ln2_b", "memory")


class OrcBlockWeights(C.Structure):
    _fields_ = [(n, _p(C.c_float)) for n in WEIGHT_FIELDS]


def _declare(L):
    f, i8, u8, i32 = _p(C.c_float), _p(C.c_int8), _p(C.c_uint8), _p(C.c_int32)
    i64, ci = C.c_int64, C.c_int
    sig = {
        "orc_num_threads": ([], ci),
        "orc_set_num_threads": ([ci], None),
        "orc_round": ([f, i64, ci], None),
        "orc_quant_int8_rows": ([f, i64, i64, i8, f], None),
        "orc_dequant_int8_rows": ([i8, f, i64, i64, ci, f], None),
        "orc_quant_int4_g128": ([f, i64, i64, u8, f, u8], None),
        "orc_dequant_int4_g128": ([u8, f, u8, i64, i64, ci, f], None),
        "orc_gemm_i8": ([i8, i8, i64, i64, i64, i32], None),
        "orc_linear_w8a8": ([i8, f, i8, f, f, ci, i64, i64, i64, f], None),
        "orc_linear_w8a32": ([f, i8, f, f, ci, i64, i64, i64, f], None),
        "orc_linear_w4a16": ([f, u8, f, u8, f, ci, i64, i64, i64, ci, f], None),
        "orc_layernorm_x2": ([f, i64, i64, f, f, f], None),
        "orc_rope_table": ([ci, ci, f], None),
        "orc_attention": ([f, i64, f, f, i64, ci, ci, ci, ci, ci, ci, ci, ci, f, i64], None),
        "orc_memory_store": ([f, f, i64, f, i64, i64, f, ci, ci, ci, C.c_float, ci, ci], None),
        "orc_activation": ([f, i64, ci, f], None),
        "orc_calib_minmax": ([f, i64, f, f], None),
        "orc_calib_percentile": ([f, i64, C.c_float, f, f], None),
        "orc_calib_mse_error": ([f, i64, C.c_float], C.c_double),
        "orc_calib_mse": ([f, i64, f, f], None),
        "orc_quant_int8_static": ([f, i64, C.c_float, i8], None),
        "orc_ema_rows": ([f, ci, i64, f, f, ci], None),
        "orc_block_forward": ([_p(OrcBlockCfg), _p(OrcBlockWeights), f, f, f, ci, ci], ci),
        "orc_block_forward_kv": ([_p(OrcBlockCfg), _p(OrcBlockWeights), f, f, f, ci, ci, f], ci),
        "orc_block_kvm": ([_p(OrcBlockCfg), _p(OrcBlockWeights), f, f], ci),
        "orc_block_decode_step": ([_p(OrcBlockCfg), _p(OrcBlockWeights), f, f, f, f, f, i64, ci,
                                   ci, f], ci),
        "orc_block_prepare": ([_p(OrcBlockCfg), _p(OrcBlockWeights)], C.c_void_p),
        "orc_block_release": ([C.c_void_p], None),
        "orc_block_forward_prepared": ([C.c_void_p, _p(OrcBlockCfg), _p(OrcBlockWeights), f, f,
                                        f, f, ci, ci], ci),
        "orc_block_kvm_prepared": ([C.c_void_p, _p(OrcBlockCfg), f, f], ci),
        "orc_block_decode_step_prepared": ([C.c_void_p, _p(OrcBlockCfg), _p(OrcBlockWeights), f, f,
                                            f, f, f, i64, ci, ci, f], ci),
        "orc_model_forward": ([_p(OrcBlockCfg), _p(OrcBlockWeights), _p(f), ci, f, ci, i32, f, ci,
                               ci], ci),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


def _ptr(a, t=C.c_float):
    return a.ctypes.data_as(C.POINTER(t)) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


def round_to(x, dtype: int) -> np.ndarray:
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().orc_round(_ptr(x), x.size, dtype)
    return x


def quant_int8_rows(x):
    x = _f32(x)
    rows, K = x.shape
    q = np.empty((rows, K), np.int8)
    s = np.empty(rows, np.float32)
    lib().orc_quant_int8_rows(_ptr(x), rows, K, _ptr(q, C.c_int8), _ptr(s))
    return q, s


def dequant_int8_rows(q, s, dtype=F32):
    q = np.ascontiguousarray(q, np.int8)
    s = _f32(s)
    out = np.empty(q.shape, np.float32)
    lib().orc_dequant_int8_rows(_ptr(q, C.c_int8), _ptr(s), q.shape[0], q.shape[1], dtype, _ptr(out))
    return out


def quant_int4_g128(w):
    w = _f32(w)
    N, K = w.shape
    packed = np.empty((N, K // 2), np.uint8)
    s = np.empty((N, K // 128), np.float32)
    zp = np.empty((N, K // 128), np.uint8)
    lib().orc_quant_int4_g128(_ptr(w), N, K, _ptr(packed, C.c_uint8), _ptr(s), _ptr(zp, C.c_uint8))
    return packed, s, zp


def dequant_int4_g128(packed, s, zp, dtype=F32):
    packed = np.ascontiguousarray(packed, np.uint8)
    N, K = packed.shape[0], packed.shape[1] * 2
    out = np.empty((N, K), np.float32)
    lib().orc_dequant_int4_g128(_ptr(packed, C.c_uint8), _ptr(_f32(s)),
                                _ptr(np.ascontiguousarray(zp, np.uint8), C.c_uint8), N, K, dtype,
                                _ptr(out))
    return out


def gemm_i8(qa, qw):
    qa = np.ascontiguousarray(qa, np.int8)
    qw = np.ascontiguousarray(qw, np.int8)
    M, K = qa.shape
    N = qw.shape[0]
    acc = np.empty((M, N), np.int32)
    lib().orc_gemm_i8(_ptr(qa, C.c_int8), _ptr(qw, C.c_int8), M, N, K, _ptr(acc, C.c_int32))
    return acc


def linear_w8a8(qa, sa, qw, sw, bias=None, act=ACT_NONE):
    qa = np.ascontiguousarray(qa, np.int8)
    qw = np.ascontiguousarray(qw, np.int8)
    M, K = qa.shape
    N = qw.shape[0]
    y = np.empty((M, N), np.float32)
    sa = None if sa is None else _f32(sa)
    bias = None if bias is None else _f32(bias)
    lib().orc_linear_w8a8(_ptr(qa, C.c_int8), _ptr(sa), _ptr(qw, C.c_int8), _ptr(_f32(sw)),
                          _ptr(bias), act, M, N, K, _ptr(y))
    return y


def linear_w8a32(a, qw, sw, bias=None, act=ACT_NONE):
    a = _f32(a)
    qw = np.ascontiguousarray(qw, np.int8)
    M, K = a.shape
    N = qw.shape[0]
    y = np.empty((M, N), np.float32)
    bias = None if bias is None else _f32(bias)
    lib().orc_linear_w8a32(_ptr(a), _ptr(qw, C.c_int8), _ptr(_f32(sw)), _ptr(bias), act, M, N, K,
                           _ptr(y))
    return y


def linear_w4a16(a, packed, s, zp, bias=None, act=ACT_NONE, wdtype=BF16):
    a = _f32(a)
    packed = np.ascontiguousarray(packed, np.uint8)
    M, K = a.shape
    N = packed.shape[0]
    y = np.empty((M, N), np.float32)
    bias = None if bias is None else _f32(bias)
    lib().orc_linear_w4a16(_ptr(a), _ptr(packed, C.c_uint8), _ptr(_f32(s)),
                           _ptr(np.ascontiguousarray(zp, np.uint8), C.c_uint8), _ptr(bias), act, M,
                           N, K, wdtype, _ptr(y))
    return y


def layernorm_x2(x, g, b):
    x = _f32(x)
    rows, H = x.shape
    y = np.empty_like(x)
    lib().orc_layernorm_x2(_ptr(x), rows, H, _ptr(_f32(g)), _ptr(_f32(b)), _ptr(y))
    return y


def rope_table(S: int, dh: int) -> np.ndarray:
    tab = np.empty((S, dh // 2, 2), np.float32)
    lib().orc_rope_table(S, dh, _ptr(tab))
    return tab


def attention(q, k, v, B, Sq, Skv, nh, dh, causal, dtype, kv_shared=False):
    """q: [B*Sq, nh*dh]; k, v: [B*Skv, nh*dh] (or [Skv, nh*dh] when kv_shared)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty((B * Sq, nh * dh), np.float32)
    lib().orc_attention(_ptr(q), q.shape[1], _ptr(k), _ptr(v), k.shape[1], B, Sq, Skv,
                        0 if kv_shared else Skv, nh, dh, int(causal), dtype, _ptr(out), nh * dh)
    return out


def calibrate(x, method: str, percentile: float = 99.9):
    """(min, max) of the MinMax / Percentile / MSE calibrators over x."""
    x = _f32(x).reshape(-1)
    lo, hi = C.c_float(), C.c_float()
    if method == "minmax":
        lib().orc_calib_minmax(_ptr(x), x.size, C.byref(lo), C.byref(hi))
    elif method == "percentile":
        lib().orc_calib_percentile(_ptr(x), x.size, percentile, C.byref(lo), C.byref(hi))
    elif method == "mse":
        lib().orc_calib_mse(_ptr(x), x.size, C.byref(lo), C.byref(hi))
    else:
        raise ValueError(method)
    return lo.value, hi.value


def calib_mse_error(x, clip: float) -> float:
    x = _f32(x).reshape(-1)
    return float(lib().orc_calib_mse_error(_ptr(x), x.size, clip))


def quant_int8_static(x, scale: float):
    x = _f32(x)
    q = np.empty(x.shape, np.int8)
    lib().orc_quant_int8_static(_ptr(x), x.size, scale, _ptr(q, C.c_int8))
    return q


def activation(x, act: int):
    """act(x) elementwise in fp32 (GELU-tanh or sigmoid)."""
    x = _f32(x)
    y = np.empty_like(x)
    lib().orc_activation(_ptr(x), x.size, act, _ptr(y))
    return y


def ema_rows(rows, v, w, dtype: int):
    """rows [Ms, n] (updated copy returned): (1 - w[s]) rows[s] + w[s] v, rounded."""
    rows = np.array(rows, dtype=np.float32, copy=True, order="C")
    lib().orc_ema_rows(_ptr(rows), rows.shape[0], rows.shape[1], _ptr(_f32(v)), _ptr(_f32(w)),
                       dtype)
    return rows


def memory_store(memory, keys, queries, state, nh: int, rate: float, use_scores: bool, dtype: int):
    """memory [Ms,H] (returned updated copy); keys [Ms, >=H]; queries [T, >=H]; state [H]."""
    mem = np.array(memory, dtype=np.float32, copy=True, order="C")
    keys, queries, state = _f32(keys), _f32(queries), _f32(state)
    Ms, H = mem.shape
    lib().orc_memory_store(_ptr(mem), _ptr(keys), keys.shape[1], _ptr(queries), queries.shape[1],
                           queries.shape[0], _ptr(state), Ms, H, nh, rate, int(use_scores), dtype)
    return mem


def _cfg(c: dict) -> OrcBlockCfg:
    return OrcBlockCfg(c["H"], c["F"], c["nh"], c["dh"], c["Ms"], c["scheme"], c["dtype"],
                       int(c.get("use_rotary", 1)), int(c.get("use_bias", 1)),
                       int(c.get("use_layer_norm", 1)), int(c.get("use_memory_gating", 1)),
                       int(c.get("memory_write", 0)), int(c.get("use_attention_scores", 1)),
                       float(c.get("update_rate", 0.9)))


def _weights(w: dict):
    keep = {n: _f32(w[n]) for n in WEIGHT_FIELDS if w.get(n) is not None}
    st = OrcBlockWeights(*[_ptr(keep[n]) if n in keep else None for n in WEIGHT_FIELDS])
    return st, keep


def block_forward(cfg: dict, w: dict, x, B: int, S: int, memory=None, return_kv=False):
    """TB-v1 block forward. Returns (y [B*S,H], memory after the optional write)
    and, with return_kv, the post-RoPE K | V rows [B*S, 2H] as a third item."""
    c = _cfg(cfg)
    st, keep = _weights(w)
    mem = round_to(w["memory"] if memory is None else memory, cfg["dtype"])
    x = _f32(x)
    y = np.empty_like(x)
    kv = np.empty((x.shape[0], 2 * cfg["H"]), np.float32) if return_kv else None
    r = lib().orc_block_forward_kv(C.byref(c), C.byref(st), _ptr(mem), _ptr(x), _ptr(y), B, S,
                                   _ptr(kv))
    if r != 0:
        raise RuntimeError(f"orc_block_forward failed ({r})")
    return (y, mem, kv) if return_kv else (y, mem)


def block_kvm(cfg: dict, w: dict, memory=None):
    """K_M | V_M [Ms, 2H] of a bank (the block's weights' bank by default)."""
    c = _cfg(cfg)
    st, keep = _weights(w)
    mem = round_to(w["memory"] if memory is None else memory, cfg["dtype"])
    out = np.empty((cfg["Ms"], 2 * cfg["H"]), np.float32)
    r = lib().orc_block_kvm(C.byref(c), C.byref(st), _ptr(mem), _ptr(out))
    if r != 0:
        raise RuntimeError(f"orc_block_kvm failed ({r})")
    return out


def block_decode_step(cfg: dict, w: dict, x, k_cache, v_cache, cache_len: int, memory, kvm):
    """One decode step (x [B, H], every sequence at position cache_len).
    k_cache, v_cache: float32 [B, nh, P, dh] (head-major); memory [Ms, H];
    kvm [Ms, 2H] -- all updated in place.  Returns y [B, H]."""
    c = _cfg(cfg)
    st, keep = _weights(w)
    x = _f32(x)
    B = x.shape[0]
    for a in (k_cache, v_cache, memory, kvm):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    P = k_cache.shape[2]
    y = np.empty_like(x)
    r = lib().orc_block_decode_step(C.byref(c), C.byref(st), _ptr(memory), _ptr(kvm), _ptr(x),
                                    _ptr(k_cache), _ptr(v_cache), P, cache_len, B, _ptr(y))
    if r != 0:
        raise RuntimeError(f"orc_block_decode_step failed ({r})")
    return y


class PreparedBlock:
    """A block whose quantized linears are made once, for repeated decode
    steps (same arithmetic as block_decode_step)."""

    def __init__(self, cfg: dict, w: dict):
        self.c = _cfg(cfg)
        self.st, self._keep = _weights(w)
        self.h = lib().orc_block_prepare(C.byref(self.c), C.byref(self.st))

    def decode_step(self, x, k_cache, v_cache, cache_len: int, memory, kvm):
        x = _f32(x)
        for a in (k_cache, v_cache, memory, kvm):
            assert a.dtype == np.float32 and a.flags.c_contiguous
        y = np.empty_like(x)
        r = lib().orc_block_decode_step_prepared(self.h, C.byref(self.c), C.byref(self.st),
                                                 _ptr(memory), _ptr(kvm), _ptr(x), _ptr(k_cache),
                                                 _ptr(v_cache), k_cache.shape[2], cache_len,
                                                 x.shape[0], _ptr(y))
        if r != 0:
            raise RuntimeError(f"orc_block_decode_step failed ({r})")
        return y

    def kvm(self, memory):
        """K_M | V_M [Ms, 2H] of a bank (rounded to the block's dtype)."""
        memory = _f32(memory)
        out = np.empty((memory.shape[0], 2 * memory.shape[1]), np.float32)
        r = lib().orc_block_kvm_prepared(self.h, C.byref(self.c), _ptr(memory), _ptr(out))
        if r != 0:
            raise RuntimeError(f"orc_block_kvm failed ({r})")
        return out

    def forward(self, x, B: int, S: int, memory, kvm=None):
        """Block forward with the prepared linears; kvm (K_M | V_M of the bank)
        is used as given when passed.  memory is updated in place when the
        block writes."""
        x = _f32(x)
        assert memory.dtype == np.float32 and memory.flags.c_contiguous
        y = np.empty_like(x)
        r = lib().orc_block_forward_prepared(self.h, C.byref(self.c), C.byref(self.st),
                                             _ptr(memory), _ptr(None if kvm is None else _f32(kvm)),
                                             _ptr(x), _ptr(y), B, S)
        if r != 0:
            raise RuntimeError(f"orc_block_forward_prepared failed ({r})")
        return y

    def close(self):
        if self.h:
            lib().orc_block_release(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def model_forward(cfg: dict, layers: list, embedding, tokens, B: int, S: int):
    c = _cfg(cfg)
    n = len(layers)
    sts, keeps, banks = [], [], []
    for w in layers:
        st, keep = _weights(w)
        sts.append(st)
        keeps.append(keep)
        banks.append(round_to(w["memory"], cfg["dtype"]))
    arr = (OrcBlockWeights * n)(*sts)
    bank_ptrs = (C.POINTER(C.c_float) * n)(*[_ptr(b) for b in banks])
    emb = _f32(embedding)
    tok = np.ascontiguousarray(tokens, np.int32).reshape(-1)
    y = np.empty((B * S, cfg["H"]), np.float32)
    r = lib().orc_model_forward(C.byref(c), arr, bank_ptrs, n, _ptr(emb), emb.shape[0],
                                _ptr(tok, C.c_int32), _ptr(y), B, S)
    if r != 0:
        raise RuntimeError(f"orc_model_forward failed ({r})")
    return y
