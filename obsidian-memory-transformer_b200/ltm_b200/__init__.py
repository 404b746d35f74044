"""Python caller of the B200 Titan-block C ABI (libltm_b200.so).

This module plays the role the reference's pybind module `_ltm`
(python_bindings/src/main.cpp:206-269) plays for its C++ library: it exposes
`TitanBlockConfig` with the same fields and defaults, a `TitanBlock` /
`TitanModel` pair, and the INT8/INT4 quantize, dequantize and quantized
linear entry points.  Every call goes through the C ABI declared in
include/ltm_b200.h; PyTorch only provides device memory and streams.
There is no CPU fallback: without the built library every call raises.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libltm_b200.so"

# ltm_status
OK, ERR_INVALID_ARG, ERR_CUDA, ERR_COMM, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_NO_DEVICE = range(7)
# ltm_dtype
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
# ltm_epilogue
EPI_NONE, EPI_GELU, EPI_SIGMOID = 0, 1, 2
# ltm_scheme
SCHEME_W8A32, SCHEME_W8A8, SCHEME_W4A16 = 0, 1, 2
# ltm_tp_reduction
TP_REDUCE_ACT, TP_REDUCE_EXACT = 0, 1


class LtmError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"ltm_b200 status {status}: {msg}")
        self.status = status


_lib = None


class BlockConfigC(C.Structure):
    _fields_ = [
        ("hidden_dim", C.c_int), ("ffn_dim", C.c_int), ("num_heads", C.c_int),
        ("head_dim", C.c_int), ("memory_slots", C.c_int), ("memory_dim", C.c_int),
        ("memory_update_rate", C.c_float), ("use_memory_compression", C.c_int),
        ("memory_compression_ratio", C.c_float), ("use_flash_attention", C.c_int),
        ("use_alibi", C.c_int), ("use_rotary", C.c_int), ("dropout_prob", C.c_float),
        ("use_parallel_attention", C.c_int), ("use_memory_gating", C.c_int),
        ("use_layer_norm", C.c_int), ("use_bias", C.c_int), ("fuse_operations", C.c_int),
        ("learn_memory", C.c_int), ("learn_compression", C.c_int),
        ("gradient_checkpointing", C.c_int),
    ]


class QuantConfigC(C.Structure):
    _fields_ = [("scheme", C.c_int), ("group_size", C.c_int), ("act_dtype", C.c_int),
                ("memory_write", C.c_int), ("use_attention_scores", C.c_int)]


WEIGHT_FIELDS = ("w_qkv", "b_qkv", "w_o", "b_o", "w_qm", "b_qm", "w_km", "b_km", "w_vm", "b_vm",
                 "w_om", "b_om", "w_g", "b_g", "w_1", "b_1", "w_2", "b_2", "ln1_g", "ln1_b",
                 "ln2_g", "ln2_b", "memory")


class BlockWeightsC(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_float)) for n in WEIGHT_FIELDS]


def _declare(L):
    vp, i64, ci = C.c_void_p, C.c_int64, C.c_int
    sig = {
        "ltm_version": ([], C.c_char_p),
        "ltm_last_error_string": ([], C.c_char_p),
        "ltm_device_error": ([C.POINTER(C.c_int)], ci),
        "ltm_launch_count": ([C.POINTER(C.c_uint64)], ci),
        "ltm_device_alloc_count": ([C.POINTER(C.c_uint64)], ci),
        "ltm_kernel_timer_begin": ([vp], ci),
        "ltm_kernel_timer_end": ([C.c_char_p, C.c_size_t], ci),
        "ltm_quantize_int8_per_channel": ([vp, ci, i64, i64, vp, vp, vp], ci),
        "ltm_dequantize_int8_per_channel": ([vp, vp, i64, i64, vp, ci, vp], ci),
        "ltm_quantize_act_int8_per_token": ([vp, ci, i64, i64, vp, vp, vp], ci),
        "ltm_quantize_int4_grouped": ([vp, ci, i64, i64, ci, vp, vp, vp, vp], ci),
        "ltm_dequantize_int4_grouped": ([vp, vp, vp, i64, i64, ci, vp, ci, vp], ci),
        "ltm_linear_w8a8": ([vp, vp, vp, vp, vp, ci, vp, ci, i64, i64, i64, vp], ci),
        "ltm_linear_w8a8_acc_i32": ([vp, vp, vp, i64, i64, i64, vp], ci),
        "ltm_linear_w4a16": ([vp, ci, vp, vp, vp, vp, ci, vp, i64, i64, i64, vp], ci),
        "ltm_linear_w8a32": ([vp, vp, vp, vp, ci, vp, i64, i64, i64, vp], ci),
        "ltm_layernorm_residual": ([vp, vp, vp, vp, vp, ci, i64, i64, vp], ci),
        "ltm_attention_forward": ([vp, i64, vp, i64, vp, i64, vp, i64, ci, ci, ci, i64, ci, ci, ci,
                                   ci, vp], ci),
        "ltm_memory_store": ([vp, vp, i64, vp, i64, i64, vp, ci, ci, ci, C.c_float, ci, ci, vp], ci),
        "ltm_memory_store_noalloc": ([vp, vp, i64, vp, i64, i64, vp, ci, ci, ci, C.c_float, ci,
                                      ci, vp], ci),
        "ltm_block_config_default": ([C.POINTER(BlockConfigC)], None),
        "ltm_block_create": ([C.POINTER(BlockConfigC), C.POINTER(QuantConfigC), ci,
                              C.POINTER(vp)], ci),
        "ltm_block_load_weights": ([vp, C.POINTER(BlockWeightsC)], ci),
        "ltm_block_forward": ([vp, vp, vp, vp, ci, ci, vp], ci),
        "ltm_block_get_memory": ([vp, vp, vp], ci),
        "ltm_block_intermediate": ([vp, C.c_char_p, vp, vp, C.POINTER(i64), C.POINTER(i64),
                                    C.POINTER(ci)], ci),
        "ltm_block_decode_step": ([vp, vp, vp, vp, vp, i64, ci, ci, vp], ci),
        "ltm_block_memory_write": ([vp, vp, vp, i64, i64, vp], ci),
        "ltm_block_destroy": ([vp], ci),
        "ltm_model_create": ([C.POINTER(BlockConfigC), C.POINTER(QuantConfigC), ci, ci, ci,
                              C.POINTER(vp)], ci),
        "ltm_model_load_embedding": ([vp, vp], ci),
        "ltm_model_load_layer": ([vp, ci, C.POINTER(BlockWeightsC)], ci),
        "ltm_model_forward": ([vp, vp, vp, ci, ci, vp], ci),
        "ltm_model_load_lm_head": ([vp, vp], ci),
        "ltm_model_lm_head": ([vp, vp, i64, i64, vp, vp], ci),
        "ltm_model_prefill": ([vp, vp, ci, ci, C.POINTER(vp), C.POINTER(vp), i64, vp, vp, vp], ci),
        "ltm_model_decode_step": ([vp, vp, vp, ci, C.POINTER(vp), C.POINTER(vp), i64, vp, vp,
                                   vp], ci),
        "ltm_greedy_next_tokens": ([vp, ci, ci, ci, vp, vp, vp], ci),
        "ltm_block_forward_with_cache": ([vp, vp, vp, ci, ci, vp, vp, i64, vp], ci),
        "ltm_block_forward_sp": ([vp, vp, vp, ci, ci, vp], ci),
        "ltm_block_set_overlap": ([vp, ci, ci], ci),
        "ltm_block_set_tp_reduction": ([vp, ci], ci),
        "ltm_calibrator_create": ([ci, C.c_float, ci, C.POINTER(vp)], ci),
        "ltm_calibrator_collect": ([vp, vp, ci, i64, vp], ci),
        "ltm_calibrator_compute_range": ([vp, C.POINTER(C.c_float), C.POINTER(C.c_float), vp],
                                         ci),
        "ltm_calibrator_reset": ([vp], ci),
        "ltm_calibrator_destroy": ([vp], ci),
        "ltm_quantize_int8_static": ([vp, ci, i64, C.c_float, vp, vp], ci),
        "ltm_block_save": ([vp, C.c_char_p], ci),
        "ltm_block_load": ([vp, C.c_char_p], ci),
        "ltm_block_save_memory": ([vp, C.c_char_p], ci),
        "ltm_block_load_memory": ([vp, C.c_char_p], ci),
        "ltm_block_decode_step_ragged": ([vp, vp, vp, vp, vp, i64, vp, ci, vp], ci),
        "ltm_model_destroy": ([vp], ci),
        "ltm_comm_unique_id": ([vp], ci),
        "ltm_comm_create": ([vp, ci, ci, ci, C.POINTER(vp)], ci),
        "ltm_comm_allreduce": ([vp, vp, vp, C.c_size_t, ci, ci, vp], ci),
        "ltm_comm_destroy": ([vp], ci),
        "ltm_block_create_tp": ([C.POINTER(BlockConfigC), C.POINTER(QuantConfigC), vp,
                                 C.POINTER(vp)], ci),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


def lib() -> C.CDLL:
    """The loaded C-ABI library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with "
                               "`python obsidian-memory-transformer_b200/build.py`")
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


def _check(status: int) -> None:
    if status != OK:
        msg = lib().ltm_last_error_string().decode(errors="replace")
        raise LtmError(status, msg)


def version() -> str:
    return lib().ltm_version().decode()


def device_error() -> int:
    code = C.c_int(0)
    _check(lib().ltm_device_error(C.byref(code)))
    return code.value


def launch_count() -> int:
    """Kernels launched by the library in this process."""
    n = C.c_uint64(0)
    _check(lib().ltm_launch_count(C.byref(n)))
    return n.value


def device_alloc_count() -> int:
    """Device allocations (cudaMalloc) the library has made in this process."""
    n = C.c_uint64(0)
    _check(lib().ltm_device_alloc_count(C.byref(n)))
    return n.value


CALIB_MINMAX, CALIB_PERCENTILE, CALIB_MSE = 0, 1, 2


class Calibrator:
    """Activation-range calibrator on the device (MinMaxCalibrator /
    PercentileCalibrator / MSECalibrator of the reference's quantizer):
    collect() CUDA tensors, then compute_range() -> (min, max); the static
    symmetric INT8 scale is max(|min|, |max|) / 127 (static_scale())."""

    def __init__(self, method: int = CALIB_MINMAX, percentile: float = 99.9, device: int = 0):
        h = C.c_void_p()
        _check(lib().ltm_calibrator_create(method, percentile, device, C.byref(h)))
        self._h = h

    def collect(self, x, stream=None) -> None:
        _need_cuda(x)
        _check(lib().ltm_calibrator_collect(self._h, _ptr(x), dtype_code(x.dtype), x.numel(),
                                            _stream(stream)))

    def compute_range(self, stream=None):
        lo, hi = C.c_float(), C.c_float()
        _check(lib().ltm_calibrator_compute_range(self._h, C.byref(lo), C.byref(hi),
                                                  _stream(stream)))
        return lo.value, hi.value

    def static_scale(self, stream=None) -> float:
        lo, hi = self.compute_range(stream)
        return float(np.float32(max(abs(lo), abs(hi))) / np.float32(127.0))

    def reset(self) -> None:
        _check(lib().ltm_calibrator_reset(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().ltm_calibrator_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def quantize_int8_static(x, scale: float, stream=None):
    """Per-tensor INT8 with a calibrated scale: clamp(round(x / scale), -127, 127)."""
    torch = _torch()
    _need_cuda(x)
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    _check(lib().ltm_quantize_int8_static(_ptr(x), dtype_code(x.dtype), x.numel(), scale, _ptr(q),
                                          _stream(stream)))
    return q


class KernelTimer:
    """Per-kernel device times of everything the library launches on a stream
    inside the `with` block: {name: (launches, total_ms)}."""

    def __init__(self, stream=None):
        self.stream = stream
        self.result = {}

    def __enter__(self):
        _check(lib().ltm_kernel_timer_begin(_stream(self.stream)))
        return self

    def __exit__(self, *exc):
        buf = C.create_string_buffer(1 << 16)
        _check(lib().ltm_kernel_timer_end(buf, len(buf)))
        for line in buf.value.decode().splitlines():
            name, n, ms = line.split()
            self.result[name] = (int(n), float(ms))
        return False


# ---------------------------------------------------------------- torch glue --
def _torch():
    import torch  # noqa: WPS433
    return torch


def dtype_code(t) -> int:
    torch = _torch()
    return {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}[t]


def torch_dtype(code: int):
    torch = _torch()
    return {DTYPE_F32: torch.float32, DTYPE_F16: torch.float16, DTYPE_BF16: torch.bfloat16}[code]


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream=None):
    torch = _torch()
    s = torch.cuda.current_stream() if stream is None else stream
    return C.c_void_p(s.cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None:
            if not t.is_cuda:
                raise ValueError("ltm_b200 operates on CUDA tensors only")
            if not t.is_contiguous():
                raise ValueError("ltm_b200 expects contiguous tensors")


# -------------------------------------------------------------- quantization --
def quantize_int8_per_channel(w, stream=None):
    """w [N,K] (f32/f16/bf16) -> (q int8 [N,K], s f32 [N])."""
    torch = _torch()
    _need_cuda(w)
    N, K = w.shape
    q = torch.empty((N, K), dtype=torch.int8, device=w.device)
    s = torch.empty((N,), dtype=torch.float32, device=w.device)
    _check(lib().ltm_quantize_int8_per_channel(_ptr(w), dtype_code(w.dtype), N, K, _ptr(q), _ptr(s),
                                               _stream(stream)))
    return q, s


def quantize_act_int8_per_token(a, stream=None):
    torch = _torch()
    _need_cuda(a)
    M, K = a.shape
    q = torch.empty((M, K), dtype=torch.int8, device=a.device)
    s = torch.empty((M,), dtype=torch.float32, device=a.device)
    _check(lib().ltm_quantize_act_int8_per_token(_ptr(a), dtype_code(a.dtype), M, K, _ptr(q),
                                                 _ptr(s), _stream(stream)))
    return q, s


def dequantize_int8_per_channel(q, s, dtype=None, stream=None):
    torch = _torch()
    _need_cuda(q, s)
    dtype = dtype or torch.float32
    out = torch.empty(q.shape, dtype=dtype, device=q.device)
    _check(lib().ltm_dequantize_int8_per_channel(_ptr(q), _ptr(s), q.shape[0], q.shape[1],
                                                 _ptr(out), dtype_code(dtype), _stream(stream)))
    return out


def quantize_int4_grouped(w, group_size: int = 128, stream=None):
    """w [N,K] -> (packed uint8 [N,K/2], s f32 [N,K/g], zp uint8 [N,K/g])."""
    torch = _torch()
    _need_cuda(w)
    N, K = w.shape
    packed = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    s = torch.empty((N, K // group_size), dtype=torch.float32, device=w.device)
    zp = torch.empty((N, K // group_size), dtype=torch.uint8, device=w.device)
    _check(lib().ltm_quantize_int4_grouped(_ptr(w), dtype_code(w.dtype), N, K, group_size,
                                           _ptr(packed), _ptr(s), _ptr(zp), _stream(stream)))
    return packed, s, zp


def dequantize_int4_grouped(packed, s, zp, group_size: int = 128, dtype=None, stream=None):
    torch = _torch()
    _need_cuda(packed, s, zp)
    dtype = dtype or torch.float32
    N, K = packed.shape[0], packed.shape[1] * 2
    out = torch.empty((N, K), dtype=dtype, device=packed.device)
    _check(lib().ltm_dequantize_int4_grouped(_ptr(packed), _ptr(s), _ptr(zp), N, K, group_size,
                                             _ptr(out), dtype_code(dtype), _stream(stream)))
    return out


# ------------------------------------------------------------------- linears --
def linear_w8a8(qa, sa, qw, sw, bias=None, act: int = EPI_NONE, out_dtype=None, stream=None):
    torch = _torch()
    _need_cuda(qa, sa, qw, sw, bias)
    out_dtype = out_dtype or torch.float16
    M, K = qa.shape
    N = qw.shape[0]
    y = torch.empty((M, N), dtype=out_dtype, device=qa.device)
    _check(lib().ltm_linear_w8a8(_ptr(qa), _ptr(sa), _ptr(qw), _ptr(sw), _ptr(bias), act, _ptr(y),
                                 dtype_code(out_dtype), M, N, K, _stream(stream)))
    return y


def linear_w8a8_acc_i32(qa, qw, stream=None):
    torch = _torch()
    _need_cuda(qa, qw)
    M, K = qa.shape
    N = qw.shape[0]
    acc = torch.empty((M, N), dtype=torch.int32, device=qa.device)
    _check(lib().ltm_linear_w8a8_acc_i32(_ptr(qa), _ptr(qw), _ptr(acc), M, N, K, _stream(stream)))
    return acc


def linear_w4a16(a, packed, s, zp, bias=None, act: int = EPI_NONE, stream=None):
    torch = _torch()
    _need_cuda(a, packed, s, zp, bias)
    M, K = a.shape
    N = packed.shape[0]
    y = torch.empty((M, N), dtype=a.dtype, device=a.device)
    _check(lib().ltm_linear_w4a16(_ptr(a), dtype_code(a.dtype), _ptr(packed), _ptr(s), _ptr(zp),
                                  _ptr(bias), act, _ptr(y), M, N, K, _stream(stream)))
    return y


def linear_w8a32(a, qw, sw, bias=None, act: int = EPI_NONE, stream=None):
    torch = _torch()
    _need_cuda(a, qw, sw, bias)
    M, K = a.shape
    N = qw.shape[0]
    y = torch.empty((M, N), dtype=torch.float32, device=a.device)
    _check(lib().ltm_linear_w8a32(_ptr(a), _ptr(qw), _ptr(sw), _ptr(bias), act, _ptr(y), M, N, K,
                                  _stream(stream)))
    return y


# ----------------------------------------------------------------------- ops --
def layernorm_residual(x, r, gamma, beta, stream=None):
    """y = LN(x + r) * gamma + beta over the last dim (eps 1e-5)."""
    torch = _torch()
    _need_cuda(x, r, gamma, beta)
    H = x.shape[-1]
    y = torch.empty_like(x)
    _check(lib().ltm_layernorm_residual(_ptr(x), _ptr(r), _ptr(gamma), _ptr(beta), _ptr(y),
                                        dtype_code(x.dtype), x.numel() // H, H, _stream(stream)))
    return y


def attention(q, k, v, B: int, Sq: int, Skv: int, num_heads: int, head_dim: int, causal: bool,
              kv_shared: bool = False, out=None, stream=None):
    """q: [B*Sq, ldq] head-sliced rows; k, v: [B*Skv, ld] (or [Skv, ld] when kv_shared).
    Returns o [B*Sq, num_heads*head_dim]."""
    torch = _torch()
    for t in (q, k, v):
        if not t.is_cuda or t.stride(-1) != 1:
            raise ValueError("attention operands must be CUDA tensors with unit column stride")
    if out is None:
        out = torch.empty((B * Sq, num_heads * head_dim), dtype=q.dtype, device=q.device)
    _check(lib().ltm_attention_forward(_ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v),
                                       v.stride(0), _ptr(out), out.stride(0), B, Sq, Skv,
                                       0 if kv_shared else Skv, num_heads, head_dim, int(causal),
                                       dtype_code(q.dtype), _stream(stream)))
    return out


def memory_store(memory, keys, queries, state, num_heads: int, update_rate: float = 0.9,
                 use_attention_scores: bool = True, stream=None):
    """MemoryBank::store: updates memory [Ms,H] in place (see ltm_memory_store).
    keys / queries: CUDA tensors with unit column stride (rows may be strided);
    state: fp32 [H]."""
    for t in (memory, keys, queries, state):
        if not t.is_cuda or t.stride(-1) != 1:
            raise ValueError("memory_store operands must be CUDA tensors with unit column stride")
    Ms, H = memory.shape
    _check(lib().ltm_memory_store(_ptr(memory), _ptr(keys), keys.stride(0), _ptr(queries),
                                  queries.stride(0), queries.shape[0], _ptr(state), Ms, H,
                                  num_heads, update_rate, int(use_attention_scores),
                                  dtype_code(memory.dtype), _stream(stream)))
    return memory


def memory_store_noalloc(memory, keys, queries, state, num_heads: int, update_rate: float = 0.9,
                         use_attention_scores: bool = True, stream=None):
    """memory_store without any device allocation by the library (for callers
    that own all device memory themselves): scratch is a fixed 256 KiB device
    array, so round_up(H, 64) + Ms <= 65536; overlapping calls race on it."""
    for t in (memory, keys, queries, state):
        if not t.is_cuda or t.stride(-1) != 1:
            raise ValueError("memory_store operands must be CUDA tensors with unit column stride")
    Ms, H = memory.shape
    _check(lib().ltm_memory_store_noalloc(_ptr(memory), _ptr(keys), keys.stride(0), _ptr(queries),
                                          queries.stride(0), queries.shape[0], _ptr(state), Ms, H,
                                          num_heads, update_rate, int(use_attention_scores),
                                          dtype_code(memory.dtype), _stream(stream)))
    return memory


# --------------------------------------------------------------------- block --
@dataclasses.dataclass
class TitanBlockConfig:
    """Field-for-field mirror of ltm::transformer::TitanBlockConfig
    (include/core/transformer/titan_inspired_block.cuh:19-50)."""
    hidden_dim: int = 768
    ffn_dim: int = 3072
    num_heads: int = 12
    head_dim: int = 64
    memory_slots: int = 512
    memory_dim: int = 64
    memory_update_rate: float = 0.9
    use_memory_compression: bool = True
    memory_compression_ratio: float = 0.5
    use_flash_attention: bool = True
    use_alibi: bool = False
    use_rotary: bool = True
    dropout_prob: float = 0.1
    use_parallel_attention: bool = True
    use_memory_gating: bool = True
    use_layer_norm: bool = True
    use_bias: bool = True
    fuse_operations: bool = True
    learn_memory: bool = True
    learn_compression: bool = True
    gradient_checkpointing: bool = True

    def to_c(self) -> BlockConfigC:
        c = BlockConfigC()
        for f in dataclasses.fields(self):
            v = getattr(self, f.name)
            setattr(c, f.name, int(v) if isinstance(v, bool) else v)
        return c


@dataclasses.dataclass
class QuantConfig:
    scheme: int = SCHEME_W8A8
    group_size: int = 128
    act_dtype: int = DTYPE_F16
    memory_write: bool = False
    use_attention_scores: bool = True

    def to_c(self) -> QuantConfigC:
        return QuantConfigC(self.scheme, self.group_size, self.act_dtype, int(self.memory_write),
                            int(self.use_attention_scores))


def _weights_c(w: dict):
    keep = {n: np.ascontiguousarray(w[n], dtype=np.float32) for n in WEIGHT_FIELDS
            if w.get(n) is not None}
    st = BlockWeightsC(*[keep[n].ctypes.data_as(C.POINTER(C.c_float)) if n in keep else None
                         for n in WEIGHT_FIELDS])
    return st, keep


COMM_ID_BYTES = 128


def comm_unique_id() -> bytes:
    """A fresh communicator id (rank 0 makes it; every rank needs the same bytes)."""
    buf = C.create_string_buffer(COMM_ID_BYTES)
    _check(lib().ltm_comm_unique_id(buf))
    return buf.raw


def broadcast_comm_id(group=None) -> bytes:
    """Group rank 0 makes a communicator id and every rank of the
    torch.distributed group receives the same bytes (host-side exchange; works
    over gloo)."""
    import torch.distributed as dist
    obj = [comm_unique_id() if dist.get_rank(group) == 0 else None]
    src = dist.get_global_rank(group, 0) if group is not None else 0
    dist.broadcast_object_list(obj, src=src, group=group)
    uid = obj[0]
    if not isinstance(uid, bytes) or len(uid) != COMM_ID_BYTES:
        raise LtmError(ERR_COMM, "malformed communicator id")
    return uid


class Comm:
    """Tensor-parallel communicator of `nranks` GPUs (ltm_comm_* over NCCL).

    `uid` is the bytes of comm_unique_id() made on rank 0 and handed to every
    rank by the caller (see `from_process_group`)."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        h = C.c_void_p()
        _check(lib().ltm_comm_create(C.c_char_p(uid), nranks, rank, device, C.byref(h)))
        self._h, self.nranks, self.rank, self.device = h, nranks, rank, device

    @classmethod
    def from_process_group(cls, device: int, group=None) -> "Comm":
        """Creates the communicator of the torch.distributed group's ranks (any
        backend; the id is broadcast from group rank 0 over it)."""
        import torch.distributed as dist
        uid = broadcast_comm_id(group)
        return cls(uid, dist.get_world_size(group), dist.get_rank(group), device)

    def allreduce(self, x, op_max: bool = False, stream=None):
        """In-place sum (or max) of a CUDA tensor over the ranks."""
        _need_cuda(x)
        _check(lib().ltm_comm_allreduce(self._h, _ptr(x), _ptr(x), x.numel(), dtype_code(x.dtype),
                                        int(op_max),
                                        _stream(stream)))
        return x

    def close(self) -> None:
        if getattr(self, "_h", None):
            _check(lib().ltm_comm_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class TitanBlock:
    """ltm::transformer::TitanBlock<T> over the C ABI (T = act dtype).

    With `comm` the block is the comm.rank-th tensor-parallel shard (on
    comm.device): load_weights still takes the full weights, forward the full
    [B,S,H] input and returns the full output on every rank."""

    def __init__(self, config: TitanBlockConfig, quant: QuantConfig | None = None, device: int = 0,
                 comm: Comm | None = None):
        self.config = config
        self.quant = quant or QuantConfig()
        self.device = comm.device if comm is not None else device
        self._comm = comm  # kept alive for the block's lifetime
        h = C.c_void_p()
        if comm is None:
            _check(lib().ltm_block_create(C.byref(config.to_c()), C.byref(self.quant.to_c()),
                                          device, C.byref(h)))
        else:
            _check(lib().ltm_block_create_tp(C.byref(config.to_c()), C.byref(self.quant.to_c()),
                                             comm._h, C.byref(h)))
        self._h = h

    def load_weights(self, w: dict) -> None:
        st, keep = _weights_c(w)
        _check(lib().ltm_block_load_weights(self._h, C.byref(st)))
        del keep

    def forward(self, x, attention_mask=None, stream=None, out=None, k_cache=None,
                v_cache=None):
        """x: CUDA tensor [B,S,H] in the act dtype -> y of the same shape
        (written into `out` when given; it must not alias x).  With k_cache /
        v_cache ([B, heads, max_positions, head_dim]) the post-RoPE keys and
        values of positions [0, S) are written there as well, so decode steps
        can follow at cache_len = S."""
        torch = _torch()
        _need_cuda(x, out, k_cache, v_cache)
        B, S, H = x.shape
        y = torch.empty_like(x) if out is None else out
        if k_cache is None and v_cache is None:
            _check(lib().ltm_block_forward(self._h, _ptr(x), _ptr(y), _ptr(attention_mask), B, S,
                                           _stream(stream)))
            return y
        if attention_mask is not None:
            raise LtmError(ERR_UNSUPPORTED, "explicit attention masks (self-attention is causal)")
        self._check_caches(k_cache, v_cache, B)
        _check(lib().ltm_block_forward_with_cache(self._h, _ptr(x), _ptr(y), B, S, _ptr(k_cache),
                                                  _ptr(v_cache), k_cache.shape[2],
                                                  _stream(stream)))
        return y

    def forward_sp(self, x_local, B: int, S: int, out=None, stream=None):
        """Sequence-parallel forward of a tensor-parallel block: x_local is
        this rank's [B*S / nranks, H] rows of the [B*S, H] activations; the
        result is this rank's rows of the block output."""
        torch = _torch()
        _need_cuda(x_local, out)
        y = torch.empty_like(x_local) if out is None else out
        _check(lib().ltm_block_forward_sp(self._h, _ptr(x_local), _ptr(y), B, S,
                                          _stream(stream)))
        return y

    def set_overlap(self, overlap=True, comm_sms: int = 16) -> None:
        """Chunked collectives overlapping the GEMMs in forward_sp (W8A8):
        True, False, or None for the library's default (off)."""
        _check(lib().ltm_block_set_overlap(self._h, -1 if overlap is None else int(overlap),
                                           comm_sms))

    def set_tp_reduction(self, exact: bool = True) -> None:
        """Row-parallel reductions of forward_sp: exact (W8A8: int32
        accumulators summed exactly, the result equal to the single-GPU
        block's) or, with exact=False, partial sums in the activation type."""
        _check(lib().ltm_block_set_tp_reduction(self._h,
                                                TP_REDUCE_EXACT if exact else TP_REDUCE_ACT))

    def _check_caches(self, k_cache, v_cache, B):
        heads = self.config.num_heads // (self._comm.nranks if self._comm is not None else 1)
        if (k_cache is None or v_cache is None or k_cache.shape != v_cache.shape
                or k_cache.dim() != 4 or k_cache.shape[0] != B or k_cache.shape[1] != heads
                or k_cache.shape[3] != self.config.head_dim):
            raise LtmError(ERR_INVALID_ARG,
                           "k_cache / v_cache must both be [B, heads, max_positions, head_dim]")
        if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
            raise LtmError(ERR_INVALID_ARG, "the caches must be contiguous")

    __call__ = forward

    def decode_step(self, x, k_cache, v_cache, cache_len: int, stream=None, out=None):
        """One decode step: x [B, H] (one new token per sequence, all at
        position cache_len) -> y [B, H].  k_cache / v_cache: CUDA tensors
        [B, heads, max_positions, head_dim] (head-major; heads = this
        block's heads) in the act dtype holding positions [0, cache_len); the
        step writes position cache_len."""
        torch = _torch()
        _need_cuda(x, k_cache, v_cache, out)
        B = x.shape[0]
        heads = self.config.num_heads // (self._comm.nranks if self._comm is not None else 1)
        if (k_cache.shape != v_cache.shape or k_cache.dim() != 4 or k_cache.shape[0] != B
                or k_cache.shape[1] != heads or k_cache.shape[3] != self.config.head_dim):
            raise LtmError(ERR_INVALID_ARG,
                           "k_cache / v_cache must both be [B, heads, max_positions, head_dim]")
        if not (k_cache.is_contiguous() and v_cache.is_contiguous() and x.is_contiguous()):
            raise LtmError(ERR_INVALID_ARG, "x and the caches must be contiguous")
        y = torch.empty_like(x) if out is None else out
        _check(lib().ltm_block_decode_step(self._h, _ptr(x), _ptr(y), _ptr(k_cache), _ptr(v_cache),
                                           k_cache.shape[2], int(cache_len), B, _stream(stream)))
        return y

    def decode_step_ragged(self, x, k_cache, v_cache, cache_lens, stream=None, out=None):
        """One decode step with a cache length per sequence: x [B, H], the
        new token of sequence b at position cache_lens[b] (CUDA int32 [B])."""
        torch = _torch()
        _need_cuda(x, k_cache, v_cache, cache_lens, out)
        B = x.shape[0]
        self._check_caches(k_cache, v_cache, B)
        if cache_lens.dtype != torch.int32 or cache_lens.numel() != B or not x.is_contiguous():
            raise LtmError(ERR_INVALID_ARG, "cache_lens must be int32 [B]; x contiguous")
        y = torch.empty_like(x) if out is None else out
        _check(lib().ltm_block_decode_step_ragged(self._h, _ptr(x), _ptr(y), _ptr(k_cache),
                                                  _ptr(v_cache), k_cache.shape[2],
                                                  _ptr(cache_lens), B, _stream(stream)))
        return y

    def memory_write(self, state, queries=None, stream=None) -> None:
        """Memory write of the block's bank towards `state` (fp32 [H]) with
        slot weights from the mean of the memory-query rows `queries` [T, Hl]
        (when use_attention_scores)."""
        _need_cuda(state, queries)
        T = 0 if queries is None else queries.shape[0]
        ldq = 0 if queries is None else queries.stride(0)
        _check(lib().ltm_block_memory_write(self._h, _ptr(state), _ptr(queries), ldq, T,
                                            _stream(stream)))

    def memory(self, stream=None):
        torch = _torch()
        out = torch.empty((self.config.memory_slots, self.config.hidden_dim),
                          dtype=torch_dtype(self.quant.act_dtype), device=f"cuda:{self.device}")
        _check(lib().ltm_block_get_memory(self._h, _ptr(out), _stream(stream)))
        return out

    def save(self, path) -> None:
        """Quantized checkpoint of the block (codes, scales, biases, LN, bank)."""
        _check(lib().ltm_block_save(self._h, str(path).encode()))

    def load(self, path) -> None:
        """Restores a checkpoint written by save() (same dimensions, scheme,
        dtype and tensor-parallel rank); the block is then ready to run."""
        _check(lib().ltm_block_load(self._h, str(path).encode()))

    def save_memory(self, path) -> None:
        _check(lib().ltm_block_save_memory(self._h, str(path).encode()))

    def load_memory(self, path) -> None:
        _check(lib().ltm_block_load_memory(self._h, str(path).encode()))

    def intermediate(self, name: str, stream=None):
        """A copy of one intermediate of the last forward / decode step
        (ltm_block_intermediate): activations in the act dtype, int8 codes,
        or fp32 per-row scales as a 1-D tensor."""
        torch = _torch()
        r, c, kind = C.c_int64(), C.c_int64(), C.c_int()
        _check(lib().ltm_block_intermediate(self._h, name.encode(), None, None, C.byref(r),
                                            C.byref(c), C.byref(kind)))
        dt = {0: torch_dtype(self.quant.act_dtype), 1: torch.int8, 2: torch.float32}[kind.value]
        out = torch.empty((r.value, c.value), dtype=dt, device=f"cuda:{self.device}")
        _check(lib().ltm_block_intermediate(self._h, name.encode(), _ptr(out), _stream(stream),
                                            C.byref(r), C.byref(c), C.byref(kind)))
        return out.reshape(-1) if kind.value == 2 else out

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().ltm_block_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class CacheManager:
    """KV caches of a stack of blocks for decoding (the reference's
    CacheManager, python_bindings/ltm/inference.py:101-128, whose native side
    is a stub): allocate(batch_size, seq_length) makes one K and one V tensor
    [batch_size, heads, seq_length, head_dim] (head-major) per layer;
    update(...) records that a step appended one position; get(index) returns
    the (keys, values, None) of layer `index`; clear() forgets the cached
    positions.

    `shared_layers` makes every layer use the same two tensors (a benchmark
    whose per-layer caches do not fit in device memory)."""

    def __init__(self, n_layers: int, heads: int, head_dim: int, dtype, device: int = 0,
                 shared_layers: bool = False):
        self.n_layers, self.heads, self.head_dim = n_layers, heads, head_dim
        self.dtype, self.device = dtype, device
        self.shared_layers = shared_layers
        self.length = 0
        self._k, self._v = [], []

    def allocate(self, batch_size: int, seq_length: int) -> None:
        torch = _torch()
        n = 1 if self.shared_layers else self.n_layers
        shape = (batch_size, self.heads, seq_length, self.head_dim)
        dev = f"cuda:{self.device}"
        self._k = [torch.empty(shape, dtype=self.dtype, device=dev) for _ in range(n)]
        self._v = [torch.empty(shape, dtype=self.dtype, device=dev) for _ in range(n)]
        self.length = 0

    @property
    def max_positions(self) -> int:
        return self._k[0].shape[2] if self._k else 0

    def update(self, key=None, value=None, memory=None) -> None:
        """Marks one appended position (the decode step wrote it in place)."""
        if self.length >= self.max_positions:
            raise LtmError(ERR_INVALID_ARG, "KV cache full")
        self.length += 1

    def get(self, index: int):
        i = 0 if self.shared_layers else index
        return self._k[i], self._v[i], None

    def clear(self) -> None:
        self.length = 0


def decode_step(blocks, x, cache: CacheManager, stream=None):
    """One decode step of a stack of blocks: x [B, H] -> hidden [B, H]; every
    layer reads and appends position cache.length of its cache, then the cache
    advances by one position."""
    cur = x
    for i, blk in enumerate(blocks):
        k, v, _ = cache.get(i)
        cur = blk.decode_step(cur, k, v, cache.length, stream=stream)
    cache.update()
    return cur


class TitanModel:
    """Embedding gather + n Titan blocks (TitanModel.forward without the LM head)."""

    def __init__(self, config: TitanBlockConfig, quant: QuantConfig, n_layers: int,
                 vocab_size: int, device: int = 0):
        self.config, self.quant, self.n_layers, self.vocab = config, quant, n_layers, vocab_size
        self.device = device
        h = C.c_void_p()
        _check(lib().ltm_model_create(C.byref(config.to_c()), C.byref(quant.to_c()), n_layers,
                                      vocab_size, device, C.byref(h)))
        self._h = h

    def load_embedding(self, emb: np.ndarray) -> None:
        e = np.ascontiguousarray(emb, dtype=np.float32)
        _check(lib().ltm_model_load_embedding(self._h, C.c_void_p(e.ctypes.data)))

    def load_layer(self, i: int, w: dict) -> None:
        st, keep = _weights_c(w)
        _check(lib().ltm_model_load_layer(self._h, i, C.byref(st)))
        del keep

    def forward(self, tokens, out=None, stream=None):
        """tokens: CUDA int32 [B,S] -> hidden [B,S,H] (act dtype)."""
        torch = _torch()
        _need_cuda(tokens)
        B, S = tokens.shape
        if out is None:
            out = torch.empty((B, S, self.config.hidden_dim), dtype=torch_dtype(self.quant.act_dtype),
                              device=tokens.device)
        _check(lib().ltm_model_forward(self._h, _ptr(tokens), _ptr(out), B, S, _stream(stream)))
        return out

    __call__ = forward

    # ------------------------------------------------------- LM head, decode --
    def load_lm_head(self, weight: np.ndarray) -> None:
        """TitanForCausalLM.lm_head: host fp32 [vocab, H], no bias."""
        w = np.ascontiguousarray(weight, dtype=np.float32)
        if w.shape != (self.vocab, self.config.hidden_dim):
            raise LtmError(ERR_INVALID_ARG, "LM head weight must be [vocab, hidden]")
        _check(lib().ltm_model_load_lm_head(self._h, C.c_void_p(w.ctypes.data)))

    def lm_head(self, hidden, out=None, stream=None):
        """logits [..., vocab] of hidden rows [..., H] (the last dim contiguous;
        rows may be strided, e.g. hidden[:, -1, :])."""
        torch = _torch()
        _need_cuda(out)
        if not hidden.is_cuda:
            raise ValueError("ltm_b200 operates on CUDA tensors only")
        H = self.config.hidden_dim
        rows = hidden.reshape(-1, H) if hidden.is_contiguous() else hidden
        if rows.dim() != 2 or rows.stride(1) != 1:
            raise LtmError(ERR_INVALID_ARG, "hidden rows must be a 2-D view with unit column stride")
        R = rows.shape[0]
        if out is None:
            out = torch.empty((R, self.vocab), dtype=torch_dtype(self.quant.act_dtype),
                              device=hidden.device)
        _check(lib().ltm_model_lm_head(self._h, _ptr(rows), R, rows.stride(0), _ptr(out),
                                       _stream(stream)))
        return out.reshape(*hidden.shape[:-1], self.vocab) if hidden.is_contiguous() else out

    def make_cache(self, batch_size: int, max_positions: int) -> "CacheManager":
        cache = CacheManager(self.n_layers, self.config.num_heads, self.config.head_dim,
                             torch_dtype(self.quant.act_dtype), device=self.device)
        cache.allocate(batch_size, max_positions)
        return cache

    @staticmethod
    def _cache_ptrs(cache: "CacheManager"):
        n = len(cache._k)
        ks = (C.c_void_p * n)(*[t.data_ptr() for t in cache._k])
        vs = (C.c_void_p * n)(*[t.data_ptr() for t in cache._v])
        return ks, vs

    def prefill(self, tokens, cache: "CacheManager", hidden_out=None, logits=True, stream=None):
        """Prompts tokens (CUDA int32 [B,S]) through the model, filling every
        layer's cache at positions [0, S); returns (hidden [B,S,H] or None,
        logits of each sequence's last position [B, vocab] or None)."""
        torch = _torch()
        _need_cuda(tokens, hidden_out)
        B, S = tokens.shape
        lg = (torch.empty((B, self.vocab), dtype=torch_dtype(self.quant.act_dtype),
                          device=tokens.device) if logits else None)
        ks, vs = self._cache_ptrs(cache)
        _check(lib().ltm_model_prefill(self._h, _ptr(tokens), B, S, ks, vs, cache.max_positions,
                                       _ptr(hidden_out), _ptr(lg), _stream(stream)))
        cache.length = S
        return hidden_out, lg

    def decode_step(self, tokens, cache_lens, cache: "CacheManager", logits=None, hidden_out=None,
                    stream=None):
        """One decode step: tokens (CUDA int32 [B]) at positions cache_lens
        (CUDA int32 [B]); returns the logits [B, vocab] (written into `logits`
        when given)."""
        torch = _torch()
        _need_cuda(tokens, cache_lens, logits, hidden_out)
        B = tokens.shape[0]
        if logits is None:
            logits = torch.empty((B, self.vocab), dtype=torch_dtype(self.quant.act_dtype),
                                 device=tokens.device)
        ks, vs = self._cache_ptrs(cache)
        _check(lib().ltm_model_decode_step(self._h, _ptr(tokens), _ptr(cache_lens), B, ks, vs,
                                           cache.max_positions, _ptr(hidden_out), _ptr(logits),
                                           _stream(stream)))
        return logits

    def greedy_next(self, logits, tokens_out, cache_lens=None, stream=None):
        """tokens_out[b] = argmax logits[b] (device); cache_lens += 1 when given."""
        _need_cuda(logits, tokens_out, cache_lens)
        _check(lib().ltm_greedy_next_tokens(_ptr(logits), dtype_code(logits.dtype),
                                            logits.shape[0], logits.shape[1], _ptr(tokens_out),
                                            _ptr(cache_lens), _stream(stream)))

    def generate_greedy(self, prompt, new_tokens: int, max_positions: int | None = None,
                        use_graph: bool = True, hidden_trace: bool = False):
        """Greedy generation of `new_tokens` tokens after the prompts (CUDA
        int32 [B,S]): a prefill that fills the caches, then one decode step
        per token on the device (captured once in a CUDA graph and replayed
        when use_graph).  Returns the generated tokens [B, new_tokens] and,
        with hidden_trace, the last layer's hidden state of every step
        [new_tokens, B, H]."""
        torch = _torch()
        B, S = prompt.shape
        P = max_positions or S + new_tokens
        cache = self.make_cache(B, P)
        dev = prompt.device
        _, logits = self.prefill(prompt, cache)
        tok = torch.empty(B, dtype=torch.int32, device=dev)
        lens = torch.full((B,), S, dtype=torch.int32, device=dev)
        out = torch.empty((B, new_tokens), dtype=torch.int32, device=dev)
        hid = torch.empty((B, self.config.hidden_dim), dtype=torch_dtype(self.quant.act_dtype),
                          device=dev)
        trace = [] if hidden_trace else None
        if new_tokens == 0:
            return out, trace
        self.greedy_next(logits, tok)  # first generated token from the prompt's last logits
        out[:, 0] = tok
        step_logits = torch.empty((B, self.vocab), dtype=logits.dtype, device=dev)

        def step():
            self.decode_step(tok, lens, cache, logits=step_logits, hidden_out=hid)
            self.greedy_next(step_logits, tok, lens)

        graph = None
        for i in range(1, new_tokens):
            if use_graph and graph is None and i >= 2:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, capture_error_mode="relaxed"):
                    step()
            if graph is not None:
                graph.replay()
            else:
                step()
            out[:, i] = tok
            if hidden_trace:
                trace.append(hid.clone())
        if hidden_trace:
            # the step of the last generated token's hidden state
            self.decode_step(tok, lens, cache, logits=step_logits, hidden_out=hid)
            trace.append(hid.clone())
        return out, trace

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().ltm_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
