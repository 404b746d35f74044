// epilogue.cuh -- the fused epilogue shared by every linear kernel.
//
// A kernel hands over 32 consecutive fp32 values of one output row (raw
// accumulators) and the epilogue applies, in this order:
//   v = acc * row_scale[m] * col_scale[n] + bias[n]     (dequant + bias)
//   v = act(v)                                           (none / GELU-tanh / sigmoid)
// then one of the modes
//   PLAIN    y = v
//   ROPE     interleaved-pair rotation of columns < rope_cols (Q and K of the
//            fused projection), position = m % seq_len
//   RESID    y = v + R[m,n]                               (FFN-down + block residual)
//   GATEMIX  g = v (sigmoid applied);  y = s + g*mem + (1-g)*x   (memory integration)
//   ACC_I32  raw int32 accumulators (exactness probe)
// and stores 32 outputs with 16-byte vector stores.
#pragma once

#include "common.cuh"

namespace ltm_b200 {

enum EpiMode : int { kEpiPlain = 0, kEpiRope = 1, kEpiResid = 2, kEpiGateMix = 3, kEpiAccI32 = 4 };

struct Epilogue {
  int act = LTM_EPI_NONE;
  const float* row_scale = nullptr;  // [M] or NULL (=1)
  const float* col_scale = nullptr;  // [N] or NULL (=1)
  const float* bias = nullptr;       // [N] or NULL (=0)
  void* out = nullptr;
  int64_t ldo = 0;  // elements
  // ROPE
  const float2* rope = nullptr;  // [seq_len, head_dim/2] of (cos, sin)
  int rope_cols = 0;
  int seq_len = 1;
  int head_dim = 64;
  // RESID (aux0 = R) / GATEMIX (aux0 = s, aux1 = mem, aux2 = x); all use ld_aux
  const void* aux0 = nullptr;
  const void* aux1 = nullptr;
  const void* aux2 = nullptr;
  int64_t ld_aux = 0;
  // GATEMIX: optional column sums of g*x over the rows (memory write), fp32 [N]
  float* colsum = nullptr;
};

// Sum over the warp's 32 rows of v[c]; lane c receives column c (31 shuffles,
// recursive halving).  Must be called by all 32 lanes.
__device__ __forceinline__ float warp_colsum32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int j = 0; j < s; ++j) {
      const float send = upper ? v[j] : v[j + s];
      const float keep = upper ? v[j + s] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // src/core/ops/fused_ops.cu:136-142
  const float cdf = 0.5f * (1.0f + tanhf(0.797885f * (x + 0.044715f * x * x * x)));
  return x * cdf;
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

template <class T>
__device__ __forceinline__ void load32(const T* p, float (&v)[32]) {
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int c = 0; c < 32 / PER; ++c) {
    uint4 raw = *reinterpret_cast<const uint4*>(p + c * PER);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < PER; ++i) v[c * PER + i] = to_f32(e[i]);
  }
}

template <class T>
__device__ __forceinline__ void store32(T* p, const float (&v)[32]) {
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int c = 0; c < 32 / PER; ++c) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < PER; ++i) e[i] = from_f32<T>(v[c * PER + i]);
    *reinterpret_cast<uint4*>(p + c * PER) = raw;
  }
}

// Applies the epilogue to 32 values of row `m`, columns [n0, n0+32) and stores.
// GATEMIX with ep.colsum: g*x is written to gx_out when given (the caller
// reduces it across the warp), else added to ep.colsum element by element.
template <int MODE, class OutT>
__device__ __forceinline__ void epilogue_store32(const Epilogue& ep, int64_t m, int64_t n0,
                                                 float (&v)[32], float* gx_out = nullptr) {
  if constexpr (MODE == kEpiAccI32) {
    int32_t* o = static_cast<int32_t*>(ep.out) + m * ep.ldo + n0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      int4 t;
      t.x = __float_as_int(v[4 * c + 0]);
      t.y = __float_as_int(v[4 * c + 1]);
      t.z = __float_as_int(v[4 * c + 2]);
      t.w = __float_as_int(v[4 * c + 3]);
      *reinterpret_cast<int4*>(o + 4 * c) = t;
    }
    return;
  } else {
    const float rs = ep.row_scale ? ep.row_scale[m] : 1.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float x = v[i] * rs;
      if (ep.col_scale) x = x * __ldg(ep.col_scale + n0 + i);
      if (ep.bias) x = x + __ldg(ep.bias + n0 + i);
      if (ep.act == LTM_EPI_GELU) x = gelu_tanh(x);
      else if (ep.act == LTM_EPI_SIGMOID) x = sigmoid_f(x);
      v[i] = x;
    }
    if constexpr (MODE == kEpiRope) {
      if (n0 < ep.rope_cols) {
        const int half = ep.head_dim >> 1;
        const int pos = static_cast<int>(m % ep.seq_len);
        const float2* tab = ep.rope + static_cast<int64_t>(pos) * half;
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int d = static_cast<int>((n0 + i) % ep.head_dim);
          const float2 cs = __ldg(tab + (d >> 1));
          const float a = v[i], b = v[i + 1];
          v[i] = a * cs.x - b * cs.y;
          v[i + 1] = a * cs.y + b * cs.x;
        }
      }
    } else if constexpr (MODE == kEpiResid) {
      float r[32];
      load32(static_cast<const OutT*>(ep.aux0) + m * ep.ld_aux + n0, r);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += r[i];
    } else if constexpr (MODE == kEpiGateMix) {
      float s[32], mem[32];
      load32(static_cast<const OutT*>(ep.aux0) + m * ep.ld_aux + n0, s);
      load32(static_cast<const OutT*>(ep.aux1) + m * ep.ld_aux + n0, mem);
#pragma unroll
      for (int i = 0; i < 32; ++i) s[i] = s[i] + v[i] * mem[i];
      load32(static_cast<const OutT*>(ep.aux2) + m * ep.ld_aux + n0, mem);
      if (ep.colsum) {
        if (gx_out) {
#pragma unroll
          for (int i = 0; i < 32; ++i) gx_out[i] = v[i] * mem[i];
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) atomicAdd(ep.colsum + n0 + i, v[i] * mem[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = s[i] + (1.0f - v[i]) * mem[i];
    }
    store32(static_cast<OutT*>(ep.out) + m * ep.ldo + n0, v);
  }
}

// Runtime (mode, out dtype) -> template dispatch used by the launchers.
template <class F>
void dispatch_epilogue(int mode, ltm_dtype out_dt, F&& f) {
  auto with_t = [&](auto mode_c) {
    constexpr int MODE = decltype(mode_c)::value;
    if constexpr (MODE == kEpiAccI32) {
      f(mode_c, int32_t{});
    } else {
      switch (out_dt) {
        case LTM_DTYPE_F32: f(mode_c, float{}); break;
        case LTM_DTYPE_F16: f(mode_c, __half{}); break;
        case LTM_DTYPE_BF16: f(mode_c, __nv_bfloat16{}); break;
        default: LTM_REQUIRE(false, "unknown output dtype");
      }
    }
  };
  switch (mode) {
    case kEpiPlain: with_t(std::integral_constant<int, kEpiPlain>{}); break;
    case kEpiRope: with_t(std::integral_constant<int, kEpiRope>{}); break;
    case kEpiResid: with_t(std::integral_constant<int, kEpiResid>{}); break;
    case kEpiGateMix: with_t(std::integral_constant<int, kEpiGateMix>{}); break;
    case kEpiAccI32: with_t(std::integral_constant<int, kEpiAccI32>{}); break;
    default: LTM_REQUIRE(false, "unknown epilogue mode");
  }
}

}  // namespace ltm_b200
