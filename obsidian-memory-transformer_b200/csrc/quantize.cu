// quantize.cu -- INT8 per-row (weights per output channel, activations per
// token) and INT4 grouped asymmetric quantize/pack/dequantize kernels.
//
// Bandwidth-bound: one warp owns one row (INT8) or one 128-element group
// (INT4); loads are 128-bit where the row layout allows, reductions are warp
// shuffles.  Codes equal IEEE round-to-nearest division followed by
// round-half-away-from-zero (roundf), the arithmetic of the reference kernels
// src/core/quantization/quantizer.cu:94-142, so they are bit-exact against a
// CPU evaluation of the same formula (INT8 uses the reciprocal fast path of
// quant_i8_exact, which falls back to the division near rounding ties).
#include <type_traits>

#include <algorithm>

#include "block.cuh"

namespace ltm_b200 {
namespace {

template <class T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}


// One warp per row: s = absmax/127, q = clamp(round(x/s)).
template <class T, bool VEC>
__global__ void __launch_bounds__(256) rowwise_int8_kernel(const T* __restrict__ x, int64_t rows,
                                                           int64_t K, int8_t* __restrict__ q,
                                                           float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * K;
  int8_t* qr = q + row * K;
  float amax = 0.0f;
  if constexpr (VEC) {
    constexpr int V = Vec16<T>::N;
    const int64_t nv = K / V;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    for (int64_t j = lane; j < nv; j += 32) {
      uint4 raw = __ldg(xv + j);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < V; ++i) amax = fmaxf(amax, fabsf(to_f32(e[i])));
    }
    amax = warp_max(amax);
    const float s = __fdiv_rn(amax, 127.0f);
    const float inv = recip_or_zero(s);
    for (int64_t j = lane; j < nv; j += 32) {
      uint4 raw = __ldg(xv + j);
      const T* e = reinterpret_cast<const T*>(&raw);
      int8_t out[V];
#pragma unroll
      for (int i = 0; i < V; ++i) out[i] = quant_i8_exact(to_f32(e[i]), s, inv);
      if constexpr (V == 8) {
        *reinterpret_cast<uint2*>(qr + j * V) = *reinterpret_cast<const uint2*>(out);
      } else {
        *reinterpret_cast<uint32_t*>(qr + j * V) = *reinterpret_cast<const uint32_t*>(out);
      }
    }
    if (lane == 0) scales[row] = s;
  } else {
    for (int64_t j = lane; j < K; j += 32) amax = fmaxf(amax, fabsf(to_f32(xr[j])));
    amax = warp_max(amax);
    const float s = __fdiv_rn(amax, 127.0f);
    const float inv = recip_or_zero(s);
    for (int64_t j = lane; j < K; j += 32) qr[j] = quant_i8_exact(to_f32(xr[j]), s, inv);
    if (lane == 0) scales[row] = s;
  }
}

// Persistent row quantizers with the next row's loads in flight while the
// current row is reduced and quantized.  WPR warps share one row (WPR = 1:
// every warp owns its rows; WPR = 4: a 128-thread CTA owns a row and reduces
// the row max through shared memory); lane l of the row group holds the
// 16-byte vectors l, l + 32*WPR, ... (NV of them).  WPR = 8 / 32: a 256- /
// 1024-thread CTA per row.
template <class T, int NV>
__device__ __forceinline__ void load_row_vecs(const T* __restrict__ x, int64_t row, int64_t K,
                                              int nvec, int gl, int stride, uint4 (&raw)[NV]) {
  const uint4* xv = reinterpret_cast<const uint4*>(x + row * K);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int vi = gl + stride * j;
    raw[j] = vi < nvec ? __ldg(xv + vi) : make_uint4(0, 0, 0, 0);
  }
}

template <class T, int NV, int WPR>
__global__ void __launch_bounds__(WPR == 1 ? 256 : 32 * WPR) rowwise_int8_pipe_kernel(
    const T* __restrict__ x, int64_t rows, int64_t K, int8_t* __restrict__ q,
    float* __restrict__ scales) {
  constexpr int V = Vec16<T>::N;
  constexpr int STRIDE = 32 * WPR;
  __shared__ float red[2][WPR];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gl = (WPR == 1) ? lane : static_cast<int>(threadIdx.x);  // lane within the row group
  const int64_t groups_per_cta = (WPR == 1) ? (blockDim.x >> 5) : 1;
  const int64_t g0 = static_cast<int64_t>(blockIdx.x) * groups_per_cta + (WPR == 1 ? warp : 0);
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * groups_per_cta;
  const int nvec = static_cast<int>(K / V);
  uint4 cur[NV], nxt[NV];
  if (g0 < rows) load_row_vecs<T, NV>(x, g0, K, nvec, gl, STRIDE, cur);
  int parity = 0;
  for (int64_t row = g0; row < rows; row += gstride) {
    const int64_t next = row + gstride;
    if (next < rows) load_row_vecs<T, NV>(x, next, K, nvec, gl, STRIDE, nxt);
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const T* e = reinterpret_cast<const T*>(&cur[j]);
#pragma unroll
      for (int i = 0; i < V; ++i) amax = fmaxf(amax, fabsf(to_f32(e[i])));
    }
    amax = warp_max(amax);
    if constexpr (WPR > 1) {
      if (lane == 0) red[parity][warp] = amax;
      __syncthreads();
#pragma unroll
      for (int w = 0; w < WPR; ++w) amax = fmaxf(amax, red[parity][w]);
      parity ^= 1;
    }
    const float s = __fdiv_rn(amax, 127.0f);
    const float inv = recip_or_zero(s);
    int8_t* qr = q + row * K;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int vi = gl + STRIDE * j;
      const T* e = reinterpret_cast<const T*>(&cur[j]);
      float f[V];
#pragma unroll
      for (int i = 0; i < V; ++i) f[i] = to_f32(e[i]);
      int8_t out[V];
      quant_i8_exact_warp<V>(f, s, inv, out);
      if (vi < nvec) {
        if constexpr (V == 8)
          *reinterpret_cast<uint2*>(qr + vi * V) = *reinterpret_cast<const uint2*>(out);
        else
          *reinterpret_cast<uint32_t*>(qr + vi * V) = *reinterpret_cast<const uint32_t*>(out);
      }
    }
    if (gl == 0) scales[row] = s;
#pragma unroll
    for (int j = 0; j < NV; ++j) cur[j] = nxt[j];
  }
}

template <class T>
__global__ void __launch_bounds__(256) dequant_int8_kernel(const int8_t* __restrict__ q,
                                                           const float* __restrict__ s,
                                                           int64_t N, int64_t K, T* __restrict__ out) {
  const int64_t total = N * K;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / K;
    out[i] = from_f32<T>(static_cast<float>(q[i]) * s[n]);
  }
}

// One warp per (row, 128-element group); lane l owns elements 4l..4l+3.
template <class T>
__global__ void __launch_bounds__(256) int4_group_quant_kernel(const T* __restrict__ w, int64_t N,
                                                               int64_t K, uint8_t* __restrict__ packed,
                                                               float* __restrict__ scales,
                                                               uint8_t* __restrict__ zeros) {
  const int lane = threadIdx.x & 31;
  const int64_t groups_per_row = K / 128;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gid >= N * groups_per_row) return;
  const int64_t n = gid / groups_per_row;
  const int64_t g = gid - n * groups_per_row;
  const T* src = w + n * K + g * 128 + lane * 4;
  float v[4];
  if constexpr (sizeof(T) == 4) {
    float4 t = __ldg(reinterpret_cast<const float4*>(src));
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    uint2 raw = __ldg(reinterpret_cast<const uint2*>(src));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = to_f32(e[i]);
  }
  float mn = fminf(fminf(v[0], v[1]), fminf(v[2], v[3]));
  float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
  mn = fminf(warp_min(mn), 0.0f);
  mx = fmaxf(warp_max(mx), 0.0f);
  const float s = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
  float zp = 0.0f;
  uint32_t code[4] = {0, 0, 0, 0};
  if (s != 0.0f) {
    zp = fminf(fmaxf(roundf(__fdiv_rn(-mn, s)), 0.0f), 15.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float r = roundf(__fadd_rn(__fdiv_rn(v[i], s), zp));
      r = fminf(fmaxf(r, 0.0f), 15.0f);
      code[i] = static_cast<uint32_t>(r);
    }
  }
  const uint16_t two = static_cast<uint16_t>((code[0] | (code[1] << 4)) |
                                             ((code[2] | (code[3] << 4)) << 8));
  *reinterpret_cast<uint16_t*>(packed + n * (K / 2) + g * 64 + lane * 2) = two;
  if (lane == 0) {
    scales[n * groups_per_row + g] = s;
    zeros[n * groups_per_row + g] = static_cast<uint8_t>(zp);
  }
}

template <class T>
__global__ void __launch_bounds__(256) int4_dequant_kernel(const uint8_t* __restrict__ packed,
                                                           const float* __restrict__ s,
                                                           const uint8_t* __restrict__ zp,
                                                           int64_t N, int64_t K, int group,
                                                           T* __restrict__ out) {
  const int64_t total_bytes = N * K / 2;
  const int64_t gpr = K / group;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total_bytes;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = 2 * i;
    const int64_t n = e / K;
    const int64_t k = e - n * K;
    const int64_t gi = n * gpr + k / group;
    const float sc = s[gi];
    const float z = static_cast<float>(zp[gi]);
    const uint8_t b = packed[i];
    out[e] = from_f32<T>((static_cast<float>(b & 0xF) - z) * sc);
    out[e + 1] = from_f32<T>((static_cast<float>(b >> 4) - z) * sc);
  }
}

// int4_dequant_kernel on 32 weights (16 packed bytes, one group's quarter)
// per thread: W[n,k] = T((q - zp) * s), the same arithmetic; K % 128 == 0.
template <class T>
__global__ void __launch_bounds__(256) int4_dequant_rows_kernel(const uint8_t* __restrict__ packed,
                                                                const float* __restrict__ s,
                                                                const uint8_t* __restrict__ zp,
                                                                int64_t N, int K,
                                                                T* __restrict__ out) {
  const int cpr = K / 32;  // 32-weight chunks per row
  const int64_t total = N * cpr;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / cpr;
    const int c = static_cast<int>(i - n * cpr);
    const int64_t gi = n * (K / 128) + c / 4;
    const float sc = __ldg(s + gi);
    const float z = static_cast<float>(__ldg(zp + gi));
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(packed + n * (K / 2)) + c);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint4 o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      T* e = reinterpret_cast<T*>(&o[j]);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (w[j] >> (8 * b)) & 0xFFu;
        e[2 * b] = from_f32<T>((static_cast<float>(byte & 0xFu) - z) * sc);
        e[2 * b + 1] = from_f32<T>((static_cast<float>(byte >> 4) - z) * sc);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + n * K) + c * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = o[j];
  }
}

int elementwise_grid(int64_t total) {
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
  return static_cast<int>(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap);
}

}  // namespace

void launch_rowwise_int8(const void* x, ltm_dtype dt, int64_t rows, int64_t K, int8_t* q,
                         float* s, cudaStream_t stream) {
  if (rows == 0 || K == 0) return;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    const bool vec = ((K * sizeof(T)) % 16 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(q) & 7) == 0);
    const int64_t nvec = K / Vec16<T>::N;
    auto warp_launch = [&](auto nv_c) {  // one warp per row, 8 rows per CTA in flight
      constexpr int NV = decltype(nv_c)::value;
      auto kern = rowwise_int8_pipe_kernel<T, NV, 1>;
      const int grid = persistent_grid(kern, 256, 0, (rows + 7) / 8);
      kern<<<grid, 256, 0, stream>>>(static_cast<const T*>(x), rows, K, q, s);
    };
    auto cta_launch = [&](auto nv_c) {  // four warps per row
      constexpr int NV = decltype(nv_c)::value;
      auto kern = rowwise_int8_pipe_kernel<T, NV, 4>;
      const int grid = persistent_grid(kern, 128, 0, rows);
      kern<<<grid, 128, 0, stream>>>(static_cast<const T*>(x), rows, K, q, s);
    };
    if (vec && nvec <= 4 * 32) {
      const int64_t nv = (nvec + 31) / 32;
      if (nv <= 1) warp_launch(std::integral_constant<int, 1>{});
      else if (nv <= 2) warp_launch(std::integral_constant<int, 2>{});
      else if (nv <= 3) warp_launch(std::integral_constant<int, 3>{});
      else warp_launch(std::integral_constant<int, 4>{});
    } else if (vec && nvec > 4 * 128 && nvec <= 4 * 256) {
      // eight warps per row (rows of 4096-8192 16-bit values): twice the
      // throughput of four warps with eight vectors each at 8192 (measured,
      // same codes)
      auto kern = rowwise_int8_pipe_kernel<T, 4, 8>;
      const int grid = persistent_grid(kern, 256, 0, rows);
      kern<<<grid, 256, 0, stream>>>(static_cast<const T*>(x), rows, K, q, s);
    } else if (vec && nvec > 8 * 128 && nvec <= 4 * 1024) {
      // a 1024-thread CTA per row for rows of 8K-32K 16-bit values (the FFN
      // hidden of the hidden-8192 block): one pass over the row instead of
      // the two-pass kernel, 11% faster at 28672 (measured, same codes)
      auto wide = [&](auto nv_c) {
        constexpr int NV = decltype(nv_c)::value;
        auto kern = rowwise_int8_pipe_kernel<T, NV, 32>;
        const int grid = persistent_grid(kern, 1024, 0, rows);
        kern<<<grid, 1024, 0, stream>>>(static_cast<const T*>(x), rows, K, q, s);
      };
      const int64_t nv = (nvec + 1023) / 1024;
      if (nv <= 2) wide(std::integral_constant<int, 2>{});
      else if (nv <= 3) wide(std::integral_constant<int, 3>{});
      else wide(std::integral_constant<int, 4>{});
    } else if (vec && nvec <= 8 * 128) {
      const int64_t nv = (nvec + 127) / 128;
      if (nv <= 2) cta_launch(std::integral_constant<int, 2>{});
      else if (nv <= 3) cta_launch(std::integral_constant<int, 3>{});
      else if (nv <= 4) cta_launch(std::integral_constant<int, 4>{});
      else if (nv <= 6) cta_launch(std::integral_constant<int, 6>{});
      else cta_launch(std::integral_constant<int, 8>{});
    } else if (vec)
      rowwise_int8_kernel<T, true><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), rows, K, q, s);
    else
      rowwise_int8_kernel<T, false><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), rows, K, q, s);
  });
  check_launch("rowwise_int8_kernel", stream);
}

namespace {

// Split form of the per-token quantizer for a row whose columns are spread
// over tensor-parallel ranks: row_absmax_kernel gives this rank's row maxima,
// the ranks combine them with an allreduce-max, and rowwise_int8_amax_kernel
// quantizes the local columns with s = global max / 127 -- the codes and
// scales the unsplit row would get.  One warp per row.
template <class T, bool VEC>
__global__ void __launch_bounds__(256) row_absmax_kernel(const T* __restrict__ x, int64_t rows,
                                                         int64_t K, float* __restrict__ amax) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * K;
  float m = 0.0f;
  if constexpr (VEC) {
    constexpr int V = Vec16<T>::N;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    const int64_t nv = K / V;
    int64_t j = lane;
    for (; j + 96 < nv; j += 128) {  // four independent 16-byte loads in flight per lane
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) raw[u] = __ldg(xv + j + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
        for (int i = 0; i < V; ++i) m = fmaxf(m, fabsf(to_f32(e[i])));
      }
    }
    for (; j < nv; j += 32) {
      const uint4 raw = __ldg(xv + j);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < V; ++i) m = fmaxf(m, fabsf(to_f32(e[i])));
    }
  } else {
    for (int64_t j = lane; j < K; j += 32) m = fmaxf(m, fabsf(to_f32(xr[j])));
  }
  m = warp_max(m);
  if (lane == 0) amax[row] = m;
}

template <class T, bool VEC>
__global__ void __launch_bounds__(256) rowwise_int8_amax_kernel(const T* __restrict__ x,
                                                                int64_t rows, int64_t K,
                                                                const float* __restrict__ amax,
                                                                int8_t* __restrict__ q,
                                                                float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * K;
  int8_t* qr = q + row * K;
  const float s = __fdiv_rn(amax[row], 127.0f);
  const float inv = recip_or_zero(s);
  if constexpr (VEC) {
    constexpr int V = Vec16<T>::N;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    const int64_t nv = K / V;
    auto put = [&](int64_t jj, const uint4& raw) {
      const T* e = reinterpret_cast<const T*>(&raw);
      int8_t out[V];
#pragma unroll
      for (int i = 0; i < V; ++i) out[i] = quant_i8_exact(to_f32(e[i]), s, inv);
      if constexpr (V == 8)
        *reinterpret_cast<uint2*>(qr + jj * V) = *reinterpret_cast<const uint2*>(out);
      else
        *reinterpret_cast<uint32_t*>(qr + jj * V) = *reinterpret_cast<const uint32_t*>(out);
    };
    int64_t j = lane;
    for (; j + 96 < nv; j += 128) {  // four independent 16-byte loads in flight per lane
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) raw[u] = __ldg(xv + j + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) put(j + 32 * u, raw[u]);
    }
    for (; j < nv; j += 32) put(j, __ldg(xv + j));
  } else {
    for (int64_t j = lane; j < K; j += 32) qr[j] = quant_i8_exact(to_f32(xr[j]), s, inv);
  }
  if (lane == 0) scales[row] = s;
}

}  // namespace

void launch_row_absmax(const void* x, ltm_dtype dt, int64_t rows, int64_t K, float* amax,
                       cudaStream_t stream) {
  if (rows == 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
    const bool vec = (K * sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (vec)
      row_absmax_kernel<T, true><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), rows, K, amax);
    else
      row_absmax_kernel<T, false><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), rows, K, amax);
  });
  check_launch("row_absmax_kernel", stream);
}

void launch_rowwise_int8_amax(const void* x, ltm_dtype dt, int64_t rows, int64_t K,
                              const float* amax, int8_t* q, float* s, cudaStream_t stream) {
  if (rows == 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
    const bool vec = (K * sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(q) & 7) == 0;
    if (vec)
      rowwise_int8_amax_kernel<T, true><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), rows,
                                                                    K, amax, q, s);
    else
      rowwise_int8_amax_kernel<T, false><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x),
                                                                     rows, K, amax, q, s);
  });
  check_launch("rowwise_int8_amax_kernel", stream);
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_quantize_int8_per_channel(const void* w, ltm_dtype w_dtype, int64_t N,
                                                    int64_t K, int8_t* q, float* s, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(N >= 0 && K >= 0, "negative size");
    LTM_REQUIRE((N == 0 || K == 0) || (w && q && s), "NULL pointer");
    if (N > 0 && K == 0) {
      LTM_CUDA_TRY(cudaMemsetAsync(s, 0, N * sizeof(float), as_stream(stream)));
      return;
    }
    launch_rowwise_int8(w, w_dtype, N, K, q, s, as_stream(stream));
  });
}

extern "C" ltm_status ltm_quantize_act_int8_per_token(const void* a, ltm_dtype a_dtype, int64_t M,
                                                      int64_t K, int8_t* q, float* s, void* stream) {
  return ltm_quantize_int8_per_channel(a, a_dtype, M, K, q, s, stream);
}

extern "C" ltm_status ltm_dequantize_int8_per_channel(const int8_t* q, const float* s, int64_t N,
                                                      int64_t K, void* out, ltm_dtype out_dtype,
                                                      void* stream) {
  return guarded([&] {
    LTM_REQUIRE(N >= 0 && K >= 0, "negative size");
    if (N == 0 || K == 0) return;
    LTM_REQUIRE(q && s && out, "NULL pointer");
    dispatch_dtype(out_dtype, [&](auto tag) {
      using T = decltype(tag);
      dequant_int8_kernel<T><<<elementwise_grid(N * K), 256, 0, as_stream(stream)>>>(
          q, s, N, K, static_cast<T*>(out));
    });
    check_launch("dequant_int8_kernel", as_stream(stream));
  });
}

extern "C" ltm_status ltm_quantize_int4_grouped(const void* w, ltm_dtype w_dtype, int64_t N,
                                                int64_t K, int group_size, uint8_t* packed,
                                                float* s, uint8_t* zp, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(N >= 0 && K >= 0, "negative size");
    if (group_size != 128) LTM_UNSUPPORTED("INT4 group_size must be 128");
    LTM_REQUIRE(K % 128 == 0, "K must be a multiple of the group size");
    if (N == 0 || K == 0) return;
    LTM_REQUIRE(w && packed && s && zp, "NULL pointer");
    const int64_t groups = N * (K / 128);
    const unsigned blocks = static_cast<unsigned>((groups + 7) / 8);
    dispatch_dtype(w_dtype, [&](auto tag) {
      using T = decltype(tag);
      LTM_REQUIRE((reinterpret_cast<uintptr_t>(w) & (4 * sizeof(T) - 1)) == 0,
                  "weight pointer misaligned for 4-element loads");
      int4_group_quant_kernel<T><<<blocks, 256, 0, as_stream(stream)>>>(
          static_cast<const T*>(w), N, K, packed, s, zp);
    });
    check_launch("int4_group_quant_kernel", as_stream(stream));
  });
}

namespace ltm_b200 {
void launch_int4_dequant_rows(const uint8_t* packed, const float* s, const uint8_t* zp, int64_t N,
                              int64_t K, void* out, ltm_dtype dt, cudaStream_t st) {
  LTM_REQUIRE(K % 128 == 0 && K < (1ll << 31), "K must be a multiple of 128");
  LTM_REQUIRE(dt != LTM_DTYPE_F32, "16-bit dequantised weights");
  LTM_REQUIRE((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(out)) % 16 == 0,
              "packed weights and output must be 16-byte aligned");
  const int64_t total = N * (K / 32);
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, device_sm_count() * 16));
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    int4_dequant_rows_kernel<T><<<grid, 256, 0, st>>>(packed, s, zp, N, static_cast<int>(K),
                                                      static_cast<T*>(out));
  });
  check_launch("int4_dequant_rows_kernel", st);
}
}  // namespace ltm_b200

extern "C" ltm_status ltm_dequantize_int4_grouped(const uint8_t* packed, const float* s,
                                                  const uint8_t* zp, int64_t N, int64_t K,
                                                  int group_size, void* out, ltm_dtype out_dtype,
                                                  void* stream) {
  return guarded([&] {
    LTM_REQUIRE(N >= 0 && K >= 0, "negative size");
    LTM_REQUIRE(group_size > 0 && group_size % 2 == 0 && K % group_size == 0,
                "group_size must be even and divide K");
    if (N == 0 || K == 0) return;
    LTM_REQUIRE(packed && s && zp && out, "NULL pointer");
    dispatch_dtype(out_dtype, [&](auto tag) {
      using T = decltype(tag);
      int4_dequant_kernel<T><<<elementwise_grid(N * K / 2), 256, 0, as_stream(stream)>>>(
          packed, s, zp, N, K, group_size, static_cast<T*>(out));
    });
    check_launch("int4_dequant_kernel", as_stream(stream));
  });
}
