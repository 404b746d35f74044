// calibrate.cu -- activation-range calibrators for static INT8 scales
// (QuantizationCalibrator and its MinMax / Percentile / MSE subclasses,
// include/core/quantization/quantizer.cuh:124-175,
// src/core/quantization/calibrator.cu:61-264), on the device.
//
//   MinMax      running min and max of everything collected
//               (calibrator.cu:61-95); an order-preserving integer image of
//               each float makes the device atomics exact for negative values.
//   Percentile  the order statistics at the reference's indices
//               lo = (size_t)((100 - p) * n / 100), hi = (size_t)(p * n / 100)
//               in fp32 arithmetic (calibrator.cu:127-142; hi clamped to
//               n - 1), found by a 4-pass radix select over the collected
//               values (8 bits per pass, a 256-bin histogram each): exact,
//               no sort.
//   MSE         the clipping range [-c a, c a] (a = max |x|) of the 100 trials
//               c = 1/100 .. 100/100 whose symmetric INT8 quantize-dequantize
//               has the least squared error over the collected values (the
//               reference's loop, calibrator.cu:176-246, repeats one trial
//               100 times and keeps the data's min / max; the search it
//               stands for is restated here, first minimum wins).
//
// Collected values are kept on the device as fp32 (Percentile, MSE) in a
// buffer that grows by doubling; MinMax keeps two words.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

#include "block.cuh"

struct ltm_calibrator {
  int method = 0;
  float percentile = 99.9f;
  int device = 0;
  ltm_b200::DevBuf minmax;  // 2 x uint32 order-preserving images (min, max)
  ltm_b200::DevBuf values;  // fp32 [capacity]
  int64_t count = 0, capacity = 0;
  ltm_b200::DevBuf hist;    // 256 x uint32 (radix select) / 100 x double (MSE)
};

namespace ltm_b200 {
namespace {

// float -> uint32 whose unsigned order is the float order (NaNs above +inf).
__device__ __forceinline__ uint32_t ordered(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
inline float unordered(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

template <class T>
__global__ void __launch_bounds__(256) minmax_kernel(const T* __restrict__ x, int64_t n,
                                                     uint32_t* __restrict__ mm) {
  uint32_t lo = 0xffffffffu, hi = 0u;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t k = ordered(to_f32(x[i]));
    lo = min(lo, k);
    hi = max(hi, k);
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, s));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, s));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(mm, lo);
    atomicMax(mm + 1, hi);
  }
}

template <class T>
__global__ void __launch_bounds__(256) append_f32_kernel(const T* __restrict__ x, int64_t n,
                                                         float* __restrict__ dst) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = to_f32(x[i]);
}

// Histogram of bits [shift, shift + 8) of the keys whose bits above shift
// equal `prefix` (mask selects those bits).
__global__ void __launch_bounds__(256) radix_hist_kernel(const float* __restrict__ v, int64_t n,
                                                         uint32_t prefix, uint32_t mask, int shift,
                                                         uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[256];
  h[threadIdx.x] = 0;
  __syncthreads();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t k = ordered(v[i]);
    if ((k & mask) == prefix) atomicAdd(&h[(k >> shift) & 255u], 1u);
  }
  __syncthreads();
  if (h[threadIdx.x]) atomicAdd(&hist[threadIdx.x], h[threadIdx.x]);
}

// Squared error of the symmetric INT8 quantize-dequantize of v at each of
// the trial scales (blockIdx.y = trial), summed in fp64.
__global__ void __launch_bounds__(256) mse_trials_kernel(const float* __restrict__ v, int64_t n,
                                                         float amax, double* __restrict__ err) {
  const int t = blockIdx.y;
  const float clip = amax * static_cast<float>(t + 1) / 100.0f;
  const float s = clip / 127.0f;
  double acc = 0.0;
  if (s > 0.0f) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const float x = v[i];
      const float q = fminf(fmaxf(roundf(__fdiv_rn(x, s)), -127.0f), 127.0f);
      const float d = x - q * s;
      acc += static_cast<double>(d) * d;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(err + t, acc);
}

int grid_for(int64_t n) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256,
                                                                   device_sm_count() * 8)));
}

float order_statistic(ltm_calibrator* c, int64_t k, cudaStream_t st) {
  c->hist.ensure(256 * sizeof(uint32_t));
  uint32_t prefix = 0, mask = 0;
  uint32_t h[256];
  for (int shift = 24; shift >= 0; shift -= 8) {
    LTM_CUDA_TRY(cudaMemsetAsync(c->hist.ptr, 0, 256 * sizeof(uint32_t), st));
    radix_hist_kernel<<<grid_for(c->count), 256, 0, st>>>(c->values.as<float>(), c->count, prefix,
                                                          mask, shift, c->hist.as<uint32_t>());
    check_launch("radix_hist_kernel", st);
    LTM_CUDA_TRY(cudaMemcpyAsync(h, c->hist.ptr, sizeof(h), cudaMemcpyDeviceToHost, st));
    LTM_CUDA_TRY(cudaStreamSynchronize(st));
    int b = 0;
    for (; b < 256; ++b) {
      if (k < static_cast<int64_t>(h[b])) break;
      k -= h[b];
    }
    LTM_REQUIRE(b < 256, "radix select lost its rank");
    prefix |= static_cast<uint32_t>(b) << shift;
    mask |= 255u << shift;
  }
  return unordered(prefix);
}

// Static (calibrated) per-tensor INT8: q = clamp(round_half_away(x / scale),
// -127, 127) with IEEE division; scale 0 gives 0 (symmetricQuantizeKernel,
// src/core/quantization/quantizer.cu:93-105, with the clamp of the block's
// quantizers).
template <class T>
__global__ void __launch_bounds__(256) quant_static_kernel(const T* __restrict__ x, int64_t n,
                                                           float scale, int8_t* __restrict__ q) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float r = 0.0f;
    if (scale != 0.0f) r = fminf(fmaxf(roundf(__fdiv_rn(to_f32(x[i]), scale)), -127.0f), 127.0f);
    q[i] = static_cast<int8_t>(static_cast<int>(r));
  }
}

}  // namespace

void launch_quant_int8_static(const void* x, ltm_dtype dt, int64_t n, float scale, int8_t* q,
                              cudaStream_t st) {
  if (n == 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    quant_static_kernel<T><<<grid_for(n), 256, 0, st>>>(static_cast<const T*>(x), n, scale, q);
  });
  check_launch("quant_static_kernel", st);
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_calibrator_create(int method, float percentile, int device,
                                            ltm_calibrator** out) {
  return guarded([&] {
    LTM_REQUIRE(out, "out is NULL");
    LTM_REQUIRE(method >= LTM_CALIB_MINMAX && method <= LTM_CALIB_MSE, "unknown calibration method");
    LTM_REQUIRE(method != LTM_CALIB_PERCENTILE || (percentile >= 50.0f && percentile <= 100.0f),
                "percentile must lie in [50, 100]");
    auto c = std::make_unique<ltm_calibrator>();
    c->method = method;
    c->percentile = percentile;
    c->device = device;
    *out = c.release();
    LTM_REQUIRE(ltm_calibrator_reset(*out) == LTM_OK, "calibrator reset failed");
  });
}

extern "C" ltm_status ltm_calibrator_reset(ltm_calibrator* c) {
  return guarded([&] {
    LTM_REQUIRE(c, "NULL calibrator");
    c->count = 0;
    if (c->method == LTM_CALIB_MINMAX) {
      int prev = 0;
      LTM_CUDA_TRY(cudaGetDevice(&prev));
      LTM_CUDA_TRY(cudaSetDevice(c->device));
      c->minmax.ensure(2 * sizeof(uint32_t));
      const uint32_t init[2] = {0xffffffffu, 0u};
      LTM_CUDA_TRY(cudaMemcpy(c->minmax.ptr, init, sizeof(init), cudaMemcpyHostToDevice));
      cudaSetDevice(prev);
    }
  });
}

extern "C" ltm_status ltm_calibrator_collect(ltm_calibrator* c, const void* data, ltm_dtype dtype,
                                             int64_t n, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(c, "NULL calibrator");
    LTM_REQUIRE(n >= 0, "negative size");
    if (n == 0) return;
    LTM_REQUIRE(data, "NULL data");
    cudaStream_t st = as_stream(stream);
    if (c->method == LTM_CALIB_MINMAX) {
      dispatch_dtype(dtype, [&](auto tag) {
        using T = decltype(tag);
        minmax_kernel<T><<<grid_for(n), 256, 0, st>>>(static_cast<const T*>(data), n,
                                                       c->minmax.as<uint32_t>());
      });
      check_launch("minmax_kernel", st);
      c->count += n;
      return;
    }
    if (c->count + n > c->capacity) {  // grow by doubling, keeping what was collected
      int64_t cap = std::max<int64_t>(c->capacity * 2, c->count + n);
      cap = std::max<int64_t>(cap, 1 << 20);
      DevBuf grown;
      grown.ensure(static_cast<size_t>(cap) * sizeof(float));
      if (c->count)
        LTM_CUDA_TRY(cudaMemcpyAsync(grown.ptr, c->values.ptr, c->count * sizeof(float),
                                     cudaMemcpyDeviceToDevice, st));
      LTM_CUDA_TRY(cudaStreamSynchronize(st));
      std::swap(grown.ptr, c->values.ptr);
      std::swap(grown.bytes, c->values.bytes);
      c->capacity = cap;
    }
    dispatch_dtype(dtype, [&](auto tag) {
      using T = decltype(tag);
      append_f32_kernel<T><<<grid_for(n), 256, 0, st>>>(static_cast<const T*>(data), n,
                                                         c->values.as<float>() + c->count);
    });
    check_launch("calib_append_kernel", st);
    c->count += n;
  });
}

extern "C" ltm_status ltm_calibrator_compute_range(ltm_calibrator* c, float* min_val,
                                                   float* max_val, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(c && min_val && max_val, "NULL argument");
    cudaStream_t st = as_stream(stream);
    if (c->count == 0) {  // nothing collected: the reference's initial range
      *min_val = 0.0f;
      *max_val = 0.0f;
      return;
    }
    if (c->method == LTM_CALIB_MINMAX) {
      uint32_t mm[2];
      LTM_CUDA_TRY(cudaMemcpyAsync(mm, c->minmax.ptr, sizeof(mm), cudaMemcpyDeviceToHost, st));
      LTM_CUDA_TRY(cudaStreamSynchronize(st));
      *min_val = unordered(mm[0]);
      *max_val = unordered(mm[1]);
      return;
    }
    const int64_t n = c->count;
    if (c->method == LTM_CALIB_PERCENTILE) {
      const float p = c->percentile;
      int64_t lo = static_cast<int64_t>((100.0f - p) * static_cast<float>(n) / 100.0f);
      int64_t hi = static_cast<int64_t>(p * static_cast<float>(n) / 100.0f);
      lo = std::min<int64_t>(std::max<int64_t>(lo, 0), n - 1);
      hi = std::min<int64_t>(std::max<int64_t>(hi, 0), n - 1);
      *min_val = order_statistic(c, lo, st);
      *max_val = order_statistic(c, hi, st);
      return;
    }
    // MSE: amax over the values, then the 100 clipping trials
    DevBuf mm;
    mm.ensure(2 * sizeof(uint32_t));
    const uint32_t init[2] = {0xffffffffu, 0u};
    LTM_CUDA_TRY(cudaMemcpyAsync(mm.ptr, init, sizeof(init), cudaMemcpyHostToDevice, st));
    minmax_kernel<float><<<grid_for(n), 256, 0, st>>>(c->values.as<float>(), n, mm.as<uint32_t>());
    check_launch("minmax_kernel", st);
    uint32_t h[2];
    LTM_CUDA_TRY(cudaMemcpyAsync(h, mm.ptr, sizeof(h), cudaMemcpyDeviceToHost, st));
    LTM_CUDA_TRY(cudaStreamSynchronize(st));
    const float amax = std::max(std::fabs(unordered(h[0])), std::fabs(unordered(h[1])));
    c->hist.ensure(100 * sizeof(double));
    LTM_CUDA_TRY(cudaMemsetAsync(c->hist.ptr, 0, 100 * sizeof(double), st));
    const int gx = std::max(1, grid_for(n) / 8);
    mse_trials_kernel<<<dim3(gx, 100), 256, 0, st>>>(c->values.as<float>(), n, amax,
                                                      c->hist.as<double>());
    check_launch("mse_trials_kernel", st);
    double err[100];
    LTM_CUDA_TRY(cudaMemcpyAsync(err, c->hist.ptr, sizeof(err), cudaMemcpyDeviceToHost, st));
    LTM_CUDA_TRY(cudaStreamSynchronize(st));
    int best = 99;
    for (int t = 0; t < 100; ++t)
      if (err[t] < err[best] || (err[t] == err[best] && t < best)) best = t;
    const float clip = amax * static_cast<float>(best + 1) / 100.0f;
    *min_val = -clip;
    *max_val = clip;
  });
}

extern "C" ltm_status ltm_quantize_int8_static(const void* x, ltm_dtype dtype, int64_t n,
                                               float scale, int8_t* q, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(n >= 0 && std::isfinite(scale) && scale >= 0.0f, "bad size or scale");
    if (n == 0) return;
    LTM_REQUIRE(x && q, "NULL pointer");
    launch_quant_int8_static(x, dtype, n, scale, q, as_stream(stream));
  });
}

extern "C" ltm_status ltm_calibrator_destroy(ltm_calibrator* c) {
  return guarded([&] {
    if (!c) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    delete c;
    cudaSetDevice(prev);
  });
}
