// ref_launch.cu -- launchers (test infrastructure only) for the reference's own
// kernels, which oracle/ref_kernels.py copies verbatim from the reference tree
// into _ref/ref_kernels_extracted.cuh.  Each launcher uses the launch shape
// of the reference host function that calls the kernel:
//   symmetric / per-channel / linear quantize, dequantize: 256-thread blocks
//     over the elements (src/core/quantization/quantizer.cu:193-318)
//   layerNormResidualKernel: a block of 256 threads per row, 2 x 256 floats of
//     dynamic shared memory (src/core/ops/fused_ops.cu:233-259)
//   biasActivationKernel<T, GELU>: 256-thread blocks over the elements
//     (src/core/ops/fused_ops.cu:287-307)
//   storeStateKernel: a block per slot, a thread per hidden element
//     (src/core/ltm/memory_bank.cu:242-260)
// dtype: 0 = float, 1 = half (the reference instantiates these two).
// Every launcher returns the cudaError_t of the launch.
#include <memory>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "core/utils/cuda_utils.cuh"

namespace ltm {
namespace refk {
#include "ref_kernels_extracted.cuh"
}  // namespace refk
}  // namespace ltm

using namespace ltm::refk;

namespace {
inline int blocks_of(long n) { return static_cast<int>((n + 255) / 256); }
}  // namespace

#define REF_DISPATCH(dtype, CALL_F32, CALL_F16) \
  do {                                          \
    if ((dtype) == 0) {                         \
      CALL_F32;                                 \
    } else if ((dtype) == 1) {                  \
      CALL_F16;                                 \
    } else {                                    \
      return static_cast<int>(cudaErrorInvalidValue); \
    }                                           \
    return static_cast<int>(cudaGetLastError()); \
  } while (0)

extern "C" int ref_symmetric_quantize(const void* x, int dtype, int8_t* q, float scale, int n,
                                      void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n <= 0) return 0;
  REF_DISPATCH(dtype,
               (symmetricQuantizeKernel<float><<<blocks_of(n), 256, 0, st>>>(
                   static_cast<const float*>(x), q, scale, n)),
               (symmetricQuantizeKernel<half><<<blocks_of(n), 256, 0, st>>>(
                   static_cast<const half*>(x), q, scale, n)));
}

extern "C" int ref_linear_quantize(const void* x, int dtype, int8_t* q, float scale,
                                   float zero_point, int n, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n <= 0) return 0;
  REF_DISPATCH(dtype,
               (linearQuantizeKernel<float><<<blocks_of(n), 256, 0, st>>>(
                   static_cast<const float*>(x), q, scale, zero_point, n)),
               (linearQuantizeKernel<half><<<blocks_of(n), 256, 0, st>>>(
                   static_cast<const half*>(x), q, scale, zero_point, n)));
}

extern "C" int ref_per_channel_quantize(const void* x, int dtype, int8_t* q, const float* scales,
                                        const float* zero_points, int size, int channels,
                                        int elements_per_channel, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (size <= 0) return 0;
  REF_DISPATCH(dtype,
               (perChannelQuantizeKernel<float><<<blocks_of(size), 256, 0, st>>>(
                   static_cast<const float*>(x), q, scales, zero_points, size, channels,
                   elements_per_channel)),
               (perChannelQuantizeKernel<half><<<blocks_of(size), 256, 0, st>>>(
                   static_cast<const half*>(x), q, scales, zero_points, size, channels,
                   elements_per_channel)));
}

extern "C" int ref_per_channel_dequantize(const int8_t* q, void* out, int dtype,
                                          const float* scales, const float* zero_points, int size,
                                          int channels, int elements_per_channel, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (size <= 0) return 0;
  REF_DISPATCH(dtype,
               (perChannelDequantizeKernel<float><<<blocks_of(size), 256, 0, st>>>(
                   q, static_cast<float*>(out), scales, zero_points, size, channels,
                   elements_per_channel)),
               (perChannelDequantizeKernel<half><<<blocks_of(size), 256, 0, st>>>(
                   q, static_cast<half*>(out), scales, zero_points, size, channels,
                   elements_per_channel)));
}

extern "C" int ref_layernorm_residual(const void* x, const void* residual, const void* gamma,
                                      const void* beta, void* out, int dtype, int batch,
                                      int hidden, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (batch <= 0) return 0;
  const int smem = 2 * 256 * static_cast<int>(sizeof(float));
  REF_DISPATCH(dtype,
               (layerNormResidualKernel<float><<<batch, 256, smem, st>>>(
                   static_cast<const float*>(x), static_cast<const float*>(residual),
                   static_cast<const float*>(gamma), static_cast<const float*>(beta),
                   static_cast<float*>(out), batch, hidden)),
               (layerNormResidualKernel<half><<<batch, 256, smem, st>>>(
                   static_cast<const half*>(x), static_cast<const half*>(residual),
                   static_cast<const half*>(gamma), static_cast<const half*>(beta),
                   static_cast<half*>(out), batch, hidden)));
}

extern "C" int ref_bias_gelu(const void* x, const void* bias, void* out, int dtype, int batch,
                             int hidden, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long n = static_cast<long>(batch) * hidden;
  if (n <= 0) return 0;
  REF_DISPATCH(dtype,
               (biasActivationKernel<float, GELU><<<blocks_of(n), 256, 0, st>>>(
                   static_cast<const float*>(x), static_cast<const float*>(bias),
                   static_cast<float*>(out), batch, hidden)),
               (biasActivationKernel<half, GELU><<<blocks_of(n), 256, 0, st>>>(
                   static_cast<const half*>(x), static_cast<const half*>(bias),
                   static_cast<half*>(out), batch, hidden)));
}

// scores may be NULL (rate-only update).  slot_dim <= 1024 (one thread per
// element of a slot).
extern "C" int ref_store_state(void* memory, const void* state, const void* scores, float rate,
                               int num_slots, int slot_dim, int dtype, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (num_slots <= 0 || slot_dim <= 0) return 0;
  if (slot_dim > 1024) return static_cast<int>(cudaErrorInvalidValue);
  REF_DISPATCH(dtype,
               (storeStateKernel<float><<<num_slots, slot_dim, 0, st>>>(
                   static_cast<float*>(memory), static_cast<const float*>(state),
                   static_cast<const float*>(scores), rate, num_slots, slot_dim)),
               (storeStateKernel<half><<<num_slots, slot_dim, 0, st>>>(
                   static_cast<half*>(memory), static_cast<const half*>(state),
                   static_cast<const half*>(scores), rate, num_slots, slot_dim)));
}
