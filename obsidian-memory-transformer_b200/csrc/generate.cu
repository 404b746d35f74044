// generate.cu -- device side of a greedy generation loop: the next token of
// every sequence is the argmax of its logits row (ties: the lowest index), and
// its cache length moves on by one, all on the device, so a captured decode
// step plus this kernel can be replayed without the host in the loop.
//
// The reference's generation (python_bindings/ltm/inference.py:131-260)
// samples on the host with torch; greedy argmax is the temperature -> 0 case.
#include "block.cuh"

namespace ltm_b200 {
namespace {

template <class T>
__global__ void __launch_bounds__(256) greedy_next_kernel(const T* __restrict__ logits,
                                                          int64_t ld, int vocab,
                                                          int32_t* __restrict__ tokens,
                                                          int32_t* __restrict__ lens) {
  const int b = blockIdx.x;
  const T* row = logits + b * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = to_f32(row[i]);
    if (v > best || (v == best && i < bi)) {  // NaN never wins
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, s);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, s);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[8];
  __shared__ int si[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    tokens[b] = bi == 0x7fffffff ? 0 : bi;  // a row of NaNs yields token 0
    if (lens != nullptr) lens[b] += 1;
  }
}

}  // namespace

void launch_greedy_next(const void* logits, int64_t ld, ltm_dtype dt, int B, int vocab,
                        int32_t* tokens, int32_t* lens, cudaStream_t st) {
  if (B == 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    greedy_next_kernel<T><<<B, 256, 0, st>>>(static_cast<const T*>(logits), ld, vocab, tokens,
                                             lens);
  });
  check_launch("greedy_next_kernel", st);
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_greedy_next_tokens(const void* logits, ltm_dtype dtype, int B,
                                             int vocab, int32_t* tokens_out,
                                             int32_t* cache_lens, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(B >= 0 && vocab > 0, "bad size");
    if (B == 0) return;
    LTM_REQUIRE(logits && tokens_out, "NULL pointer");
    launch_greedy_next(logits, vocab, dtype, B, vocab, tokens_out, cache_lens, as_stream(stream));
  });
}
