// norm.cu -- LayerNorm of (x + x) with an optional fused per-token INT8
// quantization of its output and of the raw input, plus the embedding gather.
//
// LN follows src/core/ops/fused_ops.cu:15-86 as TitanBlock::layerNorm calls
// it (residual = input, src/core/transformer/titan_inspired_block.cu:374-389):
// v = x + x, two-pass mean / variance over the row, eps 1e-5,
// y = (v - mean) * rsqrt(var + eps) * gamma + beta.  One CTA per row, each
// thread owns one 16-byte vector of the row in registers, so the row is read
// from HBM exactly once; reductions are warp shuffles + one shared-memory hop.
#include <type_traits>

#include "block.cuh"

namespace ltm_b200 {
namespace {

template <int NW>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < NW; ++i) t += (i * 32 < static_cast<int>(blockDim.x)) ? red[i] : 0.0f;
  return t;
}

template <int NW>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < NW; ++i) t = fmaxf(t, (i * 32 < static_cast<int>(blockDim.x)) ? red[i] : 0.0f);
  return t;
}


// Warp-uniform quantize + store of V values (all lanes call; `valid` lanes store).
template <int V>
__device__ __forceinline__ void store_q_warp(int8_t* dst, const float (&v)[V], float s, float inv,
                                             bool valid) {
  int8_t o[V];
  quant_i8_exact_warp<V>(v, s, inv, o);
  if (!valid) return;
  if constexpr (V == 8)
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
  else
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(o);
}

template <class T, int V>
__device__ __forceinline__ void store_q(int8_t* dst, const float (&v)[V], float s, float inv) {
  int8_t o[V];
#pragma unroll
  for (int i = 0; i < V; ++i) o[i] = quant_i8_exact(v[i], s, inv);
  if constexpr (V == 8)
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
  else
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(o);
}

// One CTA per row; thread t owns elements [t*V, t*V+V).  NW = max warps.
template <class T, int NW>
__global__ void __launch_bounds__(NW * 32) ln_x2_kernel(const T* __restrict__ x,
                                                        const T* __restrict__ res, int H,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ beta,
                                                        T* __restrict__ y, int8_t* __restrict__ yq,
                                                        float* __restrict__ ys,
                                                        int8_t* __restrict__ xq,
                                                        float* __restrict__ xs, int do_norm) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[NW];
  const int64_t row = blockIdx.x;
  const int e0 = threadIdx.x * V;
  const bool active = e0 < H;
  float xv[V], rv[V];
#pragma unroll
  for (int i = 0; i < V; ++i) xv[i] = rv[i] = 0.0f;
  if (active) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + row * H + e0));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) xv[i] = to_f32(e[i]);
    if (res == x) {
#pragma unroll
      for (int i = 0; i < V; ++i) rv[i] = xv[i];
    } else {
      uint4 rr = __ldg(reinterpret_cast<const uint4*>(res + row * H + e0));
      const T* er = reinterpret_cast<const T*>(&rr);
#pragma unroll
      for (int i = 0; i < V; ++i) rv[i] = to_f32(er[i]);
    }
  }
  if (xq) {
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) am = fmaxf(am, fabsf(xv[i]));
    am = block_max<NW>(am, red);
    const float s = __fdiv_rn(am, 127.0f);
    if (active) store_q<T, V>(xq + row * H + e0, xv, s, recip_or_zero(s));
    if (threadIdx.x == 0) xs[row] = s;
  }
  float yv[V];
  if (do_norm) {
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) sum += xv[i] + rv[i];
    const float mean = block_sum<NW>(sum, red) / static_cast<float>(H);
    float sq = 0.0f;
    if (active) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float d = (xv[i] + rv[i]) - mean;
        sq += d * d;
      }
    }
    const float var = block_sum<NW>(sq, red) / static_cast<float>(H);
    const float rstd = rsqrtf(var + 1e-5f);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = active ? e0 + i : 0;
      yv[i] = ((xv[i] + rv[i]) - mean) * rstd * __ldg(gamma + c) + __ldg(beta + c);
    }
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) yv[i] = xv[i];
  }
  if (y && active) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) e[i] = from_f32<T>(yv[i]);
    *reinterpret_cast<uint4*>(y + row * H + e0) = raw;
  }
  if (yq) {
    float am = 0.0f;
    if (active) {
#pragma unroll
      for (int i = 0; i < V; ++i) am = fmaxf(am, fabsf(yv[i]));
    }
    am = block_max<NW>(am, red);
    const float s = __fdiv_rn(am, 127.0f);
    if (active) store_q<T, V>(yq + row * H + e0, yv, s, recip_or_zero(s));
    if (threadIdx.x == 0) ys[row] = s;
  }
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per row, the row resident in registers: lane l owns the 16-byte
// vectors l, l+32, ... (NV of them).  Same arithmetic as ln_x2_kernel; all
// reductions are warp shuffles.  Persistent grid (8 warps per CTA, grid-stride
// over rows) with the next row prefetched.  SAME: residual == x.
// Row reductions of ln_x2_warp_kernel: a warp-shuffle tree, then (WPR = 8:
// the CTA's eight warps share the row) the eight warp results in order
// through a double-buffered shared array, one barrier per reduction.
template <int WPR>
struct RowReduce {
  float* red;  // [2][WPR]
  int par = 0;
  __device__ __forceinline__ float sum(float v) {
    v = warp_sum_f(v);
    if constexpr (WPR == 1) {
      return v;
    } else {
      if ((threadIdx.x & 31) == 0) red[par * WPR + (threadIdx.x >> 5)] = v;
      __syncthreads();
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < WPR; ++w) t += red[par * WPR + w];
      par ^= 1;
      return t;
    }
  }
  __device__ __forceinline__ float max(float v) {
    v = warp_max_f(v);
    if constexpr (WPR == 1) {
      return v;
    } else {
      if ((threadIdx.x & 31) == 0) red[par * WPR + (threadIdx.x >> 5)] = v;
      __syncthreads();
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < WPR; ++w) t = fmaxf(t, red[par * WPR + w]);
      par ^= 1;
      return t;
    }
  }
};

// Three 256-thread CTAs per SM (80 registers) where that spills nothing:
// more rows in flight, 1.7x the throughput at hidden 8192 (measured; codes
// and scales unchanged).
template <class T, int NV, bool SAME, int WPR>
constexpr int ln_min_blocks() {
  return (SAME && (NV <= 3 || (WPR == 8 && NV <= 4))) ? 3 : 1;
}

template <class T, int NV, bool SAME, int WPR = 1>
__global__ void __launch_bounds__(256, (ln_min_blocks<T, NV, SAME, WPR>())) ln_x2_warp_kernel(const T* __restrict__ x,
                                                         const T* __restrict__ res, int64_t rows,
                                                         int H, const float* __restrict__ gamma,
                                                         const float* __restrict__ beta,
                                                         T* __restrict__ y, int8_t* __restrict__ yq,
                                                         float* __restrict__ ys,
                                                         int8_t* __restrict__ xq,
                                                         float* __restrict__ xs, int do_norm) {
  constexpr int V = 16 / sizeof(T);
  constexpr int GROUPS = 8 / WPR;    // row groups per 256-thread CTA
  constexpr int STRIDE = 32 * WPR;   // vectors between a lane's consecutive vectors
  static_assert(WPR == 1 || WPR == 8, "one warp or the whole CTA per row");
  __shared__ float red_s[2 * WPR];
  RowReduce<WPR> rr_{red_s};
  // lane: this thread's index within its row group
  const int lane = (WPR == 1) ? static_cast<int>(threadIdx.x & 31) : static_cast<int>(threadIdx.x);
  const int64_t g0 = static_cast<int64_t>(blockIdx.x) * GROUPS + (WPR == 1 ? (threadIdx.x >> 5) : 0);
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * GROUPS;
  const int nvec = H / V;
  // persistent: the next row's loads are in flight while this row is processed
  constexpr int NR = SAME ? 1 : NV;
  uint4 cx[NV], cr[NR], nx[NV], nr[NR];
  auto load = [&](int64_t rr, uint4 (&ax)[NV], uint4 (&ar)[NR]) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int vi = lane + STRIDE * j;
      ax[j] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(x + rr * H) + vi) : make_uint4(0, 0, 0, 0);
      if constexpr (!SAME)
        ar[j] = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(res + rr * H) + vi)
                          : make_uint4(0, 0, 0, 0);
    }
  };
  if (g0 < rows) load(g0, cx, cr);
  for (int64_t row = g0; row < rows; row += gstride) {
  if (row + gstride < rows) load(row + gstride, nx, nr);
  // xv holds x; sv holds x + residual (the LN input) unless SAME
  float xv[NV][V], sv[SAME ? 1 : NV][V];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const T* e = reinterpret_cast<const T*>(&cx[j]);
#pragma unroll
    for (int i = 0; i < V; ++i) xv[j][i] = to_f32(e[i]);
    if constexpr (!SAME) {
      const T* er = reinterpret_cast<const T*>(&cr[j]);
#pragma unroll
      for (int i = 0; i < V; ++i) sv[j][i] = xv[j][i] + to_f32(er[i]);
    }
  }
  auto lnin = [&](int j, int i) -> float {
    if constexpr (SAME) return xv[j][i] + xv[j][i];
    else return sv[j][i];
  };
  if (xq) {
    float am = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int i = 0; i < V; ++i) am = fmaxf(am, fabsf(xv[j][i]));
    am = rr_.max(am);
    const float s = __fdiv_rn(am, 127.0f);
    const float inv = recip_or_zero(s);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int vi = lane + STRIDE * j;
      store_q_warp<V>(xq + row * H + vi * V, xv[j], s, inv, vi < nvec);
    }
    if (lane == 0) xs[row] = s;
  }
  if (do_norm) {
    // the LN arithmetic on packed fp32 pairs (two IEEE operations per
    // instruction); the sums run as two interleaved partial sums per lane
    static_assert(V % 2 == 0, "values in pairs");
    uint64_t in2[NV][V / 2];
    uint64_t sum2 = f2_pack(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int i = 0; i < V; i += 2) {
        in2[j][i / 2] = f2_pack(lnin(j, i), lnin(j, i + 1));
        sum2 = f2_add(sum2, in2[j][i / 2]);
      }
    float s0, s1;
    f2_unpack(sum2, s0, s1);
    const float mean = rr_.sum(s0 + s1) / static_cast<float>(H);
    const uint64_t mean2 = f2_pack(mean, mean);
    uint64_t sq2 = f2_pack(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (lane + STRIDE * j < nvec) {
#pragma unroll
        for (int i = 0; i < V / 2; ++i) {
          const uint64_t d = f2_sub(in2[j][i], mean2);
          sq2 = f2_fma(d, d, sq2);
        }
      }
    }
    f2_unpack(sq2, s0, s1);
    const float var = rr_.sum(s0 + s1) / static_cast<float>(H);
    const float rstd = rsqrtf(var + 1e-5f);
    const uint64_t rstd2 = f2_pack(rstd, rstd);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int vi = lane + STRIDE * j;
      const int c0 = vi < nvec ? vi * V : 0;
#pragma unroll
      for (int i = 0; i < V; i += 4) {  // gamma / beta are 16-byte aligned (checked by the launcher)
        const float4 g4 = __ldg(reinterpret_cast<const float4*>(gamma + c0 + i));
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(beta + c0 + i));
        const uint64_t n0 = f2_mul(f2_sub(in2[j][i / 2], mean2), rstd2);
        const uint64_t n1 = f2_mul(f2_sub(in2[j][i / 2 + 1], mean2), rstd2);
        f2_unpack(f2_fma(n0, f2_pack(g4.x, g4.y), f2_pack(b4.x, b4.y)), xv[j][i], xv[j][i + 1]);
        f2_unpack(f2_fma(n1, f2_pack(g4.z, g4.w), f2_pack(b4.z, b4.w)), xv[j][i + 2], xv[j][i + 3]);
      }
    }
  } else if constexpr (!SAME) {
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int i = 0; i < V; ++i) xv[j][i] = sv[j][i];
  }
  if (y) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int vi = lane + STRIDE * j;
      if (vi < nvec) {
        uint4 raw;
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int i = 0; i < V; ++i) e[i] = from_f32<T>(xv[j][i]);
        *(reinterpret_cast<uint4*>(y + row * H) + vi) = raw;
      }
    }
  }
  if (yq) {
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (lane + STRIDE * j >= nvec)
#pragma unroll
        for (int i = 0; i < V; ++i) xv[j][i] = 0.0f;
    float am = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int i = 0; i < V; ++i) am = fmaxf(am, fabsf(xv[j][i]));
    am = rr_.max(am);
    const float s = __fdiv_rn(am, 127.0f);
    const float inv = recip_or_zero(s);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int vi = lane + STRIDE * j;
      store_q_warp<V>(yq + row * H + vi * V, xv[j], s, inv, vi < nvec);
    }
    if (lane == 0) ys[row] = s;
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    cx[j] = nx[j];
    if constexpr (!SAME) cr[j] = nr[j];
  }
  }  // rows
}

template <class T>
__global__ void __launch_bounds__(256) embed_gather_kernel(const T* __restrict__ table, int vocab,
                                                           int H, const int32_t* __restrict__ tok,
                                                           int64_t T_, T* __restrict__ out, int* err) {
  constexpr int V = 16 / sizeof(T);
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T_) return;
  const int lane = threadIdx.x & 31;
  const int id = tok[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && lane == 0) atomicCAS(err, 0, 16);
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<int64_t>(ok ? id : 0) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + t * H);
  for (int j = lane; j < H / V; j += 32) dst[j] = ok ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
}

}  // namespace

// y (optional, dtype T) = LN(x + x); yq/ys (optional) = per-token int8 of the
// fp32 LN output; xq/xs (optional) = per-token int8 of x.  do_norm = 0 skips
// the normalisation (y = x).
void launch_ln_x2(const void* x, ltm_dtype dt, int64_t rows, int H, const float* gamma,
                  const float* beta, void* y, int8_t* yq, float* ys, int8_t* xq, float* xs,
                  bool do_norm, cudaStream_t stream, const void* residual) {
  if (rows == 0) return;
  const int V = static_cast<int>(16 / dtype_size(dt));
  LTM_REQUIRE(H % V == 0, "hidden size must be a multiple of 16 bytes");
  const int threads = ((H / V + 31) / 32) * 32;  // fallback: one thread per vector
  LTM_REQUIRE(H / V <= 2048, "hidden size too large for the row-resident LayerNorm");
  LTM_REQUIRE(!do_norm || ((reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0,
              "LayerNorm gamma / beta must be 16-byte aligned");
  const int nv = (H / V + 31) / 32;  // 16-byte vectors per lane, warp-per-row layout
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    const T* xt = static_cast<const T*>(x);
    const T* rt = static_cast<const T*>(residual ? residual : x);
    const int64_t want_blocks = (rows + 7) / 8;
    auto warp_launch = [&](auto nv_c, auto wpr_c) {
      constexpr int NV = decltype(nv_c)::value;
      constexpr int WPR = decltype(wpr_c)::value;
      const int64_t want = WPR == 1 ? want_blocks : rows;
      if (rt == xt) {
        auto kern = ln_x2_warp_kernel<T, NV, true, WPR>;
        kern<<<persistent_grid(kern, 256, 0, want), 256, 0, stream>>>(
            xt, rt, rows, H, gamma, beta, static_cast<T*>(y), yq, ys, xq, xs, do_norm ? 1 : 0);
      } else {
        auto kern = ln_x2_warp_kernel<T, NV, false, WPR>;
        kern<<<persistent_grid(kern, 256, 0, want), 256, 0, stream>>>(
            xt, rt, rows, H, gamma, beta, static_cast<T*>(y), yq, ys, xq, xs, do_norm ? 1 : 0);
      }
    };
    using W1 = std::integral_constant<int, 1>;
    using W8 = std::integral_constant<int, 8>;
    const int nv8 = (H / V + 255) / 256;  // 16-byte vectors per thread, CTA-per-row layout
    if (nv <= 8) {
      switch (nv) {
        case 1: warp_launch(std::integral_constant<int, 1>{}, W1{}); break;
        case 2: warp_launch(std::integral_constant<int, 2>{}, W1{}); break;
        case 3: warp_launch(std::integral_constant<int, 3>{}, W1{}); break;
        case 4: warp_launch(std::integral_constant<int, 4>{}, W1{}); break;
        case 5: case 6: warp_launch(std::integral_constant<int, 6>{}, W1{}); break;
        default: warp_launch(std::integral_constant<int, 8>{}, W1{}); break;
      }
    } else if (nv8 <= 8) {  // a 256-thread CTA per row (hidden up to 2048 vectors)
      switch (nv8) {
        case 2: warp_launch(std::integral_constant<int, 2>{}, W8{}); break;
        case 3: warp_launch(std::integral_constant<int, 3>{}, W8{}); break;
        case 4: warp_launch(std::integral_constant<int, 4>{}, W8{}); break;
        case 5: case 6: warp_launch(std::integral_constant<int, 6>{}, W8{}); break;
        default: warp_launch(std::integral_constant<int, 8>{}, W8{}); break;
      }
    } else {
      LTM_REQUIRE(threads <= 1024, "hidden size too large for the row-resident LayerNorm");
      ln_x2_kernel<T, 32><<<static_cast<unsigned>(rows), threads, 0, stream>>>(
          xt, rt, H, gamma, beta, static_cast<T*>(y), yq, ys, xq, xs, do_norm ? 1 : 0);
    }
  });
  check_launch("ln_x2_kernel", stream);
}

void launch_embed_gather(const void* table, ltm_dtype dt, int vocab, int H, const int32_t* tok,
                         int64_t T, void* out, cudaStream_t stream) {
  if (T == 0) return;
  LTM_REQUIRE((H * dtype_size(dt)) % 16 == 0, "hidden size must be a multiple of 16 bytes");
  dispatch_dtype(dt, [&](auto tag) {
    using TT = decltype(tag);
    embed_gather_kernel<TT><<<static_cast<unsigned>((T + 7) / 8), 256, 0, stream>>>(
        static_cast<const TT*>(table), vocab, H, tok, T, static_cast<TT*>(out), device_error_ptr());
  });
  check_launch("embed_gather_kernel", stream);
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_layernorm_residual(const void* x, const void* r, const float* gamma,
                                             const float* beta, void* y, ltm_dtype dtype,
                                             int64_t rows, int64_t H, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(rows >= 0 && H > 0 && H < (1 << 20), "bad size");
    if (rows == 0) return;
    LTM_REQUIRE(x && r && gamma && beta && y, "NULL pointer");
    const uintptr_t mis = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(r) |
                          reinterpret_cast<uintptr_t>(y);
    LTM_REQUIRE((mis & 15) == 0, "operands must be 16-byte aligned");
    launch_ln_x2(x, dtype, rows, static_cast<int>(H), gamma, beta, y, nullptr, nullptr, nullptr,
                 nullptr, true, as_stream(stream), r);
  });
}
