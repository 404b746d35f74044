// attention.cu -- causal self-attention and memory attention (queries x
// memory slots) as online-softmax flash kernels.
//
//   o[t, h*D:(h+1)*D] = softmax_j( q_t . k_j / sqrt(D) ) v_j      (fp32 softmax/accum)
//
// replacing chunkAttentionKernel (src/core/attention/flash_attention.cu:188-268;
// scale 1/sqrt(head_dim) :241) and the memory-attention scores / softmax / PV
// chain (src/core/attention/memory_attention.cu:38-88,416-510).  TB-v1 adds
// the max subtraction and the causal mask the reference omits.
//
// Q, K, V are read in place from the projection outputs (row stride ld*,
// head h at column h*D); K/V may be shared by all batch rows (memory bank:
// kv_batch_rows = 0).  16-bit data runs on the tcgen05 kernel of
// attention_tc.cu; this file holds the fp32 SIMT kernel (one warp per query
// row) and the dispatch.
#include <type_traits>

#include "block.cuh"

namespace ltm_b200 {
namespace {

// fp32 SIMT attention: one warp per (query row, head); key tiles of K and V
// staged in shared memory (K rows padded to avoid bank conflicts); each lane
// scores KPL keys of a tile, the output dims are spread over the lanes.
template <int D, bool CAUSAL>
__global__ void __launch_bounds__(128) flash_fwd_f32_kernel(AttnParams p) {
  constexpr int BN = (D <= 64) ? 64 : 32, KPL = BN / 32, DP = D + 1, PER = D / 32;
  __shared__ float sK[BN * DP];
  __shared__ float sV[BN * D];
  __shared__ float sQ[4][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int q_base = blockIdx.x * 4;  // 4 queries per CTA, one per warp
  const int qi = q_base + warp;
  const float* kg = static_cast<const float*>(p.k) + (b * p.kv_batch_rows) * p.ldk + h * D;
  const float* vg = static_cast<const float*>(p.v) + (b * p.kv_batch_rows) * p.ldv + h * D;
  const bool qok = qi < p.Sq;
  {
    const float* qg = static_cast<const float*>(p.q) + (b * p.q_batch_rows + (qok ? qi : 0)) * p.ldq + h * D;
#pragma unroll
    for (int i = 0; i < PER; ++i) sQ[warp][lane + 32 * i] = qg[lane + 32 * i];
  }
  int kv_end = p.Skv;
  if (CAUSAL) kv_end = min(p.Skv, q_base + 4 + p.causal_offset);
  float m = -INFINITY, l = 0.0f, acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.0f;
  for (int k0 = 0; k0 < kv_end; k0 += BN) {
    __syncthreads();
    for (int i = threadIdx.x; i < BN * D; i += 128) {
      const int r = i / D, c = i % D;
      const bool ok = k0 + r < p.Skv;
      sK[r * DP + c] = ok ? kg[static_cast<int64_t>(k0 + r) * p.ldk + c] : 0.0f;
      sV[r * D + c] = ok ? vg[static_cast<int64_t>(k0 + r) * p.ldv + c] : 0.0f;
    }
    __syncthreads();
    float sc[KPL];
    float mx = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < KPL; ++jj) {
      const int j = lane + 32 * jj;
      float d = 0.0f;
#pragma unroll 8
      for (int e = 0; e < D; ++e) d += sQ[warp][e] * sK[j * DP + e];
      const int key = k0 + j;
      float v = d * p.scale_log2;
      if (key >= p.Skv || (CAUSAL && key > qi + p.causal_offset)) v = -INFINITY;
      sc[jj] = v;
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mnew = fmaxf(m, mx);
    const float mref = mnew == -INFINITY ? 0.0f : mnew;
    const float corr = exp2f(m - mref);
    float ps = 0.0f;
#pragma unroll
    for (int jj = 0; jj < KPL; ++jj) {
      sc[jj] = exp2f(sc[jj] - mref);
      ps += sc[jj];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l = l * corr + ps;
    m = mnew;
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] *= corr;
#pragma unroll
    for (int jj = 0; jj < KPL; ++jj) {
      for (int j = 0; j < 32; ++j) {
        const float pj = __shfl_sync(0xffffffffu, sc[jj], j);
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[i] += pj * sV[(jj * 32 + j) * D + lane + 32 * i];
      }
    }
  }
  if (qok) {
    float* og = static_cast<float*>(p.o) + (b * p.q_batch_rows + qi) * p.ldo + h * D;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) og[lane + 32 * i] = acc[i] * inv;
  }
}

template <int D, bool CAUSAL>
void launch_f32(const AttnParams& p, int B, cudaStream_t stream) {
  dim3 grid((p.Sq + 3) / 4, p.nh, B);
  flash_fwd_f32_kernel<D, CAUSAL><<<grid, 128, 0, stream>>>(p);
  check_launch("flash_fwd_f32_kernel", stream);
}

}  // namespace

void launch_attention(const AttnParams& p_in, int B, int D, bool causal, ltm_dtype dt,
                      cudaStream_t stream) {
  if (B == 0 || p_in.Sq == 0 || p_in.nh == 0) return;
  AttnParams p = p_in;
  p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  LTM_REQUIRE(D == 64 || D == 128, "head_dim must be 64 or 128");
  if (dt != LTM_DTYPE_F32) {
    const uintptr_t mis = reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
                          reinterpret_cast<uintptr_t>(p.v) | reinterpret_cast<uintptr_t>(p.o);
    LTM_REQUIRE((mis & 15) == 0, "attention operands must be 16-byte aligned");
    LTM_REQUIRE(p.ldq % 8 == 0 && p.ldk % 8 == 0 && p.ldv % 8 == 0 && p.ldo % 8 == 0,
                "attention row strides must be multiples of 8 elements");
  }
  if (dt != LTM_DTYPE_F32) {
    launch_attention_tc(p, B, D, causal, dt, stream);
    return;
  }
  auto go = [&](auto d_c, auto c_c) {
    constexpr int DD = decltype(d_c)::value;
    constexpr bool CC = decltype(c_c)::value;
    launch_f32<DD, CC>(p, B, stream);
  };
  using I64 = std::integral_constant<int, 64>;
  using I128 = std::integral_constant<int, 128>;
  using T_ = std::true_type;
  using F_ = std::false_type;
  if (D == 64) causal ? go(I64{}, T_{}) : go(I64{}, F_{});
  else causal ? go(I128{}, T_{}) : go(I128{}, F_{});
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_attention_forward(const void* q, int64_t ldq, const void* k, int64_t ldk,
                                            const void* v, int64_t ldv, void* o, int64_t ldo, int B,
                                            int Sq, int Skv, int64_t kv_batch_rows, int num_heads,
                                            int head_dim, int causal, ltm_dtype dtype,
                                            void* stream) {
  return guarded([&] {
    LTM_REQUIRE(B >= 0 && Sq >= 0 && Skv >= 0 && num_heads >= 0 && kv_batch_rows >= 0, "bad size");
    if (B == 0 || Sq == 0 || num_heads == 0) return;
    LTM_REQUIRE(q && k && v && o, "NULL pointer");
    LTM_REQUIRE(ldq >= static_cast<int64_t>(num_heads) * head_dim &&
                    ldk >= static_cast<int64_t>(num_heads) * head_dim &&
                    ldv >= static_cast<int64_t>(num_heads) * head_dim &&
                    ldo >= static_cast<int64_t>(num_heads) * head_dim,
                "row strides smaller than num_heads * head_dim");
    if (head_dim != 64 && head_dim != 128) LTM_UNSUPPORTED("head_dim must be 64 or 128");
    AttnParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o;
    p.ldq = ldq;
    p.ldk = ldk;
    p.ldv = ldv;
    p.ldo = ldo;
    p.q_batch_rows = Sq;
    p.kv_batch_rows = kv_batch_rows;
    p.Sq = Sq;
    p.Skv = Skv;
    p.nh = num_heads;
    p.causal_offset = Skv - Sq;
    launch_attention(p, B, head_dim, causal != 0, dtype, as_stream(stream));
  });
}
