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
// kv_batch_rows = 0).  16-bit path: 8 warps x 16 query rows per CTA
// (128-query tiles), 64-key tiles double-buffered with cp.async into
// XOR-swizzled shared memory, QK^T and PV on m16n8k16 tensor-core MMAs, P
// kept in registers.  fp32 path: SIMT kernel, one warp per query row.
#include <type_traits>

#include "block.cuh"

namespace ltm_b200 {



namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <class T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <class T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  T a = from_f32<T>(lo), b = from_f32<T>(hi);
  uint16_t ua = *reinterpret_cast<uint16_t*>(&a), ub = *reinterpret_cast<uint16_t*>(&b);
  return static_cast<uint32_t>(ua) | (static_cast<uint32_t>(ub) << 16);
}

// element offset of (row, 16-byte chunk) in a [rows, D] tile with the chunk
// index XOR-swizzled by (row & 7): conflict-free ldmatrix and cp.async.
template <int D>
__device__ __forceinline__ int swz(int row, int chunk) {
  return row * D + ((chunk ^ (row & 7)) << 3);
}

template <class T, int D, bool CAUSAL>
__global__ void __launch_bounds__(256, (D <= 64 ? 2 : 1)) flash_fwd_tc_kernel(AttnParams p) {
  constexpr int BM = 128, BN = 64, CH = D / 8, KS = D / 16;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  T* sQ = reinterpret_cast<T*>(smem_raw);
  T* sK = sQ + BM * D;       // 2 stages
  T* sV = sK + 2 * BN * D;   // 2 stages

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // heaviest causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * BM;

  const T* qg = static_cast<const T*>(p.q) + (b * p.q_batch_rows + q0) * p.ldq + h * D;
  const T* kg = static_cast<const T*>(p.k) + (b * p.kv_batch_rows) * p.ldk + h * D;
  const T* vg = static_cast<const T*>(p.v) + (b * p.kv_batch_rows) * p.ldv + h * D;

  int kv_end = p.Skv;
  if (CAUSAL) kv_end = min(p.Skv, q0 + BM + p.causal_offset);
  const int ntiles = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;

  for (int i = tid; i < BM * CH; i += 256) {
    const int r = i / CH, c = i % CH;
    const bool ok = q0 + r < p.Sq;
    cp_async16(sQ + swz<D>(r, c), qg + (ok ? static_cast<int64_t>(r) * p.ldq + c * 8 : 0), ok);
  }
  auto load_kv = [&](int t, int st) {
    const int k0 = t * BN;
    T* dk = sK + st * BN * D;
    T* dv = sV + st * BN * D;
    for (int i = tid; i < BN * CH; i += 256) {
      const int r = i / CH, c = i % CH;
      const bool ok = k0 + r < p.Skv;
      const int64_t rr = ok ? static_cast<int64_t>(k0 + r) : 0;
      cp_async16(dk + swz<D>(r, c), kg + rr * p.ldk + c * 8, ok);
      cp_async16(dv + swz<D>(r, c), vg + rr * p.ldv + c * 8, ok);
    }
  };
  if (ntiles > 0) load_kv(0, 0);
  cp_async_commit();

  uint32_t qf[KS][4];
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};
  const int row_a = q0 + warp * 16 + (lane >> 2);  // query index of c0/c1; +8 for c2/c3

  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) load_kv(t + 1, (t + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(qf[ks], sQ + swz<D>(r, c));
      }
    }
    const T* cK = sK + (t & 1) * BN * D;
    const T* cV = sV + (t & 1) * BN * D;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t kb[4];
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(kb, cK + swz<D>(r, c));
        mma16816<T>(s[2 * jp], qf[ks], kb[0], kb[1]);
        mma16816<T>(s[2 * jp + 1], qf[ks], kb[2], kb[3]);
      }
    }
    // scale, mask, online softmax (rows row_a and row_a + 8)
    const int k0 = t * BN;
    const bool need_mask = (k0 + BN > p.Skv) || (CAUSAL && k0 + BN - 1 > q0 + p.causal_offset);
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * p.scale_log2;
        if (need_mask) {
          const int key = k0 + j * 8 + (lane & 3) * 2 + (e & 1);
          const int qi = row_a + ((e >> 1) << 3);
          if (key >= p.Skv || (CAUSAL && key > qi + p.causal_offset)) v = -INFINITY;
        }
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mref = (mx[r] == -INFINITY) ? 0.0f : mx[r];
      corr[r] = exp2f(m_r[r] - mref);
      m_r[r] = mx[r];
      mx[r] = mref;
    }
    float rs[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = exp2f(s[j][e] - mx[e >> 1]);
        s[j][e] = pe;
        rs[e >> 1] += pe;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_r[r] = l_r[r] * corr[r] + rs[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t vb[4];
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp * 2 + (lane >> 4);
        ldsm_x4_t(vb, cV + swz<D>(r, c));
        mma16816<T>(o[2 * dp], pa, vb[0], vb[1]);
        mma16816<T>(o[2 * dp + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // finalize: reduce row sums across the quad, normalise, stage through sQ
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  const float inv0 = l_r[0] > 0.0f ? 1.0f / l_r[0] : 0.0f;
  const float inv1 = l_r[1] > 0.0f ? 1.0f / l_r[1] : 0.0f;
  __syncthreads();
  {
    const int r0 = warp * 16 + (lane >> 2);
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int col = i * 8 + (lane & 3) * 2;
      const int ch = col >> 3, within = col & 7;
      *reinterpret_cast<uint32_t*>(sQ + swz<D>(r0, ch) + within) = pack2<T>(o[i][0] * inv0, o[i][1] * inv0);
      *reinterpret_cast<uint32_t*>(sQ + swz<D>(r0 + 8, ch) + within) =
          pack2<T>(o[i][2] * inv1, o[i][3] * inv1);
    }
  }
  __syncthreads();
  T* og = static_cast<T*>(p.o) + (b * p.q_batch_rows + q0) * p.ldo + h * D;
  for (int i = tid; i < BM * CH; i += 256) {
    const int r = i / CH, c = i % CH;
    if (q0 + r < p.Sq)
      *reinterpret_cast<uint4*>(og + static_cast<int64_t>(r) * p.ldo + c * 8) =
          *reinterpret_cast<const uint4*>(sQ + swz<D>(r, c));
  }
}

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

template <class T, int D, bool CAUSAL>
void launch_tc(const AttnParams& p, int B, cudaStream_t stream) {
  constexpr int BM = 128, BN = 64;
  const size_t smem = (BM * D + 4 * BN * D) * sizeof(T);
  auto kern = flash_fwd_tc_kernel<T, D, CAUSAL>;
  LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  dim3 grid((p.Sq + BM - 1) / BM, p.nh, B);
  kern<<<grid, 256, smem, stream>>>(p);
  check_launch("flash_fwd_tc_kernel");
}

template <int D, bool CAUSAL>
void launch_f32(const AttnParams& p, int B, cudaStream_t stream) {
  dim3 grid((p.Sq + 3) / 4, p.nh, B);
  flash_fwd_f32_kernel<D, CAUSAL><<<grid, 128, 0, stream>>>(p);
  check_launch("flash_fwd_f32_kernel");
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
  auto go = [&](auto d_c, auto c_c) {
    constexpr int DD = decltype(d_c)::value;
    constexpr bool CC = decltype(c_c)::value;
    if (dt == LTM_DTYPE_F16) launch_tc<__half, DD, CC>(p, B, stream);
    else if (dt == LTM_DTYPE_BF16) launch_tc<__nv_bfloat16, DD, CC>(p, B, stream);
    else launch_f32<DD, CC>(p, B, stream);
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
