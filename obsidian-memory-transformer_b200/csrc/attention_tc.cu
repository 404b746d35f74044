// attention_tc.cu -- flash attention on the 5th-generation tensor cores
// (16-bit inputs, fp32 softmax and accumulation).
//
//   o[t, h*D:(h+1)*D] = softmax_j( q_t . k_j / sqrt(D) ) v_j
//
// One CTA owns 128 queries of one (batch, head) and walks 128-key tiles:
//   warp 0     TMA: the Q tile once, K tiles into a 2-stage ring
//   warp 2     TMA: V tiles (single buffer, reloaded once P.V has consumed it)
//   warp 1     TMEM allocator + MMA issuer:
//                S  = Q K^T      kind::f16, M=128 N=128 K=D, Q and K K-major
//                PV = P V        kind::f16, M=128 N=D K=128, P K-major (smem),
//                                V MN-major (the [keys x D] tile as loaded)
//   warps 4-7  softmax (thread = query row = TMEM lane): two passes over its S
//              row in TMEM (raw row max, then p = 2^(s*scale - max*scale) on
//              FFMA + MUFU.EX2 and the row sum), P written as
//              16-bit into the 128-byte-swizzled K-major smem tile, the
//              previous tile's PV folded into the register accumulator O with
//              the online-softmax correction; O / l stored at the end.
// TMEM: S at columns [0,128), PV at [128, 128+D) (256 columns allocated), so
// two CTAs share an SM for D = 64.  Every mbarrier wait is bounded.
//
// Replaces chunkAttentionKernel (src/core/attention/flash_attention.cu:188-268,
// scale 1/sqrt(head_dim) :241) and the memory-attention score / softmax / PV
// chain (src/core/attention/memory_attention.cu:38-88,416-510); TB-v1 adds the
// max subtraction and the causal mask.
#include <type_traits>

#include "block.cuh"

namespace ltm_b200 {
namespace {

constexpr int kQM = 128;   // queries per CTA
constexpr int kKN = 128;   // keys per tile
constexpr uint32_t kChunk = 128 * 128;  // one [128 rows x 128 bytes] swizzled chunk

template <int D>
struct AttnSmem {
  static constexpr int DC = D / 64;                 // 128-byte chunks per row
  static constexpr uint32_t kQ = DC * kChunk;
  static constexpr uint32_t kK = DC * kChunk;
  static constexpr uint32_t kV = DC * kChunk;
  static constexpr uint32_t kP = 2 * kChunk;        // 128 x 128 16-bit
  static constexpr uint32_t kOffK = kQ;
  static constexpr uint32_t kOffV = kOffK + 2 * kK;
  static constexpr uint32_t kOffP = kOffV + kV;
  static constexpr uint32_t kOffBar = kOffP + kP;
  static constexpr uint32_t kBytes = kOffBar + 256 + 1024;
};

enum AttnBar : int {
  kBarQFull = 0, kBarKFull0, kBarKFull1, kBarKEmpty0, kBarKEmpty1, kBarVFull, kBarVEmpty,
  kBarSFull, kBarSFree, kBarPFull, kBarPVFull, kBarDrain, kNumBars
};


// Two floats rounded to a packed pair of 16-bit values (one paired convert).
template <class T>
__device__ __forceinline__ uint32_t pack2_16(float lo, float hi) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <class T, int D, bool CAUSAL>
__global__ void __launch_bounds__(256, (D <= 64 ? 2 : 1))
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, AttnParams p, int* err) {
  using L = AttnSmem<D>;
  constexpr int DC = L::DC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + L::kOffK;
  uint8_t* sV = smem + L::kOffV;
  uint8_t* sP = smem + L::kOffP;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = CAUSAL ? (gridDim.x - 1 - blockIdx.x) : blockIdx.x;  // heavy causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kQM;
  const int qrow0 = static_cast<int>(b * p.q_batch_rows) + q0;
  const int krow0 = static_cast<int>(b * p.kv_batch_rows);
  int kv_end = p.Skv;
  if (CAUSAL) kv_end = min(p.Skv, q0 + kQM + p.causal_offset);
  const int ntiles = kv_end > 0 ? (kv_end + kKN - 1) / kKN : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(bar + i, (i == kBarSFree || i == kBarPFull) ? 4 : 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) tmem_alloc(tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tPV = tmem + 128;

  if (warp == 0) {
    if (lane == 0 && ntiles > 0) {
      mbar_arrive_expect_tx(bar + kBarQFull, L::kQ);
      for (int c = 0; c < DC; ++c)
        tma_load_2d(sQ + c * kChunk, &tmQ, bar + kBarQFull, h * D + c * 64, qrow0);
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        if (!mbar_wait_bounded(bar + kBarKEmpty0 + s, ((j >> 1) & 1) ^ 1, abort_flag, err,
                               kErrWaitEmpty))
          break;
        mbar_arrive_expect_tx(bar + kBarKFull0 + s, L::kK);
        for (int c = 0; c < DC; ++c)
          tma_load_2d(sK + s * L::kK + c * kChunk, &tmK, bar + kBarKFull0 + s, h * D + c * 64,
                      krow0 + j * kKN);
        ++issued;
      }
      if (*abort_flag) {
        volatile int never = 0;
        mbar_wait_bounded(bar + kBarQFull, 0, &never, err, kErrWaitOther);
        for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
          mbar_wait_bounded(bar + kBarKFull0 + (j & 1), (j >> 1) & 1, &never, err, kErrWaitOther);
      }
    }
  } else if (warp == 2) {
    if (lane == 0 && ntiles > 0) {
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        if (!mbar_wait_bounded(bar + kBarVEmpty, (j & 1) ^ 1, abort_flag, err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(bar + kBarVFull, L::kV);
        for (int c = 0; c < DC; ++c)
          tma_load_2d(sV + c * kChunk, &tmV, bar + kBarVFull, h * D + c * 64, krow0 + j * kKN);
        ++issued;
      }
      if (*abort_flag && issued > 0) {
        volatile int never = 0;
        mbar_wait_bounded(bar + kBarVFull, (issued - 1) & 1, &never, err, kErrWaitOther);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && ntiles > 0) {
      constexpr bool kBF = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idS = idesc_f16(kQM, kKN, kBF);
      constexpr uint32_t idPV = idesc_f16(kQM, D, kBF, /*b_mn_major=*/true);
      const uint32_t aQ = smem_u32(sQ), aP = smem_u32(sP), aV = smem_u32(sV);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait_bounded(bar + kBarPFull, i & 1, abort_flag, err, kErrWaitFull)) return false;
        if (!mbar_wait_bounded(bar + kBarVFull, i & 1, abort_flag, err, kErrWaitFull)) return false;
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < kKN / 16; ++t)
          tc_mma_f16(tPV, make_desc_kmajor_sw128(aP + (t >> 2) * kChunk + (t & 3) * 32),
                     make_desc_mnmajor_sw128(aV + t * 2048, kChunk), idPV, t != 0);
        tc_commit(bar + kBarPVFull);
        tc_commit(bar + kBarVEmpty);
        return true;
      };
      bool ok = mbar_wait_bounded(bar + kBarQFull, 0, abort_flag, err, kErrWaitFull);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j & 1;
        if (!mbar_wait_bounded(bar + kBarKFull0 + s, (j >> 1) & 1, abort_flag, err, kErrWaitFull)) {
          ok = false;
          break;
        }
        if (j > 0 && !mbar_wait_bounded(bar + kBarSFree, (j - 1) & 1, abort_flag, err, kErrWaitOther)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + s * L::kK);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          tc_mma_f16(tS, make_desc_kmajor_sw128(aQ + (k >> 2) * kChunk + (k & 3) * 32),
                     make_desc_kmajor_sw128(aK + (k >> 2) * kChunk + (k & 3) * 32), idS, k != 0);
        tc_commit(bar + kBarSFull);
        tc_commit(bar + kBarKEmpty0 + s);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(ntiles - 1);
      if (*abort_flag) {
        volatile int never = 0;
        tc_commit(bar + kBarDrain);
        mbar_wait_bounded(bar + kBarDrain, 0, &never, err, kErrWaitOther);
      }
    }
  } else if (warp >= 4) {
    // ---- softmax warpgroup: thread = query row r = TMEM lane r
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.0f;
    float m = -INFINITY, l = 0.0f, corr_prev = 0.0f;
    bool ok = true;  // with no key tile at all the output is written as zeros
    for (int j = 0; ok && j < ntiles; ++j) {
      if (!mbar_wait_bounded(bar + kBarSFull, j & 1, abort_flag, err, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * kKN;
      const bool need_mask = (k0 + kKN > p.Skv) || (CAUSAL && k0 + kKN - 1 > q0 + p.causal_offset);
      const int kmax = CAUSAL ? min(p.Skv - 1, qi + p.causal_offset) : p.Skv - 1;  // last visible key
      // pass 1: row max of the raw scores (the positive scale commutes with max)
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kKN / 32; ++c) {
        uint32_t sr[32];
        tmem_ld_32x32b_x32(tS + lane_off + c * 32, sr);
        tmem_wait_ld();
        if (!need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, __uint_as_float(sr[i]));
        } else {
          const int kb = k0 + c * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            mx = fmaxf(mx, kb + i <= kmax ? __uint_as_float(sr[i]) : -INFINITY);
        }
      }
      const float m_new = fmaxf(m, mx);  // raw-score units
      const float msc = (m_new == -INFINITY) ? 0.0f : m_new * p.scale_log2;
      const float corr = ex2_approx(fmaf(m, p.scale_log2, -msc));  // m = -inf -> 0
      // fold the previous tile's P.V (relative to the previous max)
      if (j > 0) {
        if (!mbar_wait_bounded(bar + kBarPVFull, (j - 1) & 1, abort_flag, err, kErrWaitAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t pv[32];
          tmem_ld_32x32b_x32(tPV + lane_off + c * 32, pv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], corr_prev, __uint_as_float(pv[i]));
        }
      }
      // pass 2: P = 2^(s * scale - max * scale) as 16-bit into the swizzled K-major tile
      float rs = 0.0f;
#pragma unroll 1
      for (int c = 0; c < kKN / 32; ++c) {
        uint32_t sr[32];
        tmem_ld_32x32b_x32(tS + lane_off + c * 32, sr);
        tmem_wait_ld();
        float pv[32];
        if (!need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) pv[i] = ex2_approx(fmaf(__uint_as_float(sr[i]), p.scale_log2, -msc));
        } else {
          const int kb = k0 + c * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            pv[i] = kb + i <= kmax ? ex2_approx(fmaf(__uint_as_float(sr[i]), p.scale_log2, -msc)) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) rs += pv[i];
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // 4 x 16-byte chunks = 32 keys
          const int cc = c * 4 + u;      // 16-byte chunk index within the 256-byte row
          uint4 w;
          w.x = pack2_16<T>(pv[8 * u + 0], pv[8 * u + 1]);
          w.y = pack2_16<T>(pv[8 * u + 2], pv[8 * u + 3]);
          w.z = pack2_16<T>(pv[8 * u + 4], pv[8 * u + 5]);
          w.w = pack2_16<T>(pv[8 * u + 6], pv[8 * u + 7]);
          *reinterpret_cast<uint4*>(sP + (cc >> 3) * kChunk + r * 128 + (((cc & 7) ^ (r & 7)) << 4)) = w;
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar + kBarSFree);
        mbar_arrive(bar + kBarPFull);
      }
      l = l * corr + rs;
      m = m_new;
      corr_prev = corr;
    }
    if (ok && ntiles > 0) {
      ok = mbar_wait_bounded(bar + kBarPVFull, (ntiles - 1) & 1, abort_flag, err, kErrWaitAccum);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t pv[32];
          tmem_ld_32x32b_x32(tPV + lane_off + c * 32, pv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], corr_prev, __uint_as_float(pv[i]));
        }
      }
    }
    if (ok && qi < p.Sq && !*abort_flag) {
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      T* og = static_cast<T*>(p.o) + (b * p.q_batch_rows + qi) * p.ldo + h * D;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        uint4 w;
        w.x = pack2_16<T>(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
        w.y = pack2_16<T>(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
        w.z = pack2_16<T>(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
        w.w = pack2_16<T>(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
        *reinterpret_cast<uint4*>(og + 8 * c) = w;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <class T, int D, bool CAUSAL>
void launch_inst(const AttnParams& p, int B, cudaStream_t stream) {
  using L = AttnSmem<D>;
  const CUtensorMapDataType dt = std::is_same<T, __nv_bfloat16>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t width = static_cast<uint64_t>(p.nh) * D;
  const uint64_t q_rows = static_cast<uint64_t>(B) * p.q_batch_rows;
  const uint64_t kv_rows = p.kv_batch_rows == 0 ? static_cast<uint64_t>(p.Skv)
                                                : static_cast<uint64_t>(B) * p.kv_batch_rows;
  CUtensorMap tq, tk, tv;
  make_tma_2d(&tq, p.q, dt, 2, q_rows, width, p.ldq, 64, kQM);
  make_tma_2d(&tk, p.k, dt, 2, kv_rows, width, p.ldk, 64, kKN);
  make_tma_2d(&tv, p.v, dt, 2, kv_rows, width, p.ldv, 64, kKN);
  auto kern = attn_tc_kernel<T, D, CAUSAL>;
  LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  dim3 grid((p.Sq + kQM - 1) / kQM, p.nh, B);
  kern<<<grid, 256, L::kBytes, stream>>>(tq, tk, tv, p, device_error_ptr());
  check_launch(CAUSAL ? "attn_tc_kernel/causal" : "attn_tc_kernel/full", stream);
}

}  // namespace

// 16-bit flash attention on tcgen05 (head_dim 64 or 128).  p.scale_log2 set.
void launch_attention_tc(const AttnParams& p, int B, int D, bool causal, ltm_dtype dt,
                         cudaStream_t stream) {
  LTM_REQUIRE(dt == LTM_DTYPE_F16 || dt == LTM_DTYPE_BF16, "tensor-core attention needs 16-bit data");
  LTM_REQUIRE(B * p.q_batch_rows < (1ll << 31) && B * p.kv_batch_rows < (1ll << 31),
              "attention rows exceed int32");
  auto go = [&](auto tag, auto d_c, auto c_c) {
    using T = decltype(tag);
    launch_inst<T, decltype(d_c)::value, decltype(c_c)::value>(p, B, stream);
  };
  auto by_t = [&](auto d_c, auto c_c) {
    if (dt == LTM_DTYPE_BF16) go(__nv_bfloat16{}, d_c, c_c);
    else go(__half{}, d_c, c_c);
  };
  using I64 = std::integral_constant<int, 64>;
  using I128 = std::integral_constant<int, 128>;
  if (D == 64) causal ? by_t(I64{}, std::true_type{}) : by_t(I64{}, std::false_type{});
  else causal ? by_t(I128{}, std::true_type{}) : by_t(I128{}, std::false_type{});
}

}  // namespace ltm_b200
