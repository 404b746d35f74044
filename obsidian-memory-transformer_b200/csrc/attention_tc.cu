// attention_tc.cu -- flash attention on the 5th-generation tensor cores
// (16-bit inputs, fp32 softmax and accumulation).
//
//   o[t, h*D:(h+1)*D] = softmax_j( q_t . k_j / sqrt(D) ) v_j
//
// One CTA owns 128 queries of one (batch, head) and walks 64-key tiles:
//   warp 0     TMA: the Q tile once, K tiles into a 2-stage ring
//   warp 2     TMA: V tiles into a 2-stage ring
//   warp 1     TMEM allocator + MMA issuer, in the order S(0), S(1), S(2),
//              PV(0), S(3), PV(1), ... (S(j+2) as soon as the softmax has read
//              S(j)) so that the tensor core computes the scores of later tiles
//              while tile j is in the softmax:
//                S[j%2] = Q K^T  kind::f16, M=128 N=64 K=D (Q, K K-major)
//                O     += P V    kind::f16, M=128 N=D K=64 (P K-major in
//                                smem, V MN-major as loaded)
//   warps 4-7  softmax (thread = query row = TMEM lane): one TMEM read of its
//              S row into registers (the S buffer is released right after),
//              the row max, p = 2^(s*scale - m_ref*scale) on FFMA + MUFU.EX2
//              and the row sum, P written as 16-bit into the 128-byte-swizzled
//              K-major smem tile.  O accumulates in TMEM across tiles; m_ref is
//              the row's reference max, raised -- with O and the sum rescaled in
//              place -- only when the running max exceeds it by more than 2^8
//              (so p <= 256; the final O / l is the same for any reference).
// TMEM: S0 [0,64), S1 [64,128), O [128, 128+D) of 256 columns, so two CTAs
// share an SM.  Every mbarrier wait is bounded.
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
constexpr int kKN = 64;    // keys per tile
constexpr uint32_t kChunk = 128 * 128;   // one [128 rows x 128 bytes] swizzled chunk (Q, P)
constexpr uint32_t kKChunk = kKN * 128;  // one [64 rows x 128 bytes] swizzled chunk (K, V)
constexpr float kRescaleLog2 = 8.0f;    // lazy-rescale threshold (log2 units)

template <int D>
struct AttnSmem {
  static constexpr int DC = D / 64;                 // 128-byte chunks per row
  // V tiles in flight: two for D = 64; one for D = 128, which keeps the CTA
  // under half of the SM's shared memory so that two CTAs share an SM
  static constexpr int VST = D <= 64 ? 2 : 1;
  // P tiles: two for D = 64 (the softmax writes P(j+1) while P(j).V(j) runs),
  // one for D = 128 (shared-memory budget of two CTAs per SM)
  static constexpr int PST = D <= 64 ? 2 : 1;
  static constexpr uint32_t kQ = DC * kChunk;
  static constexpr uint32_t kK = DC * kKChunk;
  static constexpr uint32_t kV = DC * kKChunk;
  static constexpr uint32_t kP = kChunk;            // 128 queries x 64 keys, 16-bit
  static constexpr uint32_t kOffK = kQ;
  static constexpr uint32_t kOffV = kOffK + 2 * kK;
  static constexpr uint32_t kOffP = kOffV + VST * kV;
  static constexpr uint32_t kOffBar = kOffP + PST * kP;
  static constexpr uint32_t kBytes = kOffBar + 256 + 1024;
};

enum AttnBar : int {
  kBarQFull = 0, kBarKFull0, kBarKFull1, kBarKEmpty0, kBarKEmpty1, kBarVFull0, kBarVFull1,
  kBarVEmpty0, kBarVEmpty1, kBarSFull0, kBarSFull1, kBarSFree0, kBarSFree1, kBarPFull0,
  kBarPFull1, kBarPVDone0, kBarPVDone1, kBarDrain, kNumBars
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
__global__ void __launch_bounds__(256, 2)
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
    for (int i = 0; i < kNumBars; ++i) {
      const bool per_warp = i == kBarSFree0 || i == kBarSFree1 || i == kBarPFull0 ||
                            i == kBarPFull1;
      mbar_init(bar + i, per_warp ? 4 : 1);
    }
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
  const uint32_t tO = tmem + 2 * kKN;

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
          tma_load_2d(sK + s * L::kK + c * kKChunk, &tmK, bar + kBarKFull0 + s, h * D + c * 64,
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
        const int s = j % L::VST;
        const uint32_t use = static_cast<uint32_t>(j / L::VST);
        if (!mbar_wait_bounded(bar + kBarVEmpty0 + s, (use & 1) ^ 1, abort_flag, err,
                               kErrWaitEmpty))
          break;
        mbar_arrive_expect_tx(bar + kBarVFull0 + s, L::kV);
        for (int c = 0; c < DC; ++c)
          tma_load_2d(sV + s * L::kV + c * kKChunk, &tmV, bar + kBarVFull0 + s, h * D + c * 64,
                      krow0 + j * kKN);
        ++issued;
      }
      if (*abort_flag) {
        volatile int never = 0;
        for (int j = (issued > L::VST ? issued - L::VST : 0); j < issued; ++j)
          mbar_wait_bounded(bar + kBarVFull0 + (j % L::VST), (j / L::VST) & 1, &never, err,
                            kErrWaitOther);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && ntiles > 0) {
      constexpr bool kBF = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idS = idesc_f16(kQM, kKN, kBF);
      constexpr uint32_t idPV = idesc_f16(kQM, D, kBF, /*b_mn_major=*/true);
      const uint32_t aQ = smem_u32(sQ), aP = smem_u32(sP);
      // S(j) = Q K(j)^T into S buffer j % 2 (the softmax has released it)
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait_bounded(bar + kBarKFull0 + s, (j >> 1) & 1, abort_flag, err, kErrWaitFull))
          return false;
        if (j >= 2 && !mbar_wait_bounded(bar + kBarSFree0 + s, ((j - 2) >> 1) & 1, abort_flag, err,
                                         kErrWaitOther))
          return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + s * L::kK);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          tc_mma_f16(tmem + s * kKN, make_desc_kmajor_sw128(aQ + (k >> 2) * kChunk + (k & 3) * 32),
                     make_desc_kmajor_sw128(aK + (k >> 2) * kKChunk + (k & 3) * 32), idS, k != 0);
        tc_commit(bar + kBarSFull0 + s);
        tc_commit(bar + kBarKEmpty0 + s);
        return true;
      };
      // O (+)= P(i) V(i) once the softmax has written P(i) (and rescaled O)
      auto issue_pv = [&](int i) -> bool {
        const int s = i % L::VST;
        const int pb = i % L::PST;
        if (!mbar_wait_bounded(bar + kBarPFull0 + pb, (i / L::PST) & 1, abort_flag, err,
                               kErrWaitFull))
          return false;
        if (!mbar_wait_bounded(bar + kBarVFull0 + s, (i / L::VST) & 1, abort_flag, err,
                               kErrWaitFull))
          return false;
        tc_fence_after();
        const uint32_t aV = smem_u32(sV + s * L::kV);
        const uint32_t aPb = aP + pb * L::kP;
#pragma unroll
        for (int t = 0; t < kKN / 16; ++t)
          tc_mma_f16(tO, make_desc_kmajor_sw128(aPb + t * 32),
                     make_desc_mnmajor_sw128(aV + t * 2048, kKChunk), idPV, (i | t) != 0);
        tc_commit(bar + kBarPVDone0 + pb);
        tc_commit(bar + kBarVEmpty0 + s);
        return true;
      };
      bool ok = mbar_wait_bounded(bar + kBarQFull, 0, abort_flag, err, kErrWaitFull);
      if (ok) ok = issue_s(0);
      if (ok && ntiles > 1) ok = issue_s(1);
      // S(j+2) as soon as the softmax has read S(j) (early in its tile), then
      // P(j).V(j) once it has written P(j): the scores of tile j+2 are computed
      // during tile j's exponentials
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 2 < ntiles) ok = issue_s(j + 2);
        if (ok) ok = issue_pv(j);
      }
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
    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY, l = 0.0f;
    // waits whose outcome is the same for the whole warp (the TMEM accesses
    // that follow are warp-collective)
    auto wait_warp = [&](int bi, uint32_t parity, int code) -> bool {
      const bool r = mbar_wait_bounded(bar + bi, parity, abort_flag, err, code);
      return __all_sync(0xffffffffu, r);
    };
    bool ok = true;  // with no key tile at all the output is written as zeros
    for (int j = 0; ok && j < ntiles; ++j) {
      const int sb = j & 1;
      if (!wait_warp(kBarSFull0 + sb, (j >> 1) & 1, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      constexpr int NC = kKN / 32;
      uint32_t sr[NC][32];
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_ld_32x32b_x32(tmem + sb * kKN + lane_off + c * 32, sr[c]);
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_wait_ld_tie(sr[c]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar + kBarSFree0 + sb);  // S buffer may be overwritten
      const int k0 = j * kKN;
      const bool need_mask = (k0 + kKN > p.Skv) || (CAUSAL && k0 + kKN - 1 > q0 + p.causal_offset);
      if (need_mask) {
        const int kmax = CAUSAL ? min(p.Skv - 1, qi + p.causal_offset) : p.Skv - 1;
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (k0 + c * 32 + i > kmax) sr[c][i] = __float_as_uint(-INFINITY);
      }
      // row max: eight independent partial maxima (short dependency chains)
      float pm[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pm[u] = -INFINITY;
#pragma unroll
      for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) pm[i & 7] = fmaxf(pm[i & 7], __uint_as_float(sr[c][i]));
      const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      // raise the reference max (and rescale O, l) only past the threshold
      const bool raise = (m_ref == -INFINITY) ? (mx > -INFINITY)
                                              : ((mx - m_ref) * sl2 > kRescaleLog2);
      bool pv_waited = false;
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        const float m_new = fmaxf(m_ref, mx);
        const float f = (m_ref == -INFINITY) ? 0.0f : ex2_approx((m_ref - m_new) * sl2);
        // O is final up to P(j-1).V(j-1)
        if (!wait_warp(kBarPVDone0 + (j - 1) % L::PST, ((j - 1) / L::PST) & 1, kErrWaitAccum)) {
          ok = false;
          break;
        }
        pv_waited = true;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tO + lane_off + c * 32, ov);
          tmem_wait_ld_tie(ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * f);
          tmem_st_32x32b_x32(tO + lane_off + c * 32, ov);
        }
        tmem_wait_st();
        l *= f;
        m_ref = m_new;
      } else if (j == 0) {
        m_ref = mx;
      }
      const float msc = (m_ref == -INFINITY) ? 0.0f : m_ref * sl2;
      // P = 2^(s*scale - m_ref*scale), the row sum, and P as 16-bit pairs
      float ps[8];  // eight independent partial row sums
#pragma unroll
      for (int u = 0; u < 8; ++u) ps[u] = 0.0f;
      uint32_t pk[NC * 16];
#pragma unroll
      for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float a = ex2_approx(fmaf(__uint_as_float(sr[c][i]), sl2, -msc));
          const float bb = ex2_approx(fmaf(__uint_as_float(sr[c][i + 1]), sl2, -msc));
          ps[(i >> 1) & 7] += a + bb;
          pk[c * 16 + i / 2] = pack2_16<T>(a, bb);
        }
      l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      // P buffer j % PST is free once P(j-PST).V(j-PST) has completed
      if (j >= L::PST && !pv_waited &&
          !wait_warp(kBarPVDone0 + j % L::PST, ((j - L::PST) / L::PST) & 1, kErrWaitAccum)) {
        ok = false;
        break;
      }
#pragma unroll
      uint8_t* sPb = sP + (j % L::PST) * L::kP;
#pragma unroll
      for (int cc = 0; cc < NC * 4; ++cc) {  // 16-byte unit cc of the row's 128 bytes
        uint4 w;
        w.x = pk[cc * 4 + 0];
        w.y = pk[cc * 4 + 1];
        w.z = pk[cc * 4 + 2];
        w.w = pk[cc * 4 + 3];
        *reinterpret_cast<uint4*>(sPb + r * 128 + ((cc ^ (r & 7)) << 4)) = w;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar + kBarPFull0 + j % L::PST);
    }
    if (ok && ntiles > 0)  // the last P.V (and, in order, every earlier one) has completed
      ok = wait_warp(kBarPVDone0 + (ntiles - 1) % L::PST, ((ntiles - 1) / L::PST) & 1,
                     kErrWaitAccum);
    const bool aborted = __shfl_sync(0xffffffffu, *abort_flag, 0) != 0;
    // The TMEM reads are warp-collective (.sync.aligned): the whole warp takes
    // this branch (ok, ntiles and the abort flag are the same for its lanes)
    // and only the global stores depend on the lane's row.
    if (ok && ntiles > 0 && !aborted) {
      tc_fence_after();
      const bool store = qi < p.Sq;
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      T* og = static_cast<T*>(p.o) + (b * p.q_batch_rows + (store ? qi : 0)) * p.ldo + h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(tO + lane_off + c * 32, ov);
        tmem_wait_ld_tie(ov);
        if (store) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w;
            w.x = pack2_16<T>(__uint_as_float(ov[8 * u + 0]) * inv, __uint_as_float(ov[8 * u + 1]) * inv);
            w.y = pack2_16<T>(__uint_as_float(ov[8 * u + 2]) * inv, __uint_as_float(ov[8 * u + 3]) * inv);
            w.z = pack2_16<T>(__uint_as_float(ov[8 * u + 4]) * inv, __uint_as_float(ov[8 * u + 5]) * inv);
            w.w = pack2_16<T>(__uint_as_float(ov[8 * u + 6]) * inv, __uint_as_float(ov[8 * u + 7]) * inv);
            *reinterpret_cast<uint4*>(og + c * 32 + 8 * u) = w;
          }
        }
      }
    } else if (ok && ntiles == 0 && qi < p.Sq) {
      T* og = static_cast<T*>(p.o) + (b * p.q_batch_rows + qi) * p.ldo + h * D;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) *reinterpret_cast<uint4*>(og + 8 * c) = make_uint4(0, 0, 0, 0);
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
