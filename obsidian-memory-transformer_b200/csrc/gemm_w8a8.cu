// gemm_w8a8.cu -- W8A8 linear on the 5th-generation tensor cores.
//
//   acc[m,n] = sum_k qa[m,k] * qw[n,k]     int8 x int8 -> exact int32 in TMEM
//   y        = epilogue(acc)                dequant, bias, act, rope/resid/gate-mix
//
// The same kernels, instantiated on 16-bit operands (kind::f16, fp32
// accumulators; the stage tiling is in bytes, so a 128-byte K row holds 64
// elements), are the GEMM of the W4A16 linear at large M: the INT4 weight is
// dequantised once per call into a 16-bit scratch and contracted here
// (launch_gemm_f16).
//
// Persistent kernel, one CTA per SM, static round-robin over 128 x BN output
// tiles (N-tile fastest, so the CTAs in flight share activation rows and the
// whole weight stays L2-resident; for weights too large for L2 -- the 16-bit
// instantiation at hidden 4096 -- M-tile fastest inside groups of gm row
// blocks, so a group's activation band stays L2-resident while the weight
// streams once per group).  Warp roles (320 threads):
//   warp 0      TMA producer: 128 x 128-byte tiles of qa and BN x 128-byte
//               tiles of qw into a STAGES-deep ring (128-byte swizzle); runs
//               ahead across tile boundaries
//   warp 1      TMEM allocator + MMA issuer: 4 x tcgen05.mma kind::i8 (K = 32)
//               per stage into one of two TMEM accumulators (2 x BN columns),
//               tcgen05.commit frees the stage / publishes the accumulator
//   warps 2..9  epilogue (two warpgroups, each half of the tile's columns):
//               tcgen05.ld of the int32 accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), fused epilogue, staged coalesced
//               stores; overlaps the next tile's main loop
// Every mbarrier wait is bounded (common.cuh); an expired wait records a code
// in the device error word and the CTA unwinds, releasing its TMEM.
//
// Replaces the CUTLASS 2.x Sm80 half GEMM of the reference
// (src/core/ops/mma_ops.cu:20-92) for the quantized linears.
#include <algorithm>
#include <type_traits>

#include "block.cuh"
#include "epilogue.cuh"

namespace ltm_b200 {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage = one 128-byte swizzle row
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN, int STAGES>
struct W8A8Smem {
  static constexpr uint32_t kA = kBM * kBK;
  static constexpr uint32_t kB = BN * kBK;
  static constexpr uint32_t kStage = kA + kB;  // multiple of 1024
  static constexpr uint32_t kStgOff = STAGES * kStage;
  static constexpr uint32_t kStgWarp = 2 * 32 * 128;  // two 4 KiB TMA-store boxes per warp
  static constexpr uint32_t kColOff = kStgOff + kEpiWarps * kStgWarp;
  static constexpr uint32_t kColWarp = 2 * (BN / 2) * 4;  // scale + bias of the warp's columns
  static constexpr uint32_t kBarOff = kColOff + kEpiWarps * kColWarp;
  static constexpr uint32_t kBytes = kBarOff + 256 + 1024;  // barriers + alignment slack
};

// MMA of one 32-byte K slice: int8 (kind::i8) or 16-bit (kind::f16) operands.
template <class AT, bool PAIR>
__device__ __forceinline__ void mma_k32(uint32_t tacc, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  if constexpr (sizeof(AT) == 1) {
    if constexpr (PAIR) tc_mma_i8_pair(tacc, a, b, idesc, acc);
    else tc_mma_i8(tacc, a, b, idesc, acc);
  } else {
    if constexpr (PAIR) tc_mma_f16_pair(tacc, a, b, idesc, acc);
    else tc_mma_f16(tacc, a, b, idesc, acc);
  }
}

template <class AT>
__host__ __device__ constexpr uint32_t idesc_of(int M, int N) {
  if constexpr (sizeof(AT) == 1) return idesc_i8(M, N);
  else return idesc_f16(M, N, std::is_same<AT, __nv_bfloat16>::value);
}

// Row / column block of tile t: N fastest when gm <= 0, else M fastest
// inside groups of gm row blocks (the last group may be shorter).
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int gm, int& mb,
                                            int& nb) {
  if (gm <= 0) {
    mb = t / num_n;
    nb = t - mb * num_n;
    return;
  }
  const int per = gm * num_n;
  const int g = t / per, r = t - g * per;
  const int mg = min(gm, num_m - g * gm);
  mb = g * gm + r % mg;
  nb = r / mg;
}

template <int BN, int STAGES, int MODE, class OutT, class AT>
__global__ void __launch_bounds__(kThreads, 1)
    w8a8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, int M, int N, int K, int gm, Epilogue ep,
                   int* err) {
  using L = W8A8Smem<BN, STAGES>;
  constexpr int kKe = kBK / static_cast<int>(sizeof(AT));  // K elements per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2] accumulator ready
  uint64_t* acce = accf + 2;        // [2] accumulator drained by the epilogue
  uint64_t* drain = acce + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_n = (N + BN - 1) / BN;
  const int num_m = (M + kBM - 1) / kBM;
  const int tiles = num_m * num_n;
  const int nkb = (K + kKe - 1) / kKe;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) tmem_alloc(tslot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, gm, mb, nb);
        const int m0 = mb * kBM, n0 = nb * BN;
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(empty + s, ph ^ 1, abort_flag, err, kErrWaitEmpty)) break;
          uint8_t* a_dst = smem + s * L::kStage;
          mbar_arrive_expect_tx(full + s, L::kStage);
          tma_load_2d(a_dst, &tmA, full + s, kb * kKe, m0);
          tma_load_2d(a_dst + L::kA, &tmB, full + s, kb * kKe, n0);
          ++it;
        }
      }
      if (*abort_flag) {
        // Drain this CTA's copies still in flight before the CTA unwinds.
        volatile int never = 0;
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
          mbar_wait_bounded(full + (j % STAGES), (j / STAGES) & 1, &never, err, kErrWaitOther);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_of<AT>(kBM, BN);
      int it = 0, lt = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++lt) {
        const int b = lt & 1;
        const uint32_t use = static_cast<uint32_t>(lt >> 1);
        if (!mbar_wait_bounded(acce + b, (use & 1) ^ 1, abort_flag, err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint32_t tacc = tmem + b * BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(full + s, ph, abort_flag, err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * L::kStage);
          const uint32_t b_addr = a_addr + L::kA;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            mma_k32<AT, false>(tacc, make_desc_kmajor_sw128(a_addr + k * 32),
                               make_desc_kmajor_sw128(b_addr + k * 32), idesc, (kb | k) != 0);
          }
          tc_commit(empty + s);
          ++it;
        }
        if (!ok) break;
        tc_commit(accf + b);
      }
      if (*abort_flag) {
        volatile int never = 0;
        tc_commit(drain);
        mbar_wait_bounded(drain, 0, &never, err, kErrWaitOther);
      }
    }
  } else {
    // Epilogue warps 2..9: TMEM lane quarter q = warp % 4 (tile rows
    // 32q..32q+31), column half (warp - 2) / 4 of the tile.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stg = smem + L::kStgOff + (warp - 2) * L::kStgWarp;
    float* cvec = reinterpret_cast<float*>(smem + L::kColOff + (warp - 2) * L::kColWarp);
    TmaTileEpilogue<MODE, OutT, BN / 2, sizeof(AT) == 1> epi;
    auto rows_of = [&](int t) {
      int mb, nb;
      tile_coords(t, num_m, num_n, gm, mb, nb);
      return mb * kBM + q * 32;
    };
    auto cols_of = [&](int t) {
      int mb, nb;
      tile_coords(t, num_m, num_n, gm, mb, nb);
      return nb * BN + half * (BN / 2);
    };
    if (static_cast<int>(blockIdx.x) < tiles)
      epi.prefetch(ep, rows_of(blockIdx.x) + lane, cols_of(blockIdx.x), M, N, lane);
    int lt = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++lt) {
      const int b = lt & 1;
      const uint32_t use = static_cast<uint32_t>(lt >> 1);
      const int row0 = rows_of(t), nw = cols_of(t);
      // warp-uniform outcome: the epilogue's TMEM loads are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(accf + b, use & 1, abort_flag, err,
                                                     kErrWaitAccum)))
        break;
      tc_fence_after();
      // publish this tile's column vectors, then fetch the next tile's
      epi.run(ep, &tmO, tmem + b * BN + half * (BN / 2) + (static_cast<uint32_t>(q * 32) << 16),
              row0 + lane, row0, nw, M, N, cvec, stg, lane,
              [&] {
                if (lane == 0) mbar_arrive(acce + b);
                const int tn = t + static_cast<int>(gridDim.x);
                if (tn < tiles) epi.prefetch(ep, rows_of(tn) + lane, cols_of(tn), M, N, lane);
              });
    }
    if (lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2).  The pair computes a
// 256 x 256 tile: per stage each CTA loads its own 128 rows of qa and 128 of
// the tile's 256 rows of qw (32 KiB; 4 stages beside the epilogue staging)
// and keeps its 128 x 256 int32 accumulator in its own TMEM.  The
// even-rank CTA issues the MMAs (M = 256); both CTAs' stage bytes complete on
// its full barriers, and its commits arrive on the stage / accumulator
// barriers of both CTAs.  Both CTAs' epilogue warps release an accumulator on
// the even CTA's barrier.  Per SM this halves the weight bytes per stage, so
// more of the L2 round trip is covered by queued MMA work.
// ---------------------------------------------------------------------------
constexpr int kPairStages = 4;
constexpr int kPairBN = 256;
constexpr int kPairAccBufs = 2;  // TMEM accumulators per CTA (kPairAccBufs x 256 columns)
constexpr int kShortK = 2048;    // int8 K up to which the pair kernel runs 16 epilogue warps

// EW epilogue warps per CTA (8: two column halves of the tile; 16: four
// column quarters, for 16-bit outputs only: one 4 KiB staging box per warp).
template <int EW>
struct W8A8PairSmem {
  static constexpr int kParts = EW / 4;                // column parts of the tile
  static constexpr int kCW = kPairBN / kParts;         // columns per epilogue warp
  static constexpr uint32_t kA = kBM * kBK;            // this CTA's 128 rows of qa
  static constexpr uint32_t kB = (kPairBN / 2) * kBK;  // this CTA's 128 rows of qw
  static constexpr uint32_t kStage = kA + kB;          // multiple of 1024
  static constexpr uint32_t kStgOff = kPairStages * kStage;
  static constexpr uint32_t kStgWarp = (EW == 8 ? 2 : 1) * 32 * 128;  // 4 KiB TMA-store boxes
  static constexpr uint32_t kColOff = kStgOff + EW * kStgWarp;
  static constexpr uint32_t kColWarp = 2 * kCW * 4;
  static constexpr uint32_t kBarOff = kColOff + EW * kColWarp;
  static constexpr uint32_t kBytes = kBarOff + 256 + 1024;
};

template <int MODE, class OutT, class AT, int EW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(64 + 32 * EW, 1)
    w8a8_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO, int M, int N, int K, int gm,
                        Epilogue ep, int* err) {
  using L = W8A8PairSmem<EW>;
  static_assert(EW == 8 || (EW == 16 && MODE != kEpiAccI32 && sizeof(OutT) == 2),
                "16 epilogue warps stage one box of 16-bit values per tile");
  constexpr int BN = kPairBN;
  constexpr int CW = L::kCW;
  constexpr int STAGES = kPairStages;
  constexpr int kKe = kBK / static_cast<int>(sizeof(AT));  // K elements per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2] accumulator ready (both CTAs)
  uint64_t* acce = accf + 2;        // [2] accumulator drained (even CTA: both CTAs' warps)
  uint64_t* drain = acce + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int num_n = (N + BN - 1) / BN;
  const int num_m = (M + 2 * kBM - 1) / (2 * kBM);
  const int tiles = num_m * num_n;
  const int nkb = (K + kKe - 1) / kKe;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, 2 * EW);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) tmem_alloc_pair(tslot, kPairAccBufs * BN);
  tc_fence_before();
  cluster_sync();  // barriers initialised pair-wide before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(full, 0);  // the even CTA's full[0]
      int it = 0;
      for (int t = pair; t < tiles && !*abort_flag; t += npairs) {
        int mb, nb;
        tile_coords(t, num_m, num_n, gm, mb, nb);
        const int m0 = mb * (2 * kBM) + static_cast<int>(rank) * kBM;
        const int n0 = nb * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(empty + s, ph ^ 1, abort_flag, err, kErrWaitEmpty)) break;
          uint8_t* a_dst = smem + s * L::kStage;
          if (leader) mbar_arrive_expect_tx(full + s, 2 * L::kStage);
          const uint32_t fb = full0 + static_cast<uint32_t>(s) * 8u;
          tma_load_2d_pair(a_dst, &tmA, fb, kb * kKe, m0);
          tma_load_2d_pair(a_dst + L::kA, &tmB, fb, kb * kKe, n0);
          ++it;
        }
      }
      if (*abort_flag && leader) {
        // Drain the pair's copies still in flight before the CTAs unwind.
        volatile int never = 0;
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
          mbar_wait_bounded(full + (j % STAGES), (j / STAGES) & 1, &never, err, kErrWaitOther);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_of<AT>(2 * kBM, BN);
      int it = 0, lt = 0;
      for (int t = pair; t < tiles && !*abort_flag; t += npairs, ++lt) {
        const int b = lt % kPairAccBufs;
        const uint32_t use = static_cast<uint32_t>(lt / kPairAccBufs);
        if (!mbar_wait_bounded(acce + b, (use & 1) ^ 1, abort_flag, err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint32_t tacc = tmem + b * BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(full + s, ph, abort_flag, err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * L::kStage);
          const uint32_t b_addr = a_addr + L::kA;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            mma_k32<AT, true>(tacc, make_desc_kmajor_sw128(a_addr + k * 32),
                              make_desc_kmajor_sw128(b_addr + k * 32), idesc, (kb | k) != 0);
          }
          tc_commit_pair_mc(empty + s, 0x3);
          ++it;
        }
        if (!ok) break;
        tc_commit_pair_mc(accf + b, 0x3);
      }
      if (*abort_flag) {
        volatile int never = 0;
        tc_commit_pair_mc(drain, 0x1);
        mbar_wait_bounded(drain, 0, &never, err, kErrWaitOther);
      }
    }
  } else {
    // Epilogue warps 2..EW+1 of each CTA: TMEM lane quarter q = warp % 4
    // (this CTA's tile rows 32q..32q+31), column part (warp - 2) / 4 of CW
    // columns.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stg = smem + L::kStgOff + (warp - 2) * L::kStgWarp;
    float* cvec = reinterpret_cast<float*>(smem + L::kColOff + (warp - 2) * L::kColWarp);
    const uint32_t acce0 = mapa_shared(acce, 0);  // the even CTA's acce[0]
    TmaTileEpilogue<MODE, OutT, CW, sizeof(AT) == 1, 128> epi;
    auto rows_of = [&](int t) {
      int mb, nb;
      tile_coords(t, num_m, num_n, gm, mb, nb);
      return mb * (2 * kBM) + static_cast<int>(rank) * kBM + q * 32;
    };
    auto cols_of = [&](int t) {
      int mb, nb;
      tile_coords(t, num_m, num_n, gm, mb, nb);
      return nb * BN + half * CW;
    };
    if (pair < tiles) epi.prefetch(ep, rows_of(pair) + lane, cols_of(pair), M, N, lane);
    int lt = 0;
    for (int t = pair; t < tiles; t += npairs, ++lt) {
      const int b = lt % kPairAccBufs;
      const uint32_t use = static_cast<uint32_t>(lt / kPairAccBufs);
      const int row0 = rows_of(t), nw = cols_of(t);
      // warp-uniform outcome: the epilogue's TMEM loads are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(accf + b, use & 1, abort_flag, err,
                                                     kErrWaitAccum)))
        break;
      tc_fence_after();
      epi.run(ep, &tmO, tmem + b * BN + half * CW + (static_cast<uint32_t>(q * 32) << 16),
              row0 + lane, row0, nw, M, N, cvec, stg, lane,
              [&] {
                if (lane == 0) mbar_arrive_cluster(acce0 + static_cast<uint32_t>(b) * 8u);
                const int tn = t + npairs;
                if (tn < tiles) epi.prefetch(ep, rows_of(tn) + lane, cols_of(tn), M, N, lane);
              });
    }
    if (lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  cluster_sync();  // the pair's MMAs, copies and remote arrives are finished
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kPairAccBufs * BN);
  }
}

constexpr const char* kNamesI8[] = {"w8a8_tc_kernel/plain", "w8a8_tc_kernel/rope",
                                     "w8a8_tc_kernel/resid", "w8a8_tc_kernel/gatemix",
                                     "w8a8_tc_kernel/acc_i32"};
constexpr const char* kNamesF16[] = {"gemm_f16_tc_kernel/plain", "gemm_f16_tc_kernel/rope",
                                      "gemm_f16_tc_kernel/resid", "gemm_f16_tc_kernel/gatemix",
                                      "gemm_f16_tc_kernel/acc"};

template <class AT>
void operand_maps(CUtensorMap* ta, CUtensorMap* tb, const void* qa, const void* qw, int M, int N,
                  int K, int b_rows) {
  constexpr int el = static_cast<int>(sizeof(AT));
  make_tma_2d(ta, qa, tma_dtype_of<AT>(), el, M, K, K, kBK / el, kBM);
  make_tma_2d(tb, qw, tma_dtype_of<AT>(), el, N, K, K, kBK / el, b_rows);
}

// Row-block group of the rasterization: N fastest (0) while the weight fits
// a third of L2; else the number of row blocks whose activation band fits a
// 48 MiB share of L2.
template <class AT>
int raster_group(int rows_per_block, int N, int K) {
  const int64_t el = sizeof(AT);
  if (static_cast<int64_t>(N) * K * el <= (42ll << 20)) return 0;
  const int64_t band = static_cast<int64_t>(rows_per_block) * K * el;
  return static_cast<int>(std::max<int64_t>(1, (48ll << 20) / band));
}

template <int MODE, class OutT, class AT, int EW = 8>
void launch_w8a8_pair(const void* qa, const void* qw, int M, int N, int K, const Epilogue& ep,
                      cudaStream_t stream) {
  using StoreT = typename std::conditional<MODE == kEpiAccI32, int32_t, OutT>::type;
  using L = W8A8PairSmem<EW>;
  static_assert(L::kBytes <= 232448, "shared memory budget exceeded");
  CUtensorMap ta, tb, to;
  operand_maps<AT>(&ta, &tb, qa, qw, M, N, K, kPairBN / 2);
  constexpr int ob = static_cast<int>(sizeof(StoreT));
  make_tma_2d(&to, ep.out, tma_dtype_of<StoreT>(), ob, M, N, ep.ldo, 128 / ob, 32);
  auto kern = w8a8_tc_pair_kernel<MODE, OutT, AT, EW>;
  LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  const int tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kPairBN - 1) / kPairBN);
  const int pairs_max = device_sm_count() / 2;
  const int grid = 2 * (tiles < pairs_max ? tiles : pairs_max);
  const int gm = raster_group<AT>(2 * kBM, N, K);
  kern<<<grid, 64 + 32 * EW, L::kBytes, stream>>>(ta, tb, to, M, N, K, gm, ep,
                                                   device_error_ptr());
  check_launch(sizeof(AT) == 1 ? kNamesI8[MODE] : kNamesF16[MODE], stream);
}

template <int BN, int STAGES, int MODE, class OutT, class AT>
void launch_w8a8_inst(const void* qa, const void* qw, int M, int N, int K, const Epilogue& ep,
                      cudaStream_t stream) {
  using StoreT = typename std::conditional<MODE == kEpiAccI32, int32_t, OutT>::type;
  using L = W8A8Smem<BN, STAGES>;
  static_assert(L::kBytes <= 232448, "shared memory budget exceeded");
  CUtensorMap ta, tb, to;
  operand_maps<AT>(&ta, &tb, qa, qw, M, N, K, BN);
  constexpr int ob = static_cast<int>(sizeof(StoreT));
  make_tma_2d(&to, ep.out, tma_dtype_of<StoreT>(), ob, M, N, ep.ldo, 128 / ob, 32);
  auto kern = w8a8_tc_kernel<BN, STAGES, MODE, OutT, AT>;
  LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int grid = tiles < device_sm_count() ? tiles : device_sm_count();
  const int gm = raster_group<AT>(kBM, N, K);
  kern<<<grid, kThreads, L::kBytes, stream>>>(ta, tb, to, M, N, K, gm, ep, device_error_ptr());
  check_launch(sizeof(AT) == 1 ? kNamesI8[MODE] : kNamesF16[MODE], stream);
}

void check_gemm_args(const void* qa, const void* qw, int64_t M, int64_t N, int64_t K, int mode,
                     ltm_dtype out_dt, const Epilogue& ep) {
  LTM_REQUIRE(M >= 0 && N >= 0 && K >= 0, "negative size");
  LTM_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "size exceeds int32");
  LTM_REQUIRE(K > 0, "K must be positive");
  LTM_REQUIRE(K % 16 == 0, "K must be a multiple of 16");
  LTM_REQUIRE(N % 32 == 0, "N must be a multiple of 32");
  LTM_REQUIRE(qa && qw && ep.out, "NULL pointer");
  const size_t osz = (mode == kEpiAccI32) ? 4 : dtype_size(out_dt);
  LTM_REQUIRE((reinterpret_cast<uintptr_t>(ep.out) & 15) == 0, "output must be 16-byte aligned");
  LTM_REQUIRE((ep.ldo * osz) % 16 == 0, "output row stride must be a multiple of 16 bytes");
  LTM_REQUIRE((reinterpret_cast<uintptr_t>(ep.col_scale) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(ep.bias) & 15) == 0,
              "weight scales and bias must be 16-byte aligned");
  if (mode == kEpiResid || mode == kEpiGateMix) {
    LTM_REQUIRE((ep.ld_aux * osz) % 16 == 0, "aux row stride must be a multiple of 16 bytes");
  }
}

template <class AT>
void launch_gemm_tc(const void* qa, const void* qw, int64_t M, int64_t N, int64_t K, int mode,
                    ltm_dtype out_dt, const Epilogue& ep, cudaStream_t stream) {
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  dispatch_epilogue(mode, out_dt, [&](auto mode_c, auto out_tag) {
    constexpr int MODE = decltype(mode_c)::value;
    using OutT = decltype(out_tag);
    if constexpr (sizeof(AT) == 1 || (MODE != kEpiAccI32 && !std::is_same<OutT, float>::value)) {
      // (plain epilogues: the operand-carrying modes would spill at the
      // 96 registers a 576-thread CTA leaves)
      constexpr bool kEpi16 = sizeof(AT) == 1 && MODE == kEpiPlain && sizeof(OutT) == 2;
      if (N % 256 == 0 && M >= 2 * kBM) {
        // short K: the tile's epilogue outlasts its MMAs, so sixteen
        // epilogue warps share it
        if constexpr (kEpi16) {
          if (K <= kShortK) {
            launch_w8a8_pair<MODE, OutT, AT, 16>(qa, qw, m, n, k, ep, stream);
            return;
          }
        }
        launch_w8a8_pair<MODE, OutT, AT>(qa, qw, m, n, k, ep, stream);
      }
      else if (N % 256 == 0)
        launch_w8a8_inst<256, 3, MODE, OutT, AT>(qa, qw, m, n, k, ep, stream);
      else
        launch_w8a8_inst<128, 4, MODE, OutT, AT>(qa, qw, m, n, k, ep, stream);
    } else {
      LTM_REQUIRE(false, "16-bit GEMM stores 16-bit outputs");
    }
  });
}

}  // namespace

// Launches the W8A8 GEMM with the given epilogue. qa: [M,K], qw: [N,K].
void launch_w8a8(const int8_t* qa, const int8_t* qw, int64_t M, int64_t N, int64_t K, int mode,
                 ltm_dtype out_dt, const Epilogue& ep, cudaStream_t stream) {
  if (M == 0 || N == 0) return;
  check_gemm_args(qa, qw, M, N, K, mode, out_dt, ep);
  launch_gemm_tc<int8_t>(qa, qw, M, N, K, mode, out_dt, ep, stream);
}

// 16-bit GEMM (f16 or bf16 operands a [M,K], w [N,K] of dtype dt; fp32
// accumulation) with the fused epilogue, output in dt.
void launch_gemm_f16(const void* a, const void* w, int64_t M, int64_t N, int64_t K, int mode,
                     ltm_dtype dt, const Epilogue& ep, cudaStream_t stream) {
  if (M == 0 || N == 0) return;
  LTM_REQUIRE(dt == LTM_DTYPE_F16 || dt == LTM_DTYPE_BF16, "16-bit GEMM operands are f16 or bf16");
  LTM_REQUIRE(mode != kEpiAccI32, "no raw accumulator mode on the 16-bit GEMM");
  check_gemm_args(a, w, M, N, K, mode, dt, ep);
  LTM_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0,
              "operands must be 16-byte aligned");
  if (dt == LTM_DTYPE_BF16)
    launch_gemm_tc<__nv_bfloat16>(a, w, M, N, K, mode, dt, ep, stream);
  else
    launch_gemm_tc<__half>(a, w, M, N, K, mode, dt, ep, stream);
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_linear_w8a8(const int8_t* qa, const float* sa, const int8_t* qw,
                                      const float* sw, const float* bias, ltm_epilogue act, void* y,
                                      ltm_dtype y_dtype, int64_t M, int64_t N, int64_t K,
                                      void* stream) {
  return guarded([&] {
    LTM_REQUIRE(act == LTM_EPI_NONE || act == LTM_EPI_GELU || act == LTM_EPI_SIGMOID,
                "unknown epilogue");
    Epilogue ep;
    ep.act = act;
    ep.row_scale = sa;
    ep.col_scale = sw;
    ep.bias = bias;
    ep.out = y;
    ep.ldo = N;
    launch_w8a8(qa, qw, M, N, K, kEpiPlain, y_dtype, ep, as_stream(stream));
  });
}

extern "C" ltm_status ltm_linear_w8a8_acc_i32(const int8_t* qa, const int8_t* qw, int32_t* acc,
                                              int64_t M, int64_t N, int64_t K, void* stream) {
  return guarded([&] {
    Epilogue ep;
    ep.out = acc;
    ep.ldo = N;
    launch_w8a8(qa, qw, M, N, K, kEpiAccI32, LTM_DTYPE_F32, ep, as_stream(stream));
  });
}
