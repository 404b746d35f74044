// gemm_w4a16.cu -- W4A16 linear on the 5th-generation tensor cores.
//
//   W[n,k] = T((q[n,k] - zp[n,g]) * s[n,g]),  g = k / 128   (dequantised to the
//            activation type T, as Quantizer::dequantize writes T:
//            src/core/quantization/quantizer.cu:76-90,144-161)
//   y      = epilogue(a @ W^T)                  fp32 accumulation in TMEM
//
// One CTA computes a 128 x 128 tile; K advances 64 elements (128 bytes) per
// stage; the epilogue stages the tile in shared memory for coalesced stores.  Warp roles (192 threads):
//   warp 0      TMA producer: the 128 x 64 activation tile (128-byte swizzle)
//               and the 128 x 32-byte packed int4 weight tile
//   warp 1      TMEM allocator + MMA issuer (4 x tcgen05.mma kind::f16, K=16)
//   warps 2..5  transform: unpack nibbles, apply zero-point and scale, write
//               the T weight tile in the UMMA K-major 128-byte-swizzled layout,
//               fence it to the async proxy; then the fused epilogue
// All waits are bounded (common.cuh).
//
// Split-K for grids smaller than the GPU (decode, M <= 128): CTA z of the
// grid's third dimension reduces the K-blocks [z*kps, (z+1)*kps) and dumps its
// raw fp32 accumulator tile to partials[z] (the int32 store mode of the
// epilogue, bit for bit); splitk_epilogue_kernel sums the slices in order and
// applies the fused epilogue.
#include <memory>
#include <mutex>
#include <type_traits>
#include <vector>

#include "block.cuh"
#include "epilogue.cuh"

namespace ltm_b200 {
namespace {

constexpr int kBM = 128, kBN = 128, kBKe = 64;  // K elements per stage
constexpr int kStages = 3;

struct W4Smem {
  static constexpr uint32_t kA = kBM * 128;     // 128 rows x 128 bytes
  static constexpr uint32_t kB = kBN * 128;     // dequantised weight tile
  static constexpr uint32_t kP = kBN * 32;      // packed int4 tile
  static constexpr uint32_t kStage = kA + kB + kP;
  static constexpr uint32_t kBarOff = kStages * kStage;
  static constexpr uint32_t kBytes = kBarOff + 256 + 1024;
};

// Two floats rounded to a packed pair of 16-bit values (one paired convert;
// each half rounded to nearest-even as the single conversions do).
template <class T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <class T, int MODE>
__global__ void __launch_bounds__(192, 2)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmP,
                    const float* __restrict__ s4, const uint8_t* __restrict__ z4, int M, int N, int K,
                    int kps, Epilogue ep, int* err) {
  using L = W4Smem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* bready = full + kStages;
  uint64_t* empty = bready + kStages;
  uint64_t* accf = empty + kStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const int kb0 = blockIdx.z * kps;                // this CTA's K-blocks [kb0, kb0 + nkb)
  const int nkb = min(K / kBKe - kb0, kps);
  const int G = K / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(bready + s, 4);
      mbar_init(empty + s, 1);
    }
    mbar_init(accf, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmP);
  }
  if (warp == 1) tmem_alloc(tslot, kBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait_bounded(empty + s, ph ^ 1, abort_flag, err, kErrWaitEmpty)) break;
        uint8_t* st = smem + s * L::kStage;
        mbar_arrive_expect_tx(full + s, L::kA + L::kP);
        tma_load_2d(st, &tmA, full + s, (kb0 + kb) * kBKe, m0);
        tma_load_2d(st + L::kA + L::kB, &tmP, full + s, (kb0 + kb) * (kBKe / 2), n0);
        ++issued;
      }
      if (*abort_flag) {
        volatile int never = 0;
        for (int j = (issued > kStages ? issued - kStages : 0); j < issued; ++j)
          mbar_wait_bounded(full + (j % kStages), (j / kStages) & 1, &never, err, kErrWaitOther);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBM, kBN, std::is_same<T, __nv_bfloat16>::value);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait_bounded(bready + s, ph, abort_flag, err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * L::kStage);
        const uint32_t b_addr = a_addr + L::kA;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(tmem, make_desc_kmajor_sw128(a_addr + k * 32),
                     make_desc_kmajor_sw128(b_addr + k * 32), idesc, (kb | k) != 0);
        tc_commit(empty + s);
      }
      tc_commit(accf);
      if (*abort_flag) {
        volatile int never = 0;
        mbar_wait_bounded(accf, 0, &never, err, kErrWaitOther);
      }
    }
  } else {
    const int t = threadIdx.x - 64;  // 0..127: weight-tile row
    const int q = warp & 3;
    // ---- transform: packed int4 -> T, 128-byte swizzled K-major rows
    {
      const int n = n0 + t;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        const bool ok = mbar_wait_bounded(full + s, ph, abort_flag, err, kErrWaitFull);
        if (ok) {
          uint8_t* st = smem + s * L::kStage;
          const uint8_t* prow = st + L::kA + L::kB + t * 32;
          uint8_t* brow = st + L::kA + t * 128;
          float sc = 0.0f, zp = 0.0f;
          if (n < N) {
            const int64_t gi = static_cast<int64_t>(n) * G + ((kb0 + kb) >> 1);
            sc = __ldg(s4 + gi);
            zp = static_cast<float>(__ldg(z4 + gi));
          }
          // q - zp without an int->float conversion: the float with bits
          // 0x4B000000 | q is 2^23 + q exactly, and (2^23 + q) - (2^23 + zp) is
          // exact for 0 <= q, zp <= 15; then one rounding in the multiply, as
          // in (q - zp) * s
          const float bias_zp = 8388608.0f + zp;
          const uint4 p0 = *reinterpret_cast<const uint4*>(prow);
          const uint4 p1 = *reinterpret_cast<const uint4*>(prow + 16);
          const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t w = words[c];  // 8 nibbles: k = c*8 .. c*8+7, low nibble first
            uint4 out;
            uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo =
                  (__uint_as_float(((w >> (8 * e)) & 0xFu) | 0x4B000000u) - bias_zp) * sc;
              const float hi =
                  (__uint_as_float(((w >> (8 * e + 4)) & 0xFu) | 0x4B000000u) - bias_zp) * sc;
              o[e] = pack_pair<T>(lo, hi);
            }
            *reinterpret_cast<uint4*>(brow + ((c ^ (t & 7)) << 4)) = out;
          }
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bready + s);
        if (!ok) break;
      }
    }
    // ---- epilogue: the pipeline stages are free once the accumulator is
    // complete, so stage 0 doubles as the output staging buffer
    // warp-uniform outcome: the epilogue's TMEM loads are warp-collective
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(accf, 0, abort_flag, err,
                                                              kErrWaitAccum) &&
                                                !*abort_flag);
    tc_fence_after();
    using StoreT = typename std::conditional<MODE == kEpiAccI32, int32_t, T>::type;
    Epilogue pe = ep;
    if constexpr (MODE == kEpiAccI32)  // split-K slice: raw fp32 bits into partials[z]
      pe.out = static_cast<int32_t*>(ep.out) + static_cast<int64_t>(blockIdx.z) * M * N;
    if (ok)
      tc_tile_epilogue_passes<MODE, T, kBN, false>(pe, tmem, q, lane, m0, n0, M, N,
                                                   smem + q * 32 * epi_stage_row_bytes<StoreT>());
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kBN);
  }
}

// Sum of the split-K slices: one warp per 32-column row chunk, lane j summing
// column j over the slices (coalesced 128-byte reads), then lane 0 applies
// the fused epilogue to the chunk and stores it.
template <int MODE, class OutT>
__global__ void __launch_bounds__(256) splitk_epilogue_kernel(const float* __restrict__ part,
                                                              int splits, int M, int N,
                                                              Epilogue ep) {
  const int nch = N / 32;
  const int64_t chunk = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (chunk >= static_cast<int64_t>(M) * nch) return;  // whole warps leave together
  const int m = static_cast<int>(chunk / nch);
  const int c = static_cast<int>(chunk - static_cast<int64_t>(m) * nch);
  const float* p = part + static_cast<int64_t>(m) * N + c * 32 + lane;
  const int64_t slice = static_cast<int64_t>(M) * N;
  float acc = 0.0f;
  int z = 0;
  for (; z + 4 <= splits; z += 4) {
    const float a0 = __ldg(p + z * slice), a1 = __ldg(p + (z + 1) * slice);
    const float a2 = __ldg(p + (z + 2) * slice), a3 = __ldg(p + (z + 3) * slice);
    acc += a0;
    acc += a1;
    acc += a2;
    acc += a3;
  }
  for (; z < splits; ++z) acc += __ldg(p + z * slice);
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __shfl_sync(0xffffffffu, acc, i);
  if (lane == 0) epilogue_store32<MODE, OutT>(ep, m, static_cast<int64_t>(c) * 32, v);
}

}  // namespace

void launch_w4a16(const void* a, ltm_dtype dt, const uint8_t* q4, const float* s4, const uint8_t* z4,
                  int64_t M, int64_t N, int64_t K, int mode, const Epilogue& ep, cudaStream_t stream,
                  DevBuf* splitk_ws) {
  LTM_REQUIRE(M >= 0 && N >= 0 && K >= 0, "negative size");
  LTM_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "size exceeds int32");
  if (M == 0 || N == 0) return;
  LTM_REQUIRE(dt == LTM_DTYPE_F16 || dt == LTM_DTYPE_BF16, "W4A16 activations must be f16 or bf16");
  LTM_REQUIRE(K > 0 && K % 128 == 0, "K must be a positive multiple of 128");
  LTM_REQUIRE(N % 32 == 0, "N must be a multiple of 32");
  LTM_REQUIRE(a && q4 && s4 && z4 && ep.out, "NULL pointer");
  LTM_REQUIRE(mode != kEpiAccI32, "no int32 accumulator mode on the W4A16 path");
  LTM_REQUIRE((reinterpret_cast<uintptr_t>(ep.out) & 15) == 0, "output must be 16-byte aligned");
  LTM_REQUIRE((ep.ldo * 2) % 16 == 0, "output row stride must be a multiple of 16 bytes");
  LTM_REQUIRE((reinterpret_cast<uintptr_t>(ep.bias) & 15) == 0, "bias must be 16-byte aligned");
  CUtensorMap ta, tp;
  make_tma_2d(&ta, a, dt == LTM_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
              2, M, K, K, kBKe, kBM);
  make_tma_2d(&tp, q4, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, kBKe / 2, kBN,
              CU_TENSOR_MAP_SWIZZLE_NONE);
  const int tiles_n = static_cast<int>((N + kBN - 1) / kBN), tiles_m = static_cast<int>((M + kBM - 1) / kBM);
  const int nkb = static_cast<int>(K / kBKe);
  // split K when the tile grid leaves most SMs idle (two CTAs fit per SM),
  // with at least 8 K-blocks per slice
  int splits = 1;
  if (splitk_ws != nullptr) {
    const int want = 2 * device_sm_count() / (tiles_n * tiles_m);
    splits = std::max(1, std::min(want, nkb / 8));
  }
  const int kps = (nkb + splits - 1) / splits;
  splits = (nkb + kps - 1) / kps;
  dim3 grid(tiles_n, tiles_m, splits);
  if (splits > 1) {
    const size_t need = static_cast<size_t>(splits) * M * N * sizeof(float);
    splitk_ws->ensure(need);
    Epilogue pe;
    pe.out = splitk_ws->ptr;
    pe.ldo = N;
    dispatch_dtype(dt, [&](auto tag) {
      using T = decltype(tag);
      if constexpr (!std::is_same<T, float>::value) {
        auto kern = w4a16_tc_kernel<T, kEpiAccI32>;
        LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          W4Smem::kBytes));
        kern<<<grid, 192, W4Smem::kBytes, stream>>>(ta, tp, s4, z4, static_cast<int>(M),
                                                     static_cast<int>(N), static_cast<int>(K), kps,
                                                     pe, device_error_ptr());
      }
    });
    check_launch("w4a16_tc_kernel/splitk", stream);
    const int64_t threads = M * N;  // one warp per 32-column row chunk
    dispatch_epilogue(mode, dt, [&](auto mode_c, auto out_tag) {
      using OutT = decltype(out_tag);
      constexpr int MODE = decltype(mode_c)::value;
      if constexpr (MODE != kEpiAccI32 && !std::is_same<OutT, float>::value)
        splitk_epilogue_kernel<MODE, OutT><<<static_cast<unsigned>((threads + 255) / 256), 256, 0,
                                             stream>>>(splitk_ws->as<float>(), splits,
                                                       static_cast<int>(M), static_cast<int>(N), ep);
    });
    check_launch("splitk_epilogue_kernel", stream);
    return;
  }
  auto go = [&](auto tag, auto mode_c) {
    using T = decltype(tag);
    constexpr int MODE = decltype(mode_c)::value;
    auto kern = w4a16_tc_kernel<T, MODE>;
    LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, W4Smem::kBytes));
    kern<<<grid, 192, W4Smem::kBytes, stream>>>(ta, tp, s4, z4, static_cast<int>(M),
                                                 static_cast<int>(N), static_cast<int>(K), kps, ep,
                                                 device_error_ptr());
  };
  dispatch_epilogue(mode, dt, [&](auto mode_c, auto out_tag) {
    using OutT = decltype(out_tag);
    constexpr int MODE = decltype(mode_c)::value;
    if constexpr (MODE != kEpiAccI32 && !std::is_same<OutT, float>::value) go(OutT{}, mode_c);
  });
  check_launch("w4a16_tc_kernel", stream);
}

namespace {
// Per-device split-K partials of ltm_linear_w4a16 (grown on demand, held
// until exit; calls whose GPU work overlaps on one device share it).
DevBuf& splitk_scratch(int dev) {
  static std::mutex mu;
  static std::vector<std::unique_ptr<DevBuf>> per_dev;
  std::lock_guard<std::mutex> lk(mu);
  if (static_cast<int>(per_dev.size()) <= dev) per_dev.resize(dev + 1);
  if (!per_dev[dev]) per_dev[dev] = std::make_unique<DevBuf>();
  return *per_dev[dev];
}
}  // namespace

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_linear_w4a16(const void* a, ltm_dtype a_dtype, const uint8_t* packed,
                                       const float* s, const uint8_t* zp, const float* bias,
                                       ltm_epilogue act, void* y, int64_t M, int64_t N, int64_t K,
                                       void* stream) {
  return guarded([&] {
    LTM_REQUIRE(act == LTM_EPI_NONE || act == LTM_EPI_GELU || act == LTM_EPI_SIGMOID,
                "unknown epilogue");
    Epilogue ep;
    ep.act = act;
    ep.bias = bias;
    ep.out = y;
    ep.ldo = N;
    int dev = 0;
    LTM_CUDA_TRY(cudaGetDevice(&dev));
    launch_w4a16(a, a_dtype, packed, s, zp, M, N, K, kEpiPlain, ep, as_stream(stream),
                 &splitk_scratch(dev));
  });
}
