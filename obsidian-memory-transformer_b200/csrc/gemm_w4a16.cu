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
// Split-K for grids smaller than the GPU (decode, M <= 128): the grid's third
// dimension is a thread-block cluster of up to 8 CTAs per output tile; CTA z
// reduces the K-blocks [z*kps, (z+1)*kps) and parks its fp32 accumulator tile
// in its own shared memory; after a cluster barrier CTA r sums its share of
// the tile's rows over the slices (in slice order) through distributed shared
// memory and applies the fused epilogue.
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
constexpr int kRedLd = kBN + 4;  // row stride (floats) of a split-K slice in shared memory
constexpr int kMaxSplits = 8;    // portable cluster size

__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

static_assert(kBM * (kBN + 4) * 4 <= kStages * (kBM * 128 + kBN * 128 + kBN * 32),
              "a split-K slice fits in the pipeline stages");

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
      // group scale / zero-point of this row: the current group's and the next
      // group's, loaded one group (two K-blocks) before they are needed
      const float* srow = s4 + static_cast<int64_t>(n) * G;
      const uint8_t* zrow = z4 + static_cast<int64_t>(n) * G;
      int gcur = kb0 >> 1;
      float sc = 0.0f, zp = 0.0f, sc_n = 0.0f, zp_n = 0.0f;
      if (n < N) {
        sc = __ldg(srow + gcur);
        zp = static_cast<float>(__ldg(zrow + gcur));
        if (gcur + 1 < G) {
          sc_n = __ldg(srow + gcur + 1);
          zp_n = static_cast<float>(__ldg(zrow + gcur + 1));
        }
      }
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (((kb0 + kb) >> 1) != gcur) {
          gcur = (kb0 + kb) >> 1;
          sc = sc_n;
          zp = zp_n;
          if (n < N && gcur + 1 < G) {
            sc_n = __ldg(srow + gcur + 1);
            zp_n = static_cast<float>(__ldg(zrow + gcur + 1));
          }
        }
        const bool ok = mbar_wait_bounded(full + s, ph, abort_flag, err, kErrWaitFull);
        if (ok) {
          uint8_t* st = smem + s * L::kStage;
          const uint8_t* prow = st + L::kA + L::kB + t * 32;
          uint8_t* brow = st + L::kA + t * 128;
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
    if (gridDim.z == 1) {
      if (ok)
        tc_tile_epilogue_passes<MODE, T, kBN, false>(ep, tmem, q, lane, m0, n0, M, N,
                                                     smem + q * 32 * epi_stage_row_bytes<T>());
    } else if (ok) {
      // this slice's fp32 accumulator tile into this CTA's shared memory
      // (row-major, rows padded to kRedLd floats), read by the cluster below
      float* red = reinterpret_cast<float*>(smem);
      float* row = red + (q * 32 + lane) * kRedLd;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(row + c * 32 + 4 * j) =
              make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                          __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
      }
    }
  }

  if (gridDim.z > 1) {
    // split K over the cluster's CTAs: once every slice is in its CTA's shared
    // memory, CTA r sums its share of the tile's rows over the slices (slice
    // order) through distributed shared memory and applies the epilogue
    __syncwarp();
    cluster_sync();
    if (warp >= 2) {
      const int S = static_cast<int>(gridDim.z);
      const int r = static_cast<int>(cluster_ctarank());
      const int rows = min(kBM, M - m0), nch = min(kBN, N - n0) / 32;
      const int rpc = (rows + S - 1) / S;
      const int r0 = r * rpc, r1 = min(rows, r0 + rpc);
      const float* red = reinterpret_cast<const float*>(smem);
      for (int item = threadIdx.x - 64; item < (r1 - r0) * nch; item += 128) {
        const int rr = r0 + item / nch, c = item % nch;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.0f;
        for (int p = 0; p < S; ++p) {
          const uint32_t src = mapa_shared(red + rr * kRedLd + c * 32, p);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 t = ld_cluster_f32x4(src + 16 * j);
            v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
          }
        }
        epilogue_store32<MODE, T>(ep, m0 + rr, n0 + c * 32, v);
      }
    }
    __syncwarp();
    cluster_sync();  // the peers have read this CTA's slice
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kBN);
  }
}

}  // namespace

void launch_w4a16(const void* a, ltm_dtype dt, const uint8_t* q4, const float* s4, const uint8_t* z4,
                  int64_t M, int64_t N, int64_t K, int mode, const Epilogue& ep, cudaStream_t stream,
                  bool split_k) {
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
  // with at least 8 K-blocks per slice and at most one cluster of 8 slices
  int splits = 1;
  if (split_k) {
    const int want = 2 * device_sm_count() / (tiles_n * tiles_m);
    splits = std::max(1, std::min(std::min(want, nkb / 8), kMaxSplits));
  }
  const int kps = (nkb + splits - 1) / splits;
  splits = (nkb + kps - 1) / kps;
  const dim3 grid(tiles_n, tiles_m, splits);
  auto go = [&](auto tag, auto mode_c) {
    using T = decltype(tag);
    constexpr int MODE = decltype(mode_c)::value;
    auto kern = w4a16_tc_kernel<T, MODE>;
    LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, W4Smem::kBytes));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = W4Smem::kBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = static_cast<unsigned>(splits);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LTM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tp, s4, z4, static_cast<int>(M),
                                    static_cast<int>(N), static_cast<int>(K), kps, ep,
                                    device_error_ptr()));
  };
  dispatch_epilogue(mode, dt, [&](auto mode_c, auto out_tag) {
    using OutT = decltype(out_tag);
    constexpr int MODE = decltype(mode_c)::value;
    if constexpr (MODE != kEpiAccI32 && !std::is_same<OutT, float>::value) go(OutT{}, mode_c);
  });
  check_launch(splits > 1 ? "w4a16_tc_kernel/splitk" : "w4a16_tc_kernel", stream);
}


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
    launch_w4a16(a, a_dtype, packed, s, zp, M, N, K, kEpiPlain, ep, as_stream(stream), true);
  });
}
