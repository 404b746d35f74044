// decode.cu -- one decoding step of the Titan block against a KV cache:
// appending the new token's keys / values and the self-attention read of the
// whole cache (flash decoding, HBM-bound).
//
// Cache layout (head-major): [B, heads, max_positions, head_dim] in the
// activation dtype (heads = num_heads, or this rank's heads under tensor
// parallelism): the row of position p of head h of sequence b starts at
// cache + ((b * heads + h) * max_positions + p) * head_dim, so the 64 rows of a
// tile are one contiguous block.
//
// Attention of one query row per (sequence, head) over L cached positions
// (flash decoding): the positions are split into chunks of kDChunk (the work
// items, one partial (max, sum, output) each); a persistent grid of one CTA
// per SM walks its share of the work items.  In each CTA warp 0 streams
// 64-position K and V tiles of the items (TMA, box [64 rows x head_dim], one
// contiguous block of the head-major cache) into
// a ring of shared-memory stages that never drains between items, and 8
// consumer warps run the online softmax: each takes 8 rows of a tile as 4
// groups of 8 lanes x 2 keys, lane l of a group holding the dims
// c*64 + l*8 .. +7 of q, of the output and of the rows it reads (one 16-byte
// shared load per lane and half row, 128 contiguous bytes per 8 lanes: no
// bank conflicts).  Scores are reduced over the group's 8 lanes; each group
// keeps its own (max, sum, output), merged over the warp and then over the 8
// warps at the end of an item.  decode_combine_kernel merges the chunks.
// Every key and value byte is read from HBM once.
//
#include "block.cuh"

namespace ltm_b200 {
namespace {

constexpr int kDChunk = 1024;  // cache positions per work item
constexpr int kDTile = 64;     // cache positions per TMA tile
constexpr int kDCons = 8;      // consumer warps
constexpr int kDKeys = kDTile / (kDCons * 4);  // keys per lane group per tile

// Shared memory of the decode kernel: the K | V stages, their full / empty
// barriers, the abort flag and the per-item merge scratch (double-buffered by
// item parity).
template <int D>
struct DecSmem {
  static constexpr int kTile = kDTile * D * 2;              // one K or V tile (16-bit)
  static constexpr int kStages = D == 128 ? 6 : 12;         // 192 KiB of stages
  static constexpr int kStage = 2 * kTile;
  static constexpr int kOffBar = kStages * kStage;
  static constexpr int kOffFlag = kOffBar + 2 * kStages * 8;
  static constexpr int kOffMerge = (kOffFlag + 16 + 15) / 16 * 16;
  static constexpr int kMerge = 2 * kDCons * (D + 2) * 4;
  static constexpr int kBytes = kOffMerge + kMerge + 1024;  // + alignment slack
};

// Dims of a head row held by lane gl of an 8-lane group: for each 64-dim half
// c, the 8 consecutive dims c*64 + gl*8 .. +7, so one 16-byte load per lane
// and half reads a contiguous 128-byte segment of the row across the group.
template <class T, int DL>
__device__ __forceinline__ void load_row_part(const T* row, int gl, float (&v)[DL]) {
  static_assert(sizeof(T) == 2 && DL % 8 == 0, "16-bit rows, 8 dims per 16-byte vector");
#pragma unroll
  for (int c = 0; c < DL / 8; ++c) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row + c * 64 + gl * 8));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[c * 8 + i] = to_f32(e[i]);
  }
}

__device__ __forceinline__ int part_dim(int gl, int i) { return (i >> 3) * 64 + gl * 8 + (i & 7); }

// K | V rows of the new token (columns [width, 3 width) of its fused
// projection row) into position pos (or pos_arr[b]) of every head of its
// sequence.  A per-sequence position outside [0, P) writes nothing and sets
// the device error word.
template <class T>
__global__ void __launch_bounds__(256) kv_append_kernel(const T* __restrict__ qkv, int64_t ldq,
                                                        int width, int dh, T* __restrict__ kc,
                                                        T* __restrict__ vc, int64_t P,
                                                        int64_t pos,
                                                        const int* __restrict__ pos_arr,
                                                        int* err) {
  const int b = blockIdx.x;
  if (pos_arr != nullptr) {
    pos = pos_arr[b];
    if (pos < 0 || pos >= P) {
      if (threadIdx.x == 0) atomicExch(err, kErrBadCacheLen);
      return;
    }
  }
  const int nv = width / 8, vph = dh / 8;  // 16-byte vectors per row / per head
  const int heads = width / dh;
  const uint4* ks = reinterpret_cast<const uint4*>(qkv + b * ldq + width);
  const uint4* vs = reinterpret_cast<const uint4*>(qkv + b * ldq + 2 * static_cast<int64_t>(width));
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const int h = i / vph, c = i - h * vph;
    const int64_t dst = ((static_cast<int64_t>(b) * heads + h) * P + pos) * dh;
    reinterpret_cast<uint4*>(kc + dst)[c] = ks[i];
    reinterpret_cast<uint4*>(vc + dst)[c] = vs[i];
  }
}

// K | V rows of all T = B * S prefill rows (row t at position t % S of
// sequence t / S) into the head-major caches: one block per row.
template <class T>
__global__ void __launch_bounds__(256) kv_fill_kernel(const T* __restrict__ qkv, int64_t ldq,
                                                      int width, int dh, T* __restrict__ kc,
                                                      T* __restrict__ vc, int64_t P, int S) {
  const int64_t t = blockIdx.x;
  const int64_t b = t / S, p = t - b * S;
  const int nv = width / 8, vph = dh / 8;
  const int heads = width / dh;
  const uint4* ks = reinterpret_cast<const uint4*>(qkv + t * ldq + width);
  const uint4* vs = reinterpret_cast<const uint4*>(qkv + t * ldq + 2 * static_cast<int64_t>(width));
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const int h = i / vph, c = i - h * vph;
    const int64_t dst = ((b * heads + h) * P + p) * dh;
    reinterpret_cast<uint4*>(kc + dst)[c] = ks[i];
    reinterpret_cast<uint4*>(vc + dst)[c] = vs[i];
  }
}

// Positions attended by sequence b: L, or cache_lens[b] + 1 (0 when that
// length is outside [0, P): the sequence was skipped by the append).
__device__ __forceinline__ int seq_positions(const int* cache_lens, int b, int L, int P) {
  if (cache_lens == nullptr) return L;
  const int c = cache_lens[b];
  return (c >= 0 && c < P) ? c + 1 : 0;
}

__device__ __forceinline__ void consumer_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kDCons * 32) : "memory");
}

template <class T, int D>
__global__ void __launch_bounds__(32 * (kDCons + 1), 1) decode_attn_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
    const T* __restrict__ q, int64_t ldq, int L, int P, int nh, int nchunk, int items, float sl2,
    float* __restrict__ part, const int* __restrict__ cache_lens, int* err) {
  using S = DecSmem<D>;
  constexpr int DL = D / 8;  // dims per lane
  constexpr int NS = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* empty = full + NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::kOffFlag);
  float* merge = reinterpret_cast<float*>(smem + S::kOffMerge);  // [2][kDCons][D + 2]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kDCons);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  __syncthreads();

  if (warp == 0) {
    // ---- producer: K | V tiles of this CTA's items into the ring
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
        const int c = w % nchunk, bh = w / nchunk;
        const int Lb = seq_positions(cache_lens, bh / nh, L, P);
        const int c0 = c * kDChunk, c1 = min(Lb, c0 + kDChunk);
        const int nt = c1 > c0 ? (c1 - c0 + kDTile - 1) / kDTile : 0;
        for (int t = 0; t < nt; ++t, ++it) {
          const int st = it % NS;
          if (!mbar_wait_bounded(empty + st, ((it / NS) & 1) ^ 1, abort_flag, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + st, S::kStage);
          uint8_t* dst = smem + st * S::kStage;
          const int row = bh * P + c0 + t * kDTile;  // head-major: (b * nh + h) * P + position
          tma_load_2d(dst, &tmK, full + st, 0, row);
          tma_load_2d(dst + S::kTile, &tmV, full + st, 0, row);
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        volatile int never = 0;
        for (int j = (it > NS ? it - NS : 0); j < it; ++j)
          mbar_wait_bounded(full + j % NS, (j / NS) & 1, &never, err, kErrWaitOther);
      }
    }
    return;
  }

  // ---- consumers
  const int cw = warp - 1;
  const int grp = lane >> 3, gl = lane & 7;
  int it = 0, parity = 0;
  for (int w = blockIdx.x; w < items; w += gridDim.x, parity ^= 1) {
    const int c = w % nchunk, bh = w / nchunk;
    const int h = bh % nh, b = bh / nh;
    const int Lb = seq_positions(cache_lens, b, L, P);
    const int c0 = c * kDChunk, c1 = min(Lb, c0 + kDChunk);
    const int nt = c1 > c0 ? (c1 - c0 + kDTile - 1) / kDTile : 0;
    float qv[DL];
    load_row_part<T, DL>(q + b * ldq + h * D, gl, qv);
    float m = -INFINITY, l = 0.0f, o[DL];
#pragma unroll
    for (int i = 0; i < DL; ++i) o[i] = 0.0f;
    for (int t = 0; t < nt; ++t, ++it) {
      const int st = it % NS;
      bool ok = mbar_wait_bounded(full + st, (it / NS) & 1, abort_flag, err, kErrWaitFull);
      if (!__all_sync(0xffffffffu, ok)) return;
      const T* tk = reinterpret_cast<const T*>(smem + st * S::kStage);
      const T* tv = reinterpret_cast<const T*>(smem + st * S::kStage + S::kTile);
      float sc[kDKeys];
      float vv[kDKeys][DL];
      bool valid[kDKeys];
#pragma unroll
      for (int j = 0; j < kDKeys; ++j) {
        const int r = cw * (4 * kDKeys) + 4 * j + grp;  // row of the tile
        valid[j] = c0 + t * kDTile + r < c1;
        float kr[DL];
#pragma unroll
        for (int hh = 0; hh < DL / 8; ++hh) {
          const uint4 kraw = *reinterpret_cast<const uint4*>(tk + r * D + hh * 64 + gl * 8);
          const uint4 vraw = *reinterpret_cast<const uint4*>(tv + r * D + hh * 64 + gl * 8);
          const T* ke = reinterpret_cast<const T*>(&kraw);
          const T* ve = reinterpret_cast<const T*>(&vraw);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            kr[hh * 8 + i] = to_f32(ke[i]);
            // rows past the cache may hold anything: they contribute 0 * nothing
            vv[j][hh * 8 + i] = valid[j] ? to_f32(ve[i]) : 0.0f;
          }
        }
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < DL; ++i) d = fmaf(qv[i], kr[i], d);
        sc[j] = d;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + st);  // the stage's bytes are in registers
#pragma unroll
      for (int j = 0; j < kDKeys; ++j) {  // sum over the group's 8 lanes
        sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], 1);
        sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], 2);
        sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], 4);
        if (!valid[j]) sc[j] = -INFINITY;
      }
      float mb = sc[0];
#pragma unroll
      for (int j = 1; j < kDKeys; ++j) mb = fmaxf(mb, sc[j]);
      // no branch on the group's state: the shuffles above need the whole warp
      const float m_new = fmaxf(m, mb);
      const float mu = (m_new == -INFINITY) ? 0.0f : m_new;  // nothing visible yet
      const float corr = ex2_approx((m - mu) * sl2);          // m = -inf -> 0
      l *= corr;
#pragma unroll
      for (int i = 0; i < DL; ++i) o[i] *= corr;
#pragma unroll
      for (int j = 0; j < kDKeys; ++j) {
        const float pj = ex2_approx((sc[j] - mu) * sl2);  // -inf -> 0
        l += pj;
#pragma unroll
        for (int i = 0; i < DL; ++i) o[i] = fmaf(pj, vv[j][i], o[i]);
      }
      m = m_new;
    }
    // merge the warp's 4 groups (lanes gl, gl+8, gl+16, gl+24 hold the same dims)
    float mw = m;
    mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, 8));
    mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, 16));
    const float f = (mw == -INFINITY) ? 0.0f : ex2_approx((m - mw) * sl2);
    l *= f;
#pragma unroll
    for (int i = 0; i < DL; ++i) o[i] *= f;
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
#pragma unroll
    for (int i = 0; i < DL; ++i) {
      o[i] += __shfl_xor_sync(0xffffffffu, o[i], 8);
      o[i] += __shfl_xor_sync(0xffffffffu, o[i], 16);
    }
    float* mg = merge + parity * (kDCons * (D + 2));
    if (grp == 0) {
#pragma unroll
      for (int i = 0; i < DL; ++i) mg[cw * (D + 2) + part_dim(gl, i)] = o[i];
      if (gl == 0) {
        mg[cw * (D + 2) + D] = mw;
        mg[cw * (D + 2) + D + 1] = l;
      }
    }
    consumer_bar_sync();  // merge scratch of this parity complete; the other parity is free
    // merge the warps; consumer thread ct < D writes output dim ct of the item's partial
    const int ct = threadIdx.x - 32;
    if (ct < D) {
      float mc = -INFINITY;
#pragma unroll
      for (int k = 0; k < kDCons; ++k) mc = fmaxf(mc, mg[k * (D + 2) + D]);
      float lc = 0.0f, oc = 0.0f;
#pragma unroll
      for (int k = 0; k < kDCons; ++k) {
        const float g = (mc == -INFINITY) ? 0.0f : ex2_approx((mg[k * (D + 2) + D] - mc) * sl2);
        lc += mg[k * (D + 2) + D + 1] * g;
        oc += mg[k * (D + 2) + ct] * g;
      }
      float* pp = part + static_cast<int64_t>(w) * (D + 2);
      pp[ct] = oc;
      if (ct == 0) {
        pp[D] = mc;
        pp[D + 1] = lc;
      }
    }
  }
}

template <class T, int D>
__global__ void __launch_bounds__(D) decode_combine_kernel(const float* __restrict__ part,
                                                            int nchunk, float sl2,
                                                            T* __restrict__ o, int64_t ldo) {
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  const float* pp = part + (static_cast<int64_t>(b) * gridDim.x + h) * nchunk * (D + 2);
  float M = -INFINITY;
  for (int c = 0; c < nchunk; ++c) M = fmaxf(M, pp[c * (D + 2) + D]);
  float L = 0.0f, acc = 0.0f;
  for (int c = 0; c < nchunk; ++c) {
    const float mc = pp[c * (D + 2) + D];
    const float g = (mc == -INFINITY) ? 0.0f : ex2_approx((mc - M) * sl2);
    L += pp[c * (D + 2) + D + 1] * g;
    acc += pp[c * (D + 2) + t] * g;
  }
  o[b * ldo + h * D + t] = from_f32<T>(L > 0.0f ? acc / L : 0.0f);
}

}  // namespace

size_t decode_partials_bytes(int B, int nh, int D, int64_t L) {
  const int64_t nchunk = (L + kDChunk - 1) / kDChunk;
  return static_cast<size_t>(B) * nh * nchunk * (D + 2) * sizeof(float);
}

void launch_kv_append(const void* qkv, int64_t ldq, int width, int dh, void* kc, void* vc,
                      int64_t P, int64_t pos, int B, ltm_dtype dt, cudaStream_t st,
                      const int* pos_arr) {
  LTM_REQUIRE(dt != LTM_DTYPE_F32 && dh % 8 == 0 && width % dh == 0,
              "KV append needs 16-bit rows of whole heads");
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    kv_append_kernel<T><<<B, 256, 0, st>>>(static_cast<const T*>(qkv), ldq, width, dh,
                                            static_cast<T*>(kc), static_cast<T*>(vc), P, pos,
                                            pos_arr, device_error_ptr());
  });
  check_launch("kv_append_kernel", st);
}

void launch_kv_fill(const void* qkv, int64_t ldq, int width, int dh, void* kc, void* vc, int64_t P,
                    int B, int S, ltm_dtype dt, cudaStream_t st) {
  LTM_REQUIRE(dt != LTM_DTYPE_F32 && dh % 8 == 0 && width % dh == 0,
              "KV fill needs 16-bit rows of whole heads");
  LTM_REQUIRE(S <= P, "the prompt is longer than the cache");
  const int64_t T = static_cast<int64_t>(B) * S;
  if (T == 0) return;
  LTM_REQUIRE(T < (1ll << 31), "too many rows");
  dispatch_dtype(dt, [&](auto tag) {
    using T_ = decltype(tag);
    kv_fill_kernel<T_><<<static_cast<unsigned>(T), 256, 0, st>>>(
        static_cast<const T_*>(qkv), ldq, width, dh, static_cast<T_*>(kc), static_cast<T_*>(vc),
        P, S);
  });
  check_launch("kv_fill_kernel", st);
}

void launch_decode_attention(const void* q, int64_t ldq, const void* kc, const void* vc,
                             int64_t P, int L, int B, int nh, int D, ltm_dtype dt, float* part,
                             void* o, int64_t ldo, cudaStream_t st, const int* cache_lens) {
  LTM_REQUIRE(D == 64 || D == 128, "decode attention head_dim must be 64 or 128");
  LTM_REQUIRE(L >= 1 && L <= P, "cache length outside [1, max_positions]");
  LTM_REQUIRE(dt != LTM_DTYPE_F32, "decode attention needs 16-bit activations");
  LTM_REQUIRE(static_cast<int64_t>(B) * nh * P < (1ll << 31), "cache rows exceed int32");
  const int nchunk = (L + kDChunk - 1) / kDChunk;
  const int items = B * nh * nchunk;
  const float sl2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  const CUtensorMapDataType tdt =
      dt == LTM_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tk, tv;
  const uint64_t rows = static_cast<uint64_t>(B) * nh * P;
  make_tma_2d(&tk, kc, tdt, 2, rows, D, D, D, kDTile, CU_TENSOR_MAP_SWIZZLE_NONE);
  make_tma_2d(&tv, vc, tdt, 2, rows, D, D, D, kDTile, CU_TENSOR_MAP_SWIZZLE_NONE);
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (!std::is_same<T, float>::value) {
      auto run = [&](auto dtag) {
        constexpr int DD = decltype(dtag)::value;
        auto kern = decode_attn_kernel<T, DD>;
        constexpr int smem = DecSmem<DD>::kBytes;
        LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        const int grid = persistent_grid(kern, 32 * (kDCons + 1), smem, items);
        kern<<<grid, 32 * (kDCons + 1), smem, st>>>(tk, tv, static_cast<const T*>(q), ldq, L,
                                                    static_cast<int>(P), nh, nchunk, items, sl2,
                                                    part, cache_lens, device_error_ptr());
        check_launch("decode_attn_kernel", st);
        decode_combine_kernel<T, DD><<<dim3(nh, B), DD, 0, st>>>(part, nchunk, sl2,
                                                                 static_cast<T*>(o), ldo);
        check_launch("decode_combine_kernel", st);
      };
      if (D == 64)
        run(std::integral_constant<int, 64>{});
      else
        run(std::integral_constant<int, 128>{});
    }
  });
}

}  // namespace ltm_b200
