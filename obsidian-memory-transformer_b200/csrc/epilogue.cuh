// epilogue.cuh -- the fused epilogue shared by every linear kernel.
//
// A kernel hands over 32 consecutive fp32 values of one output row (raw
// accumulators) and the epilogue applies, in this order:
//   v = acc * row_scale[m] * col_scale[n] + bias[n]     (dequant + bias)
//   v = act(v)                                           (none / GELU-tanh / sigmoid)
// then one of the modes
//   PLAIN    y = v
//   ROPE     interleaved-pair rotation of columns < rope_cols (Q and K of the
//            fused projection), position = m % seq_len
//   RESID    y = v + R[m,n]                               (FFN-down + block residual)
//   GATEMIX  g = v (sigmoid applied);  y = s + g*mem + (1-g)*x   (memory integration)
//   ACC_I32  raw int32 accumulators (exactness probe)
// and stores 32 outputs with 16-byte vector stores (tensor-core kernels stage
// the tile in shared memory first for coalesced row stores).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace ltm_b200 {

enum EpiMode : int { kEpiPlain = 0, kEpiRope = 1, kEpiResid = 2, kEpiGateMix = 3, kEpiAccI32 = 4 };

struct Epilogue {
  int act = LTM_EPI_NONE;
  const float* row_scale = nullptr;  // [M] or NULL (=1)
  const float* col_scale = nullptr;  // [N] or NULL (=1)
  const float* bias = nullptr;       // [N] or NULL (=0)
  void* out = nullptr;
  int64_t ldo = 0;  // elements
  // ROPE
  const float2* rope = nullptr;  // [seq_len, head_dim/2] of (cos, sin)
  int rope_cols = 0;
  int seq_len = 1;
  int head_dim = 64;
  // per-row positions (decode with a cache length per sequence): row m at
  // position row_pos[m] of the table, which holds rope_rows positions (a
  // position outside [0, rope_rows) is clamped; the launchers flag it)
  const int* row_pos = nullptr;
  int rope_rows = 0;
  // rows of this launch are rows row0 + m of the whole batch (a GEMM over a
  // row chunk): the position is (row0 + m) % seq_len
  int64_t rope_row0 = 0;
  // RESID (aux0 = R) / GATEMIX (aux0 = s, aux1 = mem, aux2 = x); all use ld_aux
  const void* aux0 = nullptr;
  const void* aux1 = nullptr;
  const void* aux2 = nullptr;
  int64_t ld_aux = 0;
  // GATEMIX: optional column sums of g*x over the rows (memory write), fp32 [N]
  float* colsum = nullptr;
};

// RoPE table row of output row m.
__device__ __forceinline__ int rope_row(const Epilogue& ep, int64_t m, bool row_ok) {
  if (ep.row_pos != nullptr) {
    const int p = row_ok ? __ldg(ep.row_pos + m) : 0;
    return min(max(p, 0), ep.rope_rows - 1);
  }
  return static_cast<int>(static_cast<uint64_t>(m + ep.rope_row0) %
                          static_cast<uint64_t>(ep.seq_len));
}

// Sum over the warp's 32 rows of v[c]; lane c receives column c (31 shuffles,
// recursive halving).  Must be called by all 32 lanes.
__device__ __forceinline__ float warp_colsum32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int j = 0; j < s; ++j) {
      const float send = upper ? v[j] : v[j + s];
      const float keep = upper ? v[j + s] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// GELU, tanh approximation of src/core/ops/fused_ops.cu:136-142:
//   x * 0.5 * (1 + tanh(z)),  z = 0.797885 * (x + 0.044715 x^3),
// evaluated through 0.5 * (1 + tanh(z)) = 1 / (1 + 2^(-2 z log2(e))) with the
// hardware 2^x and a fast division (relative error ~1e-6 against tanhf).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float z = 0.797885f * (x + 0.044715f * x * x * x);
  return __fdividef(x, 1.0f + ex2_approx(-2.8853900817779268f * z));
}

// 1 / (1 + e^-x) through the hardware 2^x.
__device__ __forceinline__ float sigmoid_f(float x) {
  return __fdividef(1.0f, 1.0f + ex2_approx(-1.4426950408889634f * x));
}

template <class T>
__device__ __forceinline__ void load32(const T* p, float (&v)[32]) {
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int c = 0; c < 32 / PER; ++c) {
    uint4 raw = *reinterpret_cast<const uint4*>(p + c * PER);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < PER; ++i) v[c * PER + i] = to_f32(e[i]);
  }
}

template <class T>
__device__ __forceinline__ void store32(T* p, const float (&v)[32]) {
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int c = 0; c < 32 / PER; ++c) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < PER; ++i) e[i] = from_f32<T>(v[c * PER + i]);
    *reinterpret_cast<uint4*>(p + c * PER) = raw;
  }
}

// Applies the epilogue math to 32 values of row `m`, columns [n0, n0+32);
// the results stay in v.  GATEMIX with ep.colsum: g*x is written to gx_out
// when given (the caller reduces it across the warp), else added to
// ep.colsum element by element.  ACC_I32 leaves the raw bits untouched.
template <int MODE, class OutT>
__device__ __forceinline__ void epilogue_math32(const Epilogue& ep, int64_t m, int64_t n0,
                                                float (&v)[32], float* gx_out = nullptr) {
  if constexpr (MODE != kEpiAccI32) {
    const float rs = ep.row_scale ? ep.row_scale[m] : 1.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= rs;
    if (ep.col_scale) {  // 16-byte aligned (checked by the launchers)
      const float4* cs = reinterpret_cast<const float4*>(ep.col_scale + n0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 t = __ldg(cs + j);
        v[4 * j] *= t.x; v[4 * j + 1] *= t.y; v[4 * j + 2] *= t.z; v[4 * j + 3] *= t.w;
      }
    }
    if (ep.bias) {
      const float4* bs = reinterpret_cast<const float4*>(ep.bias + n0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 t = __ldg(bs + j);
        v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
      }
    }
    if (ep.act == LTM_EPI_GELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
    } else if (ep.act == LTM_EPI_SIGMOID) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = sigmoid_f(v[i]);
    }
    if constexpr (MODE == kEpiRope) {
      if (n0 < ep.rope_cols) {
        // a 32-column chunk never crosses a head (head_dim is a multiple of 32)
        const int half = ep.head_dim >> 1;
        const int pos = rope_row(ep, m, true);
        const int d0 = static_cast<int>(static_cast<uint32_t>(n0) % static_cast<uint32_t>(ep.head_dim));
        const float2* tab = ep.rope + static_cast<int64_t>(pos) * half + (d0 >> 1);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 cs = __ldg(tab + (i >> 1));
          const float a = v[i], b = v[i + 1];
          v[i] = a * cs.x - b * cs.y;
          v[i + 1] = a * cs.y + b * cs.x;
        }
      }
    } else if constexpr (MODE == kEpiResid) {
      float r[32];
      load32(static_cast<const OutT*>(ep.aux0) + m * ep.ld_aux + n0, r);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += r[i];
    } else if constexpr (MODE == kEpiGateMix) {
      float s[32], mem[32];
      load32(static_cast<const OutT*>(ep.aux0) + m * ep.ld_aux + n0, s);
      load32(static_cast<const OutT*>(ep.aux1) + m * ep.ld_aux + n0, mem);
#pragma unroll
      for (int i = 0; i < 32; ++i) s[i] = s[i] + v[i] * mem[i];
      load32(static_cast<const OutT*>(ep.aux2) + m * ep.ld_aux + n0, mem);
      if (ep.colsum) {
        if (gx_out) {
#pragma unroll
          for (int i = 0; i < 32; ++i) gx_out[i] = v[i] * mem[i];
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) atomicAdd(ep.colsum + n0 + i, v[i] * mem[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = s[i] + (1.0f - v[i]) * mem[i];
    }
  }
}

// Converts 32 epilogue values to the output type and writes them (16-byte
// vectors) to p; ACC_I32 reinterprets v as the raw int32 accumulators.
template <int MODE, class OutT>
__device__ __forceinline__ void pack_store32(void* p, const float (&v)[32]) {
  if constexpr (MODE == kEpiAccI32) {
    int32_t* o = static_cast<int32_t*>(p);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      int4 t;
      t.x = __float_as_int(v[4 * c + 0]);
      t.y = __float_as_int(v[4 * c + 1]);
      t.z = __float_as_int(v[4 * c + 2]);
      t.w = __float_as_int(v[4 * c + 3]);
      *reinterpret_cast<int4*>(o + 4 * c) = t;
    }
  } else {
    store32(static_cast<OutT*>(p), v);
  }
}

// Math + direct store of one 32-column row chunk (SIMT kernels).
template <int MODE, class OutT>
__device__ __forceinline__ void epilogue_store32(const Epilogue& ep, int64_t m, int64_t n0,
                                                 float (&v)[32], float* gx_out = nullptr) {
  epilogue_math32<MODE, OutT>(ep, m, n0, v, gx_out);
  using StoreT = typename std::conditional<MODE == kEpiAccI32, int32_t, OutT>::type;
  pack_store32<MODE, OutT>(static_cast<StoreT*>(ep.out) + m * ep.ldo + n0, v);
}

// Epilogue of one 128 x BN accumulator tile of a tensor-core kernel (4
// epilogue warps, warp quarter q = TMEM lanes 32q..32q+31 = tile rows).  The
// tile is processed in passes of 64 columns: two 32-column TMEM loads, the
// epilogue math, conversion into this warp's staging rows in shared memory
// (rows padded by 16 bytes: conflict-free), then coalesced 16-byte stores of
// the warp's 32 rows x 64 columns (full 128-byte lines).
constexpr int kEpiPassCols = 64;

template <class StoreT>
__host__ __device__ constexpr int epi_stage_row_bytes() {
  return kEpiPassCols * static_cast<int>(sizeof(StoreT)) + 16;
}

// The same passes with the 32 accumulator values of a chunk taken from
// src(c, v) (column chunk c of this lane's row; called by every lane).
template <int MODE, class OutT, int BN, class Src>
__device__ __forceinline__ void tile_epilogue_passes_src(const Epilogue& ep, Src&& src, int q,
                                                         int lane, int64_t m0, int64_t n0, int M,
                                                         int N, uint8_t* stg) {
  using StoreT = typename std::conditional<MODE == kEpiAccI32, int32_t, OutT>::type;
  constexpr int OB = sizeof(StoreT);
  constexpr int ROWB = epi_stage_row_bytes<StoreT>();
  constexpr int CPR = kEpiPassCols * OB / 16;  // 16-byte chunks per staged row
  constexpr int EPC = 16 / OB;                 // elements per chunk
  const int64_t m = m0 + q * 32 + lane;
  StoreT* out = static_cast<StoreT*>(ep.out);
#pragma unroll 1
  for (int p = 0; p < BN / kEpiPassCols; ++p) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = p * 2 + h;
      float v[32];
      src(c, v);
      const int64_t n = n0 + c * 32;
      const bool valid = m < M && n < N;
      if constexpr (MODE == kEpiGateMix) {
        float gx[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) gx[i] = 0.0f;
        if (valid) epilogue_math32<MODE, OutT>(ep, m, n, v, gx);
        if (ep.colsum) {
          const float cs = warp_colsum32(gx);
          if (n < N) atomicAdd(ep.colsum + n + lane, cs);
        }
      } else {
        if (valid) epilogue_math32<MODE, OutT>(ep, m, n, v);
      }
      pack_store32<MODE, OutT>(stg + lane * ROWB + h * 32 * OB, v);
    }
    __syncwarp();
#pragma unroll
    for (int idx = lane; idx < 32 * CPR; idx += 32) {
      const int rr = idx / CPR, ch = idx - rr * CPR;
      const int64_t gm = m0 + q * 32 + rr;
      const int64_t gn = n0 + p * kEpiPassCols + ch * EPC;
      if (gm < M && gn < N)
        *reinterpret_cast<uint4*>(out + gm * ep.ldo + gn) =
            *reinterpret_cast<const uint4*>(stg + rr * ROWB + ch * 16);
    }
    __syncwarp();
  }
}

template <int MODE, class OutT, int BN, bool ACC_INT>
__device__ __forceinline__ void tc_tile_epilogue_passes(const Epilogue& ep, uint32_t tacc, int q,
                                                        int lane, int64_t m0, int64_t n0, int M,
                                                        int N, uint8_t* stg) {
  tile_epilogue_passes_src<MODE, OutT, BN>(
      ep,
      [&](int c, float (&v)[32]) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tacc + (static_cast<uint32_t>(q * 32) << 16) + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if constexpr (MODE == kEpiAccI32) v[i] = __int_as_float(static_cast<int>(r[i]));
          else if constexpr (ACC_INT) v[i] = static_cast<float>(static_cast<int>(r[i]));
          else v[i] = __uint_as_float(r[i]);
        }
      },
      q, lane, m0, n0, M, N, stg);
}

// Runtime (mode, out dtype) -> template dispatch used by the launchers.
template <class F>
void dispatch_epilogue(int mode, ltm_dtype out_dt, F&& f) {
  auto with_t = [&](auto mode_c) {
    constexpr int MODE = decltype(mode_c)::value;
    if constexpr (MODE == kEpiAccI32) {
      f(mode_c, int32_t{});
    } else {
      switch (out_dt) {
        case LTM_DTYPE_F32: f(mode_c, float{}); break;
        case LTM_DTYPE_F16: f(mode_c, __half{}); break;
        case LTM_DTYPE_BF16: f(mode_c, __nv_bfloat16{}); break;
        default: LTM_REQUIRE(false, "unknown output dtype");
      }
    }
  };
  switch (mode) {
    case kEpiPlain: with_t(std::integral_constant<int, kEpiPlain>{}); break;
    case kEpiRope: with_t(std::integral_constant<int, kEpiRope>{}); break;
    case kEpiResid: with_t(std::integral_constant<int, kEpiResid>{}); break;
    case kEpiGateMix: with_t(std::integral_constant<int, kEpiGateMix>{}); break;
    case kEpiAccI32: with_t(std::integral_constant<int, kEpiAccI32>{}); break;
    default: LTM_REQUIRE(false, "unknown epilogue mode");
  }
}

}  // namespace ltm_b200

namespace ltm_b200 {

// ---------------------------------------------------------------------------
// Pipelined tensor-core epilogue with TMA stores.
//
// One epilogue warp owns 32 tile rows (its TMEM lane quarter) x CW columns of
// an accumulator tile and walks them in 32-column chunks:
//   * the per-column dequant scale and bias of the warp's CW columns and the
//     per-row activation scale are fetched one tile ahead into registers and
//     published to a per-warp shared-memory vector at the tile start (read
//     back as broadcast 16-byte loads);
//   * the TMEM load of chunk c+1 and the global operands of chunk c+1 (RoPE
//     table row, residual / gate-mix tensors) are in flight while chunk c is
//     computed;
//   * results are packed into 32-row boxes of 128 or 64 bytes per row in
//     shared memory with the matching TMA swizzle (conflict-free row writes)
//     and written by one TMA store per box; two box slots per warp alternate,
//     so packing the next box overlaps the previous store.
// The TMEM accumulator is released (on_tmem_free) as soon as the last chunk
// has been read, before its math.
// ---------------------------------------------------------------------------

template <int MODE, class OutT>
struct EpiChunkAux {
  static constexpr int kVec = 32 * static_cast<int>(sizeof(OutT)) / 16;  // uint4 per 32 values
  static constexpr int kTensors = MODE == kEpiResid ? 1 : (MODE == kEpiGateMix ? 3 : 0);
  // Residual loads go one chunk ahead in a second register set; the RoPE row
  // and the three gate-mix tensors use one set, refilled for the next chunk as
  // soon as the current chunk's math has consumed it.
  static constexpr bool kAhead = MODE == kEpiResid;
  // fp32 gate-mix reads its three tensors straight from global memory at use
  // (96 staged registers would spill).
  static constexpr bool kDirect = MODE == kEpiGateMix && sizeof(OutT) == 4;
  uint4 t[(kTensors > 0 && !kDirect) ? kTensors : 1][kVec];
  float4 rope[MODE == kEpiRope ? 8 : 1];
  const OutT* src_row[kDirect ? 3 : 1];
  bool direct_ok;

  // Issues the loads chunk (m, n) needs.  Rows >= M and chunks >= N load
  // nothing (their results are never stored).
  __device__ __forceinline__ void load(const Epilogue& ep, int64_t m, int64_t n, int pos, bool row_ok,
                                       bool col_ok) {
    if constexpr (MODE == kEpiRope) {
      if (row_ok && n < ep.rope_cols) {
        const int d0 = static_cast<int>(static_cast<uint32_t>(n) % static_cast<uint32_t>(ep.head_dim));
        const float4* tab = reinterpret_cast<const float4*>(
            ep.rope + static_cast<int64_t>(pos) * (ep.head_dim >> 1) + (d0 >> 1));
#pragma unroll
        for (int j = 0; j < 8; ++j) rope[j] = __ldg(tab + j);
      }
    } else if constexpr (kDirect) {
      direct_ok = row_ok && col_ok;
      const void* src[3] = {ep.aux0, ep.aux1, ep.aux2};
#pragma unroll
      for (int a = 0; a < 3; ++a)
        src_row[a] = direct_ok ? static_cast<const OutT*>(src[a]) + m * ep.ld_aux + n : nullptr;
    } else if constexpr (kTensors > 0) {
      if (row_ok && col_ok) {
        const void* src[3] = {ep.aux0, ep.aux1, ep.aux2};
#pragma unroll
        for (int a = 0; a < kTensors; ++a) {
          const uint4* p = reinterpret_cast<const uint4*>(static_cast<const OutT*>(src[a]) +
                                                          m * ep.ld_aux + n);
#pragma unroll
          for (int j = 0; j < kVec; ++j) t[a][j] = __ldg(p + j);
        }
      }
    }
  }

  // Element i (0..31) of tensor a of the chunk, as fp32.
  __device__ __forceinline__ float at(int a, int i) const {
    if constexpr (kDirect) {
      return direct_ok ? to_f32(__ldg(src_row[a] + i)) : 0.0f;
    } else {
      constexpr int PER = 16 / sizeof(OutT);
      return to_f32(reinterpret_cast<const OutT*>(&t[a][i / PER])[i % PER]);
    }
  }
};

// BOXB: bytes per row of one staged box, 128 (128-byte swizzle, 4 KiB boxes)
// or 64 (64-byte swizzle, 2 KiB boxes); the output tensor map's box is
// BOXB / sizeof(store type) columns x 32 rows with the same swizzle.
template <int MODE, class OutT, int CW, bool ACC_INT, int BOXB = 128>
struct TmaTileEpilogue {
  using StoreT = typename std::conditional<MODE == kEpiAccI32, int32_t, OutT>::type;
  static constexpr int NCH = CW / 32;
  static constexpr int BOXC = BOXB / static_cast<int>(sizeof(StoreT));  // columns per box
  static constexpr int UPC = 32 * static_cast<int>(sizeof(StoreT)) / 16;  // 16-byte units per chunk row
  static constexpr int UPB = BOXB / 16;                                   // 16-byte units per box row
  static constexpr uint32_t kBoxBytes = 32 * BOXB;
  // Staged boxes per tile; two slots per warp.  When both boxes of a tile fit
  // (kBatched), the warp packs the whole tile, fences once and issues both
  // stores, and waits for the previous tile's stores to leave shared memory
  // only at the next tile start.  Otherwise the slots alternate box by box.
  static constexpr int kBoxesPerTile = CW * static_cast<int>(sizeof(StoreT)) / BOXB;
  static constexpr bool kBatched = kBoxesPerTile <= 2;
  static_assert(kBatched || kBoxesPerTile % 2 == 0, "slot parity must restart at each tile");
  static constexpr bool kMath = MODE != kEpiAccI32;
  static_assert(BOXB == 128 || BOXB == 64, "box rows are 64 or 128 bytes");
  static_assert(CW % BOXC == 0, "warp columns must be whole boxes");
  // shared-memory bytes of the per-warp column vectors (scale + bias)
  static constexpr uint32_t kColBytes = 2 * CW * 4;

  float rs_next = 1.0f;
  float cs_next[NCH], bs_next[NCH];

  // Fetches the row scale of row m and the scale/bias of columns nw + 32c + lane,
  // and asks L2 for the residual / gate-mix rows the tile's chunks will load
  // (one bulk prefetch per tensor of this lane's row segment), so that their
  // loads, issued a chunk ahead, meet L2 latency rather than DRAM latency.
  __device__ __forceinline__ void prefetch(const Epilogue& ep, int64_t m, int64_t nw, int M, int N,
                                           int lane) {
    if constexpr (MODE == kEpiResid || MODE == kEpiGateMix) {
      if (m < M && nw < N) {
        const int64_t ncols = (N - nw) < CW ? (N - nw) : CW;
        const uint32_t bytes = static_cast<uint32_t>(ncols * sizeof(OutT)) & ~15u;
        const void* src[3] = {ep.aux0, ep.aux1, ep.aux2};
        constexpr int kT = MODE == kEpiResid ? 1 : 3;
#pragma unroll
        for (int a = 0; a < kT; ++a) {
          const uint8_t* row = reinterpret_cast<const uint8_t*>(
              static_cast<const OutT*>(src[a]) + m * ep.ld_aux + nw);
          if (bytes && (reinterpret_cast<uintptr_t>(row) & 15u) == 0)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(row), "r"(bytes)
                         : "memory");
        }
      }
    }
    if constexpr (kMath) {
      rs_next = (ep.row_scale && m < M) ? __ldg(ep.row_scale + m) : 1.0f;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int64_t n = nw + c * 32 + lane;
        cs_next[c] = (ep.col_scale && n < N) ? __ldg(ep.col_scale + n) : 1.0f;
        bs_next[c] = (ep.bias && n < N) ? __ldg(ep.bias + n) : 0.0f;
      }
    }
  }

  // Epilogue of one tile.  tacc: TMEM address of (lane quarter, first column);
  // m: this lane's row; row0: first row of the warp's 32 rows; nw: first
  // column; cvec: per-warp column vectors (kColBytes); stg: two staging boxes
  // (1024-byte aligned).  Returns after the last box store has been issued.
  template <class OnTmemFree>
  __device__ __forceinline__ void run(const Epilogue& ep, const CUtensorMap* tmo, uint32_t tacc,
                                      int64_t m, int row0, int nw, int M, int N, float* cvec,
                                      uint8_t* stg, int lane, OnTmemFree&& on_tmem_free) {
    const float rs = rs_next;
    if constexpr (kBatched) {
      if (lane == 0) bulk_wait_group_read<0>();  // previous tile's boxes have left the slots
    }
    if constexpr (kMath) {
      __syncwarp();  // previous tile's reads of cvec are done
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        cvec[c * 32 + lane] = cs_next[c];
        cvec[CW + c * 32 + lane] = bs_next[c];
      }
      __syncwarp();
    }
    const bool row_ok = m < M;
    int pos = 0;
    if constexpr (MODE == kEpiRope) pos = rope_row(ep, m, row_ok);

    using Aux = EpiChunkAux<MODE, OutT>;
    constexpr int kAuxSets = Aux::kAhead ? 2 : 1;
    uint32_t acc[2][32];
    Aux aux[kAuxSets];
    tmem_ld_32x32b_x32(tacc, acc[0]);
    aux[0].load(ep, m, nw, pos, row_ok, nw < N);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int cur = c & 1;
      const int ax = Aux::kAhead ? cur : 0;
      const int64_t n = nw + c * 32;
      tmem_wait_ld_tie(acc[cur]);
      if (c + 1 < NCH) {
        tmem_ld_32x32b_x32(tacc + (c + 1) * 32, acc[cur ^ 1]);
        if constexpr (Aux::kAhead) aux[cur ^ 1].load(ep, m, n + 32, pos, row_ok, n + 32 < N);
      } else {
        tc_fence_before();
        __syncwarp();
        on_tmem_free();
      }
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if constexpr (!kMath) v[i] = __int_as_float(static_cast<int>(acc[cur][i]));
        else if constexpr (ACC_INT) v[i] = static_cast<float>(static_cast<int>(acc[cur][i]));
        else v[i] = __uint_as_float(acc[cur][i]);
      }
      if constexpr (kMath) {
        // (acc * rs) * cs + bs, the last two in one FMA
        const float4* cs4 = reinterpret_cast<const float4*>(cvec + c * 32);
        const float4* bs4 = reinterpret_cast<const float4*>(cvec + CW + c * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 s = cs4[j], b = bs4[j];
          v[4 * j] = fmaf(v[4 * j] * rs, s.x, b.x);
          v[4 * j + 1] = fmaf(v[4 * j + 1] * rs, s.y, b.y);
          v[4 * j + 2] = fmaf(v[4 * j + 2] * rs, s.z, b.z);
          v[4 * j + 3] = fmaf(v[4 * j + 3] * rs, s.w, b.w);
        }
        if (ep.act == LTM_EPI_GELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
        } else if (ep.act == LTM_EPI_SIGMOID) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = sigmoid_f(v[i]);
        }
        if constexpr (MODE == kEpiRope) {
          if (n < ep.rope_cols) {
            const float* rp = reinterpret_cast<const float*>(aux[ax].rope);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float cs = rp[i], sn = rp[i + 1];
              const float a = v[i], b = v[i + 1];
              v[i] = a * cs - b * sn;
              v[i + 1] = a * sn + b * cs;
            }
          }
        } else if constexpr (MODE == kEpiResid) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] += aux[ax].at(0, i);
        } else if constexpr (MODE == kEpiGateMix) {
          // y = (s + g*mem) + (1-g)*x with g = v; g*x feeds the memory write
          float gx[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float g = v[i], xv = aux[ax].at(2, i);
            const float sm = aux[ax].at(0, i) + g * aux[ax].at(1, i);
            gx[i] = row_ok ? g * xv : 0.0f;
            v[i] = sm + (1.0f - g) * xv;
          }
          if (ep.colsum) {
            const float csum = warp_colsum32(gx);
            if (n < N) atomicAdd(ep.colsum + n + lane, csum);
          }
        }
      }
      if constexpr (!Aux::kAhead) {
        if (c + 1 < NCH) aux[0].load(ep, m, n + 32, pos, row_ok, n + 32 < N);
      }
      // Pack into staging boxes.  Unit k of this chunk is unit g = c*UPC + k
      // of the warp's row, i.e. unit g % UPB of box g / UPB.  Swizzle (as the
      // TMA applies it): 128-byte rows, unit u of row r at u ^ (r & 7);
      // 64-byte rows, unit u of row r at u ^ ((r >> 1) & 3).
      constexpr int EPU = 16 / static_cast<int>(sizeof(StoreT));
#pragma unroll
      for (int k = 0; k < UPC; ++k) {
        const int g = c * UPC + k;
        const int ub = g % UPB;
        const int sb = (g / UPB) & 1;  // slot of this box (compile-time)
        if (!kBatched && ub == 0) {
          if (lane == 0) bulk_wait_group_read<1>();  // the store that last read slot sb is done
          __syncwarp();
        }
        uint4 raw;
        if constexpr (!kMath) {
          raw.x = __float_as_uint(v[k * 4 + 0]);
          raw.y = __float_as_uint(v[k * 4 + 1]);
          raw.z = __float_as_uint(v[k * 4 + 2]);
          raw.w = __float_as_uint(v[k * 4 + 3]);
        } else {
          StoreT* e = reinterpret_cast<StoreT*>(&raw);
#pragma unroll
          for (int i = 0; i < EPU; ++i) e[i] = from_f32<StoreT>(v[k * EPU + i]);
        }
        const int unit = BOXB == 128 ? (ub ^ (lane & 7)) : (ub ^ ((lane >> 1) & 3));
        *reinterpret_cast<uint4*>(stg + sb * kBoxBytes + lane * BOXB + unit * 16) = raw;
        const bool last_box_unit = kBatched ? (g == NCH * UPC - 1) : (ub == UPB - 1);
        if (last_box_unit) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            constexpr int kFirst = kBatched ? 0 : -1;
#pragma unroll
            for (int bi = (kBatched ? kFirst : g / UPB); bi <= g / UPB; ++bi) {
              const int x = nw + bi * BOXC;
              if (row0 < M && x < N)  // boxes wholly outside the output are skipped
                tma_store_2d(tmo, stg + (bi & 1) * kBoxBytes, x, row0);
            }
            bulk_commit_group();
          }
        }
      }
    }
  }
};

}  // namespace ltm_b200
