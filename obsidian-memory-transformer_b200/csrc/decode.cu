// decode.cu -- one decoding step of the Titan block against a KV cache:
// appending the new token's keys / values and the self-attention read of the
// whole cache (flash decoding, HBM-bound).
//
// Cache layout: per sequence b a [max_positions, width] row-major block of the
// activation dtype (width = hidden, or this rank's heads under tensor
// parallelism), head h at columns h*D; position p of sequence b at
// cache + b * seq_stride + p * width.
//
// Attention of one query row per (sequence, head) over L cached positions:
// the positions are split into chunks of kChunk; a 128-thread CTA reads one
// chunk of one (sequence, head): 4 warps x 4 key groups of 8 lanes, lane l of
// a group holding dims [l*D/8, (l+1)*D/8) of q, of the running output and of
// the key / value rows it reads (each group reads whole rows, the 4 groups of
// a warp consecutive rows).  Scores are reduced across the group's 8 lanes;
// every group keeps its own online-softmax state (max, sum, output), combined
// across the groups and warps of the CTA into one partial (max, sum, output)
// per chunk; decode_combine_kernel merges the chunks.  Every key and value
// byte is read once.
//
// Replaces the KV-cache decode stubs of the reference
// (python_bindings/src/main.cpp:101-135, python_bindings/ltm/inference.py:101-128)
// with the attention of flash_attention.cu:241 (scale 1/sqrt(head_dim)).
#include "block.cuh"

namespace ltm_b200 {
namespace {

constexpr int kChunk = 512;  // cache positions per CTA
constexpr int kKB = 4;       // keys per group per step

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

template <class T>
__global__ void __launch_bounds__(256) kv_append_kernel(const T* __restrict__ qkv, int64_t ldq,
                                                        int width, T* __restrict__ kc,
                                                        T* __restrict__ vc, int64_t seq_stride,
                                                        int64_t pos) {
  const int b = blockIdx.x;
  const int nv = width * static_cast<int>(sizeof(T)) / 16;
  const uint4* ks = reinterpret_cast<const uint4*>(qkv + b * ldq + width);
  const uint4* vs = reinterpret_cast<const uint4*>(qkv + b * ldq + 2 * static_cast<int64_t>(width));
  uint4* kd = reinterpret_cast<uint4*>(kc + b * seq_stride + pos * width);
  uint4* vd = reinterpret_cast<uint4*>(vc + b * seq_stride + pos * width);
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

template <class T, int D>
__global__ void __launch_bounds__(128) decode_attn_kernel(
    const T* __restrict__ q, int64_t ldq, const T* __restrict__ kc, const T* __restrict__ vc,
    int64_t seq_stride, int width, int L, float sl2, float* __restrict__ part, int nchunk) {
  constexpr int DL = D / 8;  // dims per lane
  __shared__ float sm[4][D + 2];
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, gl = lane & 7;
  float qv[DL];
  load_row_part<T, DL>(q + b * ldq + h * D, gl, qv);
  const T* kb = kc + b * seq_stride + h * D;
  const T* vb = vc + b * seq_stride + h * D;
  const int c0 = chunk * kChunk;
  const int c1 = min(L, c0 + kChunk);
  const int w0 = c0 + warp * (kChunk / 4);  // this warp's 128 positions
  float m = -INFINITY, l = 0.0f, o[DL];
#pragma unroll
  for (int i = 0; i < DL; ++i) o[i] = 0.0f;
  for (int i0 = 0; i0 < kChunk / 4; i0 += 4 * kKB) {
    float s[kKB];
    float vv[kKB][DL];
    bool valid[kKB];
#pragma unroll
    for (int j = 0; j < kKB; ++j) {
      const int k = w0 + i0 + 4 * j + grp;  // the warp's 4 groups read 4 consecutive rows
      valid[j] = k < c1;
      float kr[DL];
      if (valid[j]) {
        load_row_part<T, DL>(kb + static_cast<int64_t>(k) * width, gl, kr);
        load_row_part<T, DL>(vb + static_cast<int64_t>(k) * width, gl, vv[j]);
      } else {
#pragma unroll
        for (int i = 0; i < DL; ++i) kr[i] = vv[j][i] = 0.0f;
      }
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < DL; ++i) d = fmaf(qv[i], kr[i], d);
      s[j] = d;
    }
#pragma unroll
    for (int j = 0; j < kKB; ++j) {  // sum over the group's 8 lanes
      s[j] += __shfl_xor_sync(0xffffffffu, s[j], 1);
      s[j] += __shfl_xor_sync(0xffffffffu, s[j], 2);
      s[j] += __shfl_xor_sync(0xffffffffu, s[j], 4);
      if (!valid[j]) s[j] = -INFINITY;
    }
    float mb = s[0];
#pragma unroll
    for (int j = 1; j < kKB; ++j) mb = fmaxf(mb, s[j]);
    // no branch on the group's state: the shuffles above need the whole warp
    const float m_new = fmaxf(m, mb);
    const float mu = (m_new == -INFINITY) ? 0.0f : m_new;  // nothing visible yet
    const float corr = ex2_approx((m - mu) * sl2);  // m = -inf -> 0
    l *= corr;
#pragma unroll
    for (int i = 0; i < DL; ++i) o[i] *= corr;
#pragma unroll
    for (int j = 0; j < kKB; ++j) {
      const float pj = ex2_approx((s[j] - mu) * sl2);  // -inf -> 0
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
  if (grp == 0) {
#pragma unroll
    for (int i = 0; i < DL; ++i) sm[warp][part_dim(gl, i)] = o[i];
    if (gl == 0) {
      sm[warp][D] = mw;
      sm[warp][D + 1] = l;
    }
  }
  __syncthreads();
  // merge the 4 warps; thread t < D writes output dim t of the chunk's partial
  if (threadIdx.x < D) {
    float mc = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mc = fmaxf(mc, sm[w][D]);
    float lc = 0.0f, oc = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float g = (mc == -INFINITY) ? 0.0f : ex2_approx((sm[w][D] - mc) * sl2);
      lc += sm[w][D + 1] * g;
      oc += sm[w][threadIdx.x] * g;
    }
    float* pp = part + ((static_cast<int64_t>(b) * gridDim.y + h) * nchunk + chunk) * (D + 2);
    pp[threadIdx.x] = oc;
    if (threadIdx.x == 0) {
      pp[D] = mc;
      pp[D + 1] = lc;
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
  const int64_t nchunk = (L + kChunk - 1) / kChunk;
  return static_cast<size_t>(B) * nh * nchunk * (D + 2) * sizeof(float);
}

void launch_kv_append(const void* qkv, int64_t ldq, int width, void* kc, void* vc,
                      int64_t seq_stride, int64_t pos, int B, ltm_dtype dt, cudaStream_t st) {
  LTM_REQUIRE((width * dtype_size(dt)) % 16 == 0, "cache width must be a multiple of 16 bytes");
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    kv_append_kernel<T><<<B, 256, 0, st>>>(static_cast<const T*>(qkv), ldq, width,
                                            static_cast<T*>(kc), static_cast<T*>(vc), seq_stride,
                                            pos);
  });
  check_launch("kv_append_kernel", st);
}

void launch_decode_attention(const void* q, int64_t ldq, const void* kc, const void* vc,
                             int64_t seq_stride, int width, int L, int B, int nh, int D,
                             ltm_dtype dt, float* part, void* o, int64_t ldo, cudaStream_t st) {
  LTM_REQUIRE(D == 64 || D == 128, "decode attention head_dim must be 64 or 128");
  LTM_REQUIRE(L >= 1, "empty cache");
  LTM_REQUIRE(dt != LTM_DTYPE_F32, "decode attention needs 16-bit activations");
  const int nchunk = (L + kChunk - 1) / kChunk;
  const float sl2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (!std::is_same<T, float>::value) {
      dim3 grid(nchunk, nh, B);
      if (D == 64) {
        decode_attn_kernel<T, 64><<<grid, 128, 0, st>>>(
            static_cast<const T*>(q), ldq, static_cast<const T*>(kc), static_cast<const T*>(vc),
            seq_stride, width, L, sl2, part, nchunk);
        check_launch("decode_attn_kernel", st);
        decode_combine_kernel<T, 64><<<dim3(nh, B), 64, 0, st>>>(part, nchunk, sl2,
                                                                 static_cast<T*>(o), ldo);
      } else {
        decode_attn_kernel<T, 128><<<grid, 128, 0, st>>>(
            static_cast<const T*>(q), ldq, static_cast<const T*>(kc), static_cast<const T*>(vc),
            seq_stride, width, L, sl2, part, nchunk);
        check_launch("decode_attn_kernel", st);
        decode_combine_kernel<T, 128><<<dim3(nh, B), 128, 0, st>>>(part, nchunk, sl2,
                                                                   static_cast<T*>(o), ldo);
      }
      check_launch("decode_combine_kernel", st);
    }
  });
}

}  // namespace ltm_b200
