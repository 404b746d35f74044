// memory.cu -- memory-bank write after the read (TB-v1), bandwidth-bound.
//
//   c_j = (1/T) sum_t g[t,j] * x[t,j]      (column sums accumulated by the
//                                            gate-mix epilogue of the gate GEMM)
//   w_s = rate * (1/nh) sum_h softmax_s( qbar_h . K_M[s, h] / sqrt(dh) ),
//         qbar = (1/T) sum_t qm[t]          (use_attention_scores; else w_s = rate)
//   M[s,j] <- (1 - w_s) M[s,j] + w_s c_j
//
// Follows MemoryBank<T>::store / storeStateKernel
// (src/core/ltm/memory_bank.cu:39-68,242-274: EMA with weight
// update_rate * attention_score[slot], state broadcast to every slot) with the
// pooled state of the paper's compression (mean over the segment).
#include <memory>
#include <mutex>
#include <vector>

#include "block.cuh"

namespace ltm_b200 {
namespace {

// out[j] += sum over rows of x[t, j] (x: [T, ld] act dtype, first H columns).
template <class T>
__global__ void __launch_bounds__(256) colsum_kernel(const T* __restrict__ x, int64_t ld, int64_t rows,
                                                     int H, float* __restrict__ out) {
  __shared__ float red[8][33];
  const int cx = threadIdx.x & 31, ry = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + cx;
  const int64_t per = (rows + gridDim.y - 1) / gridDim.y;
  const int64_t r0 = blockIdx.y * per, r1 = min(rows, r0 + per);
  float acc = 0.0f;
  if (col < H)
    for (int64_t r = r0 + ry; r < r1; r += 8) acc += to_f32(x[r * ld + col]);
  red[ry][cx] = acc;
  __syncthreads();
  if (ry == 0 && col < H) {
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i][cx];
    atomicAdd(out + col, t);
  }
}

// Slot softmax of the mean memory query against K_M, one cluster of kSlotCL
// CTAs per head: CTA r of the cluster scores the slots [r*per, (r+1)*per)
// (lane groups of dh/8 lanes read one slot's 16-byte pieces of the head's key
// row: coalesced, 16 loads in flight per lane), the softmax max and sum are
// combined over the cluster through distributed shared memory, and every CTA
// adds its slots' weights rate / nh_total * softmax into wslot (the mean over
// all heads; a tensor-parallel rank adds its own heads and the ranks sum
// wslot).
constexpr int kSlotCL = 8;
constexpr int kSlotUnroll = 4;

// 8 consecutive elements (16-byte aligned) as floats.
template <class T>
__device__ __forceinline__ void load8_f32(const T* p, float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32(e[i]);
  }
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

template <class T>
__global__ void __cluster_dims__(kSlotCL, 1, 1) __launch_bounds__(256)
    slot_weight_kernel(const float* __restrict__ qsum, float inv_T, const T* __restrict__ kvm,
                       int64_t ldk, int Ms, int dh, int nh_total, float rate,
                       float* __restrict__ wslot) {
  extern __shared__ float sc[];  // [per] scores of this CTA's slots
  __shared__ __align__(16) float qh[128];
  __shared__ float red[8];
  __shared__ float stat[2];  // this CTA's (max, sum), read by the cluster
  const int h = blockIdx.y;
  const int r = static_cast<int>(cluster_ctarank());
  const int per = (Ms + kSlotCL - 1) / kSlotCL;
  const int s0 = min(Ms, r * per), s1 = min(Ms, s0 + per);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = rsqrtf(static_cast<float>(dh));
  for (int e = threadIdx.x; e < dh; e += blockDim.x) qh[e] = qsum[h * dh + e] * inv_T;
  __syncthreads();
  // lane group g of LPS = dh/8 lanes scores one slot per step
  const int lps = dh >> 3, spw = 32 / lps;  // lanes per slot, slots per warp step
  const int gl = lane % lps, g = lane / lps;
  float q8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q8[i] = qh[gl * 8 + i];
  float mx = -INFINITY;
  const int step = 8 * spw;  // slots per CTA step
  for (int sb = s0 + warp * spw; sb < s1; sb += step * kSlotUnroll) {
    float kv[kSlotUnroll][8];
#pragma unroll
    for (int u = 0; u < kSlotUnroll; ++u) {
      const int s = sb + u * step + g;
      if (s < s1) {
        load8_f32(kvm + static_cast<int64_t>(s) * ldk + h * dh + gl * 8, kv[u]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) kv[u][i] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < kSlotUnroll; ++u) {
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(q8[i], kv[u][i], d);
      for (int o = lps >> 1; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const int s = sb + u * step + g;
      if (s < s1) {
        d *= scale;
        if (gl == 0) sc[s - s0] = d;
        mx = fmaxf(mx, d);
      }
    }
  }
  // cluster max
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    stat[0] = m;
  }
  cluster_sync();
  float gmax = -INFINITY;
  for (int c = 0; c < kSlotCL; ++c) gmax = fmaxf(gmax, ld_cluster_f32(mapa_shared(&stat[0], c)));
  // cluster sum of exp(score - max)
  float sum = 0.0f;
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const float e = expf(sc[s - s0] - gmax);
    sc[s - s0] = e;
    sum += e;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < 8; ++i) t += red[i];
    stat[1] = t;
  }
  cluster_sync();
  float gsum = 0.0f;
  for (int c = 0; c < kSlotCL; ++c) gsum += ld_cluster_f32(mapa_shared(&stat[1], c));
  const float f = rate / (gsum * static_cast<float>(nh_total));
  for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) atomicAdd(wslot + s, sc[s - s0] * f);
  cluster_sync();  // no CTA leaves while the cluster still reads its stat
}

template <class T>
__global__ void __launch_bounds__(256) bank_update_kernel(T* __restrict__ mem,
                                                          const float* __restrict__ state,
                                                          float state_scale,
                                                          const float* __restrict__ wslot,
                                                          float rate, int Ms, int H) {
  const int64_t n = static_cast<int64_t>(Ms) * H;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(i / H), j = static_cast<int>(i - static_cast<int64_t>(s) * H);
    const float w = wslot ? wslot[s] : rate;
    const float c = state[j] * state_scale;
    mem[i] = from_f32<T>((1.0f - w) * to_f32(mem[i]) + w * c);
  }
}

// rows[s, :] = (1 - w_s) rows[s, :] + w_s v  (K_M | V_M following the bank's
// EMA; v = the state row's projection), 8 elements per thread.
template <class T>
__global__ void __launch_bounds__(256) rows_ema_kernel(T* __restrict__ rows, int64_t ld, int width,
                                                       const T* __restrict__ v,
                                                       const float* __restrict__ wslot, float rate,
                                                       int Ms) {
  const int nv = width / 8;
  const int64_t n = static_cast<int64_t>(Ms) * nv;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(i / nv), c = static_cast<int>(i - static_cast<int64_t>(s) * nv);
    const float w = wslot ? wslot[s] : rate;
    uint4* rp = reinterpret_cast<uint4*>(rows + s * ld) + c;
    uint4 r = *rp;
    const uint4 vv = __ldg(reinterpret_cast<const uint4*>(v) + c);
    T* re = reinterpret_cast<T*>(&r);
    const T* ve = reinterpret_cast<const T*>(&vv);
#pragma unroll
    for (int k = 0; k < 8; ++k) re[k] = from_f32<T>((1.0f - w) * to_f32(re[k]) + w * to_f32(ve[k]));
    *rp = r;
  }
}

// out[j] = state[j] * scale in the activation dtype
template <class T>
__global__ void state_row_kernel(const float* __restrict__ state, float scale, T* __restrict__ out,
                                 int H) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < H; j += gridDim.x * blockDim.x)
    out[j] = from_f32<T>(state[j] * scale);
}

// bank_update_kernel on 8 elements (16-bit, 16-byte aligned) per thread
// (H a multiple of 8); the same arithmetic per element.
template <class T>
__global__ void __launch_bounds__(256) bank_update8_kernel(T* __restrict__ mem,
                                                           const float* __restrict__ state,
                                                           float state_scale,
                                                           const float* __restrict__ wslot,
                                                           float rate, int Ms, int H) {
  const int nv = H / 8;
  const int64_t n = static_cast<int64_t>(Ms) * nv;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(i / nv), c = static_cast<int>(i - static_cast<int64_t>(s) * nv);
    const float w = wslot ? wslot[s] : rate;
    uint4* mp = reinterpret_cast<uint4*>(mem + static_cast<int64_t>(s) * H) + c;
    uint4 r = *mp;
    T* e = reinterpret_cast<T*>(&r);
    const float4 a = __ldg(reinterpret_cast<const float4*>(state + c * 8));
    const float4 b = __ldg(reinterpret_cast<const float4*>(state + c * 8) + 1);
    const float cv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 8; ++k)
      e[k] = from_f32<T>((1.0f - w) * to_f32(e[k]) + w * (cv[k] * state_scale));
    *mp = r;
  }
}

}  // namespace

void launch_rows_ema(void* rows, int64_t ld, int width, const void* v, const float* wslot,
                     float rate, int Ms, ltm_dtype dt, cudaStream_t st) {
  LTM_REQUIRE(dt != LTM_DTYPE_F32 && width % 8 == 0 && ld % 8 == 0,
              "row EMA needs 16-bit rows of a multiple of 8 elements");
  dispatch_dtype(dt, [&](auto tag) {
    using TT = decltype(tag);
    const int64_t n = static_cast<int64_t>(Ms) * (width / 8);
    const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, device_sm_count() * 8));
    rows_ema_kernel<TT><<<grid, 256, 0, st>>>(static_cast<TT*>(rows), ld, width,
                                              static_cast<const TT*>(v), wslot, rate, Ms);
    check_launch("rows_ema_kernel", st);
  });
}

void launch_state_row(const float* state, float scale, void* out, int H, ltm_dtype dt,
                      cudaStream_t st) {
  dispatch_dtype(dt, [&](auto tag) {
    using TT = decltype(tag);
    state_row_kernel<TT><<<(H + 255) / 256, 256, 0, st>>>(state, scale, static_cast<TT*>(out), H);
    check_launch("state_row_kernel", st);
  });
}

void MemoryWriteState::prepare_gate_epilogue(Epilogue& ep, int H, cudaStream_t st) {
  colsum.ensure(H * sizeof(float));
  LTM_CUDA_TRY(cudaMemsetAsync(colsum.ptr, 0, H * sizeof(float), st));
  ep.colsum = colsum.as<float>();
}

void launch_slot_weights(const void* keys, int64_t ldk, const void* queries, int64_t ldq,
                         int64_t T, int Ms, int heads, int dh, int nh_total, float rate,
                         ltm_dtype dt, float* qsum, float* wslot, cudaStream_t st) {
  const int Hq = heads * dh;
  LTM_REQUIRE(dh == 8 || dh == 16 || dh == 32 || dh == 64 || dh == 128,
              "attention-score slot weights need head_dim 8, 16, 32, 64 or 128");
  LTM_REQUIRE(reinterpret_cast<uintptr_t>(keys) % 16 == 0 && (ldk * dtype_size(dt)) % 16 == 0,
              "keys must be 16-byte aligned with a row stride of a multiple of 16 bytes");
  dispatch_dtype(dt, [&](auto tag) {
    using TT = decltype(tag);
    LTM_CUDA_TRY(cudaMemsetAsync(qsum, 0, Hq * sizeof(float), st));
    LTM_CUDA_TRY(cudaMemsetAsync(wslot, 0, Ms * sizeof(float), st));
    const int splits = static_cast<int>(std::min<int64_t>(64, (T + 63) / 64));
    dim3 g1((Hq + 31) / 32, splits);
    colsum_kernel<TT><<<g1, 256, 0, st>>>(static_cast<const TT*>(queries), ldq, T, Hq, qsum);
    check_launch("colsum_kernel", st);
    const size_t smem = static_cast<size_t>((Ms + kSlotCL - 1) / kSlotCL) * sizeof(float);
    auto kern = slot_weight_kernel<TT>;
    LTM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
    kern<<<dim3(kSlotCL, heads), 256, smem, st>>>(qsum, 1.0f / static_cast<float>(T),
                                                  static_cast<const TT*>(keys), ldk, Ms, dh,
                                                  nh_total, rate, wslot);
    check_launch("slot_weight_kernel", st);
  });
}

void launch_bank_update(void* memory, const float* state, float state_scale, const float* wslot,
                        float rate, int Ms, int H, ltm_dtype dt, cudaStream_t st) {
  dispatch_dtype(dt, [&](auto tag) {
    using TT = decltype(tag);
    const bool vec = sizeof(TT) == 2 && H % 8 == 0 && reinterpret_cast<uintptr_t>(memory) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(state) % 16 == 0;
    const int64_t n = static_cast<int64_t>(Ms) * (vec ? H / 8 : H);
    const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, device_sm_count() * 8));
    if (vec)
      bank_update8_kernel<TT><<<grid, 256, 0, st>>>(static_cast<TT*>(memory), state, state_scale,
                                                    wslot, rate, Ms, H);
    else
      bank_update_kernel<TT><<<grid, 256, 0, st>>>(static_cast<TT*>(memory), state, state_scale,
                                                   wslot, rate, Ms, H);
    check_launch("bank_update_kernel", st);
  });
}

void launch_memory_store(void* memory, const void* keys, int64_t ldk, const void* queries,
                         int64_t ldq, int64_t T, const float* state, float state_scale, int Ms,
                         int H, int nh, float rate, bool use_scores, ltm_dtype dt, float* qsum,
                         float* wslot, cudaStream_t st) {
  if (Ms == 0 || H == 0) return;
  if (use_scores)
    launch_slot_weights(keys, ldk, queries, ldq, T, Ms, nh, H / nh, nh, rate, dt, qsum, wslot, st);
  launch_bank_update(memory, state, state_scale, use_scores ? wslot : nullptr, rate, Ms, H, dt, st);
}

void validate_memory_store(const void* memory, const void* keys, int64_t ldk, const void* queries,
                           int64_t ldq, int64_t T, const float* state, int Ms, int H, int nh,
                           bool use_scores) {
  LTM_REQUIRE(Ms >= 0 && H >= 0 && T >= 0, "negative size");
  LTM_REQUIRE(memory && state, "NULL pointer");
  LTM_REQUIRE(nh > 0 && H % nh == 0, "hidden size must be a multiple of num_heads");
  if (use_scores) {
    LTM_REQUIRE(T > 0, "attention-score slot weights need at least one query row");
    LTM_REQUIRE(keys && queries, "NULL keys / queries");
    LTM_REQUIRE(ldk >= H && ldq >= H, "row strides smaller than the hidden size");
    LTM_REQUIRE(static_cast<size_t>(Ms) * sizeof(float) <= 200 * 1024,
                "memory_slots too large for the slot-weight kernel (max 51200)");
  }
}

float MemoryWriteState::update_bank(void* memory, const void* kvm, int64_t ldk, const void* qm,
                                    int64_t ldq, int64_t T, int H, int heads, int nh_total, int dh,
                                    int Ms, float rate, bool use_scores, ltm_dtype dt,
                                    ltm_comm* comm, cudaStream_t st, bool colsum_partial) {
  if (T == 0 || Ms == 0) return 0.0f;
  const int Hq = heads * dh;
  if (use_scores) {
    qsum.ensure(Hq * sizeof(float));
    wslot.ensure(Ms * sizeof(float));
    validate_memory_store(memory, kvm, ldk, qm, ldq, T, colsum.as<float>(), Ms, Hq, heads, true);
    launch_slot_weights(kvm, ldk, qm, ldq, T, Ms, heads, dh, nh_total, rate, dt, qsum.as<float>(),
                        wslot.as<float>(), st);
    if (comm && comm->nranks > 1)  // every rank adds its heads' share of the head mean
      comm_allreduce(comm, wslot.ptr, wslot.ptr, Ms, LTM_DTYPE_F32, false, st);
  }
  float state_scale = 1.0f / static_cast<float>(T);
  if (comm && comm->nranks > 1) {
    // Replicated gate: every rank accumulated the same column sums, in its
    // own atomic order, and their mean makes the state -- and so the bank --
    // identical on all ranks.  Sequence-parallel gate: each rank summed its
    // own rows, and the sum over the ranks is the total.
    comm_allreduce(comm, colsum.ptr, colsum.ptr, H, LTM_DTYPE_F32, false, st);
    if (!colsum_partial) state_scale /= static_cast<float>(comm->nranks);
  }
  launch_bank_update(memory, colsum.as<float>(), state_scale,
                     use_scores ? wslot.as<float>() : nullptr, rate, Ms, H, dt, st);
  return state_scale;
}

namespace {
// Per-device scratch of ltm_memory_store (query column sums [H], slot weights
// [Ms]); grown on demand, freed at exit.
struct StoreScratch {
  DevBuf qsum, wslot;
};
StoreScratch& store_scratch(int dev) {
  static std::mutex mu;
  static std::vector<std::unique_ptr<StoreScratch>> per_dev;
  std::lock_guard<std::mutex> lk(mu);
  if (static_cast<int>(per_dev.size()) <= dev) per_dev.resize(dev + 1);
  if (!per_dev[dev]) per_dev[dev] = std::make_unique<StoreScratch>();
  return *per_dev[dev];
}
}  // namespace

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_memory_store(void* memory, const void* keys, int64_t ldk,
                                       const void* queries, int64_t ldq, int64_t T,
                                       const float* state, int memory_slots, int hidden_dim,
                                       int num_heads, float update_rate, int use_attention_scores,
                                       ltm_dtype dtype, void* stream) {
  return guarded([&] {
    const bool scores = use_attention_scores != 0;
    validate_memory_store(memory, keys, ldk, queries, ldq, T, state, memory_slots, hidden_dim,
                          num_heads, scores);
    if (memory_slots == 0 || hidden_dim == 0) return;
    int dev = 0;
    LTM_CUDA_TRY(cudaGetDevice(&dev));
    StoreScratch& sc = store_scratch(dev);
    if (scores) {
      sc.qsum.ensure(static_cast<size_t>(hidden_dim) * sizeof(float));
      sc.wslot.ensure(static_cast<size_t>(memory_slots) * sizeof(float));
    }
    launch_memory_store(memory, keys, ldk, queries, ldq, T, state, 1.0f, memory_slots, hidden_dim,
                        num_heads, update_rate, scores, dtype, sc.qsum.as<float>(),
                        sc.wslot.as<float>(), as_stream(stream));
  });
}
