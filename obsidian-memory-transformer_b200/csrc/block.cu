// block.cu -- Titan block and multi-layer model over the kernels (C ABI).
//
// TB-v1 block forward (x, y: [B*S, H] in the activation dtype):
//   h   = LN(x + x)                      (+ per-token int8 of h and of x for W8A8)
//   qkvm= h [Wq;Wk;Wv;Wqm]^T + b         RoPE on the Q and K columns in the epilogue
//   kvm = M [Wkm;Wvm]^T + b              memory keys / values from the bank M [Ms,H]
//   os  = causal_attn(q, k, v)           om = attn(qm, K_M, V_M)   (bank shared by the batch)
//   s   = os Wo^T + bo                   m  = om Wom^T + bom
//   y   = s + g*m + (1-g)*x,  g = sigmoid(x Wg^T + bg)   (gate-mix epilogue of the gate GEMM)
//   out = y + W2 GELU(W1 LN(y + y) + b1) + b2            (residual epilogue of the FFN-down GEMM)
// with the memory write after the read (optional, see memory.cu).
// Reference: TitanBlock<T>::forward, src/core/transformer/titan_inspired_block.cu:254-345.
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

#include "block.cuh"

namespace ltm_b200 {

// ------------------------------------------------------------ device memory --
DevBuf::~DevBuf() { release(); }
void DevBuf::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
}
void DevBuf::ensure(size_t n) {
  if (n <= bytes) return;
  release();
  LTM_CUDA_TRY(cudaMalloc(&ptr, n));
  note_device_alloc();
  bytes = n;
}

namespace {

template <class T>
__global__ void f32_to_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = from_f32<T>(src[i]);
}

template <class T>
__global__ void add3_kernel(const T* __restrict__ a, const T* __restrict__ b,
                            const T* __restrict__ c, T* __restrict__ y, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = from_f32<T>(to_f32(a[i]) + to_f32(b[i]) + (c ? to_f32(c[i]) : 0.0f));
}

// int32 accumulator rows summed over the ranks' slots (4 columns per
// thread), then the tensor-core epilogue's arithmetic.
template <class T>
__global__ void sum_slots_i32_kernel(const int4* __restrict__ slots, const int4* __restrict__ own,
                                     int nslots, int own_slot, int64_t stride4,
                                     const float* __restrict__ rs, const float4* __restrict__ cs,
                                     const float4* __restrict__ bias, const T* __restrict__ add,
                                     T* __restrict__ y, int64_t rows, int64_t cols4) {
  const int64_t n = rows * cols4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols4, c4 = i - r * cols4;
    int4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < nslots) v[j] = __ldcs(j == own_slot ? own + i : slots + j * stride4 + i);
    int acc[4] = {0, 0, 0, 0};
    for (int j = 0; j < nslots; ++j) {
      const int4 w = j < 8 ? v[j] : __ldcs(j == own_slot ? own + i : slots + j * stride4 + i);
      acc[0] += w.x;
      acc[1] += w.y;
      acc[2] += w.z;
      acc[3] += w.w;
    }
    const float rsv = rs ? __ldg(rs + r) : 1.0f;
    const float4 csv = cs ? __ldg(cs + c4) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
    const float4 bv = bias ? __ldg(bias + c4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float o[4];
    o[0] = fmaf(static_cast<float>(acc[0]) * rsv, csv.x, bv.x);
    o[1] = fmaf(static_cast<float>(acc[1]) * rsv, csv.y, bv.y);
    o[2] = fmaf(static_cast<float>(acc[2]) * rsv, csv.z, bv.z);
    o[3] = fmaf(static_cast<float>(acc[3]) * rsv, csv.w, bv.w);
    if (add) {
      const uint2 w = __ldg(reinterpret_cast<const uint2*>(add) + i);
      const T* e16 = reinterpret_cast<const T*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] += to_f32(e16[e]);
    }
    uint2 out;
    T* o16 = reinterpret_cast<T*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) o16[e] = from_f32<T>(o[e]);
    reinterpret_cast<uint2*>(y)[i] = out;
  }
}

int grid_for(int64_t n) {
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  int64_t g = (n + 255) / 256;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

void upload_f32_as(const float* host, int64_t n, ltm_dtype dt, void* dev, cudaStream_t stream) {
  if (n == 0) return;
  if (dt == LTM_DTYPE_F32) {
    LTM_CUDA_TRY(cudaMemcpyAsync(dev, host, n * sizeof(float), cudaMemcpyHostToDevice, stream));
    return;
  }
  DevBuf tmp;
  tmp.ensure(n * sizeof(float));
  LTM_CUDA_TRY(cudaMemcpyAsync(tmp.ptr, host, n * sizeof(float), cudaMemcpyHostToDevice, stream));
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    f32_to_kernel<T><<<grid_for(n), 256, 0, stream>>>(static_cast<const float*>(tmp.ptr),
                                                      static_cast<T*>(dev), n);
  });
  check_launch("f32_to_kernel", stream);
  LTM_CUDA_TRY(cudaStreamSynchronize(stream));
}

void launch_add3(const void* a, const void* b, const void* c, void* y, int64_t n, ltm_dtype dt,
                 cudaStream_t stream) {
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    add3_kernel<T><<<grid_for(n), 256, 0, stream>>>(static_cast<const T*>(a), static_cast<const T*>(b),
                                                    static_cast<const T*>(c), static_cast<T*>(y), n);
  });
  check_launch("add3_kernel", stream);
}

void launch_sum_slots_i32(const int32_t* slots, const int32_t* own, int nslots, int own_slot,
                          int64_t slot_stride, const float* row_scale, const float* col_scale,
                          const float* bias, const void* add, void* y, int64_t rows, int64_t cols,
                          ltm_dtype dt, cudaStream_t stream) {
  LTM_REQUIRE(dt != LTM_DTYPE_F32, "slot sums are for 16-bit rows");
  LTM_REQUIRE(cols % 4 == 0 && slot_stride % 4 == 0, "slot rows must be whole 16-byte units");
  auto al = [](const void* q, unsigned m) { return (reinterpret_cast<uintptr_t>(q) & m) == 0; };
  LTM_REQUIRE(al(slots, 15) && al(own, 15) && al(y, 7) && (!add || al(add, 7)) &&
                  (!col_scale || al(col_scale, 15)) && (!bias || al(bias, 15)),
              "slot buffers misaligned");
  const int64_t n = rows * (cols / 4);
  if (n == 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (sizeof(T) == 2)
      sum_slots_i32_kernel<T><<<grid_for(n), 256, 0, stream>>>(
          reinterpret_cast<const int4*>(slots), reinterpret_cast<const int4*>(own), nslots,
          own_slot, slot_stride / 4, row_scale, reinterpret_cast<const float4*>(col_scale),
          reinterpret_cast<const float4*>(bias), static_cast<const T*>(add), static_cast<T*>(y),
          rows, cols / 4);
  });
  check_launch("sum_slots_i32_kernel", stream);
}

// ------------------------------------------------------------ quantized W --
void QLinear::load(const ltm_quant_config& q, const float* w_host, const float* b_host,
                   int64_t n, int64_t k, cudaStream_t stream) {
  N = n;
  K = k;
  scheme = q.scheme;
  DevBuf wd;
  wd.ensure(N * K * sizeof(float));
  LTM_CUDA_TRY(cudaMemcpyAsync(wd.ptr, w_host, N * K * sizeof(float), cudaMemcpyHostToDevice, stream));
  if (scheme == LTM_SCHEME_W4A16) {
    if (K % 128 != 0) LTM_UNSUPPORTED("W4A16 needs the input width to be a multiple of 128");
    q4.ensure(N * K / 2);
    s4.ensure(N * (K / 128) * sizeof(float));
    z4.ensure(N * (K / 128));
    LTM_REQUIRE(ltm_quantize_int4_grouped(wd.ptr, LTM_DTYPE_F32, N, K, 128, q4.as<uint8_t>(),
                                          s4.as<float>(), z4.as<uint8_t>(), stream) == LTM_OK,
                "int4 weight quantization failed");
  } else {
    q8.ensure(N * K);
    s8.ensure(N * sizeof(float));
    launch_rowwise_int8(wd.ptr, LTM_DTYPE_F32, N, K, q8.as<int8_t>(), s8.as<float>(), stream);
  }
  if (b_host) {
    bias.ensure(N * sizeof(float));
    LTM_CUDA_TRY(cudaMemcpyAsync(bias.ptr, b_host, N * sizeof(float), cudaMemcpyHostToDevice, stream));
  } else {
    bias.release();
  }
  LTM_CUDA_TRY(cudaStreamSynchronize(stream));
}

// Loads the columns [c0, c0 + nc) of a host [n, k] weight: the full matrix is
// quantized (per-output-channel scales, or group-128 int4 along K) and the
// codes / group parameters of the column range are kept, so the shard holds
// exactly the codes and scales of the unsplit weight (row-parallel
// tensor-parallel layers).  c0 and nc are multiples of 128 for W4A16.
void QLinear::load_cols(const ltm_quant_config& q, const float* w_host, const float* b_host,
                        int64_t n, int64_t k, int64_t c0, int64_t nc, cudaStream_t stream) {
  QLinear full;
  full.load(q, w_host, b_host, n, k, stream);
  N = n;
  K = nc;
  scheme = q.scheme;
  if (scheme == LTM_SCHEME_W4A16) {
    LTM_REQUIRE(c0 % 128 == 0 && nc % 128 == 0, "int4 column shard must align to 128");
    q4.ensure(N * nc / 2);
    s4.ensure(N * (nc / 128) * sizeof(float));
    z4.ensure(N * (nc / 128));
    LTM_CUDA_TRY(cudaMemcpy2DAsync(q4.ptr, nc / 2, full.q4.as<uint8_t>() + c0 / 2, k / 2, nc / 2, N,
                                   cudaMemcpyDeviceToDevice, stream));
    LTM_CUDA_TRY(cudaMemcpy2DAsync(s4.ptr, (nc / 128) * sizeof(float),
                                   full.s4.as<float>() + c0 / 128, (k / 128) * sizeof(float),
                                   (nc / 128) * sizeof(float), N, cudaMemcpyDeviceToDevice, stream));
    LTM_CUDA_TRY(cudaMemcpy2DAsync(z4.ptr, nc / 128, full.z4.as<uint8_t>() + c0 / 128, k / 128,
                                   nc / 128, N, cudaMemcpyDeviceToDevice, stream));
  } else {
    q8.ensure(N * nc);
    s8.ensure(N * sizeof(float));
    LTM_CUDA_TRY(cudaMemcpy2DAsync(q8.ptr, nc, full.q8.as<int8_t>() + c0, k, nc, N,
                                   cudaMemcpyDeviceToDevice, stream));
    LTM_CUDA_TRY(cudaMemcpyAsync(s8.ptr, full.s8.ptr, N * sizeof(float), cudaMemcpyDeviceToDevice,
                                 stream));
  }
  if (b_host) {
    bias.ensure(N * sizeof(float));
    LTM_CUDA_TRY(cudaMemcpyAsync(bias.ptr, full.bias.ptr, N * sizeof(float),
                                 cudaMemcpyDeviceToDevice, stream));
  } else {
    bias.release();
  }
  LTM_CUDA_TRY(cudaStreamSynchronize(stream));
}

// Runs y = epilogue(a W^T) for the block's scheme.  a_act: activation in the
// act dtype (W8A32 / W4A16); aq/as: its per-token int8 codes (W8A8).
// M from which a W4A16 linear dequantises its weight once into wdq and runs
// the 16-bit persistent GEMM (every weight tile then serves M / 128 row
// tiles without being dequantised again); below it the fused kernel
// dequantises tiles on the fly and reads the packed weight once.
constexpr int64_t kW4DequantM = 1024;

void QLinear::run(const void* a_act, const int8_t* aq, const float* as, int64_t M, int mode,
                  ltm_dtype dt, Epilogue ep, cudaStream_t stream, DevBuf* wdq) const {
  ep.bias = apply_bias ? bias.as<float>() : nullptr;
  if (scheme == LTM_SCHEME_W8A8) {
    ep.row_scale = as;
    ep.col_scale = s8.as<float>();
    launch_w8a8(aq, q8.as<int8_t>(), M, N, K, mode, dt, ep, stream);
  } else if (scheme == LTM_SCHEME_W8A32) {
    ep.row_scale = nullptr;
    ep.col_scale = s8.as<float>();
    launch_w8a32(static_cast<const float*>(a_act), q8.as<int8_t>(), M, N, K, mode, ep, stream);
  } else if (wdq != nullptr && M >= kW4DequantM) {
    ep.row_scale = nullptr;
    ep.col_scale = nullptr;
    wdq->ensure(static_cast<size_t>(N) * K * dtype_size(dt));
    launch_int4_dequant_rows(q4.as<uint8_t>(), s4.as<float>(), z4.as<uint8_t>(), N, K, wdq->ptr, dt,
                             stream);
    launch_gemm_f16(a_act, wdq->ptr, M, N, K, mode, dt, ep, stream);
  } else {
    ep.row_scale = nullptr;
    ep.col_scale = nullptr;
    launch_w4a16(a_act, dt, q4.as<uint8_t>(), s4.as<float>(), z4.as<uint8_t>(), M, N, K, mode, ep,
                 stream);
  }
}

}  // namespace ltm_b200

using namespace ltm_b200;

// ---------------------------------------------------------------- the block --
struct ltm_block {
  ltm_block_config cfg{};
  ltm_quant_config q{};
  int device = 0;
  int H = 0, F = 0, nh = 0, dh = 0, Ms = 0;
  // tensor parallelism: this rank's heads (nhl), their width Hl = nhl * dh
  // and FFN columns Fl; tp = 1 is the single-GPU block
  ltm_comm* comm = nullptr;
  int tp = 1, tpr = 0;
  int nhl = 0, Hl = 0, Fl = 0;
  ltm_dtype dt = LTM_DTYPE_F16;
  bool loaded = false;
  QLinear qkvm, kvm, o, om, g, w1, w2;
  DevBuf ln1_g, ln1_b, ln2_g, ln2_b;
  DevBuf memory;  // [Ms, H] act dtype
  DevBuf rope;    // [rope_S, dh/2] float2
  int rope_S = 0;
  // workspace (ws_T rows of capacity; last_T rows written by the last
  // forward or decode step)
  int64_t ws_T = 0, last_T = 0;
  DevBuf hq, hs, xq, xs, h, qkv, kvmb, mq, ms, os, om_, osq, oss, omq, oms, spm, y, zq, zs, z,
      u, uq, us, amax;
  DevBuf sploc;  // sequence parallel: this rank's rows of s | m [2, T/tp, H]
  MemoryWriteState mw;
  // decode: K_M | V_M kept resident between steps (kvm_fresh: kvmb holds them
  // for the current bank), the state row of the write and its projection,
  // split-cache attention partials
  bool kvm_fresh = false;
  DevBuf crow, cq, cs, kcv, dpart;
  DevBuf wdq;  // dequantised weight of the W4A16 GEMMs at large M (one at a time)

  size_t act_bytes() const { return dtype_size(dt); }

  // RoPE table of at least S positions (grown in steps of 4096 positions so
  // that a decode loop rebuilds it once per 4096 steps).
  void ensure_rope(int S) {
    if (S <= rope_S) return;
    S = (S + 4095) / 4096 * 4096;
    const int half = dh / 2;
    std::vector<float> tab(static_cast<size_t>(S) * dh);
    for (int p = 0; p < S; ++p)
      for (int i = 0; i < half; ++i) {
        const float inv = 1.0f / powf(10000.0f, (2.0f * static_cast<float>(i)) / static_cast<float>(dh));
        const float th = static_cast<float>(p) * inv;
        tab[2 * (static_cast<size_t>(p) * half + i)] = static_cast<float>(std::cos(static_cast<double>(th)));
        tab[2 * (static_cast<size_t>(p) * half + i) + 1] = static_cast<float>(std::sin(static_cast<double>(th)));
      }
    rope.ensure(tab.size() * sizeof(float));
    LTM_CUDA_TRY(cudaMemcpy(rope.ptr, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice));
    rope_S = S;
  }

  void ensure_ws(int64_t T) {
    if (T <= ws_T) return;
    const size_t a = act_bytes();
    const bool w8a8 = q.scheme == LTM_SCHEME_W8A8;
    if (w8a8) {
      hq.ensure(T * H);
      hs.ensure(T * 4);
      xq.ensure(T * H);
      xs.ensure(T * 4);
      osq.ensure(T * Hl);
      oss.ensure(T * 4);
      omq.ensure(T * Hl);
      oms.ensure(T * 4);
      zq.ensure(T * H);
      zs.ensure(T * 4);
      uq.ensure(T * Fl);
      us.ensure(T * 4);
      if (tp > 1) amax.ensure(2 * T * 4);
    } else {
      h.ensure(T * H * a);
      z.ensure(T * H * a);
    }
    qkv.ensure(T * 4 * Hl * a);
    os.ensure(T * Hl * a);
    om_.ensure(T * Hl * a);
    spm.ensure(2 * T * H * a);  // s | m, one allreduce under tensor parallelism
    y.ensure(T * H * a);
    u.ensure(T * Fl * a);
    ws_T = T;
  }

  // Per-token int8 of rows whose columns are split over the ranks (global row
  // maxima through an allreduce-max); the plain quantizer when tp == 1.
  void quant_rows(const void* src, int64_t T, int64_t K, int8_t* qd, float* sd, float* amx,
                  cudaStream_t st) {
    if (tp == 1) {
      launch_rowwise_int8(src, dt, T, K, qd, sd, st);
      return;
    }
    launch_row_absmax(src, dt, T, K, amx, st);
    comm_allreduce(comm, amx, amx, T, LTM_DTYPE_F32, true, st);
    launch_rowwise_int8_amax(src, dt, T, K, amx, qd, sd, st);
  }

  // K_M | V_M of the current bank into kvmb.
  void compute_kvm(cudaStream_t st) {
    if (q.scheme == LTM_SCHEME_W8A8)
      launch_rowwise_int8(memory.ptr, dt, Ms, H, mq.as<int8_t>(), ms.as<float>(), st);
    Epilogue ep;
    ep.out = kvmb.ptr;
    ep.ldo = 2 * Hl;
    kvm.run(memory.ptr, mq.as<int8_t>(), ms.as<float>(), Ms, kEpiPlain, dt, ep, st, &wdq);
    kvm_fresh = true;
  }

  // 1. LN1 (+ per-token int8 of LN1(x) and of x for W8A8); returns the
  // projection input of the non-W8A8 schemes.
  const void* ln1(const void* x, int64_t T, cudaStream_t st) {
    if (q.scheme == LTM_SCHEME_W8A8) {
      launch_ln_x2(x, dt, T, H, ln1_g.as<float>(), ln1_b.as<float>(), nullptr, hq.as<int8_t>(),
                   hs.as<float>(), xq.as<int8_t>(), xs.as<float>(), cfg.use_layer_norm != 0, st);
    } else if (cfg.use_layer_norm) {
      launch_ln_x2(x, dt, T, H, ln1_g.as<float>(), ln1_b.as<float>(), h.ptr, nullptr, nullptr,
                   nullptr, nullptr, true, st);
    }
    return (q.scheme == LTM_SCHEME_W8A8 || cfg.use_layer_norm) ? h.ptr : x;
  }

  // 3. fused Q | K | V | Qm projection with RoPE on Q, K at position
  // pos0 + (row % S), or at row_pos[row] when given (device [T])
  void qkv_proj(const void* hin, int64_t T, int S, int pos0, cudaStream_t st,
                const int* row_pos = nullptr) {
    Epilogue ep;
    ep.out = qkv.ptr;
    ep.ldo = 4 * Hl;
    ep.rope = rope.as<float2>() + (row_pos ? 0 : static_cast<int64_t>(pos0) * (dh / 2));
    ep.rope_cols = cfg.use_rotary ? 2 * Hl : 0;
    ep.seq_len = S;
    ep.head_dim = dh;
    ep.row_pos = row_pos;
    ep.rope_rows = rope_S;
    qkvm.run(hin, hq.as<int8_t>(), hs.as<float>(), T, cfg.use_rotary ? kEpiRope : kEpiPlain, dt,
             ep, st, &wdq);
  }

  // Memory attention of nb groups of sq query rows against K_M | V_M (the
  // bank is shared: every group reads the same keys).
  void mem_attention(int nb, int sq, cudaStream_t st) {
    const size_t a = act_bytes();
    AttnParams pm{};
    pm.q = static_cast<const char*>(qkv.ptr) + 3 * Hl * a;
    pm.k = kvmb.ptr;
    pm.v = static_cast<const char*>(kvmb.ptr) + Hl * a;
    pm.o = om_.ptr;
    pm.ldq = 4 * Hl;
    pm.ldk = pm.ldv = 2 * Hl;
    pm.ldo = Hl;
    pm.q_batch_rows = sq;
    pm.kv_batch_rows = 0;
    pm.Sq = sq;
    pm.Skv = Ms;
    pm.nh = nhl;
    pm.causal_offset = 0;
    launch_attention(pm, nb, dh, false, dt, st);
  }

  // 5-7. output projections, gated memory integration, FFN with residual
  // (os, om_ hold the two attention outputs of the T rows).
  void tail(const void* x, void* out, int64_t T, cudaStream_t st) {
    const bool w8a8 = q.scheme == LTM_SCHEME_W8A8;
    if (w8a8) {
      quant_rows(os.ptr, T, Hl, osq.as<int8_t>(), oss.as<float>(), amax.as<float>(), st);
      quant_rows(om_.ptr, T, Hl, omq.as<int8_t>(), oms.as<float>(),
                 tp > 1 ? amax.as<float>() + T : nullptr, st);
    }
    void* sp = spm.ptr;
    void* mp = static_cast<char*>(spm.ptr) + T * H * act_bytes();
    {
      Epilogue ep;
      ep.out = sp;
      ep.ldo = H;
      o.run(os.ptr, osq.as<int8_t>(), oss.as<float>(), T, kEpiPlain, dt, ep, st, &wdq);
      ep.out = mp;
      om.run(om_.ptr, omq.as<int8_t>(), oms.as<float>(), T, kEpiPlain, dt, ep, st, &wdq);
    }
    // row-parallel partial sums of s and m (the biases were added by rank 0)
    if (tp > 1) comm_allreduce(comm, spm.ptr, spm.ptr, 2 * T * H, dt, false, st);
    // 6. gated memory integration
    if (cfg.use_memory_gating) {
      Epilogue ep;
      ep.act = LTM_EPI_SIGMOID;
      ep.out = y.ptr;
      ep.ldo = H;
      ep.aux0 = sp;
      ep.aux1 = mp;
      ep.aux2 = x;
      ep.ld_aux = H;
      if (q.memory_write) mw.prepare_gate_epilogue(ep, H, st);
      g.run(x, xq.as<int8_t>(), xs.as<float>(), T, kEpiGateMix, dt, ep, st, &wdq);
    } else {
      launch_add3(sp, mp, x, y.ptr, T * H, dt, st);
    }
    // 7. FFN with residual
    if (w8a8) {
      launch_ln_x2(y.ptr, dt, T, H, ln2_g.as<float>(), ln2_b.as<float>(), nullptr, zq.as<int8_t>(),
                   zs.as<float>(), nullptr, nullptr, cfg.use_layer_norm != 0, st);
    } else if (cfg.use_layer_norm) {
      launch_ln_x2(y.ptr, dt, T, H, ln2_g.as<float>(), ln2_b.as<float>(), z.ptr, nullptr, nullptr,
                   nullptr, nullptr, true, st);
    }
    const void* zin = (w8a8 || cfg.use_layer_norm) ? z.ptr : y.ptr;
    {
      Epilogue ep;
      ep.act = LTM_EPI_GELU;
      ep.out = u.ptr;
      ep.ldo = Fl;
      w1.run(zin, zq.as<int8_t>(), zs.as<float>(), T, kEpiPlain, dt, ep, st, &wdq);
    }
    if (w8a8) quant_rows(u.ptr, T, Fl, uq.as<int8_t>(), us.as<float>(), amax.as<float>(), st);
    {
      // out = y + W2 u + b2; under tensor parallelism rank 0 adds y and b2 to
      // its partial product and the allreduce sums the ranks' partials
      Epilogue ep;
      ep.out = out;
      ep.ldo = H;
      ep.aux0 = y.ptr;
      ep.ld_aux = H;
      w2.run(u.ptr, uq.as<int8_t>(), us.as<float>(), T, tpr == 0 ? kEpiResid : kEpiPlain, dt, ep,
             st, &wdq);
    }
    if (tp > 1) comm_allreduce(comm, out, out, T * H, dt, false, st);
  }

  // 8. memory write after the read.  kvm_follow: K_M | V_M follow the bank's
  // EMA towards the projected state (decode keeps them resident); otherwise
  // they are recomputed from the bank before their next use.
  void write(int64_t T, bool kvm_follow, cudaStream_t st) {
    const size_t a = act_bytes();
    const float scale = mw.update_bank(memory.ptr, kvmb.ptr, 2 * Hl,
                                       static_cast<const char*>(qkv.ptr) + 3 * Hl * a, 4 * Hl, T, H,
                                       nhl, nh, dh, Ms, cfg.memory_update_rate,
                                       q.use_attention_scores != 0, dt, comm, st);
    if (!kvm_follow) {
      kvm_fresh = false;
      return;
    }
    follow_kvm(mw.colsum.as<float>(), scale,
               q.use_attention_scores ? mw.wslot.as<float>() : nullptr, st);
  }

  // K_M | V_M follow the bank's EMA (slot weights wslot, or the update rate):
  // kvm[s] = (1 - w_s) kvm[s] + w_s (c [Wkm;Wvm]^T + b) with c = state * scale
  // rounded to the activation dtype.
  void follow_kvm(const float* state, float scale, const float* wslot, cudaStream_t st) {
    const size_t a = act_bytes();
    crow.ensure(static_cast<size_t>(H) * a);
    kcv.ensure(static_cast<size_t>(2 * Hl) * a);
    launch_state_row(state, scale, crow.ptr, H, dt, st);
    if (q.scheme == LTM_SCHEME_W8A8) {
      cq.ensure(H);
      cs.ensure(sizeof(float));
      launch_rowwise_int8(crow.ptr, dt, 1, H, cq.as<int8_t>(), cs.as<float>(), st);
    }
    Epilogue ep;
    ep.out = kcv.ptr;
    ep.ldo = 2 * Hl;
    kvm.run(crow.ptr, cq.as<int8_t>(), cs.as<float>(), 1, kEpiPlain, dt, ep, st, &wdq);
    launch_rows_ema(kvmb.ptr, 2 * Hl, 2 * Hl, kcv.ptr, wslot, cfg.memory_update_rate, Ms, dt, st);
  }

  // ---- sequence parallelism
  // Collectives of the overlapped sequence-parallel forward run on a stream
  // of the block's own (every NCCL call of the block on one stream, in one
  // order on every rank), ordered against the caller's stream by events.
  // -1 (default) and 0: the collectives on the caller's stream, one per
  // phase; 1: overlapped (set by ltm_block_set_overlap).  The overlapped form
  // splits every GEMM into tp launches and reserves SMs for the collectives,
  // which cost more than the hidden transfers saved at 2 and at 8 ranks
  // (measured), so it is not the default.
  int overlap = -1;
  // row-parallel reductions of the sequence-parallel forward: 0 = partial
  // sums in the activation type, reduce-scattered by NCCL; 1 = exact (W8A8):
  // int32 accumulators exchanged rank to rank and summed at the row owner,
  // then the unsplit GEMM's epilogue, so the output equals the single-GPU
  // block's bit for bit at twice the bytes of those exchanges
  int tp_reduce = 0;
  DevBuf spi, spri;  // exact reduction: int32 partials [2, T, H] and the ranks' slots
  int comm_sms = 16;  // SMs the chunked GEMMs leave to the concurrent collectives
  cudaStream_t comm_st = nullptr;
  std::vector<cudaEvent_t> evs;

  ~ltm_block() {
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
    if (comm_st) cudaStreamDestroy(comm_st);
  }

  void ensure_comm_stream(int n_events) {
    if (!comm_st) LTM_CUDA_TRY(cudaStreamCreateWithFlags(&comm_st, cudaStreamNonBlocking));
    while (static_cast<int>(evs.size()) < n_events) {
      cudaEvent_t e = nullptr;
      LTM_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      evs.push_back(e);
    }
  }
  // `to` waits for the work issued so far on `from` (through event k).
  void order(cudaStream_t from, cudaStream_t to, int k) {
    if (from == to) return;
    LTM_CUDA_TRY(cudaEventRecord(evs[k], from));
    LTM_CUDA_TRY(cudaStreamWaitEvent(to, evs[k], 0));
  }

  // All-gather of this rank's rows [r0, r0 + Tr) of the int8 rows q [T, H]
  // and their scales s [T], as one broadcast per root rank on the comm
  // stream (event k0 + root marks its arrival).
  void gather_rows_chunked(int8_t* q, float* s, int64_t Tr, int k0) {
    for (int j = 0; j < tp; ++j) {
      comm_group_start();
      comm_broadcast_bytes(comm, q + j * Tr * H, Tr * H, j, comm_st);
      comm_broadcast_bytes(comm, s + j * Tr, Tr * sizeof(float), j, comm_st);
      comm_group_end(nullptr, comm_st);
      LTM_CUDA_TRY(cudaEventRecord(evs[k0 + j], comm_st));
    }
  }

  // Sequence-parallel tensor-parallel forward (Megatron sequence
  // parallelism): x_loc / out_loc are this rank's T / tp consecutive rows of
  // the [B*S, H] activations.  LayerNorms, the gate and the gated
  // integration run on the local rows only; the LayerNorm outputs (int8
  // codes and scales for W8A8) are all-gathered for the column-parallel
  // projections, and the row-parallel output / FFN-down partial sums are
  // reduce-scattered back to the rows' owners, so no rank repeats another's
  // row work and the bytes on NVLink are the reduce-scatter + all-gather of
  // the collectives they replace (the LayerNorm all-gathers in int8).
  //
  // Overlap (W8A8): every all-gather is a broadcast per root rank and every
  // reduce-scatter a reduce per root rank, on the block's comm stream; the
  // GEMM that consumes (or produces) the rows of root j runs as its own
  // launch, so the transfer of one rank's rows overlaps the GEMM of
  // another's (this rank's own rows first on the gathering side), with
  // comm_sms SMs left free for the collectives' kernels.
  void forward_sp(const void* x_loc, void* out_loc, int B, int S, cudaStream_t st) {
    const int64_t T = static_cast<int64_t>(B) * S;
    const int64_t Tr = T / tp, r0 = static_cast<int64_t>(tpr) * Tr;
    ensure_ws(T);
    last_T = T;
    const size_t a = act_bytes();
    sploc.ensure(static_cast<size_t>(2 * Tr) * H * a);
    if (tp_reduce == 1 && q.scheme == LTM_SCHEME_W8A8) {
      spi.ensure(static_cast<size_t>(2 * T) * H * sizeof(int32_t));
      spri.ensure(static_cast<size_t>(2 * T) * H * sizeof(int32_t));
    }
    if (cfg.use_rotary) ensure_rope(S);
    const bool w8a8 = q.scheme == LTM_SCHEME_W8A8;
    const bool ovl = overlap > 0 && w8a8;
    const bool exact = tp_reduce == 1 && w8a8;
    ensure_comm_stream(2 * tp + 8);
    cudaStream_t ns = ovl ? comm_st : st;  // the stream of the collectives
    const int kA = 8, kB = 8 + tp;    // per-root events of the two chunked phases
    // 1. LN1 of the local rows into rows [r0, r0 + Tr) of the full buffers
    //    (+ the int8 of x's local rows for the gate), then all-gather
    if (w8a8) {
      launch_ln_x2(x_loc, dt, Tr, H, ln1_g.as<float>(), ln1_b.as<float>(), nullptr,
                   hq.as<int8_t>() + r0 * H, hs.as<float>() + r0, xq.as<int8_t>(), xs.as<float>(),
                   cfg.use_layer_norm != 0, st);
      if (ovl) {
        order(st, comm_st, 0);
        gather_rows_chunked(hq.as<int8_t>(), hs.as<float>(), Tr, kA);
      } else {
        comm_group_start();
        comm_allgather_bytes(comm, hq.as<int8_t>() + r0 * H, hq.ptr, Tr * H, st);
        comm_allgather_bytes(comm, hs.as<float>() + r0, hs.ptr, Tr * sizeof(float), st);
        comm_group_end("nccl_allgather", st);
      }
    } else {
      char* hl = static_cast<char*>(h.ptr) + r0 * H * a;
      if (cfg.use_layer_norm)
        launch_ln_x2(x_loc, dt, Tr, H, ln1_g.as<float>(), ln1_b.as<float>(), hl, nullptr, nullptr,
                     nullptr, nullptr, true, st);
      else
        LTM_CUDA_TRY(cudaMemcpyAsync(hl, x_loc, Tr * H * a, cudaMemcpyDeviceToDevice, st));
      comm_allgather_bytes(comm, hl, h.ptr, Tr * H * a, st);
    }
    // 2-3. K_M | V_M (needs no gathered rows: overlaps the first transfers),
    //      Q | K | V | Qm of all T rows for this rank's heads
    compute_kvm(st);
    if (ovl) {
      ScopedSmReserve reserve(comm_sms);
      for (int i = 0; i < tp; ++i) {
        const int j = (tpr + i) % tp;  // own rows first: they need no transfer
        if (j != tpr) LTM_CUDA_TRY(cudaStreamWaitEvent(st, evs[kA + j], 0));
        qkv_rows(j * Tr, Tr, S, st);
      }
      // the remaining broadcasts read hq rows that the next layer rewrites:
      // the caller's stream has waited for all of them above
    } else {
      qkv_proj(h.ptr, T, S, 0, st);
    }
    // 4. the two attentions of this rank's heads over all T rows
    {
      AttnParams p{};
      p.q = qkv.ptr;
      p.k = static_cast<const char*>(qkv.ptr) + Hl * a;
      p.v = static_cast<const char*>(qkv.ptr) + 2 * Hl * a;
      p.o = os.ptr;
      p.ldq = p.ldk = p.ldv = 4 * Hl;
      p.ldo = Hl;
      p.q_batch_rows = S;
      p.kv_batch_rows = S;
      p.Sq = S;
      p.Skv = S;
      p.nh = nhl;
      p.causal_offset = 0;
      launch_attention(p, B, dh, true, dt, st);
      mem_attention(B, S, st);
    }
    // 5. output projections: partial sums of all rows, reduced to the rows'
    //    owners (rank 0's partial carries the biases)
    void* sp = spm.ptr;
    void* mp = static_cast<char*>(spm.ptr) + T * H * a;
    void* s_loc = sploc.ptr;
    void* m_loc = static_cast<char*>(sploc.ptr) + Tr * H * a;
    if (w8a8) {  // per-token int8 of the head-split rows: global row maxima
      float* amx = amax.as<float>();
      launch_row_absmax(os.ptr, dt, T, Hl, amx, st);
      launch_row_absmax(om_.ptr, dt, T, Hl, amx + T, st);
      order(st, ns, 1);
      comm_allreduce(comm, amx, amx, 2 * T, LTM_DTYPE_F32, true, ns);
      order(ns, st, 2);
      launch_rowwise_int8_amax(os.ptr, dt, T, Hl, amx, osq.as<int8_t>(), oss.as<float>(), st);
      launch_rowwise_int8_amax(om_.ptr, dt, T, Hl, amx + T, omq.as<int8_t>(), oms.as<float>(), st);
    }
    // Activation-type mode: the partial sums of all rows are reduce-scattered
    // to the rows' owners (NCCL, in the switch where NVLS is available).
    // Exact mode: every rank's int32 accumulators of this rank's rows land in
    // a slot of sr / mr (all-to-all), summed exactly by the owner, which then
    // applies the unsplit GEMM's epilogue.
    const size_t esz = exact ? sizeof(int32_t) : a;
    void* sp5 = exact ? spi.ptr : sp;  // partials of s | m, all rows
    void* mp5 = static_cast<char*>(sp5) + T * H * esz;
    void* sr = spri.ptr;  // exact mode only
    void* mr = static_cast<char*>(sr) + T * H * esz;
    if (ovl) {
      ScopedSmReserve reserve(comm_sms);
      for (int j = 0; j < tp; ++j) {
        out_rows(o, osq.as<int8_t>(), oss.as<float>(), Hl, j * Tr, Tr, sp5, st, exact);
        out_rows(om, omq.as<int8_t>(), oms.as<float>(), Hl, j * Tr, Tr, mp5, st, exact);
        order(st, comm_st, kB + j);
        comm_group_start();
        if (exact) {
          comm_send_recv_slots(comm, sp5, sr, Tr * H * esz, j, comm_st);
          comm_send_recv_slots(comm, mp5, mr, Tr * H * esz, j, comm_st);
        } else {
          comm_reduce(comm, static_cast<char*>(sp) + j * Tr * H * a, s_loc, Tr * H, dt, j, comm_st);
          comm_reduce(comm, static_cast<char*>(mp) + j * Tr * H * a, m_loc, Tr * H, dt, j, comm_st);
        }
        comm_group_end(nullptr, comm_st);
      }
      order(comm_st, st, 3);
    } else {
      Epilogue ep;
      ep.out = sp5;
      ep.ldo = H;
      const int mode = exact ? kEpiAccI32 : kEpiPlain;
      o.run(os.ptr, osq.as<int8_t>(), oss.as<float>(), T, mode, dt, ep, st, &wdq);
      ep.out = mp5;
      om.run(om_.ptr, omq.as<int8_t>(), oms.as<float>(), T, mode, dt, ep, st, &wdq);
      comm_group_start();
      if (exact) {
        comm_send_recv_slots(comm, sp5, sr, Tr * H * esz, -1, st);
        comm_send_recv_slots(comm, mp5, mr, Tr * H * esz, -1, st);
      } else {
        comm_reduce_scatter(comm, sp, s_loc, Tr * H, dt, st);
        comm_reduce_scatter(comm, mp, m_loc, Tr * H, dt, st);
      }
      comm_group_end(exact ? "nccl_send_recv" : "nccl_reduce_scatter", st);
    }
    if (exact) {
      launch_sum_slots_i32(static_cast<const int32_t*>(sr), static_cast<const int32_t*>(sp5) + r0 * H,
                           tp, tpr, Tr * H, oss.as<float>() + r0, o.s8.as<float>(),
                           o.bias.as<float>(), nullptr, s_loc, Tr, H, dt, st);
      launch_sum_slots_i32(static_cast<const int32_t*>(mr), static_cast<const int32_t*>(mp5) + r0 * H,
                           tp, tpr, Tr * H, oms.as<float>() + r0, om.s8.as<float>(),
                           om.bias.as<float>(), nullptr, m_loc, Tr, H, dt, st);
    }
    // 6. gate and gated integration of the local rows
    if (cfg.use_memory_gating) {
      Epilogue ep;
      ep.act = LTM_EPI_SIGMOID;
      ep.out = y.ptr;
      ep.ldo = H;
      ep.aux0 = s_loc;
      ep.aux1 = m_loc;
      ep.aux2 = x_loc;
      ep.ld_aux = H;
      if (q.memory_write) mw.prepare_gate_epilogue(ep, H, st);
      g.run(x_loc, xq.as<int8_t>(), xs.as<float>(), Tr, kEpiGateMix, dt, ep, st, &wdq);
    } else {
      launch_add3(s_loc, m_loc, x_loc, y.ptr, Tr * H, dt, st);
    }
    // 7. LN2 of the local rows, all-gathered for the column-parallel FFN-up
    if (w8a8) {
      launch_ln_x2(y.ptr, dt, Tr, H, ln2_g.as<float>(), ln2_b.as<float>(), nullptr,
                   zq.as<int8_t>() + r0 * H, zs.as<float>() + r0, nullptr, nullptr,
                   cfg.use_layer_norm != 0, st);
      if (ovl) {
        order(st, comm_st, 4);
        gather_rows_chunked(zq.as<int8_t>(), zs.as<float>(), Tr, kA);
      } else {
        comm_group_start();
        comm_allgather_bytes(comm, zq.as<int8_t>() + r0 * H, zq.ptr, Tr * H, st);
        comm_allgather_bytes(comm, zs.as<float>() + r0, zs.ptr, Tr * sizeof(float), st);
        comm_group_end("nccl_allgather", st);
      }
    } else {
      char* zl = static_cast<char*>(z.ptr) + r0 * H * a;
      if (cfg.use_layer_norm)
        launch_ln_x2(y.ptr, dt, Tr, H, ln2_g.as<float>(), ln2_b.as<float>(), zl, nullptr, nullptr,
                     nullptr, nullptr, true, st);
      else
        LTM_CUDA_TRY(cudaMemcpyAsync(zl, y.ptr, Tr * H * a, cudaMemcpyDeviceToDevice, st));
      comm_allgather_bytes(comm, zl, z.ptr, Tr * H * a, st);
    }
    if (ovl) {
      ScopedSmReserve reserve(comm_sms);
      for (int i = 0; i < tp; ++i) {
        const int j = (tpr + i) % tp;
        if (j != tpr) LTM_CUDA_TRY(cudaStreamWaitEvent(st, evs[kA + j], 0));
        Epilogue ep;
        ep.act = LTM_EPI_GELU;
        ep.out = static_cast<char*>(u.ptr) + j * Tr * Fl * a;
        ep.ldo = Fl;
        w1.run(nullptr, zq.as<int8_t>() + j * Tr * H, zs.as<float>() + j * Tr, Tr, kEpiPlain, dt,
               ep, st, &wdq);
      }
    } else {
      Epilogue ep;
      ep.act = LTM_EPI_GELU;
      ep.out = u.ptr;
      ep.ldo = Fl;
      w1.run(z.ptr, zq.as<int8_t>(), zs.as<float>(), T, kEpiPlain, dt, ep, st, &wdq);
    }
    if (w8a8) {
      float* amx = amax.as<float>();
      launch_row_absmax(u.ptr, dt, T, Fl, amx, st);
      order(st, ns, 5);
      comm_allreduce(comm, amx, amx, T, LTM_DTYPE_F32, true, ns);
      order(ns, st, 6);
      launch_rowwise_int8_amax(u.ptr, dt, T, Fl, amx, uq.as<int8_t>(), us.as<float>(), st);
    }
    // 8. FFN-down partial sums of all rows (rank 0's carry b2), reduced to
    //    the rows' owners; the owner adds its rows' residual
    if (ovl) {
      ScopedSmReserve reserve(comm_sms);
      for (int j = 0; j < tp; ++j) {
        out_rows(w2, uq.as<int8_t>(), us.as<float>(), Fl, j * Tr, Tr, sp5, st, exact);
        order(st, comm_st, kB + j);
        if (exact)
          comm_send_recv_slots(comm, sp5, sr, Tr * H * esz, j, comm_st);
        else
          comm_reduce(comm, static_cast<char*>(sp) + j * Tr * H * a, out_loc, Tr * H, dt, j,
                      comm_st);
      }
      order(comm_st, st, 7);
    } else {
      Epilogue ep;
      ep.out = sp5;
      ep.ldo = H;
      w2.run(u.ptr, uq.as<int8_t>(), us.as<float>(), T, exact ? kEpiAccI32 : kEpiPlain, dt, ep, st,
             &wdq);
      if (exact)
        comm_send_recv_slots(comm, sp5, sr, Tr * H * esz, -1, st);
      else
        comm_reduce_scatter(comm, sp, out_loc, Tr * H, dt, st);
    }
    if (exact)  // the slots' exact sum, the epilogue and the residual, rounded once
      launch_sum_slots_i32(static_cast<const int32_t*>(sr), static_cast<const int32_t*>(sp5) + r0 * H,
                           tp, tpr, Tr * H, us.as<float>() + r0, w2.s8.as<float>(),
                           w2.bias.as<float>(), y.ptr, out_loc, Tr, H, dt, st);
    else  // the owner adds its rows' residual
      launch_add3(out_loc, y.ptr, nullptr, out_loc, Tr * H, dt, st);
    // 9. memory write: column sums of the local rows, summed over the ranks
    if (q.memory_write && cfg.use_memory_gating) {
      order(st, ns, 1);
      mw.update_bank(memory.ptr, kvmb.ptr, 2 * Hl, static_cast<const char*>(qkv.ptr) + 3 * Hl * a,
                     4 * Hl, T, H, nhl, nh, dh, Ms, cfg.memory_update_rate,
                     q.use_attention_scores != 0, dt, comm, ns, /*colsum_partial=*/true);
      order(ns, st, 2);
      kvm_fresh = false;
    }
  }

  // Q | K | V | Qm (RoPE) of rows [row0, row0 + M) from the gathered int8
  // LayerNorm rows (W8A8).
  void qkv_rows(int64_t row0, int64_t M, int S, cudaStream_t st) {
    Epilogue ep;
    ep.out = static_cast<char*>(qkv.ptr) + row0 * 4 * Hl * act_bytes();
    ep.ldo = 4 * Hl;
    ep.rope = rope.as<float2>();
    ep.rope_cols = cfg.use_rotary ? 2 * Hl : 0;
    ep.seq_len = S;
    ep.head_dim = dh;
    ep.rope_rows = rope_S;
    ep.rope_row0 = row0;
    qkvm.run(nullptr, hq.as<int8_t>() + row0 * H, hs.as<float>() + row0, M,
             cfg.use_rotary ? kEpiRope : kEpiPlain, dt, ep, st, &wdq);
  }

  // Row-parallel partial sums [M, H] of rows [row0, row0 + M) (int8 inputs
  // of width K, per-token scales) into out rows [row0, row0 + M).
  void out_rows(const QLinear& lin, const int8_t* aq, const float* as, int64_t K, int64_t row0,
                int64_t M, void* out, cudaStream_t st, bool acc_i32 = false) {
    Epilogue ep;
    ep.out = static_cast<char*>(out) + row0 * H * (acc_i32 ? sizeof(int32_t) : act_bytes());
    ep.ldo = H;
    lin.run(nullptr, aq + row0 * K, as + row0, M, acc_i32 ? kEpiAccI32 : kEpiPlain, dt, ep, st,
            &wdq);
  }

  // Memory write of a caller-given state (fp32 [H]) with slot weights from
  // the mean of T memory-query rows (this rank's heads' columns, stride ldq)
  // against the current K_M; K_M | V_M follow when they are resident.
  void write_state(const float* state, const void* queries, int64_t ldq, int64_t T,
                   cudaStream_t st) {
    const bool use_scores = q.use_attention_scores != 0;
    if (use_scores) {
      if (!kvm_fresh) compute_kvm(st);
      mw.qsum.ensure(static_cast<size_t>(Hl) * sizeof(float));
      mw.wslot.ensure(static_cast<size_t>(Ms) * sizeof(float));
      launch_slot_weights(kvmb.ptr, 2 * Hl, queries, ldq, T, Ms, nhl, dh, nh,
                          cfg.memory_update_rate, dt, mw.qsum.as<float>(), mw.wslot.as<float>(),
                          st);
      if (tp > 1) comm_allreduce(comm, mw.wslot.ptr, mw.wslot.ptr, Ms, LTM_DTYPE_F32, false, st);
    }
    const float* wslot = use_scores ? mw.wslot.as<float>() : nullptr;
    launch_bank_update(memory.ptr, state, 1.0f, wslot, cfg.memory_update_rate, Ms, H, dt, st);
    if (kvm_fresh) follow_kvm(state, 1.0f, wslot, st);
  }

  // kc / vc (optional): head-major caches [B, nhl, P, dh] that receive the
  // post-RoPE keys / values of positions [0, S) of every sequence.
  void forward(const void* x, void* out, int B, int S, cudaStream_t st, void* kc = nullptr,
               void* vc = nullptr, int64_t P = 0) {
    const int64_t T = static_cast<int64_t>(B) * S;
    ensure_ws(T);
    last_T = T;
    if (cfg.use_rotary) ensure_rope(S);
    const void* hin = ln1(x, T, st);
    // 2. memory keys / values from the bank
    compute_kvm(st);
    qkv_proj(hin, T, S, 0, st);
    if (kc) launch_kv_fill(qkv.ptr, 4 * Hl, Hl, dh, kc, vc, P, B, S, dt, st);
    // 4. causal self-attention, memory attention
    {
      const size_t a = act_bytes();
      AttnParams p{};
      p.q = qkv.ptr;
      p.k = static_cast<const char*>(qkv.ptr) + Hl * a;
      p.v = static_cast<const char*>(qkv.ptr) + 2 * Hl * a;
      p.o = os.ptr;
      p.ldq = p.ldk = p.ldv = 4 * Hl;
      p.ldo = Hl;
      p.q_batch_rows = S;
      p.kv_batch_rows = S;
      p.Sq = S;
      p.Skv = S;
      p.nh = nhl;
      p.causal_offset = 0;
      launch_attention(p, B, dh, true, dt, st);
      mem_attention(B, S, st);
    }
    tail(x, out, T, st);
    if (q.memory_write && cfg.use_memory_gating) write(T, false, st);
  }

  // One decode step: x, out [B, H], every sequence's new token at position L;
  // k_cache / v_cache [B, nhl, P, dh] hold positions [0, L) and receive
  // position L.
  // cache_lens (optional, device [B]): sequence b's new token sits at
  // position cache_lens[b] (L is ignored); its launches then depend on P and
  // B only, so the step can be captured once and replayed as the lengths move.
  void decode(const void* x, void* out, void* kc, void* vc, int64_t P, int L, int B,
              cudaStream_t st, const int* cache_lens = nullptr) {
    const int64_t T = B;
    ensure_ws(T);
    last_T = T;
    if (cfg.use_rotary) ensure_rope(cache_lens ? static_cast<int>(P) : L + 1);
    if (!kvm_fresh) compute_kvm(st);
    const void* hin = ln1(x, T, st);
    qkv_proj(hin, T, 1, L, st, cache_lens);
    launch_kv_append(qkv.ptr, 4 * Hl, Hl, dh, kc, vc, P, L, B, dt, st, cache_lens);
    const size_t pb = decode_partials_bytes(B, nhl, dh, P);
    if (pb > dpart.bytes) dpart.ensure(pb);
    launch_decode_attention(qkv.ptr, 4 * Hl, kc, vc, P, cache_lens ? static_cast<int>(P) : L + 1,
                            B, nhl, dh, dt, dpart.as<float>(), os.ptr, Hl, st, cache_lens);
    mem_attention(1, B, st);  // the batch's rows share the bank: one group of B queries
    tail(x, out, T, st);
    if (q.memory_write && cfg.use_memory_gating) write(T, true, st);
  }
};

namespace ltm_b200 {

// Sizes of a QLinear's buffers for an [n, k] weight of `scheme`, with or
// without a bias; the buffers are made to hold them.
static void shape_linear(QLinear& l, int scheme, int64_t n, int64_t k, bool with_bias) {
  l.N = n;
  l.K = k;
  l.scheme = scheme;
  if (scheme == LTM_SCHEME_W4A16) {
    l.q4.ensure(n * k / 2);
    l.s4.ensure(n * (k / 128) * sizeof(float));
    l.z4.ensure(n * (k / 128));
  } else {
    l.q8.ensure(n * k);
    l.s8.ensure(n * sizeof(float));
  }
  if (with_bias)
    l.bias.ensure(n * sizeof(float));
  else
    l.bias.release();
}

static void linear_sections(std::vector<StateSection>& out, const std::string& name,
                            const QLinear& l) {
  const int64_t n = l.N, k = l.K;
  if (l.scheme == LTM_SCHEME_W4A16) {
    out.push_back({name + ".q4", l.q4.ptr, static_cast<size_t>(n * k / 2)});
    out.push_back({name + ".s4", l.s4.ptr, static_cast<size_t>(n * (k / 128) * sizeof(float))});
    out.push_back({name + ".z4", l.z4.ptr, static_cast<size_t>(n * (k / 128))});
  } else {
    out.push_back({name + ".q8", l.q8.ptr, static_cast<size_t>(n * k)});
    out.push_back({name + ".s8", l.s8.ptr, static_cast<size_t>(n * sizeof(float))});
  }
  if (l.bias.ptr) out.push_back({name + ".bias", l.bias.ptr, static_cast<size_t>(n * sizeof(float))});
}

std::vector<StateSection> block_state(ltm_block* b, bool weights, bool bank, bool allocate) {
  const int H = b->H, F = b->F, Hl = b->Hl, Fl = b->Fl;
  const bool ub = b->cfg.use_bias != 0, lead = b->tpr == 0, tp1 = b->tp == 1;
  const int sc = b->q.scheme;
  if (allocate) {
    if (weights) {
      shape_linear(b->qkvm, sc, 4 * Hl, H, ub);
      shape_linear(b->kvm, sc, 2 * Hl, H, ub);
      shape_linear(b->o, sc, H, tp1 ? H : Hl, ub);
      shape_linear(b->om, sc, H, tp1 ? H : Hl, ub);
      shape_linear(b->g, sc, H, H, ub);
      shape_linear(b->w1, sc, Fl, H, ub);
      shape_linear(b->w2, sc, H, tp1 ? F : Fl, ub);
      b->o.apply_bias = b->om.apply_bias = b->w2.apply_bias = tp1 || lead;
      if (b->cfg.use_layer_norm)
        for (DevBuf* d : {&b->ln1_g, &b->ln1_b, &b->ln2_g, &b->ln2_b}) d->ensure(H * sizeof(float));
    }
    if (bank) b->memory.ensure(static_cast<size_t>(b->Ms) * H * dtype_size(b->dt));
  }
  std::vector<StateSection> out;
  if (weights) {
    linear_sections(out, "qkvm", b->qkvm);
    linear_sections(out, "kvm", b->kvm);
    linear_sections(out, "o", b->o);
    linear_sections(out, "om", b->om);
    linear_sections(out, "gate", b->g);
    linear_sections(out, "ffn_up", b->w1);
    linear_sections(out, "ffn_down", b->w2);
    if (b->cfg.use_layer_norm) {
      out.push_back({"ln1.gamma", b->ln1_g.ptr, H * sizeof(float)});
      out.push_back({"ln1.beta", b->ln1_b.ptr, H * sizeof(float)});
      out.push_back({"ln2.gamma", b->ln2_g.ptr, H * sizeof(float)});
      out.push_back({"ln2.beta", b->ln2_b.ptr, H * sizeof(float)});
    }
  }
  if (bank)
    out.push_back({"memory", b->memory.ptr, static_cast<size_t>(b->Ms) * H * dtype_size(b->dt)});
  return out;
}

void block_state_loaded(ltm_block* b, bool weights) {
  if (weights) {
    b->kvmb.ensure(static_cast<size_t>(b->Ms) * 2 * b->Hl * dtype_size(b->dt));
    if (b->q.scheme == LTM_SCHEME_W8A8) {
      b->mq.ensure(static_cast<size_t>(b->Ms) * b->H);
      b->ms.ensure(static_cast<size_t>(b->Ms) * sizeof(float));
    }
    b->loaded = true;
  }
  b->kvm_fresh = false;  // K_M | V_M follow the (new) bank at the next use
}

void block_identity(const ltm_block* b, ltm_block_config* cfg, ltm_quant_config* q, int* tp,
                    int* tpr, int* device, bool* loaded) {
  *cfg = b->cfg;
  *q = b->q;
  *tp = b->tp;
  *tpr = b->tpr;
  *device = b->device;
  *loaded = b->loaded;
}

}  // namespace ltm_b200

namespace {

void validate(const ltm_block_config& c, const ltm_quant_config& q) {
  LTM_REQUIRE(c.hidden_dim > 0 && c.ffn_dim > 0 && c.num_heads > 0 && c.head_dim > 0 &&
                  c.memory_slots > 0,
              "block dimensions must be positive");
  LTM_REQUIRE(c.num_heads * c.head_dim == c.hidden_dim, "num_heads * head_dim must equal hidden_dim");
  if (c.head_dim != 64 && c.head_dim != 128) LTM_UNSUPPORTED("head_dim must be 64 or 128");
  LTM_REQUIRE(c.hidden_dim % 32 == 0 && c.ffn_dim % 32 == 0,
              "hidden_dim and ffn_dim must be multiples of 32");
  if (c.use_alibi) LTM_UNSUPPORTED("ALiBi position bias");
  switch (q.scheme) {
    case LTM_SCHEME_W8A32:
      LTM_REQUIRE(q.act_dtype == LTM_DTYPE_F32, "W8A32 computes in fp32 activations");
      break;
    case LTM_SCHEME_W8A8:
    case LTM_SCHEME_W4A16:
      LTM_REQUIRE(q.act_dtype == LTM_DTYPE_F16 || q.act_dtype == LTM_DTYPE_BF16,
                  "W8A8 / W4A16 compute in f16 or bf16 activations");
      break;
    default: LTM_REQUIRE(false, "unknown quantization scheme");
  }
  if (q.scheme == LTM_SCHEME_W4A16) {
    LTM_REQUIRE(q.group_size == 128, "W4A16 group size must be 128");
    LTM_REQUIRE(c.hidden_dim % 128 == 0 && c.ffn_dim % 128 == 0,
                "W4A16 needs hidden_dim and ffn_dim multiples of 128");
  }
}

std::vector<float> cat_rows(const float* a, int64_t na, const float* b, int64_t nb, int64_t k) {
  std::vector<float> r(static_cast<size_t>((na + nb) * k));
  std::memcpy(r.data(), a, sizeof(float) * na * k);
  std::memcpy(r.data() + na * k, b, sizeof(float) * nb * k);
  return r;
}

// Rows [r0, r0 + nr) of each of the `parts` consecutive [n_part, k] blocks of
// a host matrix, concatenated ([parts * nr, k]); k = 1 for a bias.
std::vector<float> take_rows(const float* w, int parts, int64_t n_part, int64_t r0, int64_t nr,
                             int64_t k) {
  std::vector<float> r(static_cast<size_t>(parts * nr * k));
  for (int p = 0; p < parts; ++p)
    std::memcpy(r.data() + p * nr * k, w + (p * n_part + r0) * k, sizeof(float) * nr * k);
  return r;
}

void load_block(ltm_block* b, const ltm_block_weights* w, cudaStream_t st) {
  const int H = b->H, F = b->F, Hl = b->Hl, Fl = b->Fl;
  const int64_t hr0 = static_cast<int64_t>(b->tpr) * Hl, fr0 = static_cast<int64_t>(b->tpr) * Fl;
  const bool ub = b->cfg.use_bias != 0;
  const bool lead = b->tpr == 0;  // adds the biases of the row-parallel layers
  LTM_REQUIRE(w && w->w_qkv && w->w_o && w->w_qm && w->w_km && w->w_vm && w->w_om && w->w_g &&
                  w->w_1 && w->w_2 && w->memory,
              "missing weight");
  if (ub)
    LTM_REQUIRE(w->b_qkv && w->b_o && w->b_qm && w->b_km && w->b_vm && w->b_om && w->b_g && w->b_1 &&
                    w->b_2,
                "missing bias");
  if (b->cfg.use_layer_norm)
    LTM_REQUIRE(w->ln1_g && w->ln1_b && w->ln2_g && w->ln2_b, "missing LayerNorm parameters");
  // Q | K | V | Qm rows of this rank's heads
  auto wq = cat_rows(take_rows(w->w_qkv, 3, H, hr0, Hl, H).data(), 3 * Hl,
                     take_rows(w->w_qm, 1, H, hr0, Hl, H).data(), Hl, H);
  std::vector<float> bq;
  if (ub)
    bq = cat_rows(take_rows(w->b_qkv, 3, H, hr0, Hl, 1).data(), 3 * Hl,
                  take_rows(w->b_qm, 1, H, hr0, Hl, 1).data(), Hl, 1);
  b->qkvm.load(b->q, wq.data(), ub ? bq.data() : nullptr, 4 * Hl, H, st);
  // K_M | V_M rows of this rank's heads
  auto wk = cat_rows(take_rows(w->w_km, 1, H, hr0, Hl, H).data(), Hl,
                     take_rows(w->w_vm, 1, H, hr0, Hl, H).data(), Hl, H);
  std::vector<float> bk;
  if (ub)
    bk = cat_rows(take_rows(w->b_km, 1, H, hr0, Hl, 1).data(), Hl,
                  take_rows(w->b_vm, 1, H, hr0, Hl, 1).data(), Hl, 1);
  b->kvm.load(b->q, wk.data(), ub ? bk.data() : nullptr, 2 * Hl, H, st);
  if (b->tp == 1) {
    b->o.load(b->q, w->w_o, ub ? w->b_o : nullptr, H, H, st);
    b->om.load(b->q, w->w_om, ub ? w->b_om : nullptr, H, H, st);
    b->w2.load(b->q, w->w_2, ub ? w->b_2 : nullptr, H, F, st);
  } else {  // row-parallel: input columns of this rank's heads / FFN columns
    // every rank keeps the full biases (the exact reduction adds them at
    // the row owner); the partial sums carry them on the first rank only
    b->o.load_cols(b->q, w->w_o, ub ? w->b_o : nullptr, H, H, hr0, Hl, st);
    b->om.load_cols(b->q, w->w_om, ub ? w->b_om : nullptr, H, H, hr0, Hl, st);
    b->w2.load_cols(b->q, w->w_2, ub ? w->b_2 : nullptr, H, F, fr0, Fl, st);
    b->o.apply_bias = b->om.apply_bias = b->w2.apply_bias = lead;
  }
  b->g.load(b->q, w->w_g, ub ? w->b_g : nullptr, H, H, st);
  b->w1.load(b->q, w->w_1 + fr0 * H, ub ? w->b_1 + fr0 : nullptr, Fl, H, st);
  if (b->cfg.use_layer_norm) {
    for (auto pr : {std::make_pair(&b->ln1_g, w->ln1_g), std::make_pair(&b->ln1_b, w->ln1_b),
                    std::make_pair(&b->ln2_g, w->ln2_g), std::make_pair(&b->ln2_b, w->ln2_b)}) {
      pr.first->ensure(H * sizeof(float));
      LTM_CUDA_TRY(cudaMemcpy(pr.first->ptr, pr.second, H * sizeof(float), cudaMemcpyHostToDevice));
    }
  }
  b->memory.ensure(static_cast<size_t>(b->Ms) * H * dtype_size(b->dt));
  upload_f32_as(w->memory, static_cast<int64_t>(b->Ms) * H, b->dt, b->memory.ptr, st);
  b->kvmb.ensure(static_cast<size_t>(b->Ms) * 2 * Hl * dtype_size(b->dt));
  if (b->q.scheme == LTM_SCHEME_W8A8) {
    b->mq.ensure(static_cast<size_t>(b->Ms) * H);
    b->ms.ensure(static_cast<size_t>(b->Ms) * sizeof(float));
  }
  LTM_CUDA_TRY(cudaStreamSynchronize(st));
  b->loaded = true;
  b->kvm_fresh = false;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    LTM_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != dev) LTM_CUDA_TRY(cudaSetDevice(dev));
  }
  ~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

ltm_block* make_block(const ltm_block_config* cfg, const ltm_quant_config* qcfg, int device) {
  LTM_REQUIRE(cfg && qcfg, "NULL config");
  validate(*cfg, *qcfg);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    set_error("no CUDA device");
    throw Fail{LTM_ERR_NO_DEVICE};
  }
  LTM_REQUIRE(device >= 0 && device < ndev, "device index out of range");
  auto b = std::make_unique<ltm_block>();
  b->cfg = *cfg;
  b->q = *qcfg;
  b->device = device;
  b->H = cfg->hidden_dim;
  b->F = cfg->ffn_dim;
  b->nh = cfg->num_heads;
  b->dh = cfg->head_dim;
  b->Ms = cfg->memory_slots;
  b->dt = qcfg->act_dtype;
  b->nhl = b->nh;
  b->Hl = b->H;
  b->Fl = b->F;
  return b.release();
}

}  // namespace

extern "C" void ltm_block_config_default(ltm_block_config* c) {
  if (!c) return;
  c->hidden_dim = 768;
  c->ffn_dim = 3072;
  c->num_heads = 12;
  c->head_dim = 64;
  c->memory_slots = 512;
  c->memory_dim = 64;
  c->memory_update_rate = 0.9f;
  c->use_memory_compression = 1;
  c->memory_compression_ratio = 0.5f;
  c->use_flash_attention = 1;
  c->use_alibi = 0;
  c->use_rotary = 1;
  c->dropout_prob = 0.1f;
  c->use_parallel_attention = 1;
  c->use_memory_gating = 1;
  c->use_layer_norm = 1;
  c->use_bias = 1;
  c->fuse_operations = 1;
  c->learn_memory = 1;
  c->learn_compression = 1;
  c->gradient_checkpointing = 1;
}

extern "C" ltm_status ltm_block_create(const ltm_block_config* cfg, const ltm_quant_config* qcfg,
                                       int device, ltm_block** out) {
  return guarded([&] {
    LTM_REQUIRE(out, "out is NULL");
    *out = make_block(cfg, qcfg, device);
  });
}

extern "C" ltm_status ltm_block_create_tp(const ltm_block_config* cfg, const ltm_quant_config* qcfg,
                                          ltm_comm* comm, ltm_block** out) {
  return guarded([&] {
    LTM_REQUIRE(out && comm, "NULL argument");
    LTM_REQUIRE(cfg && qcfg, "NULL config");
    const int n = comm->nranks;
    LTM_REQUIRE(n >= 1, "communicator without ranks");
    LTM_REQUIRE(cfg->num_heads % n == 0, "num_heads must be divisible by the tensor-parallel size");
    LTM_REQUIRE(cfg->ffn_dim % n == 0, "ffn_dim must be divisible by the tensor-parallel size");
    const int Hl = cfg->hidden_dim / n, Fl = cfg->ffn_dim / n;
    LTM_REQUIRE(Hl % 32 == 0 && Fl % 32 == 0,
                "per-rank head and FFN widths must be multiples of 32");
    if (qcfg->scheme == LTM_SCHEME_W4A16)
      LTM_REQUIRE(Hl % 128 == 0 && Fl % 128 == 0,
                  "W4A16 needs per-rank head and FFN widths that are multiples of 128");
    std::unique_ptr<ltm_block> b(make_block(cfg, qcfg, comm->device));
    b->comm = comm;
    b->tp = n;
    b->tpr = comm->rank;
    b->nhl = b->nh / n;
    b->Hl = Hl;
    b->Fl = Fl;
    *out = b.release();
  });
}

extern "C" ltm_status ltm_block_load_weights(ltm_block* blk, const ltm_block_weights* w) {
  return guarded([&] {
    LTM_REQUIRE(blk, "block is NULL");
    DeviceGuard g(blk->device);
    load_block(blk, w, nullptr);
  });
}

extern "C" ltm_status ltm_block_forward(ltm_block* blk, const void* x, void* y,
                                        const void* attention_mask, int B, int S, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded, "block not created or weights not loaded");
    if (attention_mask) LTM_UNSUPPORTED("explicit attention masks (self-attention is causal)");
    LTM_REQUIRE(B >= 0 && S >= 0, "negative batch or sequence length");
    if (B == 0 || S == 0) return;
    LTM_REQUIRE(x && y && x != y, "x and y must be distinct device buffers");
    DeviceGuard g(blk->device);
    blk->forward(x, y, B, S, as_stream(stream));
  });
}

extern "C" ltm_status ltm_block_decode_step(ltm_block* blk, const void* x, void* y, void* k_cache,
                                            void* v_cache, int64_t max_positions, int cache_len,
                                            int B, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded, "block not created or weights not loaded");
    LTM_REQUIRE(B >= 0, "negative batch");
    if (B == 0) return;
    LTM_REQUIRE(x && y && x != y, "x and y must be distinct device buffers");
    LTM_REQUIRE(k_cache && v_cache && k_cache != v_cache, "NULL or aliased KV cache");
    LTM_REQUIRE(blk->dt != LTM_DTYPE_F32, "decode needs f16 or bf16 activations (W8A8 / W4A16)");
    LTM_REQUIRE(cache_len >= 0 && static_cast<int64_t>(cache_len) < max_positions,
                "cache_len must lie in [0, max_positions)");
    LTM_REQUIRE((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 == 0,
                "KV cache must be 16-byte aligned");
    DeviceGuard g(blk->device);
    blk->decode(x, y, k_cache, v_cache, max_positions, cache_len, B, as_stream(stream));
  });
}

extern "C" ltm_status ltm_block_forward_sp(ltm_block* blk, const void* x_local, void* y_local,
                                           int B, int S, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded, "block not created or weights not loaded");
    LTM_REQUIRE(blk->tp > 1 && blk->comm, "sequence parallelism needs a tensor-parallel block");
    LTM_REQUIRE(B >= 0 && S >= 0, "negative batch or sequence length");
    if (B == 0 || S == 0) return;
    const int64_t T = static_cast<int64_t>(B) * S;
    LTM_REQUIRE(T % blk->tp == 0, "B * S must be a multiple of the tensor-parallel size");
    LTM_REQUIRE(x_local && y_local && x_local != y_local, "x and y must be distinct device buffers");
    LTM_REQUIRE(blk->dt != LTM_DTYPE_F32, "sequence parallelism needs f16 or bf16 activations");
    DeviceGuard g(blk->device);
    blk->forward_sp(x_local, y_local, B, S, as_stream(stream));
  });
}

extern "C" ltm_status ltm_block_set_tp_reduction(ltm_block* blk, int mode) {
  return guarded([&] {
    LTM_REQUIRE(blk, "block is NULL");
    LTM_REQUIRE(mode == LTM_TP_REDUCE_ACT || mode == LTM_TP_REDUCE_EXACT, "unknown reduction mode");
    LTM_REQUIRE(mode == LTM_TP_REDUCE_ACT || blk->q.scheme == LTM_SCHEME_W8A8,
                "the exact reduction needs the W8A8 scheme");
    blk->tp_reduce = mode;
  });
}

extern "C" ltm_status ltm_block_set_overlap(ltm_block* blk, int overlap, int comm_sms) {
  return guarded([&] {
    LTM_REQUIRE(blk, "block is NULL");
    LTM_REQUIRE(comm_sms >= 0 && comm_sms < 128, "comm_sms out of range");
    blk->overlap = overlap < 0 ? -1 : (overlap != 0 ? 1 : 0);
    blk->comm_sms = comm_sms;
  });
}

extern "C" ltm_status ltm_block_forward_with_cache(ltm_block* blk, const void* x, void* y, int B,
                                                   int S, void* k_cache, void* v_cache,
                                                   int64_t max_positions, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded, "block not created or weights not loaded");
    LTM_REQUIRE(B >= 0 && S >= 0, "negative batch or sequence length");
    if (B == 0 || S == 0) return;
    LTM_REQUIRE(x && y && x != y, "x and y must be distinct device buffers");
    LTM_REQUIRE(k_cache && v_cache && k_cache != v_cache, "NULL or aliased KV cache");
    LTM_REQUIRE(blk->dt != LTM_DTYPE_F32, "KV caches hold f16 or bf16 (W8A8 / W4A16)");
    LTM_REQUIRE(S <= max_positions, "the prompt is longer than the cache");
    LTM_REQUIRE((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 == 0,
                "KV cache must be 16-byte aligned");
    DeviceGuard g(blk->device);
    blk->forward(x, y, B, S, as_stream(stream), k_cache, v_cache, max_positions);
  });
}

extern "C" ltm_status ltm_block_decode_step_ragged(ltm_block* blk, const void* x, void* y,
                                                   void* k_cache, void* v_cache,
                                                   int64_t max_positions,
                                                   const int32_t* cache_lens, int B,
                                                   void* stream) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded, "block not created or weights not loaded");
    LTM_REQUIRE(B >= 0, "negative batch");
    if (B == 0) return;
    LTM_REQUIRE(x && y && x != y, "x and y must be distinct device buffers");
    LTM_REQUIRE(k_cache && v_cache && k_cache != v_cache, "NULL or aliased KV cache");
    LTM_REQUIRE(cache_lens, "NULL cache_lens");
    LTM_REQUIRE(blk->dt != LTM_DTYPE_F32, "decode needs f16 or bf16 activations (W8A8 / W4A16)");
    LTM_REQUIRE(max_positions >= 1 && max_positions < (1ll << 31), "max_positions out of range");
    LTM_REQUIRE((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 == 0,
                "KV cache must be 16-byte aligned");
    DeviceGuard g(blk->device);
    blk->decode(x, y, k_cache, v_cache, max_positions, 0, B, as_stream(stream), cache_lens);
  });
}

extern "C" ltm_status ltm_block_memory_write(ltm_block* blk, const float* state,
                                             const void* queries, int64_t ldq, int64_t T,
                                             void* stream) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded, "block not created or weights not loaded");
    LTM_REQUIRE(state, "NULL state");
    if (blk->q.use_attention_scores) {
      LTM_REQUIRE(queries && T > 0, "attention-score slot weights need at least one query row");
      LTM_REQUIRE(ldq >= blk->Hl, "query row stride smaller than the block's query width");
      LTM_REQUIRE(static_cast<size_t>(blk->Ms) * sizeof(float) <= 200 * 1024,
                  "memory_slots too large for the slot-weight kernel (max 51200)");
    }
    DeviceGuard g(blk->device);
    blk->write_state(state, queries, ldq, T, as_stream(stream));
  });
}

extern "C" ltm_status ltm_block_get_memory(ltm_block* blk, void* out, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded && out, "bad argument");
    DeviceGuard g(blk->device);
    LTM_CUDA_TRY(cudaMemcpyAsync(out, blk->memory.ptr,
                                 static_cast<size_t>(blk->Ms) * blk->H * dtype_size(blk->dt),
                                 cudaMemcpyDeviceToDevice, as_stream(stream)));
  });
}

extern "C" ltm_status ltm_block_intermediate(ltm_block* blk, const char* name, void* out,
                                             void* stream, int64_t* rows, int64_t* cols,
                                             int* kind) {
  return guarded([&] {
    LTM_REQUIRE(blk && blk->loaded && name && rows && cols && kind, "bad argument");
    LTM_REQUIRE(blk->last_T > 0, "no forward or decode step has run on this block");
    const std::string n(name);
    const int64_t T = blk->last_T;
    const int64_t H = blk->H, Hl = blk->Hl, Fl = blk->Fl;
    const size_t a = dtype_size(blk->dt);
    const bool w8a8 = blk->q.scheme == LTM_SCHEME_W8A8;
    const bool ln = blk->cfg.use_layer_norm != 0;
    struct View {
      const char* name;
      bool present;
      const void* p;
      int64_t r, c, ld;
      int kind;
    };
    const View views[] = {
        {"ln1_q", w8a8, blk->hq.ptr, T, H, H, 1},
        {"ln1_s", w8a8, blk->hs.ptr, T, 1, 1, 2},
        {"x_q", w8a8, blk->xq.ptr, T, H, H, 1},
        {"x_s", w8a8, blk->xs.ptr, T, 1, 1, 2},
        {"ln1", !w8a8 && ln, blk->h.ptr, T, H, H, 0},
        {"qkvm", true, blk->qkv.ptr, T, 4 * Hl, 4 * Hl, 0},
        {"kvm", true, blk->kvmb.ptr, blk->Ms, 2 * Hl, 2 * Hl, 0},
        {"attn_self", true, blk->os.ptr, T, Hl, Hl, 0},
        {"attn_mem", true, blk->om_.ptr, T, Hl, Hl, 0},
        {"attn_self_q", w8a8, blk->osq.ptr, T, Hl, Hl, 1},
        {"attn_self_s", w8a8, blk->oss.ptr, T, 1, 1, 2},
        {"attn_mem_q", w8a8, blk->omq.ptr, T, Hl, Hl, 1},
        {"attn_mem_s", w8a8, blk->oms.ptr, T, 1, 1, 2},
        {"s", true, blk->spm.ptr, T, H, H, 0},
        {"m", true, static_cast<const char*>(blk->spm.ptr) + T * H * a, T, H, H, 0},
        {"y", true, blk->y.ptr, T, H, H, 0},
        {"ln2_q", w8a8, blk->zq.ptr, T, H, H, 1},
        {"ln2_s", w8a8, blk->zs.ptr, T, 1, 1, 2},
        {"ln2", !w8a8 && ln, blk->z.ptr, T, H, H, 0},
        {"ffn_hidden", true, blk->u.ptr, T, Fl, Fl, 0},
        {"ffn_hidden_q", w8a8, blk->uq.ptr, T, Fl, Fl, 1},
        {"ffn_hidden_s", w8a8, blk->us.ptr, T, 1, 1, 2},
    };
    for (const View& v : views) {
      if (n != v.name) continue;
      LTM_REQUIRE(v.present && v.p, "this block's scheme has no such intermediate");
      *rows = v.r;
      *cols = v.c;
      *kind = v.kind;
      if (out) {
        const size_t es = v.kind == 0 ? a : (v.kind == 1 ? 1 : sizeof(float));
        DeviceGuard g(blk->device);
        LTM_CUDA_TRY(cudaMemcpy2DAsync(out, v.c * es, v.p, v.ld * es, v.c * es, v.r,
                                       cudaMemcpyDeviceToDevice, as_stream(stream)));
      }
      return;
    }
    LTM_REQUIRE(false, "unknown intermediate name");
  });
}

extern "C" ltm_status ltm_block_destroy(ltm_block* blk) {
  return guarded([&] {
    if (!blk) return;
    DeviceGuard g(blk->device);
    cudaDeviceSynchronize();
    delete blk;
  });
}

// ---------------------------------------------------------------- the model --
struct ltm_model {
  std::vector<std::unique_ptr<ltm_block>> layers;
  ltm_block_config cfg{};
  ltm_quant_config q{};
  int device = 0, vocab = 0;
  DevBuf emb, a, b;
  int64_t ws_T = 0;
  // LM head (TitanForCausalLM.lm_head, no bias): weight rows padded to a
  // multiple of 32 (vocab_p); rows of hidden states gathered contiguously,
  // their int8 codes / scales (W8A8), logits of the padded vocabulary when
  // vocab != vocab_p
  QLinear head;
  bool head_loaded = false;
  int vocab_p = 0;
  DevBuf hrows, hq, hs, hlog, wdq;
  int64_t head_rows = 0;

  ltm_dtype dt() const { return q.act_dtype; }

  // Makes sure the layer ping-pong buffers hold T rows.
  void ensure_ws(int64_t T) {
    if (T <= ws_T) return;
    const size_t bytes = static_cast<size_t>(T) * cfg.hidden_dim * dtype_size(dt());
    a.ensure(bytes);
    b.ensure(bytes);
    ws_T = T;
  }

  // logits [rows, vocab] (stride ld_logits) of `rows` hidden rows of stride
  // ld_hidden elements.
  void lm_head(const void* hidden, int64_t rows, int64_t ld_hidden, void* logits, int64_t ld_logits,
               cudaStream_t st) {
    const int H = cfg.hidden_dim;
    const size_t es = dtype_size(dt());
    if (rows > head_rows) {
      hrows.ensure(static_cast<size_t>(rows) * H * es);
      if (q.scheme == LTM_SCHEME_W8A8) {
        hq.ensure(static_cast<size_t>(rows) * H);
        hs.ensure(static_cast<size_t>(rows) * sizeof(float));
      }
      if (vocab_p != vocab) hlog.ensure(static_cast<size_t>(rows) * vocab_p * es);
      head_rows = rows;
    }
    const void* in = hidden;
    if (ld_hidden != H) {
      LTM_CUDA_TRY(cudaMemcpy2DAsync(hrows.ptr, H * es, hidden, ld_hidden * es, H * es, rows,
                                     cudaMemcpyDeviceToDevice, st));
      in = hrows.ptr;
    }
    if (q.scheme == LTM_SCHEME_W8A8)
      launch_rowwise_int8(in, dt(), rows, H, hq.as<int8_t>(), hs.as<float>(), st);
    Epilogue ep;
    const bool direct = vocab_p == vocab;
    ep.out = direct ? logits : hlog.ptr;
    ep.ldo = direct ? ld_logits : vocab_p;
    head.run(in, hq.as<int8_t>(), hs.as<float>(), rows, kEpiPlain, dt(), ep, st, &wdq);
    if (!direct)
      LTM_CUDA_TRY(cudaMemcpy2DAsync(logits, ld_logits * es, hlog.ptr, vocab_p * es, vocab * es,
                                     rows, cudaMemcpyDeviceToDevice, st));
  }

  void require_ready(bool need_head) const {
    LTM_REQUIRE(emb.ptr, "model not created or embedding not loaded");
    for (auto& l : layers) LTM_REQUIRE(l->loaded, "a layer has no weights");
    if (need_head) LTM_REQUIRE(head_loaded, "LM head not loaded");
  }
};

extern "C" ltm_status ltm_model_create(const ltm_block_config* cfg, const ltm_quant_config* qcfg,
                                       int n_layers, int vocab_size, int device, ltm_model** out) {
  return guarded([&] {
    LTM_REQUIRE(out && n_layers > 0 && vocab_size > 0, "bad argument");
    auto m = std::make_unique<ltm_model>();
    for (int i = 0; i < n_layers; ++i) m->layers.emplace_back(make_block(cfg, qcfg, device));
    m->cfg = *cfg;
    m->q = *qcfg;
    m->device = device;
    m->vocab = vocab_size;
    *out = m.release();
  });
}

extern "C" ltm_status ltm_model_load_embedding(ltm_model* m, const float* embedding) {
  return guarded([&] {
    LTM_REQUIRE(m && embedding, "bad argument");
    DeviceGuard g(m->device);
    const int64_t n = static_cast<int64_t>(m->vocab) * m->cfg.hidden_dim;
    m->emb.ensure(n * dtype_size(m->q.act_dtype));
    upload_f32_as(embedding, n, m->q.act_dtype, m->emb.ptr, nullptr);
  });
}

extern "C" ltm_status ltm_model_load_layer(ltm_model* m, int layer, const ltm_block_weights* w) {
  return guarded([&] {
    LTM_REQUIRE(m && layer >= 0 && layer < static_cast<int>(m->layers.size()), "bad layer index");
    DeviceGuard g(m->device);
    load_block(m->layers[layer].get(), w, nullptr);
  });
}

extern "C" ltm_status ltm_model_forward(ltm_model* m, const int32_t* tokens, void* hidden_out, int B,
                                        int S, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(m && m->emb.ptr, "model not created or embedding not loaded");
    for (auto& l : m->layers) LTM_REQUIRE(l->loaded, "a layer has no weights");
    LTM_REQUIRE(B >= 0 && S >= 0, "negative batch or sequence length");
    if (B == 0 || S == 0) return;
    LTM_REQUIRE(tokens && hidden_out, "NULL pointer");
    DeviceGuard g(m->device);
    cudaStream_t st = as_stream(stream);
    const int64_t T = static_cast<int64_t>(B) * S;
    const int H = m->cfg.hidden_dim;
    m->ensure_ws(T);
    launch_embed_gather(m->emb.ptr, m->q.act_dtype, m->vocab, H, tokens, T, m->a.ptr, st);
    const void* cur = m->a.ptr;
    const size_t L = m->layers.size();
    for (size_t i = 0; i < L; ++i) {
      void* dst = (i + 1 == L) ? hidden_out : (cur == m->a.ptr ? m->b.ptr : m->a.ptr);
      m->layers[i]->forward(cur, dst, B, S, st);
      cur = dst;
    }
  });
}

extern "C" ltm_status ltm_model_load_lm_head(ltm_model* m, const float* weight) {
  return guarded([&] {
    LTM_REQUIRE(m && weight, "bad argument");
    DeviceGuard g(m->device);
    const int H = m->cfg.hidden_dim;
    m->vocab_p = (m->vocab + 31) / 32 * 32;
    std::vector<float> wp;
    const float* w = weight;
    if (m->vocab_p != m->vocab) {  // zero rows up to a multiple of 32
      wp.assign(static_cast<size_t>(m->vocab_p) * H, 0.0f);
      std::memcpy(wp.data(), weight, sizeof(float) * static_cast<size_t>(m->vocab) * H);
      w = wp.data();
    }
    m->head.load(m->q, w, nullptr, m->vocab_p, H, nullptr);
    m->head_loaded = true;
  });
}

extern "C" ltm_status ltm_model_lm_head(ltm_model* m, const void* hidden, int64_t rows,
                                        int64_t row_stride, void* logits, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(m && m->head_loaded, "model not created or LM head not loaded");
    LTM_REQUIRE(rows >= 0 && row_stride >= m->cfg.hidden_dim, "bad rows / row stride");
    if (rows == 0) return;
    LTM_REQUIRE(hidden && logits, "NULL pointer");
    DeviceGuard g(m->device);
    m->lm_head(hidden, rows, row_stride, logits, m->vocab, as_stream(stream));
  });
}

namespace {

void check_caches(ltm_model* m, void* const* kc, void* const* vc, int64_t P) {
  LTM_REQUIRE(kc && vc, "NULL cache pointer arrays");
  LTM_REQUIRE(m->q.act_dtype != LTM_DTYPE_F32, "KV caches hold f16 or bf16 (W8A8 / W4A16)");
  LTM_REQUIRE(P >= 1 && P < (1ll << 31), "max_positions out of range");
  for (size_t i = 0; i < m->layers.size(); ++i) {
    LTM_REQUIRE(kc[i] && vc[i] && kc[i] != vc[i], "NULL or aliased KV cache");
    LTM_REQUIRE((reinterpret_cast<uintptr_t>(kc[i]) | reinterpret_cast<uintptr_t>(vc[i])) % 16 == 0,
                "KV cache must be 16-byte aligned");
  }
}

}  // namespace

extern "C" ltm_status ltm_model_prefill(ltm_model* m, const int32_t* tokens, int B, int S,
                                        void* const* k_caches, void* const* v_caches,
                                        int64_t max_positions, void* hidden_out,
                                        void* logits_last, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(m, "NULL model");
    m->require_ready(logits_last != nullptr);
    LTM_REQUIRE(B >= 0 && S >= 0, "negative batch or sequence length");
    if (B == 0 || S == 0) return;
    LTM_REQUIRE(tokens, "NULL tokens");
    LTM_REQUIRE(S <= max_positions, "the prompt is longer than the cache");
    check_caches(m, k_caches, v_caches, max_positions);
    DeviceGuard g(m->device);
    cudaStream_t st = as_stream(stream);
    const int64_t T = static_cast<int64_t>(B) * S;
    const int H = m->cfg.hidden_dim;
    m->ensure_ws(T);
    launch_embed_gather(m->emb.ptr, m->dt(), m->vocab, H, tokens, T, m->a.ptr, st);
    const void* cur = m->a.ptr;
    const size_t L = m->layers.size();
    for (size_t i = 0; i < L; ++i) {
      void* dst = (i + 1 == L && hidden_out) ? hidden_out : (cur == m->a.ptr ? m->b.ptr : m->a.ptr);
      m->layers[i]->forward(cur, dst, B, S, st, k_caches[i], v_caches[i], max_positions);
      cur = dst;
    }
    if (logits_last) {  // the last position of every sequence
      const char* last = static_cast<const char*>(cur) +
                         static_cast<size_t>(S - 1) * H * dtype_size(m->dt());
      m->lm_head(last, B, static_cast<int64_t>(S) * H, logits_last, m->vocab, st);
    }
  });
}

extern "C" ltm_status ltm_model_decode_step(ltm_model* m, const int32_t* tokens,
                                            const int32_t* cache_lens, int B,
                                            void* const* k_caches, void* const* v_caches,
                                            int64_t max_positions, void* hidden_out,
                                            void* logits, void* stream) {
  return guarded([&] {
    LTM_REQUIRE(m, "NULL model");
    m->require_ready(logits != nullptr);
    LTM_REQUIRE(B >= 0, "negative batch");
    if (B == 0) return;
    LTM_REQUIRE(tokens && cache_lens, "NULL tokens / cache_lens");
    check_caches(m, k_caches, v_caches, max_positions);
    DeviceGuard g(m->device);
    cudaStream_t st = as_stream(stream);
    const int H = m->cfg.hidden_dim;
    m->ensure_ws(B);
    launch_embed_gather(m->emb.ptr, m->dt(), m->vocab, H, tokens, B, m->a.ptr, st);
    const void* cur = m->a.ptr;
    const size_t L = m->layers.size();
    for (size_t i = 0; i < L; ++i) {
      void* dst = (i + 1 == L && hidden_out) ? hidden_out : (cur == m->a.ptr ? m->b.ptr : m->a.ptr);
      m->layers[i]->decode(cur, dst, k_caches[i], v_caches[i], max_positions, 0, B, st,
                           cache_lens);
      cur = dst;
    }
    if (logits) m->lm_head(cur, B, H, logits, m->vocab, st);
  });
}

extern "C" ltm_status ltm_model_destroy(ltm_model* m) {
  return guarded([&] {
    if (!m) return;
    DeviceGuard g(m->device);
    cudaDeviceSynchronize();
    delete m;
  });
}
