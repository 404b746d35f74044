// common.cuh -- shared host/device helpers of the B200 Titan-block library:
// status plumbing for the C ABI, dtype traits, and the sm_100a PTX wrappers
// (mbarrier, TMA, tcgen05) used by the tensor-core kernels.
#pragma once

#include <type_traits>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/ltm_b200.h"

namespace ltm_b200 {

// ------------------------------------------------------------------ status --
void set_error(const std::string& msg);
void clear_error();

struct Fail {
  ltm_status st;
};

// Device address (current device) of the error word that bounded in-kernel
// waits write when they expire (0 = none).  Kernels receive it as a parameter.
int* device_error_ptr();

enum DeviceErrorCode : int {
  kErrNone = 0,
  kErrWaitFull = 1,     // consumer waited too long for a TMA stage
  kErrWaitEmpty = 2,    // producer waited too long for a free stage
  kErrWaitAccum = 3,    // epilogue waited too long for the accumulator
  kErrWaitOther = 4,
  kErrBadCacheLen = 5,  // a per-sequence cache length outside [0, max_positions)
};

#define LTM_CUDA_TRY(expr)                                                              \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    if (_e != cudaSuccess) {                                                            \
      ::ltm_b200::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));       \
      throw ::ltm_b200::Fail{LTM_ERR_CUDA};                                             \
    }                                                                                   \
  } while (0)

#define LTM_REQUIRE(cond, msg)                                                          \
  do {                                                                                  \
    if (!(cond)) {                                                                      \
      ::ltm_b200::set_error(std::string("invalid argument: ") + (msg));                 \
      throw ::ltm_b200::Fail{LTM_ERR_INVALID_ARG};                                      \
    }                                                                                   \
  } while (0)

#define LTM_UNSUPPORTED(msg)                                                            \
  do {                                                                                  \
    ::ltm_b200::set_error(std::string("unsupported: ") + (msg));                        \
    throw ::ltm_b200::Fail{LTM_ERR_UNSUPPORTED};                                        \
  } while (0)

// Wraps a C-ABI body: converts Fail / std exceptions into a status.
template <class F>
ltm_status guarded(F&& f) {
  try {
    clear_error();
    f();
    return LTM_OK;
  } catch (const Fail& e) {
    return e.st;
  } catch (const std::exception& e) {
    set_error(e.what());
    return LTM_ERR_CUDA;
  }
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Counts a launch and, while the kernel timer is on for `stream`, records an
// event after it (the kernel's end; its start is the previous mark).
void note_launch(const char* what, cudaStream_t stream);
// Counts one device allocation made by the library (every cudaMalloc goes
// through DevBuf::ensure, which calls this).
void note_device_alloc();

inline void check_launch(const char* what, cudaStream_t stream = nullptr) {
  note_launch(what, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    throw Fail{LTM_ERR_CUDA};
  }
}

inline size_t dtype_size(ltm_dtype d) { return d == LTM_DTYPE_F32 ? 4 : 2; }

// -------------------------------------------------------------- dtype I/O --
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <class T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Symmetric INT8 code of v for scale s: clamp(round_half_away(v / s), -127, 127)
// with v / s the IEEE round-to-nearest quotient (s == 0 -> 0), bit-identical to
// evaluating that division, but with the quotient estimated as v * inv_s
// (inv_s = 1/s rounded to nearest).  The estimate is within |q| * 2^-23 of the
// exact quotient and the IEEE quotient within |q| * 2^-24, so both round to the
// same integer unless the estimate lies within |q| * 1.5 * 2^-23 of a rounding
// boundary k + 1/2; only then (margin 2^-20 here) is the division evaluated.
__device__ __forceinline__ int8_t quant_i8_exact(float v, float s, float inv_s) {
  if (s == 0.0f) return 0;
  float t = v * inv_s;
  const float a = fabsf(t);
  const float f = a - floorf(a);
  if (fabsf(f - 0.5f) <= a * 9.5367431640625e-07f) t = __fdiv_rn(v, s);  // 2^-20
  float r = roundf(t);
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}

__device__ __forceinline__ float recip_or_zero(float s) { return s == 0.0f ? 0.0f : __frcp_rn(s); }

// Packed fp32 pairs (sm_100 f32x2 instructions: two IEEE round-to-nearest
// operations per instruction, lane by lane).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Warp-cooperative form of quant_i8_exact for V values per lane; must be
// called by all 32 lanes (lanes without data pass zeros).  Off the rounding
// ties round-half-even equals round-half-away, so the common path rounds with
// the 1.5 * 2^23 shift (for |t| < 2^22, t + 1.5 * 2^23 holds round-half-even(t)
// in its low mantissa bits, whose low byte is the two's-complement int8 code)
// -- about five instructions per value, none on the conversion unit.  Its
// near-tie test is wider than quant_i8_exact's: |t| <= 127.5 makes
// |t| * 2^-20 <= 1.22e-4, so every value within 2^-20 |t| of a tie is within
// 1.22e-4 of it; a warp holding such a value takes the IEEE quotients of
// quant_i8_exact, so the codes equal quant_i8_exact's.  Requires
// |v| <= 127 |s| (s is the row's, or a larger, absmax / 127), so that codes
// stay within [-127, 127] without a clamp; s = 0 gives inv_s = 0 and code 0.
template <int V>
__device__ __forceinline__ void quant_i8_exact_warp(const float (&v)[V], float s, float inv_s,
                                                    int8_t (&out)[V]) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  constexpr float kTie = 0.5f - 1.220703125e-4f;  // 0.5 - 2^-13
  static_assert(V % 2 == 0, "values in pairs");
  float big[V];
  bool near_tie = false;
  const uint64_t inv2 = f2_pack(inv_s, inv_s), shift2 = f2_pack(kShift, kShift);
#pragma unroll
  for (int i = 0; i < V; i += 2) {  // the same per-value operations, two values per instruction
    const uint64_t t = f2_mul(f2_pack(v[i], v[i + 1]), inv2);
    const uint64_t b = f2_add(t, shift2);
    float d0, d1;
    f2_unpack(f2_sub(t, f2_sub(b, shift2)), d0, d1);
    f2_unpack(b, big[i], big[i + 1]);
    near_tie |= (fabsf(d0) >= kTie) | (fabsf(d1) >= kTie);
  }
  if (__any_sync(0xffffffffu, near_tie)) {
#pragma unroll
    for (int i = 0; i < V; ++i) out[i] = quant_i8_exact(v[i], s, inv_s);
    return;
  }
#pragma unroll
  for (int i = 0; i < V; ++i) out[i] = static_cast<int8_t>(__float_as_uint(big[i]) & 0xFFu);
}

// 2^x with the hardware approximation (MUFU.EX2, flush-to-zero); 2^-inf = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Dispatch a runtime dtype onto a template functor taking the element type.
template <class F>
void dispatch_dtype(ltm_dtype d, F&& f) {
  switch (d) {
    case LTM_DTYPE_F32: f(float{}); break;
    case LTM_DTYPE_F16: f(__half{}); break;
    case LTM_DTYPE_BF16: f(__nv_bfloat16{}); break;
    default: LTM_REQUIRE(false, "unknown dtype");
  }
}

// Number of SMs of the current device (cached per device).
// SMs the library's persistent grids may use on the current device: all of
// them, less the reserve of a ScopedSmReserve active on this thread (left to
// collectives that run concurrently on another stream).
int device_sm_count();
int device_sm_count_total();
struct ScopedSmReserve {
  explicit ScopedSmReserve(int n);
  ~ScopedSmReserve();
  ScopedSmReserve(const ScopedSmReserve&) = delete;
  ScopedSmReserve& operator=(const ScopedSmReserve&) = delete;

 private:
  int prev_;
};

// Grid size of a persistent kernel: resident CTAs per SM (from the occupancy
// calculator for this kernel, block size and dynamic smem) x SMs, capped at
// `want` (the CTAs the problem needs).
template <class K>
int persistent_grid(K kernel, int block, size_t smem, int64_t want) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, block, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t cap = static_cast<int64_t>(per_sm) * device_sm_count();
  return static_cast<int>(want < cap ? (want < 1 ? 1 : want) : cap);
}

// ------------------------------------------------------- PTX: sync/timing --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any single in-kernel wait.  Kernels that exceed it record an
// error code in the device error word and unwind instead of spinning forever.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (and
// records `code` in the device error word and the CTA abort flag) when the
// limit expires or another role of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort_flag, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      atomicCAS(err, 0, code);
      return false;
    }
  }
}

// ------------------------------------------------------------- PTX: TMA --
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ------------------------------------------------------- PTX: clusters --
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of every CTA of the cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Shared::cluster address of `p` (a shared::cta pointer of this CTA's layout)
// in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Arrive (release, cluster scope) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Tiled TMA load of a CTA pair: the box lands in this CTA's shared memory and
// its bytes complete on the mbarrier at `bar_cluster_addr`, which may be the
// peer CTA's; the data goes to this CTA only.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* desc,
                                                 uint32_t bar_cluster_addr, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

// Tiled TMA store of one box from shared memory (bulk-group completion).
// The box's smem writes must be made visible to the async proxy first
// (fence_proxy_async_smem by the writing threads, then a warp/CTA sync).
__device__ __forceinline__ void tma_store_2d(const void* desc, const void* smem_src, int32_t x,
                                             int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(desc)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N committed bulk groups of this thread still read smem.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until every committed bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// --------------------------------------------------------- PTX: tcgen05 --
__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// TMEM allocation of a CTA pair (cta_group::2): issued by one warp in each
// CTA of the pair; both CTAs receive the same column range.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 x int8 -> int32.
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` (same shared-memory offset) in every CTA of `cta_mask`
// once all tcgen05.mma of the CTA pair issued so far by this thread completed.
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// CTA-pair MMA (cta_group::2): D (M = 256 split 128 / 128 over the pair's
// TMEM) (+)= A (128 rows from each CTA's shared memory) * B^T (N/2 rows from
// each CTA's shared memory), int8 x int8 -> int32.  Issued by the pair's
// even-rank CTA only.
__device__ __forceinline__ void tc_mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// CTA-pair MMA (cta_group::2) of f16 / bf16 operands -> fp32, as
// tc_mma_i8_pair.  Issued by the pair's even-rank CTA only.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B^T, f16/bf16 inputs -> fp32.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Loads 32 consecutive 32-bit columns of this warp's 32 TMEM lanes
// (thread i of the warp receives lane base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Stores 32 consecutive 32-bit columns of this warp's 32 TMEM lanes (thread
// i writes lane base+i); complete with tmem_wait_st.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// tcgen05.wait::ld that also names the destination registers of the load it
// completes, so no use of them can be scheduled above the wait (used when the
// next load is issued before the current registers are consumed).
__device__ __forceinline__ void tmem_wait_ld_tie(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart), the
// layout a SWIZZLE_128B TMA box of 128-byte rows produces.  Fields: start
// address>>4 [0,14), leading byte offset>>4 [16,30) (unused for this layout),
// stride byte offset>>4 [32,46), descriptor version 1 [46,48), swizzle mode
// 2 = 128B [61,64).
__device__ __forceinline__ uint64_t make_desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(16 >> 4) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Shared-memory matrix descriptor of an MN-major operand tile stored with the
// 128-byte swizzle: rows of 128 bytes (64 16-bit elements) along M/N, one row
// per K index, 8-row groups 1024 bytes apart (stride byte offset), further
// 64-element M/N chunks `lbo_bytes` apart (leading byte offset).  This is the
// layout a SWIZZLE_128B TMA box of [K rows x 64 elements] produces.
__device__ __forceinline__ uint64_t make_desc_mnmajor_sw128(uint32_t smem_addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::i8 (signed x signed -> s32),
// both operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4)                       // D format: s32
         | (1u << 7)                     // A: signed 8-bit
         | (1u << 10)                    // B: signed 8-bit
         | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor of tcgen05.mma kind::f16 (f16 or bf16 inputs, fp32
// accumulate), both operands K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16, bool b_mn_major = false) {
  return (1u << 4)                                   // D format: f32
         | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((b_mn_major ? 1u : 0u) << 16)               // B major: 0 = K, 1 = MN
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// -------------------------------------------------------- TMA descriptors --
template <class T>
constexpr CUtensorMapDataType tma_dtype_of() {
  if constexpr (std::is_same<T, __half>::value) return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  else if constexpr (std::is_same<T, float>::value) return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  else if constexpr (std::is_same<T, int32_t>::value) return CU_TENSOR_MAP_DATA_TYPE_INT32;
  else return CU_TENSOR_MAP_DATA_TYPE_UINT8;
}

// 2-D tiled tensor map over a row-major [rows, cols] matrix of `elem_bytes`
// elements (128-byte swizzle unless given); box = box_cols x box_rows.
void make_tma_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

}  // namespace ltm_b200
