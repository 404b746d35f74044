// memory_noalloc.cu -- allocation-free variant of the memory-bank store.
//
// ltm_memory_store keeps its scratch (the column sums of the query rows and
// the per-slot update weights) in device memory that the library allocates on
// the first call per device and grows when a larger bank arrives.  Some
// callers cannot let a library allocate device memory at call time: a host
// framework that owns every byte of device memory through its own planned
// arena, a serving process that must keep its device footprint fixed after
// start-up, or a latency-critical loop in which a cudaMalloc would stall the
// device.  ltm_memory_store_noalloc serves them: its scratch is a fixed
// file-scope device array, so the call allocates nothing.
//
// Limits and behaviour:
//   * the array holds kNoAllocScratchFloats fp32 values (256 KiB) on every GPU
//     that loads the library, until the process exits;
//   * with use_attention_scores != 0 it fits round_up(hidden_dim, 64) +
//     memory_slots <= kNoAllocScratchFloats; larger sizes are rejected with
//     LTM_ERR_INVALID_ARG.  Rate-only calls (use_attention_scores == 0) use no
//     scratch and take any size ltm_memory_store takes;
//   * every call shares the one array and clears the parts it uses at its
//     start (in stream order), so calls whose GPU work overlaps -- different
//     streams, or different host threads without ordering -- race on it;
//   * the first call on a device looks the array's device address up
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before any stream capture.  The cached address belongs to the
//     device's primary context: after cudaDeviceReset (or anything else that
//     destroys that context) it is stale, so do not call this entry point
//     again in that process.
#include <mutex>

#include "block.cuh"

namespace ltm_b200 {
namespace {

constexpr int kNoAllocScratchFloats = 64 * 1024;
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol; kernels receive the device address looked up below.
static __device__ __align__(256) float g_store_scratch[kNoAllocScratchFloats];

// Device address of g_store_scratch on the current device, looked up once per
// device (no heap, no device allocation).
float* scratch_address() {
  static std::mutex mu;
  static float* addr[kMaxDevices] = {};
  int dev = 0;
  LTM_CUDA_TRY(cudaGetDevice(&dev));
  LTM_REQUIRE(dev >= 0 && dev < kMaxDevices, "device index beyond the scratch address table");
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_store_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error(std::string("cudaGetSymbolAddress of the memory-store scratch failed: ") +
                cudaGetErrorString(e));
      throw Fail{LTM_ERR_CUDA};
    }
    addr[dev] = static_cast<float*>(p);
  }
  return addr[dev];
}

}  // namespace
}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_memory_store_noalloc(void* memory, const void* keys, int64_t ldk,
                                               const void* queries, int64_t ldq, int64_t T,
                                               const float* state, int memory_slots,
                                               int hidden_dim, int num_heads, float update_rate,
                                               int use_attention_scores, ltm_dtype dtype,
                                               void* stream) {
  return guarded([&] {
    const bool scores = use_attention_scores != 0;
    validate_memory_store(memory, keys, ldk, queries, ldq, T, state, memory_slots, hidden_dim,
                          num_heads, scores);
    const int64_t qsum_floats = (static_cast<int64_t>(hidden_dim) + 63) / 64 * 64;
    LTM_REQUIRE(!scores || qsum_floats + memory_slots <= kNoAllocScratchFloats,
                "hidden_dim (rounded up to 64) + memory_slots exceeds the 65536-float "
                "allocation-free scratch; use ltm_memory_store");
    if (memory_slots == 0 || hidden_dim == 0) return;
    // Rate-only updates read no scratch (the bank update takes the constant
    // rate), so they need no device address either.
    float* scratch = scores ? scratch_address() : nullptr;
    launch_memory_store(memory, keys, ldk, queries, ldq, T, state, 1.0f, memory_slots, hidden_dim,
                        num_heads, update_rate, scores, dtype, scratch,
                        scores ? scratch + qsum_floats : nullptr, as_stream(stream));
  });
}
