// runtime.cu -- error strings, device error word, device properties and the
// TMA descriptor encoder (driver entry point resolved through the runtime, so
// the library needs no link-time dependency on libcuda).
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <map>
#include <mutex>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace ltm_b200 {

__device__ int g_device_error = 0;

int* device_error_ptr() {
  static std::mutex mu;
  static std::vector<int*> cache;
  int dev = 0;
  LTM_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, nullptr);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    LTM_CUDA_TRY(cudaGetSymbolAddress(&p, g_device_error));
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

namespace {
thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};
std::atomic<uint64_t> g_device_allocs{0};
}  // namespace

// Kernel timer: while on, every launch on the timed stream is followed by an
// event; a kernel's duration is the time between its event and the previous
// one (launches on one stream run back to back).
struct KernelTimer {
  std::mutex mu;
  std::atomic<bool> on{false};
  cudaStream_t stream = nullptr;
  int device = -1;
  cudaEvent_t start = nullptr;
  std::vector<std::pair<std::string, cudaEvent_t>> marks;
  std::vector<cudaEvent_t> pool;
  cudaEvent_t get() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};
KernelTimer& timer() {
  static KernelTimer t;
  return t;
}

void note_launch(const char* what, cudaStream_t stream) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  KernelTimer& t = timer();
  if (!t.on.load(std::memory_order_relaxed) || stream != t.stream) return;
  std::lock_guard<std::mutex> lk(t.mu);
  cudaEvent_t e = t.get();
  if (e && cudaEventRecord(e, stream) == cudaSuccess) t.marks.emplace_back(what, e);
}

void note_device_alloc() { g_device_allocs.fetch_add(1, std::memory_order_relaxed); }

void set_error(const std::string& msg) { t_last_error = msg; }
void clear_error() { t_last_error.clear(); }

namespace {
thread_local int t_sm_reserve = 0;
}  // namespace

ScopedSmReserve::ScopedSmReserve(int n) : prev_(t_sm_reserve) { t_sm_reserve = n; }
ScopedSmReserve::~ScopedSmReserve() { t_sm_reserve = prev_; }

int device_sm_count() {
  const int n = device_sm_count_total();
  return n - t_sm_reserve > 1 ? n - t_sm_reserve : 1;
}

int device_sm_count_total() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  LTM_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    LTM_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    cache[dev] = n;
  }
  return cache[dev];
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    throw Fail{LTM_ERR_CUDA};
  }
  return fn;
}
}  // namespace

void make_tma_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  LTM_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  LTM_REQUIRE((row_stride_elems * elem_bytes) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  if (swizzle == CU_TENSOR_MAP_SWIZZLE_128B)
    LTM_REQUIRE(box_cols * elem_bytes <= 128, "TMA box inner extent exceeds the 128-byte swizzle");
  LTM_REQUIRE((box_cols * elem_bytes) % 16 == 0, "TMA box inner extent must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)));
    throw Fail{LTM_ERR_CUDA};
  }
}

}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" const char* ltm_version(void) { return "ltm_b200 0.1.0 (sm_100a)"; }

extern "C" const char* ltm_last_error_string(void) { return t_last_error.c_str(); }

extern "C" ltm_status ltm_device_error(int* code_out) {
  return guarded([&] {
    LTM_REQUIRE(code_out != nullptr, "code_out is NULL");
    int zero = 0, v = 0;
    LTM_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
    LTM_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
    *code_out = v;
  });
}

extern "C" ltm_status ltm_launch_count(uint64_t* count_out) {
  return guarded([&] {
    LTM_REQUIRE(count_out != nullptr, "count_out is NULL");
    *count_out = g_launches.load(std::memory_order_relaxed);
  });
}

extern "C" ltm_status ltm_device_alloc_count(uint64_t* count_out) {
  return guarded([&] {
    LTM_REQUIRE(count_out != nullptr, "count_out is NULL");
    *count_out = g_device_allocs.load(std::memory_order_relaxed);
  });
}

extern "C" ltm_status ltm_kernel_timer_begin(void* stream) {
  return guarded([&] {
    KernelTimer& t = timer();
    std::lock_guard<std::mutex> lk(t.mu);
    LTM_REQUIRE(!t.on.load(), "kernel timer already running");
    for (auto& m : t.marks) t.pool.push_back(m.second);
    t.marks.clear();
    if (!t.start) LTM_CUDA_TRY(cudaEventCreate(&t.start));
    t.stream = as_stream(stream);
    LTM_CUDA_TRY(cudaEventRecord(t.start, t.stream));
    t.on.store(true);
  });
}

extern "C" ltm_status ltm_kernel_timer_end(char* report, size_t capacity) {
  return guarded([&] {
    KernelTimer& t = timer();
    std::lock_guard<std::mutex> lk(t.mu);
    LTM_REQUIRE(t.on.load(), "kernel timer not running");
    t.on.store(false);
    LTM_CUDA_TRY(cudaStreamSynchronize(t.stream));
    std::map<std::string, std::pair<int, double>> agg;
    std::vector<std::string> order;
    cudaEvent_t prev = t.start;
    for (auto& m : t.marks) {
      float ms = 0.0f;
      LTM_CUDA_TRY(cudaEventElapsedTime(&ms, prev, m.second));
      if (!agg.count(m.first)) order.push_back(m.first);
      agg[m.first].first += 1;
      agg[m.first].second += ms;
      prev = m.second;
    }
    std::string out;
    for (const auto& name : order) {
      char line[256];
      std::snprintf(line, sizeof(line), "%s %d %.6f\n", name.c_str(), agg[name].first,
                    agg[name].second);
      out += line;
    }
    LTM_REQUIRE(report && capacity > out.size(), "report buffer too small");
    std::memcpy(report, out.c_str(), out.size() + 1);
  });
}
