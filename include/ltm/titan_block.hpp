// titan_block.hpp -- C++17 drop-in for the reference's block and quantizer
// classes, over the C ABI of ltm_b200.h (header-only; link libltm_b200.so and
// the CUDA runtime).
//
//   ltm::Tensor<T>                      include/core/utils/tensor.cuh:18-315
//   ltm::transformer::TitanBlockConfig  include/core/transformer/titan_inspired_block.cuh:19-50
//   ltm::transformer::TitanBlock<T>     include/core/transformer/titan_inspired_block.cuh:61-154
//   ltm::quantization::QuantizationConfig, QuantizedTensor<T>, Quantizer<T>
//                                       include/core/quantization/quantizer.cuh:10-60,177-185
//
// T is float (W8A32: int8 weights, fp32 activations), half or __nv_bfloat16
// (W8A8 by default, W4A16 on request).  Errors surface as std::runtime_error
// carrying ltm_last_error_string(), as the reference's CUDA_CHECK does
// (include/core/utils/cuda_utils.cuh:19-45).  Tensors are device buffers
// owned by the caller; a block owns its quantized weights, bank and workspace.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <random>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

#include "../ltm_b200.h"

namespace ltm {

inline void check(ltm_status s) {
  if (s != LTM_OK) throw std::runtime_error(std::string("ltm_b200: ") + ltm_last_error_string());
}

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
struct dtype_of;
template <>
struct dtype_of<float> {
  static constexpr ltm_dtype value = LTM_DTYPE_F32;
};
template <>
struct dtype_of<half> {
  static constexpr ltm_dtype value = LTM_DTYPE_F16;
};
template <>
struct dtype_of<__nv_bfloat16> {
  static constexpr ltm_dtype value = LTM_DTYPE_BF16;
};

// Owning (or viewing) device tensor, move-only, row-major.
template <class T>
class Tensor {
 public:
  explicit Tensor(std::vector<int> shape) : shape_(std::move(shape)) { allocate(); }
  // own_memory: copy `data` from the host; else view `data` as device memory.
  Tensor(std::vector<int> shape, const T* data, bool own_memory = true)
      : shape_(std::move(shape)), own_(own_memory) {
    if (own_) {
      allocate();
      copyFromHost(data);
    } else {
      data_ = const_cast<T*>(data);
    }
  }
  Tensor(Tensor&& o) noexcept : data_(o.data_), shape_(std::move(o.shape_)), own_(o.own_) {
    o.data_ = nullptr;
    o.own_ = false;
  }
  Tensor& operator=(Tensor&& o) noexcept {
    if (this != &o) {
      release();
      data_ = o.data_;
      shape_ = std::move(o.shape_);
      own_ = o.own_;
      o.data_ = nullptr;
      o.own_ = false;
    }
    return *this;
  }
  Tensor(const Tensor&) = delete;
  Tensor& operator=(const Tensor&) = delete;
  ~Tensor() { release(); }

  T* data() const { return data_; }
  const std::vector<int>& shape() const { return shape_; }
  int64_t numel() const {
    int64_t n = 1;
    for (int d : shape_) n *= d;
    return n;
  }
  void copyFromHost(const T* host) {
    cuda_check(cudaMemcpy(data_, host, numel() * sizeof(T), cudaMemcpyHostToDevice), "H2D");
  }
  void copyToHost(T* host) const {
    cuda_check(cudaMemcpy(host, data_, numel() * sizeof(T), cudaMemcpyDeviceToHost), "D2H");
  }
  std::vector<T> toHost() const {
    std::vector<T> v(static_cast<size_t>(numel()));
    copyToHost(v.data());
    return v;
  }

 private:
  void allocate() {
    if (numel() > 0) cuda_check(cudaMalloc(&data_, numel() * sizeof(T)), "cudaMalloc");
    own_ = true;
  }
  void release() {
    if (own_ && data_) cudaFree(data_);
    data_ = nullptr;
  }
  T* data_ = nullptr;
  std::vector<int> shape_;
  bool own_ = true;
};

namespace transformer {

// TitanBlockConfig: the same fields, order and defaults as the reference
// (the bools are ints in the C layout; true / false assign as before).
struct TitanBlockConfig : ltm_block_config {
  TitanBlockConfig() { ltm_block_config_default(this); }
};

// Quantization of a block: scheme, INT4 group, memory write after the read.
struct QuantConfig : ltm_quant_config {
  template <class T>
  static QuantConfig defaults() {
    QuantConfig q;
    q.scheme = std::is_same<T, float>::value ? LTM_SCHEME_W8A32 : LTM_SCHEME_W8A8;
    q.group_size = 128;
    q.act_dtype = dtype_of<T>::value;
    q.memory_write = 0;
    q.use_attention_scores = 1;
    return q;
  }
};

// Host fp32 master weights of one block ([out, in] row-major), owning.
struct BlockWeights {
  std::vector<float> w_qkv, b_qkv, w_o, b_o, w_qm, b_qm, w_km, b_km, w_vm, b_vm, w_om, b_om, w_g,
      b_g, w_1, b_1, w_2, b_2, ln1_g, ln1_b, ln2_g, ln2_b, memory;

  // Seeded random init (weights and biases N(0, 0.02), LayerNorm gamma
  // 1 + N(0, 0.02), beta N(0, 0.02), bank N(0, 1/sqrt(H))), the role of the
  // reference's initialize() (titan_inspired_block.cuh:76).
  static BlockWeights random(const TitanBlockConfig& c, uint64_t seed) {
    const size_t H = c.hidden_dim, F = c.ffn_dim, Ms = c.memory_slots;
    std::mt19937_64 gen(seed);
    std::normal_distribution<float> n01(0.0f, 1.0f);
    auto fill = [&](std::vector<float>& v, size_t n, float std, float mean = 0.0f) {
      v.resize(n);
      for (float& x : v) x = mean + std * n01(gen);
    };
    BlockWeights w;
    fill(w.w_qkv, 3 * H * H, 0.02f); fill(w.b_qkv, 3 * H, 0.02f);
    fill(w.w_o, H * H, 0.02f);       fill(w.b_o, H, 0.02f);
    fill(w.w_qm, H * H, 0.02f);      fill(w.b_qm, H, 0.02f);
    fill(w.w_km, H * H, 0.02f);      fill(w.b_km, H, 0.02f);
    fill(w.w_vm, H * H, 0.02f);      fill(w.b_vm, H, 0.02f);
    fill(w.w_om, H * H, 0.02f);      fill(w.b_om, H, 0.02f);
    fill(w.w_g, H * H, 0.02f);       fill(w.b_g, H, 0.02f);
    fill(w.w_1, F * H, 0.02f);       fill(w.b_1, F, 0.02f);
    fill(w.w_2, H * F, 0.02f);       fill(w.b_2, H, 0.02f);
    fill(w.ln1_g, H, 0.02f, 1.0f);   fill(w.ln1_b, H, 0.02f);
    fill(w.ln2_g, H, 0.02f, 1.0f);   fill(w.ln2_b, H, 0.02f);
    fill(w.memory, Ms * H, 1.0f / std::sqrt(static_cast<float>(H)));
    return w;
  }

  ltm_block_weights view() const {
    auto p = [](const std::vector<float>& v) { return v.empty() ? nullptr : v.data(); };
    ltm_block_weights w{};
    w.w_qkv = p(w_qkv); w.b_qkv = p(b_qkv); w.w_o = p(w_o); w.b_o = p(b_o);
    w.w_qm = p(w_qm); w.b_qm = p(b_qm); w.w_km = p(w_km); w.b_km = p(b_km);
    w.w_vm = p(w_vm); w.b_vm = p(b_vm); w.w_om = p(w_om); w.b_om = p(b_om);
    w.w_g = p(w_g); w.b_g = p(b_g); w.w_1 = p(w_1); w.b_1 = p(b_1); w.w_2 = p(w_2);
    w.b_2 = p(b_2); w.ln1_g = p(ln1_g); w.ln1_b = p(ln1_b); w.ln2_g = p(ln2_g);
    w.ln2_b = p(ln2_b); w.memory = p(memory);
    return w;
  }
};

template <class T>
class TitanBlock {
  static_assert(std::is_same<T, float>::value || std::is_same<T, half>::value ||
                    std::is_same<T, __nv_bfloat16>::value,
                "TitanBlock<T>: T is float, half or __nv_bfloat16");

 public:
  explicit TitanBlock(const TitanBlockConfig& config,
                      const QuantConfig& quant = QuantConfig::defaults<T>(), int device = 0)
      : config_(config), quant_(quant) {
    if (quant_.act_dtype != dtype_of<T>::value)
      throw std::runtime_error("TitanBlock<T>: the quantization config's act dtype is not T");
    check(ltm_block_create(&config_, &quant_, device, &blk_));
  }
  TitanBlock(const TitanBlock&) = delete;
  TitanBlock& operator=(const TitanBlock&) = delete;
  ~TitanBlock() {
    if (blk_) ltm_block_destroy(blk_);
  }

  // Random init with a seed (the reference initializes on the device with
  // curand; the stream argument is kept for the signature).
  void initialize(cudaStream_t = nullptr, uint64_t seed = 0) {
    loadWeights(BlockWeights::random(config_, seed));
  }
  void loadWeights(const BlockWeights& w) {
    const ltm_block_weights v = w.view();
    check(ltm_block_load_weights(blk_, &v));
  }

  // input, output: [batch, seq, hidden]; attention_mask must be NULL (the
  // self-attention is causal).
  void forward(const Tensor<T>& input, Tensor<T>& output,
               const Tensor<T>* attention_mask = nullptr, cudaStream_t stream = nullptr) {
    const auto& s = input.shape();
    if (s.size() != 3 || s[2] != config_.hidden_dim || output.shape() != s)
      throw std::runtime_error("TitanBlock::forward: tensors must be [batch, seq, hidden_dim]");
    check(ltm_block_forward(blk_, input.data(), output.data(),
                            attention_mask ? attention_mask->data() : nullptr, s[0], s[1],
                            stream));
  }

  // One decode step, every sequence's new token at position cache_len of the
  // head-major caches [batch, heads, max_positions, head_dim].
  void decodeStep(const Tensor<T>& x, Tensor<T>& y, Tensor<T>& k_cache, Tensor<T>& v_cache,
                  int cache_len, cudaStream_t stream = nullptr) {
    check(ltm_block_decode_step(blk_, x.data(), y.data(), k_cache.data(), v_cache.data(),
                                k_cache.shape().at(2), cache_len, x.shape().at(0), stream));
  }

  const TitanBlockConfig& getConfig() const { return config_; }
  // A copy of the memory bank [memory_slots, hidden_dim] (getMemoryBank()).
  Tensor<T> getMemoryBank(cudaStream_t stream = nullptr) const {
    Tensor<T> m({config_.memory_slots, config_.hidden_dim});
    check(ltm_block_get_memory(blk_, m.data(), stream));
    cuda_check(cudaStreamSynchronize(stream), "getMemoryBank");
    return m;
  }
  void save(const std::string& path) const { check(ltm_block_save(blk_, path.c_str())); }
  void load(const std::string& path) { check(ltm_block_load(blk_, path.c_str())); }
  void saveMemory(const std::string& path) const {
    check(ltm_block_save_memory(blk_, path.c_str()));
  }
  void loadMemory(const std::string& path) { check(ltm_block_load_memory(blk_, path.c_str())); }
  ltm_block* handle() const { return blk_; }

 private:
  TitanBlockConfig config_;
  QuantConfig quant_;
  ltm_block* blk_ = nullptr;
};

}  // namespace transformer

namespace quantization {

enum class QuantizationPrecision { INT8, INT4, FP16, BF16 };

struct QuantizationConfig {
  bool enabled = true;
  QuantizationPrecision precision = QuantizationPrecision::INT8;
  bool per_channel = true;
  bool symmetric = true;
  int channel_axis = 0;
  int group_size = 128;  // INT4 groups along the input dimension
};

// Quantized codes and their parameters, on the device: INT8 codes [rows,
// cols] with fp32 scales [rows] (one row per output channel, or one for the
// whole tensor); INT4 packed nibbles [rows, cols/2] with fp32 scales and
// uint8 zero-points [rows, cols/group].
template <class T>
class QuantizedTensor {
 public:
  QuantizedTensor() = default;
  const std::vector<int>& shape() const { return shape_; }
  QuantizationPrecision precision() const { return precision_; }
  const void* data() const { return codes_.empty() ? nullptr : codes_.data(); }
  const Tensor<uint8_t>& codes() const { return codes_.front(); }
  const Tensor<float>& scales() const { return scales_.front(); }
  const Tensor<uint8_t>& zeroPoints() const { return zps_.front(); }
  int rows() const { return rows_; }
  int cols() const { return cols_; }

 private:
  template <class>
  friend class Quantizer;
  std::vector<int> shape_;
  QuantizationPrecision precision_ = QuantizationPrecision::INT8;
  int rows_ = 0, cols_ = 0;
  std::vector<Tensor<uint8_t>> codes_, zps_;
  std::vector<Tensor<float>> scales_;
};

template <class T>
class Quantizer {
 public:
  explicit Quantizer(const QuantizationConfig& config) : config_(config) {
    if (config_.precision != QuantizationPrecision::INT8 &&
        config_.precision != QuantizationPrecision::INT4)
      throw std::runtime_error("Quantizer: INT8 and INT4 are the quantized precisions");
    if (config_.precision == QuantizationPrecision::INT8 && !config_.symmetric)
      throw std::runtime_error("Quantizer: INT8 is symmetric (asymmetric is the INT4 form)");
    if (config_.channel_axis != 0)
      throw std::runtime_error("Quantizer: channels are the rows (channel_axis 0)");
  }

  void quantize(const Tensor<T>& input, QuantizedTensor<T>& output,
                cudaStream_t stream = nullptr) {
    const auto& s = input.shape();
    const int64_t n = input.numel();
    const int rows = config_.per_channel && !s.empty() ? s[0] : 1;
    const int cols = static_cast<int>(n / rows);
    output.shape_ = s;
    output.precision_ = config_.precision;
    output.rows_ = rows;
    output.cols_ = cols;
    output.codes_.clear();
    output.scales_.clear();
    output.zps_.clear();
    if (config_.precision == QuantizationPrecision::INT8) {
      output.codes_.emplace_back(std::vector<int>{rows, cols});
      output.scales_.emplace_back(std::vector<int>{rows});
      check(ltm_quantize_int8_per_channel(input.data(), dtype_of<T>::value, rows, cols,
                                          reinterpret_cast<int8_t*>(output.codes_[0].data()),
                                          output.scales_[0].data(), stream));
    } else {
      const int g = config_.group_size;
      output.codes_.emplace_back(std::vector<int>{rows, cols / 2});
      output.scales_.emplace_back(std::vector<int>{rows, cols / g});
      output.zps_.emplace_back(std::vector<int>{rows, cols / g});
      check(ltm_quantize_int4_grouped(input.data(), dtype_of<T>::value, rows, cols, g,
                                      output.codes_[0].data(), output.scales_[0].data(),
                                      output.zps_[0].data(), stream));
    }
  }

  void dequantize(const QuantizedTensor<T>& input, Tensor<T>& output,
                  cudaStream_t stream = nullptr) {
    if (output.numel() != static_cast<int64_t>(input.rows()) * input.cols())
      throw std::runtime_error("Quantizer::dequantize: output size differs");
    if (input.precision() == QuantizationPrecision::INT8)
      check(ltm_dequantize_int8_per_channel(
          reinterpret_cast<const int8_t*>(input.codes().data()), input.scales().data(),
          input.rows(), input.cols(), output.data(), dtype_of<T>::value, stream));
    else
      check(ltm_dequantize_int4_grouped(input.codes().data(), input.scales().data(),
                                        input.zeroPoints().data(), input.rows(), input.cols(),
                                        config_.group_size, output.data(), dtype_of<T>::value,
                                        stream));
  }

  const QuantizationConfig& config() const { return config_; }
  void setConfig(const QuantizationConfig& c) { config_ = c; }

 private:
  QuantizationConfig config_;
};

}  // namespace quantization
}  // namespace ltm
