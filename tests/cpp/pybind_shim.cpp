// pybind_shim.cpp -- the reference's `_ltm` pybind module
// (python_bindings/src/main.cpp:34-66,211-236) re-pointed at this library
// through the C++ drop-in header: TitanBlockConfig with the same fields and
// TitanModelImpl holding a TitanBlock.  Tensors cross as device addresses
// (torch's data_ptr()) so the module builds without torch headers.  This is
// the binding INTEGRATION.md shows; the CPU suite compiles and imports it.
#include <pybind11/pybind11.h>

#include <cstdint>

#include "ltm/titan_block.hpp"

namespace py = pybind11;
using ltm::transformer::TitanBlockConfig;

class TitanModelImpl {
 public:
  explicit TitanModelImpl(const TitanBlockConfig& config) : model_(config) {}
  void initialize(uint64_t seed) { model_.initialize(nullptr, seed); }
  void load(const std::string& path) { model_.load(path); }
  void save(const std::string& path) const { model_.save(path); }
  // input / output: device addresses of [batch, seq, hidden] fp32 tensors
  void forward(uintptr_t input, uintptr_t output, int batch, int seq, uintptr_t stream) {
    const int H = model_.getConfig().hidden_dim;
    ltm::Tensor<float> in({batch, seq, H}, reinterpret_cast<const float*>(input), false);
    ltm::Tensor<float> out({batch, seq, H}, reinterpret_cast<float*>(output), false);
    model_.forward(in, out, nullptr, reinterpret_cast<cudaStream_t>(stream));
  }

 private:
  ltm::transformer::TitanBlock<float> model_;
};

PYBIND11_MODULE(ltm_pybind_shim, m) {
  m.doc() = "The reference's _ltm module over the B200 Titan-block library";
  py::class_<TitanBlockConfig>(m, "TitanBlockConfig")
      .def(py::init<>())
      .def_readwrite("hidden_dim", &TitanBlockConfig::hidden_dim)
      .def_readwrite("ffn_dim", &TitanBlockConfig::ffn_dim)
      .def_readwrite("num_heads", &TitanBlockConfig::num_heads)
      .def_readwrite("head_dim", &TitanBlockConfig::head_dim)
      .def_readwrite("memory_slots", &TitanBlockConfig::memory_slots)
      .def_readwrite("memory_dim", &TitanBlockConfig::memory_dim)
      .def_readwrite("memory_update_rate", &TitanBlockConfig::memory_update_rate)
      .def_readwrite("use_memory_compression", &TitanBlockConfig::use_memory_compression)
      .def_readwrite("memory_compression_ratio", &TitanBlockConfig::memory_compression_ratio)
      .def_readwrite("use_flash_attention", &TitanBlockConfig::use_flash_attention)
      .def_readwrite("use_alibi", &TitanBlockConfig::use_alibi)
      .def_readwrite("use_rotary", &TitanBlockConfig::use_rotary)
      .def_readwrite("dropout_prob", &TitanBlockConfig::dropout_prob)
      .def_readwrite("use_bias", &TitanBlockConfig::use_bias)
      .def_readwrite("use_layer_norm", &TitanBlockConfig::use_layer_norm)
      .def_readwrite("fuse_operations", &TitanBlockConfig::fuse_operations);
  py::class_<TitanModelImpl>(m, "TitanModelImpl")
      .def(py::init<const TitanBlockConfig&>())
      .def("initialize", &TitanModelImpl::initialize, py::arg("seed") = 0)
      .def("load", &TitanModelImpl::load)
      .def("save", &TitanModelImpl::save)
      .def("forward", &TitanModelImpl::forward, py::arg("input"), py::arg("output"),
           py::arg("batch"), py::arg("seq"), py::arg("stream") = 0);
}
