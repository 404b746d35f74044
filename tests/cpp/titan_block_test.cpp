// titan_block_test.cpp -- the C++ drop-in (include/ltm/titan_block.hpp) on the
// GPU: TitanBlock<float / half / __nv_bfloat16> forward on weights and inputs
// written by the pytest driver (tests/test_cpp_dropin_gpu.py), checkpoint
// save / load round trip, Quantizer<T> INT8 / INT4, and error reporting as
// std::runtime_error.  Outputs go back to the driver as raw fp32 / byte
// files, which it compares with the oracle.
//
//   titan_block_test <dir>     (dir holds meta.txt, w_*.f32, x.f32)
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "ltm/titan_block.hpp"

namespace {

std::vector<float> read_f32(const std::string& path, size_t n) {
  std::vector<float> v(n);
  std::ifstream f(path, std::ios::binary);
  if (!f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(n * 4)))
    throw std::runtime_error("cannot read " + path);
  return v;
}

template <class V>
void write_raw(const std::string& path, const V& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(v.data()),
          static_cast<std::streamsize>(v.size() * sizeof(v[0])));
}

template <class T>
T cvt(float x);
template <>
float cvt<float>(float x) { return x; }
template <>
half cvt<half>(float x) { return __float2half_rn(x); }
template <>
__nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
float back(float x) { return x; }
float back(half x) { return __half2float(x); }
float back(__nv_bfloat16 x) { return __bfloat162float(x); }

template <class T>
std::vector<T> to_t(const std::vector<float>& v) {
  std::vector<T> o(v.size());
  for (size_t i = 0; i < v.size(); ++i) o[i] = cvt<T>(v[i]);
  return o;
}

template <class T>
std::vector<float> to_f32(const std::vector<T>& v) {
  std::vector<float> o(v.size());
  for (size_t i = 0; i < v.size(); ++i) o[i] = back(v[i]);
  return o;
}

template <class T>
int run_block(const std::string& dir, const std::string& tag,
              const ltm::transformer::TitanBlockConfig& cfg,
              const ltm::transformer::BlockWeights& w, const std::vector<float>& x, int B, int S) {
  using ltm::Tensor;
  using ltm::transformer::TitanBlock;
  const int H = cfg.hidden_dim;
  TitanBlock<T> blk(cfg);
  blk.loadWeights(w);
  const std::vector<T> xt = to_t<T>(x);
  Tensor<T> in({B, S, H}, xt.data());
  Tensor<T> out({B, S, H});
  blk.forward(in, out);
  ltm::cuda_check(cudaDeviceSynchronize(), "forward");
  const std::vector<float> y = to_f32(out.toHost());
  write_raw(dir + "/y_" + tag + ".f32", y);
  // checkpoint round trip: a block restored from the file, without the fp32
  // master weights, gives the same bits
  const std::string ck = dir + "/block_" + tag + ".ltm";
  blk.save(ck);
  TitanBlock<T> restored(cfg);
  restored.load(ck);
  Tensor<T> out2({B, S, H});
  restored.forward(in, out2);
  ltm::cuda_check(cudaDeviceSynchronize(), "forward (restored)");
  const std::vector<float> y2 = to_f32(out2.toHost());
  if (std::memcmp(y.data(), y2.data(), y.size() * 4) != 0) {
    std::cerr << tag << ": restored block differs\n";
    return 3;
  }
  const Tensor<T> bank = blk.getMemoryBank();
  if (bank.shape()[0] != cfg.memory_slots || bank.shape()[1] != H) return 4;
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::cerr << "usage: titan_block_test <dir>\n";
    return 2;
  }
  const std::string dir = argv[1];
  int H = 0, F = 0, nh = 0, Ms = 0, B = 0, S = 0;
  {
    std::ifstream meta(dir + "/meta.txt");
    meta >> H >> F >> nh >> Ms >> B >> S;
    if (!meta) {
      std::cerr << "bad meta.txt\n";
      return 2;
    }
  }
  try {
    ltm::transformer::TitanBlockConfig cfg;
    cfg.hidden_dim = H;
    cfg.ffn_dim = F;
    cfg.num_heads = nh;
    cfg.head_dim = H / nh;
    cfg.memory_slots = Ms;
    ltm::transformer::BlockWeights w;
    const size_t h = H, f = F, ms = Ms;
    struct Part {
      const char* name;
      std::vector<float>* v;
      size_t n;
    } parts[] = {{"w_qkv", &w.w_qkv, 3 * h * h}, {"b_qkv", &w.b_qkv, 3 * h},
                 {"w_o", &w.w_o, h * h},         {"b_o", &w.b_o, h},
                 {"w_qm", &w.w_qm, h * h},       {"b_qm", &w.b_qm, h},
                 {"w_km", &w.w_km, h * h},       {"b_km", &w.b_km, h},
                 {"w_vm", &w.w_vm, h * h},       {"b_vm", &w.b_vm, h},
                 {"w_om", &w.w_om, h * h},       {"b_om", &w.b_om, h},
                 {"w_g", &w.w_g, h * h},         {"b_g", &w.b_g, h},
                 {"w_1", &w.w_1, f * h},         {"b_1", &w.b_1, f},
                 {"w_2", &w.w_2, h * f},         {"b_2", &w.b_2, h},
                 {"ln1_g", &w.ln1_g, h},         {"ln1_b", &w.ln1_b, h},
                 {"ln2_g", &w.ln2_g, h},         {"ln2_b", &w.ln2_b, h},
                 {"memory", &w.memory, ms * h}};
    for (auto& p : parts) *p.v = read_f32(dir + "/" + p.name + ".f32", p.n);
    const std::vector<float> x = read_f32(dir + "/x.f32", static_cast<size_t>(B) * S * H);

    int rc = run_block<float>(dir, "f32", cfg, w, x, B, S);
    if (!rc) rc = run_block<half>(dir, "f16", cfg, w, x, B, S);
    if (!rc) rc = run_block<__nv_bfloat16>(dir, "bf16", cfg, w, x, B, S);
    if (rc) return rc;

    // Quantizer<T>: INT8 per channel of the FFN-up weight (half), INT4 group
    // 128 of it (bf16); the dequantized INT8 weight back as half
    using namespace ltm::quantization;
    {
      const std::vector<half> wh = to_t<half>(w.w_1);
      ltm::Tensor<half> wt({F, H}, wh.data());
      QuantizationConfig qc;
      Quantizer<half> q(qc);
      QuantizedTensor<half> qt;
      q.quantize(wt, qt);
      ltm::Tensor<half> deq({F, H});
      q.dequantize(qt, deq);
      ltm::cuda_check(cudaDeviceSynchronize(), "int8 quantize");
      write_raw(dir + "/q8_codes.i8", qt.codes().toHost());
      write_raw(dir + "/q8_scales.f32", qt.scales().toHost());
      write_raw(dir + "/q8_deq.f32", to_f32(deq.toHost()));
    }
    {
      const std::vector<__nv_bfloat16> wb = to_t<__nv_bfloat16>(w.w_1);
      ltm::Tensor<__nv_bfloat16> wt({F, H}, wb.data());
      QuantizationConfig qc;
      qc.precision = QuantizationPrecision::INT4;
      qc.symmetric = false;
      Quantizer<__nv_bfloat16> q(qc);
      QuantizedTensor<__nv_bfloat16> qt;
      q.quantize(wt, qt);
      ltm::cuda_check(cudaDeviceSynchronize(), "int4 quantize");
      write_raw(dir + "/q4_packed.u8", qt.codes().toHost());
      write_raw(dir + "/q4_scales.f32", qt.scales().toHost());
      write_raw(dir + "/q4_zp.u8", qt.zeroPoints().toHost());
    }
    // errors surface as std::runtime_error with the library's message
    bool threw = false;
    try {
      ltm::transformer::TitanBlockConfig bad = cfg;
      bad.head_dim = 96;
      bad.num_heads = H / 96 > 0 ? H / 96 : 1;
      bad.hidden_dim = bad.num_heads * 96;
      ltm::transformer::TitanBlock<half> b(bad);
    } catch (const std::runtime_error& e) {
      threw = std::string(e.what()).find("head_dim") != std::string::npos;
    }
    if (!threw) {
      std::cerr << "an unsupported head_dim did not throw\n";
      return 5;
    }
  } catch (const std::exception& e) {
    std::cerr << "error: " << e.what() << "\n";
    return 1;
  }
  std::cout << "titan_block_test ok\n";
  return 0;
}
