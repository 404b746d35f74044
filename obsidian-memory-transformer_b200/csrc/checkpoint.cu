// checkpoint.cu -- quantized checkpoints of a block: TitanBlock<T>::save / load
// (include/core/transformer/titan_inspired_block.cuh:147-154) and
// MemoryBank<T>::save / load (include/core/ltm/memory_bank.cuh:152-159), which
// the reference declares and never defines.
//
// File layout (little-endian):
//   header   magic "LTMB200\0", format version, kind (1 = block weights and
//            bank, 2 = bank only), header size, section count, the writer's
//            ltm_block_config and ltm_quant_config, tensor-parallel size and
//            rank, then an FNV-1a 64 checksum of the bytes before it;
//   sections one per device buffer of the block's state in a fixed order --
//            per linear its int8 codes and fp32 scales (W8A8 / W8A32) or
//            packed INT4 nibbles, fp32 group scales and uint8 zero-points
//            (W4A16), and its fp32 bias when it has one; the LayerNorm
//            gammas / betas; the bank [Ms, H] in the activation dtype --
//            each a 64-byte header (name, byte count, FNV-1a 64 checksum of
//            the bytes) followed by the bytes, padded to 16.
// The weights are stored quantized, so a load restores the exact codes and
// scales without requantizing, and a block saved under tensor parallelism
// holds its own shard (a load checks the size and rank).
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include "block.cuh"

namespace ltm_b200 {
namespace {

constexpr char kMagic[8] = {'L', 'T', 'M', 'B', '2', '0', '0', '\0'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kKindBlock = 1, kKindBank = 2;

struct FileHeader {
  char magic[8];
  uint32_t version;
  uint32_t kind;
  uint32_t header_bytes;
  uint32_t n_sections;
  ltm_block_config cfg;
  ltm_quant_config quant;
  int32_t tp;
  int32_t tpr;
  uint64_t checksum;  // of the bytes before this field
};

struct SectionHeader {
  char name[48];
  uint64_t bytes;
  uint64_t checksum;
};
static_assert(sizeof(SectionHeader) == 64, "section header is 64 bytes");

uint64_t fnv1a(const void* p, size_t n, uint64_t h = 1469598103934665603ull) {
  const unsigned char* b = static_cast<const unsigned char*>(p);
  for (size_t i = 0; i < n; ++i) {
    h ^= b[i];
    h *= 1099511628211ull;
  }
  return h;
}

struct File {
  FILE* f = nullptr;
  ~File() {
    if (f) std::fclose(f);
  }
};

void write_all(FILE* f, const void* p, size_t n, const char* path) {
  if (n && std::fwrite(p, 1, n, f) != n) {
    set_error(std::string("checkpoint write failed: ") + path);
    throw Fail{LTM_ERR_INVALID_ARG};
  }
}

void read_all(FILE* f, void* p, size_t n, const char* path) {
  if (n && std::fread(p, 1, n, f) != n) {
    set_error(std::string("checkpoint truncated: ") + path);
    throw Fail{LTM_ERR_INVALID_ARG};
  }
}

size_t pad16(size_t n) { return (16 - n % 16) % 16; }

// Makes `dev` current for a scope and restores the caller's device on every
// exit, the error paths included.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int dev) {
    LTM_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != dev) LTM_CUDA_TRY(cudaSetDevice(dev));
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

void save(ltm_block* b, const char* path, uint32_t kind) {
  LTM_REQUIRE(b && path, "NULL argument");
  ltm_block_config cfg;
  ltm_quant_config q;
  int tp = 1, tpr = 0, device = 0;
  bool loaded = false;
  block_identity(b, &cfg, &q, &tp, &tpr, &device, &loaded);
  const bool weights = kind == kKindBlock;
  LTM_REQUIRE(loaded, "block not loaded: nothing to save");
  DeviceScope on(device);
  LTM_CUDA_TRY(cudaDeviceSynchronize());  // the state of all work issued so far
  const std::vector<StateSection> secs = block_state(b, weights, true, false);
  FileHeader h;
  std::memset(&h, 0, sizeof(h));
  std::memcpy(h.magic, kMagic, sizeof(kMagic));
  h.version = kVersion;
  h.kind = kind;
  h.header_bytes = sizeof(FileHeader);
  h.n_sections = static_cast<uint32_t>(secs.size());
  h.cfg = cfg;
  h.quant = q;
  h.tp = tp;
  h.tpr = tpr;
  h.checksum = fnv1a(&h, offsetof(FileHeader, checksum));
  File out;
  out.f = std::fopen(path, "wb");
  if (!out.f) {
    set_error(std::string("cannot open checkpoint for writing: ") + path);
    throw Fail{LTM_ERR_INVALID_ARG};
  }
  write_all(out.f, &h, sizeof(h), path);
  std::vector<unsigned char> host;
  const unsigned char zeros[16] = {};
  for (const StateSection& s : secs) {
    LTM_REQUIRE(s.ptr != nullptr, "a state buffer is missing");
    host.resize(s.bytes);
    LTM_CUDA_TRY(cudaMemcpy(host.data(), s.ptr, s.bytes, cudaMemcpyDeviceToHost));
    SectionHeader sh;
    std::memset(&sh, 0, sizeof(sh));
    std::strncpy(sh.name, s.name.c_str(), sizeof(sh.name) - 1);
    sh.bytes = s.bytes;
    sh.checksum = fnv1a(host.data(), host.size());
    write_all(out.f, &sh, sizeof(sh), path);
    write_all(out.f, host.data(), host.size(), path);
    write_all(out.f, zeros, pad16(host.size()), path);
  }
  if (std::fflush(out.f) != 0) {
    set_error(std::string("checkpoint write failed: ") + path);
    throw Fail{LTM_ERR_INVALID_ARG};
  }
}

void load(ltm_block* b, const char* path, uint32_t kind) {
  LTM_REQUIRE(b && path, "NULL argument");
  ltm_block_config cfg;
  ltm_quant_config q;
  int tp = 1, tpr = 0, device = 0;
  bool loaded = false;
  block_identity(b, &cfg, &q, &tp, &tpr, &device, &loaded);
  File in;
  in.f = std::fopen(path, "rb");
  if (!in.f) {
    set_error(std::string("cannot open checkpoint: ") + path);
    throw Fail{LTM_ERR_INVALID_ARG};
  }
  FileHeader h;
  read_all(in.f, &h, sizeof(h), path);
  LTM_REQUIRE(std::memcmp(h.magic, kMagic, sizeof(kMagic)) == 0, "not a Titan-block checkpoint");
  LTM_REQUIRE(h.version == kVersion, "unsupported checkpoint format version");
  LTM_REQUIRE(h.header_bytes == sizeof(FileHeader), "checkpoint header size mismatch");
  LTM_REQUIRE(h.checksum == fnv1a(&h, offsetof(FileHeader, checksum)),
              "checkpoint header checksum mismatch");
  LTM_REQUIRE(h.kind == kind, kind == kKindBlock ? "the file holds a bank only, not a block"
                                                 : "the file holds a block, not a bank");
  const ltm_block_config& c = h.cfg;
  LTM_REQUIRE(c.hidden_dim == cfg.hidden_dim && c.ffn_dim == cfg.ffn_dim &&
                  c.num_heads == cfg.num_heads && c.head_dim == cfg.head_dim &&
                  c.memory_slots == cfg.memory_slots,
              "checkpoint dimensions differ from the block's");
  LTM_REQUIRE(h.quant.act_dtype == q.act_dtype, "checkpoint activation dtype differs");
  const bool weights = kind == kKindBlock;
  if (weights) {
    LTM_REQUIRE(c.use_bias == cfg.use_bias && c.use_layer_norm == cfg.use_layer_norm,
                "checkpoint bias / LayerNorm flags differ from the block's");
    LTM_REQUIRE(h.quant.scheme == q.scheme && h.quant.group_size == q.group_size,
                "checkpoint quantization scheme differs from the block's");
    LTM_REQUIRE(h.tp == tp && h.tpr == tpr,
                "checkpoint tensor-parallel size / rank differ from the block's");
  }
  DeviceScope on(device);
  const std::vector<StateSection> secs = block_state(b, weights, true, true);
  LTM_REQUIRE(h.n_sections == secs.size(), "checkpoint section count differs from the block's");
  // Two passes over the sections: the first checks every name, size and
  // checksum, the second copies; a damaged file fails before any of the
  // block's buffers is written, so the block keeps its previous state.
  const long first = std::ftell(in.f);
  LTM_REQUIRE(first >= 0, "checkpoint file is not seekable");
  std::vector<unsigned char> host;
  unsigned char pad[16];
  for (int pass = 0; pass < 2; ++pass) {
    LTM_REQUIRE(std::fseek(in.f, first, SEEK_SET) == 0, "checkpoint file is not seekable");
    for (const StateSection& s : secs) {
      SectionHeader sh;
      read_all(in.f, &sh, sizeof(sh), path);
      sh.name[sizeof(sh.name) - 1] = '\0';
      LTM_REQUIRE(s.name == sh.name, "checkpoint section order differs: expected " + s.name);
      LTM_REQUIRE(sh.bytes == s.bytes, "checkpoint section size differs: " + s.name);
      host.resize(s.bytes);
      read_all(in.f, host.data(), host.size(), path);
      read_all(in.f, pad, pad16(host.size()), path);
      LTM_REQUIRE(fnv1a(host.data(), host.size()) == sh.checksum,
                  "checkpoint section checksum mismatch: " + s.name);
      if (pass == 1) LTM_CUDA_TRY(cudaMemcpy(s.ptr, host.data(), s.bytes, cudaMemcpyHostToDevice));
    }
  }
  block_state_loaded(b, weights);
}

}  // namespace
}  // namespace ltm_b200

using namespace ltm_b200;

extern "C" ltm_status ltm_block_save(ltm_block* blk, const char* path) {
  return guarded([&] { save(blk, path, kKindBlock); });
}

extern "C" ltm_status ltm_block_load(ltm_block* blk, const char* path) {
  return guarded([&] { load(blk, path, kKindBlock); });
}

extern "C" ltm_status ltm_block_save_memory(ltm_block* blk, const char* path) {
  return guarded([&] { save(blk, path, kKindBank); });
}

extern "C" ltm_status ltm_block_load_memory(ltm_block* blk, const char* path) {
  return guarded([&] { load(blk, path, kKindBank); });
}
