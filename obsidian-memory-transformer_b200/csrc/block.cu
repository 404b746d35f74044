// block.cu -- Titan block / model orchestration over the kernels (C ABI).
#include "common.cuh"

using namespace ltm_b200;

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

#define LTM_PENDING(name, ...)                                                 \
  extern "C" ltm_status name(__VA_ARGS__) {                                    \
    return guarded([&] { LTM_UNSUPPORTED(#name " is not built yet"); });       \
  }

LTM_PENDING(ltm_linear_w4a16, const void*, ltm_dtype, const uint8_t*, const float*, const uint8_t*,
            const float*, ltm_epilogue, void*, int64_t, int64_t, int64_t, void*)
LTM_PENDING(ltm_linear_w8a32, const float*, const int8_t*, const float*, const float*, ltm_epilogue,
            float*, int64_t, int64_t, int64_t, void*)
LTM_PENDING(ltm_block_create, const ltm_block_config*, const ltm_quant_config*, int, ltm_block**)
LTM_PENDING(ltm_block_load_weights, ltm_block*, const ltm_block_weights*)
LTM_PENDING(ltm_block_forward, ltm_block*, const void*, void*, const void*, int, int, void*)
LTM_PENDING(ltm_block_get_memory, ltm_block*, void*, void*)
LTM_PENDING(ltm_block_destroy, ltm_block*)
LTM_PENDING(ltm_model_create, const ltm_block_config*, const ltm_quant_config*, int, int, int,
            ltm_model**)
LTM_PENDING(ltm_model_load_embedding, ltm_model*, const float*)
LTM_PENDING(ltm_model_load_layer, ltm_model*, int, const ltm_block_weights*)
LTM_PENDING(ltm_model_forward, ltm_model*, const int32_t*, void*, int, int, void*)
LTM_PENDING(ltm_model_destroy, ltm_model*)
