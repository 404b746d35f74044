/*
 * tb_oracle.h -- CPU oracle of the quantized Titan-block forward ("TB-v1").
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain C++ restatement of the
 * reference's per-op formulas (Obsidian-Memory-Transformer; file:line
 * citations in tb_oracle.cpp), composed into the block semantics the B200
 * library implements.  It is the checker for the parity tests and the timed
 * CPU baseline of the bench; the product never links or calls it.
 *
 * Parity is unpinned by the reference itself: the reference ships no tests,
 * fixtures or golden vectors, and none of its sources compile, so this
 * restatement cannot be cross-checked against reference outputs.
 *
 * All activations are float arrays holding values representable in the
 * storage dtype (0 = f32, 1 = f16, 2 = bf16); outputs are rounded to that
 * dtype wherever the device path stores to memory.
 */
#ifndef TB_ORACLE_H
#define TB_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };
enum { ORC_ACT_NONE = 0, ORC_ACT_GELU = 1, ORC_ACT_SIGMOID = 2 };
enum { ORC_W8A32 = 0, ORC_W8A8 = 1, ORC_W4A16 = 2 };

int orc_num_threads(void);
void orc_set_num_threads(int n);

/* storage rounding of n floats in place */
void orc_round(float* x, int64_t n, int dtype);

/* INT8 symmetric per row (weights: per output channel; activations: per token) */
void orc_quant_int8_rows(const float* x, int64_t rows, int64_t K, int8_t* q, float* s);
void orc_dequant_int8_rows(const int8_t* q, const float* s, int64_t rows, int64_t K, int dtype,
                           float* out);
/* INT4 asymmetric, group 128, two nibbles per byte (low = even k) */
void orc_quant_int4_g128(const float* w, int64_t N, int64_t K, uint8_t* packed, float* s,
                         uint8_t* zp);
void orc_dequant_int4_g128(const uint8_t* packed, const float* s, const uint8_t* zp, int64_t N,
                           int64_t K, int dtype, float* out);

/* exact int32 accumulators of qa[M,K] . qw[N,K]^T */
void orc_gemm_i8(const int8_t* qa, const int8_t* qw, int64_t M, int64_t N, int64_t K, int32_t* acc);
/* fp32 results (before storage rounding) */
void orc_linear_w8a8(const int8_t* qa, const float* sa, const int8_t* qw, const float* sw,
                     const float* bias, int act, int64_t M, int64_t N, int64_t K, float* y);
void orc_linear_w8a32(const float* a, const int8_t* qw, const float* sw, const float* bias, int act,
                      int64_t M, int64_t N, int64_t K, float* y);
void orc_linear_w4a16(const float* a, const uint8_t* packed, const float* s, const uint8_t* zp,
                      const float* bias, int act, int64_t M, int64_t N, int64_t K, int wdtype,
                      float* y);

/* LN(x + x) over rows of H, eps 1e-5 */
void orc_layernorm_x2(const float* x, int64_t rows, int64_t H, const float* g, const float* b,
                      float* y);
/* RoPE table [S, dh/2] of (cos, sin) pairs */
void orc_rope_table(int S, int dh, float* tab);
/* attention over head-sliced rows: q row t of batch b at q + (b*Sq+t)*ldq + h*dh;
 * k,v rows at k + (b*kv_bstride_rows + j)*ldk; causal when causal != 0;
 * out [B*Sq, nh*dh] rounded to dtype */
void orc_attention(const float* q, int64_t ldq, const float* k, const float* v, int64_t ldk,
                   int B, int Sq, int Skv, int kv_batch_stride_rows, int nh, int dh, int causal,
                   int dtype, float* out, int64_t ldo);

/* memory-bank store: slot weights from the mean query row against the keys
 * (use_scores) or update_rate; memory[s,:] = (1-w_s) memory[s,:] + w_s state,
 * rounded to dtype.  keys rows of stride ldk, queries [T, ldq], state [H]. */
// calibrators: data range (MinMax), the reference's percentile order
// statistics, the least-squared-error symmetric INT8 clipping of 100 trials
void orc_calib_minmax(const float* x, int64_t n, float* mn, float* mx);
void orc_calib_percentile(const float* x, int64_t n, float p, float* lo, float* hi);
double orc_calib_mse_error(const float* x, int64_t n, float clip);
void orc_calib_mse(const float* x, int64_t n, float* lo, float* hi);
// static per-tensor INT8 with a given scale
void orc_quant_int8_static(const float* x, int64_t n, float scale, int8_t* q);
// y = act(x) elementwise (ORC_ACT_GELU: tanh form; ORC_ACT_SIGMOID)
void orc_activation(const float* x, int64_t n, int act, float* y);
// rows[s, :] = (1 - w[s]) rows[s, :] + w[s] v, rounded to dtype (rows [Ms, n])
void orc_ema_rows(float* rows, int Ms, int64_t n, const float* v, const float* w, int dtype);
void orc_memory_store(float* memory, const float* keys, int64_t ldk, const float* queries,
                      int64_t ldq, int64_t T, const float* state, int Ms, int H, int nh,
                      float rate, int use_scores, int dtype);

typedef struct orc_block_cfg {
  int H, F, nh, dh, Ms;
  int scheme;    /* ORC_W8A32 / ORC_W8A8 / ORC_W4A16 */
  int dtype;     /* activation storage dtype */
  int use_rotary, use_bias, use_layer_norm, use_memory_gating;
  int memory_write, use_attention_scores;
  float update_rate;
} orc_block_cfg;

/* same field order as ltm_block_weights */
typedef struct orc_block_weights {
  const float *w_qkv, *b_qkv, *w_o, *b_o, *w_qm, *b_qm, *w_km, *b_km, *w_vm, *b_vm, *w_om, *b_om,
      *w_g, *b_g, *w_1, *b_1, *w_2, *b_2, *ln1_g, *ln1_b, *ln2_g, *ln2_b;
  const float* memory;
} orc_block_weights;

/* One block forward.  x, y: [B*S, H].  memory_inout: [Ms, H] bank in the
 * storage dtype, initialised by the caller from weights->memory and updated
 * in place when memory_write != 0.  Returns 0 on success. */
int orc_block_forward(const orc_block_cfg* c, const orc_block_weights* w, float* memory_inout,
                      const float* x, float* y, int B, int S);

/* orc_block_forward that also writes the post-RoPE K | V rows of every token
 * ([B*S, 2H], rounded) into kv_out when it is not NULL. */
int orc_block_forward_kv(const orc_block_cfg* c, const orc_block_weights* w, float* memory_inout,
                         const float* x, float* y, int B, int S, float* kv_out);

/* K_M | V_M of a bank: [Ms, 2H], rounded. */
int orc_block_kvm(const orc_block_cfg* c, const orc_block_weights* w, const float* memory,
                  float* kvm_out);

/* One decode step: x, y [B, H] (one new token per sequence, all at position
 * cache_len); k_cache, v_cache [B, nh, max_positions, dh] (head-major) hold
 * positions [0, cache_len) and receive the new token's K, V at cache_len; kvm_inout
 * [Ms, 2H] is the resident K_M | V_M.  With memory_write the bank and K_M |
 * V_M follow the same EMA (K_M | V_M towards c [Wkm;Wvm]^T + b). */
int orc_block_decode_step(const orc_block_cfg* c, const orc_block_weights* w, float* memory_inout,
                          float* kvm_inout, const float* x, float* k_cache, float* v_cache,
                          int64_t max_positions, int cache_len, int B, float* y);

/* The block's quantized linears made once (orc_block_prepare) for repeated
 * decode steps (the same step as orc_block_decode_step; w still supplies the
 * LayerNorm parameters). */
void* orc_block_prepare(const orc_block_cfg* c, const orc_block_weights* w);
void orc_block_release(void* prepared);
int orc_block_decode_step_prepared(const void* prepared, const orc_block_cfg* c,
                                   const orc_block_weights* w, float* memory_inout,
                                   float* kvm_inout, const float* x, float* k_cache,
                                   float* v_cache, int64_t max_positions, int cache_len, int B,
                                   float* y);

/* Embedding gather + n_layers blocks (weights[l], banks[l]).  tokens [B*S]. */
// Forward with a prepared block; kvm_in ([Ms, 2H] K_M | V_M of the bank) is
// used as given when not NULL (else made from the bank).
int orc_block_forward_prepared(const void* prepared, const orc_block_cfg* c,
                               const orc_block_weights* w, float* memory_inout,
                               const float* kvm_in, const float* x, float* y, int B, int S);
int orc_block_kvm_prepared(const void* prepared, const orc_block_cfg* c, const float* memory,
                           float* kvm_out);
int orc_model_forward(const orc_block_cfg* c, const orc_block_weights* w, float** banks,
                      int n_layers, const float* embedding, int vocab, const int32_t* tokens,
                      float* y, int B, int S);

#ifdef __cplusplus
}
#endif
#endif
