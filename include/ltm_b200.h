/*
 * ltm_b200.h -- C ABI of the B200-native quantized Titan-block forward.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, returns an
 * ltm_status and never throws.  Device pointers are CUDA global-memory
 * pointers on the current device; `stream` is a cudaStream_t passed as void*
 * (NULL = legacy default stream).  All launches are asynchronous on `stream`.
 * On error, ltm_last_error_string() describes the failure of the calling
 * thread's last call.
 *
 * The reference interfaces each group replaces (paths inside the
 * Obsidian-Memory-Transformer project) are cited beside the declarations,
 * with the formula each one computes.
 */
#ifndef LTM_B200_H
#define LTM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LTM_API __attribute__((visibility("default")))
#else
#define LTM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status -- */
/* Replaces CUDA_CHECK -> std::runtime_error (include/core/utils/cuda_utils.cuh:19-45):
 * no exception crosses the ABI; the C++ wrapper rethrows. */
typedef enum ltm_status {
  LTM_OK = 0,
  LTM_ERR_INVALID_ARG = 1,
  LTM_ERR_CUDA = 2,
  LTM_ERR_COMM = 3,
  LTM_ERR_TIMEOUT = 4,   /* a bounded in-kernel wait expired (device error word) */
  LTM_ERR_UNSUPPORTED = 5,
  LTM_ERR_NO_DEVICE = 6
} ltm_status;

typedef enum ltm_dtype {
  LTM_DTYPE_F32 = 0,
  LTM_DTYPE_F16 = 1,
  LTM_DTYPE_BF16 = 2
} ltm_dtype;

/* Activation fused into a linear's epilogue. GELU is the tanh form of
 * src/core/ops/fused_ops.cu:136-142; SIGMOID is 1/(1+exp(-x)). */
typedef enum ltm_epilogue {
  LTM_EPI_NONE = 0,
  LTM_EPI_GELU = 1,
  LTM_EPI_SIGMOID = 2
} ltm_epilogue;

/* Weight/activation quantization scheme of a block (extension of
 * QuantizationConfig, include/core/quantization/quantizer.cuh:24-52). */
typedef enum ltm_scheme {
  LTM_SCHEME_W8A32 = 0, /* int8 per-output-channel weights, fp32 activations   */
  LTM_SCHEME_W8A8 = 1,  /* int8 weights, per-token dynamic int8 activations     */
  LTM_SCHEME_W4A16 = 2  /* int4 group-128 asymmetric weights, 16-bit activations */
} ltm_scheme;

LTM_API const char* ltm_version(void);
/* Message of the calling thread's last failed call ("" if none). */
LTM_API const char* ltm_last_error_string(void);
/* Reads and clears the device error word set by bounded in-kernel waits on
 * the current device (0 = none; otherwise the code of the wait that expired). */
LTM_API ltm_status ltm_device_error(int* code_out);

/* Number of kernels this library has launched in this process (all devices). */
LTM_API ltm_status ltm_launch_count(uint64_t* count_out);

/* Number of device allocations (cudaMalloc) the library has made in this
 * process (all devices): workspaces, weights, banks, scratch. */
LTM_API ltm_status ltm_device_alloc_count(uint64_t* count_out);

/* In-library kernel timer.  Between begin and end, every kernel the library
 * launches on `stream` is followed by a CUDA event; end synchronizes the
 * stream and writes one line per kernel name, "name launches total_ms\n", in
 * first-launch order (a kernel's time is measured from the previous mark, so
 * launches on the stream should run back to back). */
LTM_API ltm_status ltm_kernel_timer_begin(void* stream);
LTM_API ltm_status ltm_kernel_timer_end(char* report, size_t capacity);

/* ---------------------------------------------------------- quantization -- */
/* Replaces Quantizer<T>::quantize with per_channel=true, symmetric=true,
 * channel_axis=0 (include/core/quantization/quantizer.cuh:183,
 * src/core/quantization/quantizer.cu:263-310):
 *   s[n] = max_k |w[n,k]| / 127 ;  q[n,k] = clamp(round_half_away(w/s[n]), -127, 127)
 *   (s[n] == 0  =>  q[n,:] = 0).  Scales live on the device.
 * w: [N,K] row-major in w_dtype; q: int8 [N,K]; s: fp32 [N]. */
LTM_API ltm_status ltm_quantize_int8_per_channel(const void* w, ltm_dtype w_dtype, int64_t N, int64_t K,
                                         int8_t* q, float* s, void* stream);

/* Replaces Quantizer<T>::dequantize, per-channel symmetric
 * (src/core/quantization/quantizer.cu:144-161,312-328):  out[n,k] = q[n,k] * s[n]. */
LTM_API ltm_status ltm_dequantize_int8_per_channel(const int8_t* q, const float* s, int64_t N, int64_t K,
                                           void* out, ltm_dtype out_dtype, void* stream);

/* Per-token dynamic activation quantization (same formula as the per-channel
 * weight quantizer, rows = tokens): a: [M,K] in a_dtype -> q int8 [M,K], s fp32 [M].
 * New entry point; the reference declares dynamic ranges only
 * (include/core/quantization/quantizer.cuh:38-39,191). */
LTM_API ltm_status ltm_quantize_act_int8_per_token(const void* a, ltm_dtype a_dtype, int64_t M, int64_t K,
                                           int8_t* q, float* s, void* stream);

/* INT4 asymmetric group quantization + packing; implements
 * QuantizationPrecision::INT4 (include/core/quantization/quantizer.cuh:12),
 * following the asymmetric form of src/core/quantization/quantizer.cu:291-293
 * for unsigned nibbles.  Per (row n, group g of `group_size` consecutive k):
 *   mn = min(0, min w), mx = max(0, max w), s = (mx - mn) / 15,
 *   zp = clamp(round_half_away(-mn / s), 0, 15),
 *   q  = clamp(round_half_away(w / s + zp), 0, 15)      (s == 0 => q = zp = 0)
 *   packed[n, k/2] = q[n,2j] | q[n,2j+1] << 4            (low nibble = even k)
 * w: [N,K]; packed: uint8 [N,K/2]; s: fp32 [N,K/group]; zp: uint8 [N,K/group].
 * group_size must be 128 and divide K. */
LTM_API ltm_status ltm_quantize_int4_grouped(const void* w, ltm_dtype w_dtype, int64_t N, int64_t K,
                                     int group_size, uint8_t* packed, float* s, uint8_t* zp,
                                     void* stream);

/* out[n,k] = (q[n,k] - zp[n,g]) * s[n,g], g = k / group_size. */
LTM_API ltm_status ltm_dequantize_int4_grouped(const uint8_t* packed, const float* s, const uint8_t* zp,
                                       int64_t N, int64_t K, int group_size, void* out,
                                       ltm_dtype out_dtype, void* stream);

/* ----------------------------------------------------------- calibration -- */
/* Activation-range calibrators for static INT8 scales: QuantizationCalibrator
 * and its MinMax / Percentile / MSE subclasses
 * (include/core/quantization/quantizer.cuh:124-175,
 * src/core/quantization/calibrator.cu:61-264), on the device.
 *   MINMAX      min and max of everything collected;
 *   PERCENTILE  the sorted values at lo = (size_t)((100 - p) * n / 100) and
 *               hi = (size_t)(p * n / 100) (fp32 arithmetic, hi <= n - 1),
 *               exact (radix select, no sort);
 *   MSE         [-c a, c a] for the c in {1/100, ..., 100/100} (a = max |x|)
 *               whose symmetric INT8 quantize-dequantize has the least
 *               squared error over the collected values (first minimum).
 * compute_range writes host floats (it synchronizes the stream); with nothing
 * collected it gives [0, 0].  A static symmetric scale is then
 * max(|min|, |max|) / 127. */
typedef enum ltm_calibration {
  LTM_CALIB_MINMAX = 0,
  LTM_CALIB_PERCENTILE = 1,
  LTM_CALIB_MSE = 2
} ltm_calibration;
typedef struct ltm_calibrator ltm_calibrator;
LTM_API ltm_status ltm_calibrator_create(int method, float percentile, int device,
                                         ltm_calibrator** out);
LTM_API ltm_status ltm_calibrator_collect(ltm_calibrator* c, const void* data, ltm_dtype dtype,
                                          int64_t n, void* stream);
LTM_API ltm_status ltm_calibrator_compute_range(ltm_calibrator* c, float* min_val,
                                                float* max_val, void* stream);
LTM_API ltm_status ltm_calibrator_reset(ltm_calibrator* c);
LTM_API ltm_status ltm_calibrator_destroy(ltm_calibrator* c);
/* Static per-tensor INT8 with a calibrated scale (symmetricQuantizeKernel,
 * src/core/quantization/quantizer.cu:93-105, plus the clamp):
 *   q = clamp(round_half_away(x / scale), -127, 127), IEEE division;
 *   scale == 0 => q = 0. */
LTM_API ltm_status ltm_quantize_int8_static(const void* x, ltm_dtype dtype, int64_t n, float scale,
                                            int8_t* q, void* stream);

/* --------------------------------------------------------------- linears -- */
/* Quantized replacements of ops::matmul + bias add (src/core/ops/mma_ops.cu:59-92,
 * src/core/ops/fused_ops.cu:187-210) and of the per-token FFN kernel
 * (src/core/transformer/titan_inspired_block.cu:39-98).  Weights are [N,K]
 * row-major (out x in), matching the reference kernels' indexing.
 *
 * W8A8:  acc[m,n] = sum_k qa[m,k]*qw[n,k] (exact int32);
 *        y[m,n]   = act(acc * sa[m] * sw[n] + bias[n])  stored as y_dtype.
 *        sa may be NULL (= 1); bias may be NULL (= 0).  Requires K % 16 == 0,
 *        N % 32 == 0.  tcgen05 kind::i8 tensor-core GEMM on sm_100a. */
LTM_API ltm_status ltm_linear_w8a8(const int8_t* qa, const float* sa, const int8_t* qw, const float* sw,
                           const float* bias, ltm_epilogue act, void* y, ltm_dtype y_dtype,
                           int64_t M, int64_t N, int64_t K, void* stream);

/* Exactness probe of the W8A8 GEMM: writes the raw int32 accumulators. */
LTM_API ltm_status ltm_linear_w8a8_acc_i32(const int8_t* qa, const int8_t* qw, int32_t* acc, int64_t M,
                                   int64_t N, int64_t K, void* stream);

/* W4A16: y = act(a @ dequant(W)^T + bias), a: [M,K] f16/bf16; the weight is
 * dequantized to a_dtype (as Quantizer::dequantize writes T) and contracted
 * on tcgen05 kind::f16 with fp32 accumulation; y stored as a_dtype.
 * Requires K % 128 == 0 (group 128), N % 32 == 0.  This entry point
 * dequantises weight tiles in shared memory at every M (K split over a
 * thread-block cluster when the tile grid is small) and allocates nothing;
 * a W4A16 Titan block at M >= 1024 tokens instead dequantises each weight once
 * into its own workspace and runs the persistent 16-bit GEMM. */
LTM_API ltm_status ltm_linear_w4a16(const void* a, ltm_dtype a_dtype, const uint8_t* packed,
                            const float* s, const uint8_t* zp, const float* bias,
                            ltm_epilogue act, void* y, int64_t M, int64_t N, int64_t K,
                            void* stream);

/* W8A32: y = act((a @ qw^T) * sw[n] + bias[n]) with fp32 a and y (the fp32
 * TitanBlock<float> path with int8 per-channel weights). */
LTM_API ltm_status ltm_linear_w8a32(const float* a, const int8_t* qw, const float* sw, const float* bias,
                            ltm_epilogue act, float* y, int64_t M, int64_t N, int64_t K,
                            void* stream);

/* ------------------------------------------------------------------- ops -- */
/* y = LN(x + r) * gamma + beta over rows of H, eps 1e-5, two-pass mean /
 * variance; replaces ops::layerNormResidual (src/core/ops/fused_ops.cu:15-86,
 * 233-259).  TitanBlock::layerNorm passes r = x
 * (src/core/transformer/titan_inspired_block.cu:374-389).  gamma, beta: fp32 [H]. */
LTM_API ltm_status ltm_layernorm_residual(const void* x, const void* r, const float* gamma,
                                          const float* beta, void* y, ltm_dtype dtype,
                                          int64_t rows, int64_t H, void* stream);

/* o = softmax(q k^T / sqrt(head_dim)) v per head, fp32 softmax and accumulation;
 * the attention core of FlashAttention<T>::forward
 * (src/core/attention/flash_attention.cu:188-268,380-445; TB-v1 adds the max
 * subtraction and the causal mask) and of MemoryAttention<T>::forward
 * (src/core/attention/memory_attention.cu:38-88,416-510: queries x memory slots).
 * Rows are head-sliced: query t of batch b, head h is q[(b*Sq + t)*ldq + h*head_dim ..];
 * key j is k[(b*kv_batch_rows + j)*ldk + h*head_dim ..] (kv_batch_rows = 0 shares
 * K/V across the batch, as the memory bank does); same for v / ldv and o / ldo.
 * causal: key j is visible to query t iff j <= t + (Skv - Sq).  head_dim 64 or 128. */
LTM_API ltm_status ltm_attention_forward(const void* q, int64_t ldq, const void* k, int64_t ldk,
                                         const void* v, int64_t ldv, void* o, int64_t ldo, int B,
                                         int Sq, int Skv, int64_t kv_batch_rows, int num_heads,
                                         int head_dim, int causal, ltm_dtype dtype, void* stream);

/* Memory-bank write: MemoryBank<T>::store (src/core/ltm/memory_bank.cu:39-68,
 * 242-274: every slot blends towards the stored state with weight
 * update_rate * score[slot]) with the slot scores of the TB-v1 write:
 *   qbar     = mean over the T rows of `queries`            (memory queries Q_m)
 *   score[s] = mean over heads h of softmax_s(qbar_h . keys[s]_h / sqrt(head_dim))
 *   w_s      = update_rate * score[s]   (update_rate alone when use_attention_scores = 0)
 *   memory[s,:] = (1 - w_s) * memory[s,:] + w_s * state
 * memory: [memory_slots, hidden_dim] in dtype, updated in place; keys: rows of
 * stride ldk (the bank's memory keys K_M); queries: [T, ldq]; state: fp32
 * [hidden_dim] (the pooled gated input mean_t g_t * x_t).  The query column
 * sums and slot weights live in library-owned device scratch, allocated on the
 * first call per device and grown on demand.  memory_slots <= 51200. */
LTM_API ltm_status ltm_memory_store(void* memory, const void* keys, int64_t ldk,
                                    const void* queries, int64_t ldq, int64_t T,
                                    const float* state, int memory_slots, int hidden_dim,
                                    int num_heads, float update_rate, int use_attention_scores,
                                    ltm_dtype dtype, void* stream);

/* Allocation-free variant of ltm_memory_store (same arguments, same result).
 * It has no counterpart in the reference.  It is for callers that cannot let
 * a library allocate device memory at call time -- a framework that plans all
 * device memory itself, a server whose device footprint must stay fixed after
 * start-up, a latency-critical loop where cudaMalloc would stall the device.
 * Its scratch is one fixed 256 KiB device array per GPU that loads the library
 * (held until exit), so with use_attention_scores != 0, hidden_dim rounded up
 * to 64 plus memory_slots must not exceed 65536 (else LTM_ERR_INVALID_ARG);
 * rate-only calls (use_attention_scores == 0) use no scratch and have no such
 * limit.  All calls share that array and clear it at their start: calls whose
 * GPU work overlaps (other streams or unordered host threads) race.  The first
 * call on a device looks up the array's device address in the device's
 * primary context and caches it; make it before any stream capture, and do
 * not call this entry point again after cudaDeviceReset in the same process
 * (the cached address is then stale). */
LTM_API ltm_status ltm_memory_store_noalloc(void* memory, const void* keys, int64_t ldk,
                                            const void* queries, int64_t ldq, int64_t T,
                                            const float* state, int memory_slots,
                                            int hidden_dim, int num_heads, float update_rate,
                                            int use_attention_scores, ltm_dtype dtype,
                                            void* stream);

/* ----------------------------------------------------------------- block -- */
/* Field-for-field mirror of ltm::transformer::TitanBlockConfig
 * (include/core/transformer/titan_inspired_block.cuh:19-50): same names, same
 * order, same defaults (ltm_block_config_default).  bools are int (0/1). */
typedef struct ltm_block_config {
  int hidden_dim;
  int ffn_dim;
  int num_heads;
  int head_dim;
  int memory_slots;
  int memory_dim;
  float memory_update_rate;
  int use_memory_compression;
  float memory_compression_ratio;
  int use_flash_attention;
  int use_alibi;
  int use_rotary;
  float dropout_prob;
  int use_parallel_attention;
  int use_memory_gating;
  int use_layer_norm;
  int use_bias;
  int fuse_operations;
  int learn_memory;
  int learn_compression;
  int gradient_checkpointing;
} ltm_block_config;

/* Quantization extension of the block (kept separate so the field layout of
 * ltm_block_config stays that of TitanBlockConfig). */
typedef struct ltm_quant_config {
  ltm_scheme scheme;
  int group_size;           /* INT4 group (128) */
  ltm_dtype act_dtype;      /* F32 for W8A32; F16 or BF16 otherwise */
  int memory_write;         /* 1: write the bank after the read (TB-v1 write) */
  int use_attention_scores; /* 1: slot weights from the mean memory query */
} ltm_quant_config;

/* Host fp32 master weights of one block, all row-major [out, in].  Biases may
 * be NULL when use_bias == 0.  `memory` is the bank [memory_slots, hidden_dim]. */
typedef struct ltm_block_weights {
  const float *w_qkv, *b_qkv;   /* [3H,H], [3H]: rows Q | K | V, head h at rows h*dh.. */
  const float *w_o, *b_o;       /* [H,H] */
  const float *w_qm, *b_qm;     /* memory-attention query  [H,H] */
  const float *w_km, *b_km;     /* memory-attention key    [H,H] (applied to the bank) */
  const float *w_vm, *b_vm;     /* memory-attention value  [H,H] (applied to the bank) */
  const float *w_om, *b_om;     /* memory-attention output [H,H] */
  const float *w_g, *b_g;       /* compression gate        [H,H] */
  const float *w_1, *b_1;       /* FFN up   [F,H] */
  const float *w_2, *b_2;       /* FFN down [H,F] */
  const float *ln1_g, *ln1_b;   /* [H] */
  const float *ln2_g, *ln2_b;   /* [H] */
  const float* memory;          /* [Ms,H] */
} ltm_block_weights;

typedef struct ltm_block ltm_block;

LTM_API void ltm_block_config_default(ltm_block_config* cfg);

/* Replaces `explicit TitanBlock(const TitanBlockConfig&)` + initialize()
 * (titan_inspired_block.cuh:69,76).  Weights are supplied by
 * ltm_block_load_weights instead of curand init. */
LTM_API ltm_status ltm_block_create(const ltm_block_config* cfg, const ltm_quant_config* qcfg, int device,
                            ltm_block** out);
/* Quantizes and uploads the host fp32 master weights (synchronous). */
LTM_API ltm_status ltm_block_load_weights(ltm_block* blk, const ltm_block_weights* w);

/* Replaces TitanBlock<T>::forward (titan_inspired_block.cuh:86-91,
 * titan_inspired_block.cu:254-345) with the TB-v1 semantics.  x, y: device
 * [B,S,H] in act_dtype (x and y must not alias).  attention_mask must be NULL
 * (self-attention is causal; an explicit mask returns LTM_ERR_UNSUPPORTED).
 * Workspace grows on the first call at a new B*S and is reused afterwards. */
LTM_API ltm_status ltm_block_forward(ltm_block* blk, const void* x, void* y, const void* attention_mask,
                             int B, int S, void* stream);

/* One batched decode step against a KV cache.  No callable counterpart in the
 * reference: it replaces the KV-cache stubs CacheManagerImpl::allocate /
 * update / get (python_bindings/src/main.cpp:101-135) and CacheManager
 * (python_bindings/ltm/inference.py:101-128) with the TB-v1 block applied to
 * one new token per sequence:
 *   x, y     device [B, H] in act_dtype (f16 / bf16; distinct buffers);
 *   k_cache, v_cache  device [B, heads, max_positions, head_dim] in
 *            act_dtype (head-major; heads = num_heads, or this rank's
 *            num_heads / n under tensor parallelism), 16-byte aligned;
 *            positions [0, cache_len) hold the post-RoPE keys and the values
 *            of the tokens before; the step writes the new token's K and V at
 *            position cache_len of every head of every sequence;
 *   the new token's RoPE position is cache_len; its self-attention reads the
 *   cache_len + 1 positions [0, cache_len];
 *   the memory attention reads K_M | V_M, which the block keeps resident
 *   between decode steps (computed from the bank on the first step after
 *   load_weights or after a forward that wrote the bank);
 *   with memory_write the bank is written after the read (state = mean over
 *   the batch of g * x) and K_M | V_M follow the same EMA towards
 *   state [Wkm;Wvm]^T + b.
 * 0 <= cache_len < max_positions.  Workspace grows on the first call at a new
 * B or max_positions; the RoPE table grows in steps of 4096 positions. */
LTM_API ltm_status ltm_block_decode_step(ltm_block* blk, const void* x, void* y, void* k_cache,
                                         void* v_cache, int64_t max_positions, int cache_len, int B,
                                         void* stream);

/* The decode step with a cache length per sequence (the continuous-batching
 * form of the CacheManager stubs, python_bindings/src/main.cpp:101-135):
 * cache_lens is a device int32 [B]; sequence b's new token sits at position
 * cache_lens[b], is written there and attends positions [0, cache_lens[b]].
 * The launches depend only on B and max_positions, not on the lengths, so
 * one step can be captured in a CUDA graph once (after a first, uncaptured
 * call has sized the workspace) and replayed while the lengths move on the
 * device.  A length outside [0, max_positions) skips that sequence's cache
 * write and attention (its attention output is 0) and sets the device error
 * word (ltm_device_error: 5). */
LTM_API ltm_status ltm_block_decode_step_ragged(ltm_block* blk, const void* x, void* y,
                                                void* k_cache, void* v_cache,
                                                int64_t max_positions, const int32_t* cache_lens,
                                                int B, void* stream);

/* Prefill that also fills the decode KV caches: ltm_block_forward plus the
 * post-RoPE K and V of positions [0, S) of every sequence written to the
 * head-major caches [B, heads, max_positions, head_dim] (this rank's heads
 * under tensor parallelism), so decode steps can follow at cache_len = S. */
LTM_API ltm_status ltm_block_forward_with_cache(ltm_block* blk, const void* x, void* y, int B,
                                                int S, void* k_cache, void* v_cache,
                                                int64_t max_positions, void* stream);

/* Memory write of the block's own bank: MemoryBank<T>::store
 * (src/core/ltm/memory_bank.cu:242-274) with a caller-given state (fp32 [H],
 * device) and, with use_attention_scores, slot weights from the mean of the T
 * memory-query rows `queries` (device, act_dtype, row stride ldq; this rank's
 * heads' columns under tensor parallelism) against the block's K_M.  The
 * resident K_M | V_M of the decode step follow the same EMA. */
LTM_API ltm_status ltm_block_memory_write(ltm_block* blk, const float* state, const void* queries,
                                          int64_t ldq, int64_t T, void* stream);

/* Copies the memory bank [Ms,H] (act_dtype) to a device buffer
 * (getMemoryBank(), titan_inspired_block.cuh:133). */
LTM_API ltm_status ltm_block_get_memory(ltm_block* blk, void* out, void* stream);

/* Stage-by-stage inspection (no counterpart in the reference, whose block
 * keeps its intermediates private): the shape of one intermediate of the last
 * forward / decode step on this handle and, when out is not NULL, a copy of it
 * into out (device memory, rows x cols packed, on stream).  kind: 0 =
 * activation in act_dtype, 1 = int8 codes, 2 = fp32 per-row scales
 * ([rows, 1]).  Names: "qkvm" [T, 4H] (post-RoPE
 * Q|K|V|Qm), "kvm" [Ms, 2H] (K_M|V_M), "attn_self", "attn_mem" [T, H], "s",
 * "m" [T, H] (output projections), "y" [T, H] (gated integration),
 * "ffn_hidden" [T, F] (GELU output); W8A8 adds the per-token int8 codes and
 * scales "ln1_q"/"ln1_s", "x_q"/"x_s", "attn_self_q"/"_s", "attn_mem_q"/"_s",
 * "ln2_q"/"ln2_s", "ffn_hidden_q"/"_s"; the other schemes "ln1", "ln2".
 * Under tensor parallelism H and F are this rank's widths (s, m: full H). */
LTM_API ltm_status ltm_block_intermediate(ltm_block* blk, const char* name, void* out,
                                          void* stream, int64_t* rows, int64_t* cols, int* kind);
/* Quantized checkpoints: TitanBlock<T>::save / load
 * (include/core/transformer/titan_inspired_block.cuh:147-154) and
 * MemoryBank<T>::save / load (include/core/ltm/memory_bank.cuh:152-159),
 * declared but never defined in the reference.  A versioned little-endian
 * file: a header (magic "LTMB200", format version, kind, the writer's block
 * and quantization configs, tensor-parallel size / rank, FNV-1a 64 header
 * checksum) and one checksummed section per device buffer -- the quantized
 * codes, scales, zero-points and biases of every linear, the LayerNorm
 * parameters and the bank.  load restores the exact codes (no requantizing)
 * into a block created with the same dimensions, scheme, dtype and
 * tensor-parallel rank (LTM_ERR_INVALID_ARG otherwise, or on a checksum
 * mismatch); after it the block is ready without ltm_block_load_weights.
 * The *_memory pair saves / loads the bank [Ms, H] alone. */
LTM_API ltm_status ltm_block_save(ltm_block* blk, const char* path);
LTM_API ltm_status ltm_block_load(ltm_block* blk, const char* path);
LTM_API ltm_status ltm_block_save_memory(ltm_block* blk, const char* path);
LTM_API ltm_status ltm_block_load_memory(ltm_block* blk, const char* path);
LTM_API ltm_status ltm_block_destroy(ltm_block* blk);

/* ------------------------------------------------------ tensor parallel -- */
/* No counterpart in the reference (single GPU only).  A communicator of
 * nranks GPUs (NCCL, loaded at run time from libnccl.so.2) for the
 * tensor-parallel block: rank 0 creates a 128-byte unique id, the caller
 * distributes it to every rank over its own channel, each rank creates its
 * communicator on its device. */
typedef struct ltm_comm ltm_comm;
#define LTM_COMM_ID_BYTES 128
LTM_API ltm_status ltm_comm_unique_id(void* id_out /* LTM_COMM_ID_BYTES */);
LTM_API ltm_status ltm_comm_create(const void* id, int nranks, int rank, int device, ltm_comm** out);
/* In-place allowed (send == recv); op_max != 0: maximum, else sum. */
LTM_API ltm_status ltm_comm_allreduce(ltm_comm* comm, const void* send, void* recv, size_t count,
                              ltm_dtype dtype, int op_max, void* stream);
LTM_API ltm_status ltm_comm_destroy(ltm_comm* comm);

/* Tensor-parallel block on the communicator's device (rank r of n): Q/K/V/
 * Q_m, K_M/V_M and W1 are split by heads / FFN columns, W_o, W_om and W2 by
 * their input columns (partial sums joined by one allreduce each), the gate
 * and LayerNorms are replicated, the bank is replicated and updated
 * identically on every rank.  ltm_block_load_weights takes the FULL host
 * weights on every rank and keeps this rank's shard; per-channel weight
 * scales and per-token activation scales are those of the unsplit matrices
 * (global row maxima), so the int8 codes equal the single-GPU block's.
 * ltm_block_forward's x and y are the full [B,S,H] on every rank.  Needs
 * num_heads and ffn_dim divisible by n.  The communicator must outlive the
 * block. */
LTM_API ltm_status ltm_block_create_tp(const ltm_block_config* cfg, const ltm_quant_config* qcfg,
                               ltm_comm* comm, ltm_block** out);
/* Sequence-parallel forward of a tensor-parallel block (f16 / bf16): x_local
 * and y_local are this rank's B*S / nranks consecutive rows [T / nranks, H]
 * of the [B*S, H] activations (B*S a multiple of nranks).  The LayerNorms,
 * the gate and the gated integration run on the local rows; the LayerNorm
 * outputs (int8 codes + scales for W8A8) are all-gathered for the
 * column-parallel projections and the row-parallel partial sums are
 * reduce-scattered to the rows' owners, so no rank repeats another's row
 * work.  Consecutive layers chain y_local -> x_local with no gather. */
LTM_API ltm_status ltm_block_forward_sp(ltm_block* blk, const void* x_local, void* y_local, int B,
                                        int S, void* stream);
/* Overlap of ltm_block_forward_sp (W8A8): the all-gathers run as one
 * broadcast per root rank and the row-block exchanges as one gather per root
 * rank on a stream of the block's own, each overlapping the GEMM of another
 * rank's rows, whose grids leave comm_sms SMs (default 16) to the
 * collectives.  overlap = 1: on; 0 or -1 (default): the plain collectives on
 * the caller's stream (measured faster at 2 and 8 ranks). */
LTM_API ltm_status ltm_block_set_overlap(ltm_block* blk, int overlap, int comm_sms);
/* Row-parallel reductions of ltm_block_forward_sp.  LTM_TP_REDUCE_ACT
 * (default): the ranks' partial sums in the activation type, reduce-scattered
 * by NCCL (16-bit adds along the way).  LTM_TP_REDUCE_EXACT (W8A8 only): the
 * int32 GEMM accumulators are exchanged and summed exactly and the unsplit
 * GEMM's epilogue (scales, bias, residual) is applied at the owner, so
 * forward_sp's rows equal the single-GPU block's bit for bit (the memory-bank
 * update aside, whose column sums are accumulated in no fixed order); the
 * three row-parallel exchanges carry twice the bytes. */
typedef enum { LTM_TP_REDUCE_ACT = 0, LTM_TP_REDUCE_EXACT = 1 } ltm_tp_reduction;
LTM_API ltm_status ltm_block_set_tp_reduction(ltm_block* blk, int mode);

/* ----------------------------------------------------------------- model -- */
/* Multi-layer model (token embedding gather + n_layers Titan blocks), the
 * forward of TitanModel (python_bindings/ltm/model.py:159-215), plus the LM
 * head of TitanForCausalLM (python_bindings/ltm/model.py:217-231,261) and a
 * prefill / decode-step pair over per-layer KV caches (the generation loop
 * of python_bindings/ltm/inference.py:131-260 with its CacheManager stubs,
 * python_bindings/src/main.cpp:101-135). */
typedef struct ltm_model ltm_model;
LTM_API ltm_status ltm_model_create(const ltm_block_config* cfg, const ltm_quant_config* qcfg,
                            int n_layers, int vocab_size, int device, ltm_model** out);
/* embedding: host fp32 [vocab, H] */
LTM_API ltm_status ltm_model_load_embedding(ltm_model* m, const float* embedding);
LTM_API ltm_status ltm_model_load_layer(ltm_model* m, int layer, const ltm_block_weights* w);
/* tokens: device int32 [B,S]; hidden_out: device [B,S,H] act_dtype. */
LTM_API ltm_status ltm_model_forward(ltm_model* m, const int32_t* tokens, void* hidden_out, int B, int S,
                             void* stream);
/* LM head weight: host fp32 [vocab, H] (nn.Linear(H, vocab, bias=False)),
 * quantized like the blocks' linears (W8A8: int8 per row, the hidden rows
 * quantized per token; W4A16: int4 group 128; W8A32: int8, fp32 rows). */
LTM_API ltm_status ltm_model_load_lm_head(ltm_model* m, const float* weight);
/* logits [rows, vocab] (act_dtype, device) = hidden rows (device, row stride
 * row_stride elements, e.g. S * H for the last position of each sequence)
 * times the LM head weight. */
LTM_API ltm_status ltm_model_lm_head(ltm_model* m, const void* hidden, int64_t rows,
                                     int64_t row_stride, void* logits, void* stream);
/* Prefill of B prompts of S tokens (device int32 [B,S]): the model forward
 * with every layer writing the post-RoPE K / V of positions [0, S) into its
 * caches k_caches[l] / v_caches[l] (host arrays of n_layers device pointers to
 * [B, heads, max_positions, head_dim] act_dtype); hidden_out ([B,S,H], or
 * NULL) receives the last layer's output, logits_last ([B, vocab], or NULL)
 * the LM head of each sequence's last position. */
LTM_API ltm_status ltm_model_prefill(ltm_model* m, const int32_t* tokens, int B, int S,
                                     void* const* k_caches, void* const* v_caches,
                                     int64_t max_positions, void* hidden_out, void* logits_last,
                                     void* stream);
/* One decode step of the model: tokens (device int32 [B]) at positions
 * cache_lens[b] (device int32 [B]; ltm_block_decode_step_ragged for every
 * layer), hidden_out ([B, H] or NULL), logits ([B, vocab] or NULL).  The
 * launches depend on B and max_positions only: after one uncaptured call the
 * step (with ltm_greedy_next_tokens) can be captured in a CUDA graph and
 * replayed for a whole greedy generation. */
LTM_API ltm_status ltm_model_decode_step(ltm_model* m, const int32_t* tokens,
                                         const int32_t* cache_lens, int B, void* const* k_caches,
                                         void* const* v_caches, int64_t max_positions,
                                         void* hidden_out, void* logits, void* stream);
/* Greedy next tokens: tokens_out[b] = argmax of logits row b ([B, vocab],
 * dtype; lowest index on ties); cache_lens[b] += 1 when cache_lens is not
 * NULL (device int32 [B]). */
LTM_API ltm_status ltm_greedy_next_tokens(const void* logits, ltm_dtype dtype, int B, int vocab,
                                          int32_t* tokens_out, int32_t* cache_lens, void* stream);
LTM_API ltm_status ltm_model_destroy(ltm_model* m);

#ifdef __cplusplus
}
#endif
#endif /* LTM_B200_H */
