// block.cuh -- internal interfaces between the kernels and the block
// orchestration (device buffers, quantized weights, launchers).
#pragma once

#include <string>
#include <vector>

#include "common.cuh"
#include "epilogue.cuh"

// Tensor-parallel communicator (comm.cu): an NCCL communicator of `nranks`
// GPUs; this process is `rank`, on `device`.
struct ltm_comm {
  void* handle = nullptr;
  int nranks = 1, rank = 0, device = 0;
};

namespace ltm_b200 {

// In-stream allreduce (sum, or max) over the communicator; send == recv allowed.
void comm_allreduce(ltm_comm* c, const void* send, void* recv, size_t count, ltm_dtype dt,
                    bool max_op, cudaStream_t st);
// All-gather of bytes_per_rank bytes from every rank into recv (rank order);
// in place when send == recv + rank * bytes_per_rank.
void comm_allgather_bytes(ltm_comm* c, const void* send, void* recv, size_t bytes_per_rank,
                          cudaStream_t st);
// Reduce-scatter (sum): rank r receives the sum of every rank's block r of
// count_per_rank elements of send.
void comm_reduce_scatter(ltm_comm* c, const void* send, void* recv, size_t count_per_rank,
                         ltm_dtype dt, cudaStream_t st);
// In-place broadcast of `bytes` bytes at buf from rank root.
void comm_broadcast_bytes(ltm_comm* c, void* buf, size_t bytes, int root, cudaStream_t st);
// Sum of every rank's send into recv on rank root (recv unused elsewhere).
void comm_reduce(ltm_comm* c, const void* send, void* recv, size_t count, ltm_dtype dt, int root,
                 cudaStream_t st);
// Rank-to-rank exchange of row blocks (all-to-all, no reduction): for every
// peer j, block j of `send` (`bytes` bytes) goes to rank j and rank j's
// block for this rank lands in slot j of `recv` ([nranks, bytes]; this
// rank's own slot is left untouched).  root >= 0 restricts it to the
// transfers into rank `root` (the blocks of one row owner).
void comm_send_recv_slots(ltm_comm* c, const void* send, void* recv, size_t bytes, int root,
                          cudaStream_t st);
// Rows [rows, cols] of int32 GEMM accumulators summed over the ranks' slots
// (exact), then the W8A8 epilogue of the unsplit GEMM: y = round(fma(acc *
// row_scale[r], col_scale[c], bias[c]) (+ add[r, c])), the arithmetic of the
// tensor-core epilogue, so the rows equal the single-GPU GEMM's bit for bit.
void launch_sum_slots_i32(const int32_t* slots, const int32_t* own, int nslots, int own_slot,
                          int64_t slot_stride, const float* row_scale, const float* col_scale,
                          const float* bias, const void* add, void* y, int64_t rows, int64_t cols,
                          ltm_dtype dt, cudaStream_t stream);
// NCCL group brackets: the collectives between them launch as one (at the
// end, which marks them for the kernel timer under `what` on stream st).
void comm_group_start();
void comm_group_end(const char* what, cudaStream_t st);

// Owning device allocation (grow-only).
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf();
  void ensure(size_t n);
  void release();
  template <class T>
  T* as() const {
    return static_cast<T*>(ptr);
  }
};

// A quantized weight [N,K] with per-channel int8 or group-128 int4 codes.
struct QLinear {
  int64_t N = 0, K = 0;
  int scheme = LTM_SCHEME_W8A8;
  DevBuf q8, s8, q4, s4, z4, bias;
  // false: run() leaves the bias out (the row-parallel shards of ranks other
  // than the first, whose partial sums are added to the first rank's)
  bool apply_bias = true;
  void load(const ltm_quant_config& q, const float* w_host, const float* b_host, int64_t n,
            int64_t k, cudaStream_t stream);
  // Input columns [c0, c0 + nc) of a host [n, k] weight with the unsplit
  // weight's scales (row-parallel tensor-parallel layers).
  void load_cols(const ltm_quant_config& q, const float* w_host, const float* b_host, int64_t n,
                 int64_t k, int64_t c0, int64_t nc, cudaStream_t stream);
  // wdq: scratch for the dequantised weight of the W4A16 path at large M
  // (NULL: the fused dequantising kernel at every M).
  void run(const void* a_act, const int8_t* aq, const float* as, int64_t M, int mode, ltm_dtype dt,
           Epilogue ep, cudaStream_t stream, DevBuf* wdq = nullptr) const;
};

// One device buffer of a block's state (a checkpoint section).
struct StateSection {
  std::string name;
  void* ptr;
  size_t bytes;
};

}  // namespace ltm_b200

struct ltm_block;

namespace ltm_b200 {

// The device buffers of a block's weights (quantized codes, scales,
// zero-points, biases, LayerNorm parameters) and / or its bank, in a fixed
// order; with allocate they are sized for the block's config first (before
// a load from a checkpoint).
std::vector<StateSection> block_state(ltm_block* b, bool weights, bool bank, bool allocate);
// After the sections were written: the block counts as loaded (weights) and
// its resident K_M | V_M are recomputed at the next use.
void block_state_loaded(ltm_block* b, bool weights);
void block_identity(const ltm_block* b, ltm_block_config* cfg, ltm_quant_config* q, int* tp,
                    int* tpr, int* device, bool* loaded);

struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t ldq, ldk, ldv, ldo;
  int64_t q_batch_rows;
  int64_t kv_batch_rows;
  int Sq, Skv, nh;
  int causal_offset;
  float scale_log2;
};

// Memory-bank write after the read (TB-v1):
//   c   = mean_t g_t * x_t                 (accumulated by the gate-mix epilogue)
//   w_s = rate * mean_heads softmax_s(qbar_h . K_M[s,h] / sqrt(dh))   (or rate)
//   M_s = (1 - w_s) M_s + w_s c
struct MemoryWriteState {
  DevBuf colsum, qsum, wslot;
  void prepare_gate_epilogue(Epilogue& ep, int H, cudaStream_t st);
  // kvm: K_M [Ms, heads*dh] with row stride ldk; qm: memory queries [T,
  // heads*dh] with row stride ldq (this rank's `heads` of nh_total; comm
  // sums the slot weights over the ranks when given).
  // Returns the factor that turns colsum into the state c (1 / T, and the
  // mean over the ranks under tensor parallelism).
  // colsum_partial: each rank's column sums cover only its own rows
  // (sequence-parallel gate), so the ranks' sums add up to the total.
  float update_bank(void* memory, const void* kvm, int64_t ldk, const void* qm, int64_t ldq,
                    int64_t T, int H, int heads, int nh_total, int dh, int Ms, float rate,
                    bool use_scores, ltm_dtype dt, ltm_comm* comm, cudaStream_t st,
                    bool colsum_partial = false);
};

// The state c = state * scale as one row [H] in the activation dtype.
void launch_state_row(const float* state, float scale, void* out, int H, ltm_dtype dt,
                      cudaStream_t st);

// rows[s, :width] = (1 - w_s) rows[s, :width] + w_s v  (w_s = wslot[s], or
// rate when wslot is NULL); rows of stride ld, 16-bit activations.
void launch_rows_ema(void* rows, int64_t ld, int width, const void* v, const float* wslot,
                     float rate, int Ms, ltm_dtype dt, cudaStream_t st);

// Decode step, head-major caches [B, width / dh, P, dh]: the new token's K | V
// rows (columns [width, 3 width) of the fused projection rows, stride ldq) to
// position pos of every head of its sequence.
// pos_arr (device [B], optional): a position per sequence instead of pos;
// positions outside [0, P) write nothing and set the device error word.
void launch_kv_append(const void* qkv, int64_t ldq, int width, int dh, void* kc, void* vc,
                      int64_t P, int64_t pos, int B, ltm_dtype dt, cudaStream_t st,
                      const int* pos_arr = nullptr);
// Prefill: the K | V rows of all B * S rows (positions 0 .. S-1 of each
// sequence) into the head-major caches.
void launch_kv_fill(const void* qkv, int64_t ldq, int width, int dh, void* kc, void* vc, int64_t P,
                    int B, int S, ltm_dtype dt, cudaStream_t st);
// Self-attention of one query row per (sequence, head) over the first L of
// the P cached positions (split into chunks, partials in `part`, then merged
// into o).
size_t decode_partials_bytes(int B, int nh, int D, int64_t L);
// cache_lens (device [B], optional): sequence b attends cache_lens[b] + 1
// positions (L is then the upper bound max_positions).
void launch_decode_attention(const void* q, int64_t ldq, const void* kc, const void* vc,
                             int64_t P, int L, int B, int nh, int D, ltm_dtype dt, float* part,
                             void* o, int64_t ldo, cudaStream_t st,
                             const int* cache_lens = nullptr);

// Slot weights of `heads` heads (rate / nh_total per head, summed into wslot;
// qsum [heads*dh] and wslot [Ms] are cleared here) and the bank EMA.
void launch_slot_weights(const void* keys, int64_t ldk, const void* queries, int64_t ldq,
                         int64_t T, int Ms, int heads, int dh, int nh_total, float rate,
                         ltm_dtype dt, float* qsum, float* wslot, cudaStream_t st);
void launch_bank_update(void* memory, const float* state, float state_scale, const float* wslot,
                        float rate, int Ms, int H, ltm_dtype dt, cudaStream_t st);

// Memory-bank store: slot weights from the mean of the query rows against the
// keys (use_scores) and the EMA of every slot towards state * state_scale.
// qsum [H] and wslot [Ms] are fp32 scratch, cleared here.
void launch_memory_store(void* memory, const void* keys, int64_t ldk, const void* queries,
                         int64_t ldq, int64_t T, const float* state, float state_scale, int Ms,
                         int H, int nh, float rate, bool use_scores, ltm_dtype dt, float* qsum,
                         float* wslot, cudaStream_t st);
void validate_memory_store(const void* memory, const void* keys, int64_t ldk, const void* queries,
                           int64_t ldq, int64_t T, const float* state, int Ms, int H, int nh,
                           bool use_scores);

void launch_rowwise_int8(const void* x, ltm_dtype dt, int64_t rows, int64_t K, int8_t* q, float* s,
                         cudaStream_t stream);
// Tensor-parallel per-token quantization: local row maxima, then codes with
// s = amax / 127 from the (allreduced) maxima.
void launch_row_absmax(const void* x, ltm_dtype dt, int64_t rows, int64_t K, float* amax,
                       cudaStream_t stream);
void launch_rowwise_int8_amax(const void* x, ltm_dtype dt, int64_t rows, int64_t K,
                              const float* amax, int8_t* q, float* s, cudaStream_t stream);
void launch_w8a8(const int8_t* qa, const int8_t* qw, int64_t M, int64_t N, int64_t K, int mode,
                 ltm_dtype out_dt, const Epilogue& ep, cudaStream_t stream);
// 16-bit GEMM on the persistent tcgen05 kernels (operands a [M,K], w [N,K]
// in dt, fp32 accumulation, fused epilogue, output in dt).
void launch_gemm_f16(const void* a, const void* w, int64_t M, int64_t N, int64_t K, int mode,
                     ltm_dtype dt, const Epilogue& ep, cudaStream_t stream);
// INT4 group-128 weight [N,K] dequantised to dt (T((q - zp) * s)).
void launch_int4_dequant_rows(const uint8_t* packed, const float* s, const uint8_t* zp, int64_t N,
                              int64_t K, void* out, ltm_dtype dt, cudaStream_t st);
void launch_w8a32(const float* a, const int8_t* qw, int64_t M, int64_t N, int64_t K, int mode,
                  const Epilogue& ep, cudaStream_t stream);
// split_k: grids smaller than the GPU split K over a cluster of CTAs per
// output tile (reduced through distributed shared memory).
void launch_w4a16(const void* a, ltm_dtype dt, const uint8_t* q4, const float* s4, const uint8_t* z4,
                  int64_t M, int64_t N, int64_t K, int mode, const Epilogue& ep, cudaStream_t stream,
                  bool split_k = true);
void launch_ln_x2(const void* x, ltm_dtype dt, int64_t rows, int H, const float* gamma,
                  const float* beta, void* y, int8_t* yq, float* ys, int8_t* xq, float* xs,
                  bool do_norm, cudaStream_t stream, const void* residual = nullptr);
void launch_embed_gather(const void* table, ltm_dtype dt, int vocab, int H, const int32_t* tok,
                         int64_t T, void* out, cudaStream_t stream);
void launch_attention(const AttnParams& p, int B, int D, bool causal, ltm_dtype dt,
                      cudaStream_t stream);
void launch_attention_tc(const AttnParams& p, int B, int D, bool causal, ltm_dtype dt,
                         cudaStream_t stream);
// Next token of each of B rows of logits (stride ld): argmax (lowest index
// on ties); lens[b] += 1 when lens is given.
void launch_greedy_next(const void* logits, int64_t ld, ltm_dtype dt, int B, int vocab,
                        int32_t* tokens, int32_t* lens, cudaStream_t st);
void launch_add3(const void* a, const void* b, const void* c, void* y, int64_t n, ltm_dtype dt,
                 cudaStream_t stream);
void upload_f32_as(const float* host, int64_t n, ltm_dtype dt, void* dev, cudaStream_t stream);

}  // namespace ltm_b200
