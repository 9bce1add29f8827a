// Internal launcher interfaces shared by the kernel files and the engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ms_engine.h"

namespace ms {

struct AttnArgs {
  const void *q;
  const void *k_pool;
  const void *v_pool;
  const int32_t *block_tables;
  int max_blocks_per_seq;
  const int32_t *row_table;
  const int32_t *row_ctx;
  int num_rows;
  int max_ctx;
  void *out;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int block_size;
  float scale;
  int part_blocks;
  void *workspace;
  int64_t workspace_bytes;
  int dtype;
  unsigned *status;  // device status word (may be null)
  // Tensor maps (CUtensorMap, host memory) describing k_pool / v_pool for the
  // 16-bit tensor-core build; null -> encoded per call.  pool_tiles = pages x
  // kv heads held by the pools (0 -> unknown).
  const void *k_map = nullptr;
  const void *v_map = nullptr;
  int64_t pool_tiles = 0;
  // launch row i attends for packed row row_index[i] (q, out, row_ctx,
  // row_table are indexed by the packed row); null -> identity
  const int32_t *row_index = nullptr;
};

// Encode the TMA tensor map of one paged pool for the tensor-core attention
// build (64-element inner boxes, 128-byte swizzle).  Returns false if the
// driver entry point is unavailable or the encode fails.
bool encode_pool_tensor_map(void *map_out, const void *pool, int dtype, int head_dim, int64_t pool_tiles);

cudaError_t launch_paged_attention(const AttnArgs &a, cudaStream_t stream);
// The current device's status word for kernels launched without an engine
// (see ms_kernel_status); looked up on every call.
cudaError_t standalone_status_word(unsigned **out);

// K3p: ragged causal prefill over the paged pool (16-bit, tensor cores).
// tiles [num_tiles][4] = (first packed row, rows, position of the first row,
// block-table row); rows of a tile are consecutive tokens of one sequence.
struct PrefillArgs {
  const void *q;
  const void *k_pool;
  const void *v_pool;
  const int32_t *block_tables;
  int max_blocks_per_seq;
  const int32_t *tiles;
  int num_tiles;
  void *out;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int block_size;
  float scale;
  int dtype;
  unsigned *status = nullptr;
};
cudaError_t launch_paged_prefill(const PrefillArgs &a, cudaStream_t stream);
// true when the 16-bit tensor-core decode / prefill kernels serve this shape
bool attention_tc_available(int dtype, int head_dim, int group);
int prefill_tokens_per_tile(int group);
// Host: split prefill sequences into tiles of prefill_tokens_per_tile(group)
// tokens; returns the tile count or -1 if capacity is exceeded.
int build_prefill_tiles(const int32_t *seq_row0, const int32_t *seq_ntok, const int32_t *seq_start,
                        const int32_t *seq_trow, int num_seqs, int group, int32_t *tiles_out, int capacity);
int choose_partition_blocks(int num_rows, int num_kv_heads, int max_ctx, long long total_blocks);
int64_t attention_workspace_bytes(int num_rows, int num_heads, int max_ctx, int part_blocks);

cudaError_t launch_add_rmsnorm(const void *x, const void *r, const int32_t *row_index, const void *w,
                               void *resid_out, void *norm_out, int rows, int hidden, float eps,
                               int dtype, cudaStream_t stream);

cudaError_t launch_qk_norm_rope_append(const void *qkv, const void *bias, const void *q_norm_w,
                                       const void *k_norm_w, const void *cos_table,
                                       const void *sin_table, const int32_t *positions,
                                       const int64_t *slot_mapping, void *q_out, void *k_pool,
                                       void *v_pool, int num_tokens, int num_heads, int num_kv_heads,
                                       int head_dim, int block_size, float eps, int dtype,
                                       cudaStream_t stream, unsigned *status = nullptr);

cudaError_t launch_silu_mul(const void *gate_up, void *out, int rows, int inter, int dtype,
                            cudaStream_t stream);
// K6b sampling (ms_sample.cu).  seeds, or seed_lo/seed_hi halves, or neither (0).
struct SampleArgs {
  const float *logits = nullptr;  // [rows, vocab]
  int rows = 0, vocab = 0;
  const float *temperature = nullptr;  // [rows]; < 1e-7 leaves out[row] untouched
  const float *top_p = nullptr;        // [rows] or null
  const uint64_t *seeds = nullptr;
  const uint32_t *seed_lo = nullptr, *seed_hi = nullptr;
  int32_t *out = nullptr;               // [rows]
  const int32_t *row_slot = nullptr;    // with slot_last: also record the token per slot
  int32_t *slot_last = nullptr;
  unsigned *status = nullptr;           // kStatus* bits; null: the standalone status word
};
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t st);
cudaError_t launch_argmax(const float *logits, int rows, int vocab, int32_t *out,
                          const int32_t *row_slot, int32_t *slot_last_token, cudaStream_t stream);
cudaError_t launch_embedding(const int32_t *tokens, const void *table, void *out, int rows,
                             int hidden, int dtype, cudaStream_t stream);
cudaError_t launch_convert(const void *src, int src_dtype, void *dst, int dst_dtype, int64_t n,
                           cudaStream_t stream);

// NCCL, resolved at run time (ms_nccl.cu)
bool nccl_available();
int nccl_allreduce_sum(void *buf, size_t count, int dtype, void *comm, cudaStream_t stream);
int nccl_allgather_bytes(void *buf, size_t bytes, int rank, void *comm, cudaStream_t stream);
int nccl_allreduce_min_i32(int32_t *buf, void *comm, cudaStream_t stream);
int nccl_async_error(void *comm);
void nccl_abort(void *comm);

struct PackArgs {
  const int32_t *seq_row;    // [nseq] block-table row (engine slot) of each sequence
  const int32_t *seq_ntok;   // [nseq] tokens this step
  const int32_t *seq_start;  // [nseq] position of the first token
  int num_seqs;
  const int32_t *delta_row;
  const int32_t *delta_idx;
  const int32_t *delta_block;
  int num_deltas;                  // capacity of the delta arrays
  const int32_t *num_deltas_dev;   // when set, the delta count is read here (<= num_deltas)
  int32_t *block_tables;  // [rows][max_blocks_per_seq]
  int max_blocks_per_seq;
  int block_size;
  int32_t *cu_seqlens;    // [nseq+1]
  int32_t *positions;     // [T]
  int64_t *slot_mapping;  // [T]
  int32_t *row_table;     // [T]
  int32_t *row_ctx;       // [T]
  // optional engine extras
  int32_t *last_index;          // [nseq] packed index of each sequence's last token
  int32_t *tokens;              // [T] input tokens (rewritten for device-fed decode rows)
  const int32_t *slot_last_tok; // [rows] last token produced per slot (device-fed decode)
  int tokens_from_device;
  unsigned *status;
  int64_t pool_blocks;
};
cudaError_t launch_pack(const PackArgs &a, cudaStream_t stream);

}  // namespace ms
