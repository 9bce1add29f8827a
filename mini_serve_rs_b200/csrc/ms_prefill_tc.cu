// K3p launcher and tile planning: the ragged paged causal prefill attention
// (the prefill branch of Attention::forward, src/backends/qwen2.rs:329-345,
// with the causal mask of :476-503 including the seqlen_offset columns of a
// cached prefix) runs as the tcgen05 kernel of ms_prefill_tc5.cu.  This file
// checks the launch arguments, supplies the standalone status word, and cuts
// each step's prompt chunks into tiles ordered longest causal range first.
#include <algorithm>
#include <array>
#include <vector>

#include "ms_attention_common.cuh"

namespace ms {
namespace attn {
// tcgen05 kernel (ms_prefill_tc5.cu)
int prefill_tc5_tokens_per_tile(int group);
cudaError_t launch_prefill_tc5(const void *q, void *out, const int32_t *block_tables, int max_blocks_per_seq,
                               const int32_t *tiles, int num_tiles, int num_kv_heads, int group, int head_dim,
                               float scale, unsigned *status, int dtype, const void *k_pool, const void *v_pool,
                               cudaStream_t stream);
}  // namespace attn

int prefill_tokens_per_tile(int group) { return attn::prefill_tc5_tokens_per_tile(group); }

cudaError_t launch_paged_prefill(const PrefillArgs &a, cudaStream_t stream) {
  if (a.num_tiles == 0) return cudaSuccess;
  if (a.num_tiles < 0 || a.num_heads <= 0 || a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads != 0 ||
      a.block_size != attn::kBS)
    return cudaErrorInvalidValue;
  const int group = a.num_heads / a.num_kv_heads;
  if (!attn::attention_tc_supported(a.dtype, a.head_dim, group)) return cudaErrorInvalidValue;
  unsigned *status = a.status;
  if (!status) {
    cudaError_t e = standalone_status_word(&status);
    if (e != cudaSuccess) return e;
  }
  return attn::launch_prefill_tc5(a.q, a.out, a.block_tables, a.max_blocks_per_seq, a.tiles, a.num_tiles,
                                  a.num_kv_heads, group, a.head_dim, a.scale, status, a.dtype, a.k_pool, a.v_pool,
                                  stream);
}

// Tiles in decreasing order of their causal range (position of the first row
// + rows), ties in input order: the CTAs that sweep the most keys start
// first, so short tiles fill the last wave.
int build_prefill_tiles(const int32_t *seq_row0, const int32_t *seq_ntok, const int32_t *seq_start,
                        const int32_t *seq_trow, int num_seqs, int group, int32_t *tiles_out, int capacity) {
  const int tpb = prefill_tokens_per_tile(group);
  std::vector<std::array<int32_t, 4>> tl;
  for (int i = 0; i < num_seqs; ++i) {
    for (int j = 0; j < seq_ntok[i]; j += tpb) {
      if (int(tl.size()) >= capacity) return -1;
      tl.push_back({seq_row0[i] + j, std::min(tpb, seq_ntok[i] - j), seq_start[i] + j, seq_trow[i]});
    }
  }
  std::stable_sort(tl.begin(), tl.end(), [](const std::array<int32_t, 4> &a, const std::array<int32_t, 4> &b) {
    return a[2] + a[1] > b[2] + b[1];
  });
  for (size_t n = 0; n < tl.size(); ++n)
    for (int k = 0; k < 4; ++k) tiles_out[4 * n + k] = tl[n][k];
  return int(tl.size());
}

}  // namespace ms

extern "C" int ms_launch_paged_prefill(const void *q, const void *k_pool, const void *v_pool,
                                       const int32_t *block_tables, int32_t max_blocks_per_seq,
                                       const int32_t *tiles, int32_t num_tiles, void *out, int32_t num_heads,
                                       int32_t num_kv_heads, int32_t head_dim, int32_t block_size, float scale,
                                       int32_t dtype, void *stream) {
  ms::PrefillArgs a{};
  a.q = q;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.block_tables = block_tables;
  a.max_blocks_per_seq = max_blocks_per_seq;
  a.tiles = tiles;
  a.num_tiles = num_tiles;
  a.out = out;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  return int(ms::launch_paged_prefill(a, static_cast<cudaStream_t>(stream)));
}

extern "C" int ms_prefill_tiles(const int32_t *seq_row0, const int32_t *seq_ntok, const int32_t *seq_start,
                                const int32_t *seq_table_row, int32_t num_seqs, int32_t num_heads,
                                int32_t num_kv_heads, int32_t *tiles_out, int32_t capacity) {
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return -1;
  return ms::build_prefill_tiles(seq_row0, seq_ntok, seq_start, seq_table_row, num_seqs, num_heads / num_kv_heads,
                                 tiles_out, capacity);
}
