// K1: on-GPU ragged batch packer.
//
// Replaces the host-side tensor building of the reference's step
// (src/backends/candle.rs:603-630: decode ids and positions
// prompt + outputs - 1; src/backends/qwen2.rs:649-655: the positions tensor)
// and the contiguous per-request cache addressing (qwen2.rs:349-361).  Block
// tables live on the device, one row per engine sequence slot, and are
// updated from the scheduler's block deltas (KVCache::allocate /
// allocate_block results, src/cache/kv_cache.rs:61-99) before the slots are
// computed as block_table[row][pos / 16] * 16 + pos % 16 -- the addressing of
// the prototype kernels (docs/colab_cuda_kernels/mini_serve_kernels.cu:219-223).
//
// Integer-only and tiny: one CTA of 1024 threads applies the deltas, scans
// the per-sequence token counts into cu_seqlens (kept in shared memory), then
// fills the per-token arrays with a binary search over cu_seqlens.
#include "ms_common.cuh"
#include "ms_internal.h"

namespace ms {
namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int *warp_tot, int &total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tot[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(kFull, wi, o);
      if (lane >= o) wi += n;
    }
    warp_tot[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) warp_tot[32] = wi;
  }
  __syncthreads();
  total = warp_tot[32];
  const int r = warp_tot[warp] + incl - v;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kThreads) pack_kernel(PackArgs a) {
  extern __shared__ int cu_s[];  // [num_seqs + 1]
  __shared__ int warp_tot[33];
  const int tid = threadIdx.x;

  // 1. block-table deltas (count from device memory when the launch is replayed from a graph)
  const int nd = a.num_deltas_dev ? min(*a.num_deltas_dev, a.num_deltas) : a.num_deltas;
  for (int i = tid; i < nd; i += kThreads) {
    const int row = a.delta_row[i], idx = a.delta_idx[i], blk = a.delta_block[i];
    const bool ok = row >= 0 && idx >= 0 && idx < a.max_blocks_per_seq && blk >= 0 &&
                    (a.pool_blocks <= 0 || blk < a.pool_blocks);
    if (ok) a.block_tables[size_t(row) * a.max_blocks_per_seq + idx] = blk;
    else if (a.status) atomicOr(a.status, kStatusBadIndex);
  }

  // 2. cu_seqlens: each thread scans a contiguous run of sequences
  const int per = (a.num_seqs + kThreads - 1) / kThreads;
  const int s0 = min(a.num_seqs, tid * per), s1 = min(a.num_seqs, s0 + per);
  int local = 0;
  for (int i = s0; i < s1; ++i) local += a.seq_ntok[i];
  int total = 0;
  int run = block_exclusive_scan(local, warp_tot, total);
  for (int i = s0; i < s1; ++i) {
    cu_s[i] = run;
    run += a.seq_ntok[i];
  }
  if (tid == 0) cu_s[a.num_seqs] = total;
  __syncthreads();  // deltas and cu_s visible to the whole CTA
  for (int i = tid; i <= a.num_seqs; i += kThreads) a.cu_seqlens[i] = cu_s[i];
  if (a.last_index)
    for (int i = tid; i < a.num_seqs; i += kThreads) a.last_index[i] = cu_s[i + 1] - 1;

  // 3. per-token metadata
  for (int t = tid; t < total; t += kThreads) {
    int lo = 0, hi = a.num_seqs - 1;  // largest i with cu_s[i] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cu_s[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int i = lo;
    const int row = a.seq_row[i];
    const int pos = a.seq_start[i] + (t - cu_s[i]);
    const int li = pos / a.block_size;
    int64_t slot = 0;
    if (pos >= 0 && li < a.max_blocks_per_seq) {
      const int blk = a.block_tables[size_t(row) * a.max_blocks_per_seq + li];
      slot = int64_t(blk) * a.block_size + pos % a.block_size;
    } else if (a.status) {
      atomicOr(a.status, kStatusBadIndex);
    }
    a.positions[t] = pos;
    a.slot_mapping[t] = slot;
    a.row_table[t] = row;
    a.row_ctx[t] = pos + 1;
    if (a.tokens && a.slot_last_tok && a.tokens[t] < 0) a.tokens[t] = a.slot_last_tok[row];
  }
}

}  // namespace

cudaError_t launch_pack(const PackArgs &a, cudaStream_t st) {
  if (a.num_seqs <= 0) return cudaErrorInvalidValue;
  if (a.block_size <= 0 || a.max_blocks_per_seq <= 0) return cudaErrorInvalidValue;
  const size_t smem = size_t(a.num_seqs + 1) * sizeof(int);
  if (smem > 160 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  pack_kernel<<<1, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace ms

extern "C" int ms_launch_pack(const int32_t *seq_row, const int32_t *seq_ntok, const int32_t *seq_start,
                              int32_t num_seqs, const int32_t *delta_row, const int32_t *delta_idx,
                              const int32_t *delta_block, int32_t num_deltas, int32_t *block_tables,
                              int32_t max_blocks_per_seq, int32_t block_size, int32_t *cu_seqlens,
                              int32_t *positions, int64_t *slot_mapping, int32_t *row_table, int32_t *row_ctx,
                              void *stream) {
  ms::PackArgs a{};
  a.seq_row = seq_row;
  a.seq_ntok = seq_ntok;
  a.seq_start = seq_start;
  a.num_seqs = num_seqs;
  a.delta_row = delta_row;
  a.delta_idx = delta_idx;
  a.delta_block = delta_block;
  a.num_deltas = num_deltas;
  a.block_tables = block_tables;
  a.max_blocks_per_seq = max_blocks_per_seq;
  a.block_size = block_size;
  a.cu_seqlens = cu_seqlens;
  a.positions = positions;
  a.slot_mapping = slot_mapping;
  a.row_table = row_table;
  a.row_ctx = row_ctx;
  a.pool_blocks = 0;
  return int(ms::launch_pack(a, static_cast<cudaStream_t>(stream)));
}
