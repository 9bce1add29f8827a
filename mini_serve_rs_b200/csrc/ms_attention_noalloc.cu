// Paged GQA decode attention that never allocates device memory.
//
// launch_paged_gqa_decode_tiled_bf16 grows a cached workspace with cudaMalloc
// the first time a batch needs more split-K scratch than it has.  Some callers
// cannot allow that: a serving process whose allocator has already reserved
// nearly all of HBM for its KV pages (a cudaMalloc there fails or evicts
// cached pages), or a runtime that forbids cudaMalloc / cudaFree on its hot
// path because both can synchronise the whole device and stall the other
// streams that are decoding at that moment.  This variant gives them the same
// kernel with its split-K scratch in a fixed buffer that is part of the
// library image.
//
// The buffer is a file-scope __device__ array of kScratchBytes (16 MiB).  The
// CUDA runtime reserves it on a device when it loads this file's module
// there: with CUDA's default lazy module loading that is the first call of
// this entry point on the device (or an earlier use of the symbol), with
// CUDA_MODULE_LOADING=EAGER it is when the library's first CUDA call
// initialises the device.  It stays reserved until the process exits.  A
// caller whose allocator claims nearly all of HBM must therefore make one
// call per device before that (any small batch will do), or the load itself
// can fail with an out-of-memory error; make that first call before any
// stream capture as well.  Host code cannot use the array's name as a device
// address: every call asks the runtime for the current device's address with
// cudaGetSymbolAddress (cheap once loaded, and never stale after a context is
// torn down and recreated).  All calls share the one buffer and it keeps the
// last call's contents: calls that can overlap on the GPU (different streams
// without ordering between them) race on it and must be serialised by the
// caller.  Nothing in the buffer has to start at zero: each call writes every
// partial result it later reads.  A kernel-side failure (a bounded wait that
// ran out) is recorded in the per-device status word that ms_kernel_status
// reads and clears.
#include <algorithm>

#include "ms_common.cuh"
#include "ms_internal.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

}  // namespace

extern "C" int launch_paged_gqa_decode_tiled_bf16_noalloc(const void *d_q, const void *d_k_pool,
                                                          const void *d_v_pool, const int *d_block_tables,
                                                          const int *d_seq_lens, void *d_out, int batch_size,
                                                          int num_heads, int num_kv_heads,
                                                          int max_blocks_per_seq, float scale) {
  // the argument checks of the allocating entry point
  if (batch_size <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return int(cudaErrorInvalidValue);
  if (max_blocks_per_seq <= 0) return int(cudaErrorInvalidValue);
  // same partition choice as launch_paged_gqa_decode_tiled_bf16, so the two agree
  const int max_ctx = max_blocks_per_seq * 16;
  const int part = ms::choose_partition_blocks(batch_size, num_kv_heads, max_ctx,
                                               (long long)batch_size * max_blocks_per_seq / 2);
  const int64_t need = ms::attention_workspace_bytes(batch_size, num_heads, max_ctx, part);
  if (need > int64_t(kScratchBytes)) return int(cudaErrorMemoryAllocation);  // beyond the fixed scratch

  // the current device's copy of the buffer (loads this module on the first call there)
  void *scratch = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
  if (e != cudaSuccess) return int(e);
  ms::AttnArgs a{};
  a.q = d_q;
  a.k_pool = d_k_pool;
  a.v_pool = d_v_pool;
  a.block_tables = d_block_tables;
  a.max_blocks_per_seq = max_blocks_per_seq;
  a.row_table = nullptr;
  a.row_ctx = d_seq_lens;
  a.num_rows = batch_size;
  a.max_ctx = max_ctx;
  a.out = d_out;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = 128;
  a.block_size = 16;
  a.scale = scale;
  a.part_blocks = part;
  a.workspace = scratch;
  a.workspace_bytes = int64_t(kScratchBytes);
  a.dtype = MS_DTYPE_BF16;
  a.status = nullptr;
  return int(ms::launch_paged_attention(a, 0));
}
