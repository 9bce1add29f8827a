// K3, tensor-core build for 16-bit K/V (bf16 / f16): split-K paged GQA
// attention where each page's scores and its P.V product run on mma.sync.
//
// Same decomposition as the SIMT build (one CTA of 4 warps per (query row,
// KV head, partition), pages round-robin over warps, per-warp TMA ring,
// cross-warp merge, log-sum-exp partition combine) -- restating
// decode_attention_gqa_zero_copy (src/backends/qwen2.rs:182-203) for every
// packed row.  Per page and warp:
//   * the K and V tiles arrive by TMA tensor copies (cp.async.bulk.tensor,
//     no multicast) as 16-token x 64-dim boxes with 128-byte swizzle, so the
//     ldmatrix reads below are bank-conflict free;
//   * S[16 x 16] = Q[16 x D] K^T: the kv head's G query heads are rows 0..G-1
//     of the m16 tile (the rest zero), 2 n-tiles x D/16 k-steps of
//     mma.m16n8k16 with f32 accumulation;
//   * online softmax in base 2 on each lane's four scores (row gid);
//   * O[16 x D] += P V: P (rounded to the K/V type, as FlashAttention does)
//     is reused in registers as the A operand, V^T fragments come from
//     ldmatrix.trans, D/8 n-tiles.
// That is ~120 instructions per page per warp instead of ~930 for the SIMT
// scoring, which leaves the kernel bound by HBM instead of by issue.
// The contraction per page is 16 x 16 x D -- far below one tcgen05 tile
// (M >= 64) -- so the warp-level MMA keeps it in registers.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "ms_attention_common.cuh"

namespace ms {
namespace attn {
namespace {

constexpr int kHalfBytes = 16 * 64 * 2;  // one 16-token x 64-dim box of 16-bit elements

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

// byte offset of (token, dim) inside one tile stored as D/64 boxes of
// [16 tokens][64 dims] with the 128-byte swizzle (16-byte chunk ^ token % 8)
__device__ __forceinline__ uint32_t tile_off(int token, int dim) {
  const int dh = dim >> 6, c = (dim & 63) >> 3;
  return uint32_t(dh * kHalfBytes + token * 128 + ((c ^ (token & 7)) << 4));
}

template <typename T, int D, int G, int NSTAGE>
__global__ void __launch_bounds__(kWarps * 32)
    paged_attention_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                              Params p) {
  static_assert(G >= 1 && G <= 8, "query heads per kv head must fit rows 0..7 of the m16 tile");
  constexpr int NDH = D / 64;
  constexpr int TILE_BYTES = NDH * kHalfBytes;
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int KSTEPS = D / 16;
  constexpr int NTD = D / 8;

  extern __shared__ unsigned char smem_dyn[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + size_t(kWarps) * NSTAGE * STAGE_BYTES);

  const int ri = blockIdx.x;
  const int row = p.row_index ? p.row_index[ri] : ri;
  const int kvh = blockIdx.y;
  const int part = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;

  const int ctx = p.row_ctx[row];
  const int nblk = max(0, (ctx + kBS - 1) / kBS);
  int nparts = max(1, (nblk + p.part_blocks - 1) / p.part_blocks);
  if (nparts > p.max_parts) {  // row_ctx beyond the launch's max_ctx: flag, do not fault
    if (threadIdx.x == 0 && part == 0) atomicOr(p.status, kStatusBadIndex);
    nparts = p.max_parts;
  }
  if (part >= nparts) return;
  const int blk0 = part * p.part_blocks;
  const int blk1 = min(blk0 + p.part_blocks, nblk);
  const int trow = p.row_table ? p.row_table[row] : row;
  const int32_t *table = p.block_tables + size_t(trow) * p.max_blocks_per_seq;
  const int nb_w = (blk1 - blk0 - warp + kWarps - 1) / kWarps;  // pages blk0 + warp + k * kWarps
  unsigned char *my_stage = smem + size_t(warp) * NSTAGE * STAGE_BYTES;
  uint64_t *my_bar = bars + warp * NSTAGE;

  if (lane == 0) {
    for (int s = 0; s < NSTAGE; ++s) mbar_init(&my_bar[s], 1);
    fence_barrier_init();
    fence_proxy_async();
  }
  __syncwarp();

  int page_reg = 0;  // lane k holds the page id of this warp's k-th page (32 at a time)
  auto page_of = [&](int k) -> int { return __shfl_sync(kFull, page_reg, k & 31); };
  auto refill_pages = [&](int k0) {
    const int k = k0 + lane;
    page_reg = (k < nb_w) ? table[blk0 + warp + k * kWarps] : 0;
  };
  auto issue = [&](int s, int page) {
    if (lane == 0) {
      unsigned char *st = my_stage + size_t(s) * STAGE_BYTES;
      const int tile = page * p.num_kv_heads + kvh;
      mbar_expect_tx(&my_bar[s], STAGE_BYTES);
#pragma unroll
      for (int dh = 0; dh < NDH; ++dh) {
        tma_load_4d(st + dh * kHalfBytes, &kmap, 0, dh, 0, tile, &my_bar[s]);
        tma_load_4d(st + TILE_BYTES + dh * kHalfBytes, &vmap, 0, dh, 0, tile, &my_bar[s]);
      }
    }
  };

  // Q as the A operand: row gid < G is query head kvh*G + gid, other rows zero
  uint32_t qa[KSTEPS][2];
  {
    const T *qrow = static_cast<const T *>(p.q) +
                    (size_t(row) * p.num_kv_heads * G + size_t(kvh) * G + (gid < G ? gid : 0)) * D;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      qa[kk][0] = gid < G ? *reinterpret_cast<const uint32_t *>(qrow + kk * 16 + 2 * tig) : 0u;
      qa[kk][1] = gid < G ? *reinterpret_cast<const uint32_t *>(qrow + kk * 16 + 8 + 2 * tig) : 0u;
    }
  }
  float o[NTD][4];
#pragma unroll
  for (int nd = 0; nd < NTD; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  // ldmatrix lane roles: matrix mi = lane / 8, row lr = lane % 8
  const int mi = lane >> 3, lr = lane & 7;

  bool failed = false;
  int issued = 0, kfail = 0;
  if (nb_w > 0) {
    refill_pages(0);
    const int pro = min(NSTAGE, nb_w);
    for (int k = 0; k < pro; ++k) issue(k, page_of(k));
    issued = pro;
  }

  for (int k = 0; k < nb_w; ++k) {
    const int s = k % NSTAGE;
    // the whole warp agrees before leaving, so no lane is left waiting in a shuffle
    if (!__all_sync(kFull, mbar_wait_bounded(&my_bar[s], (k / NSTAGE) & 1, p.wait_limit))) {
      failed = true;
      kfail = k;
      break;
    }
    unsigned char *st = my_stage + size_t(s) * STAGE_BYTES;
    const uint32_t kb = smem_addr(st), vb = kb + TILE_BYTES;
    const int blk = blk0 + warp + k * kWarps;
    const int valid = min(kBS, ctx - blk * kBS);

    if (valid < kBS) {
      // tokens past the context hold stale pool data (possibly NaN): zero
      // their V rows so P = 0 cannot turn them into NaN in the P.V product
      uint4 *vz = reinterpret_cast<uint4 *>(st + TILE_BYTES);
      for (int i = lane; i < NDH * (kBS - valid) * 8; i += 32) {
        const int dh = i / ((kBS - valid) * 8), rem = i % ((kBS - valid) * 8);
        const int tok = valid + rem / 8, ch = rem % 8;
        vz[(dh * kHalfBytes + tok * 128) / 16 + ch] = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }

    // S = Q K^T for tokens 0..7 (sc[0]) and 8..15 (sc[1])
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      uint32_t b[4];
      const int token = (mi >> 1) * 8 + lr;
      ldmatrix_x4(b, kb + tile_off(token, kk * 16 + (mi & 1) * 8));
      const uint32_t a[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
      mma_16816<T>(sc[0], a, b[0], b[1]);
      mma_16816<T>(sc[1], a, b[2], b[3]);
    }
    // online softmax over this page for row gid (lanes gid*4 .. gid*4+3)
    float sv[4] = {sc[0][0], sc[0][1], sc[1][0], sc[1][1]};
    const int tk[4] = {2 * tig, 2 * tig + 1, 8 + 2 * tig, 9 + 2 * tig};
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sv[j] = (tk[j] < valid) ? sv[j] * p.qscale : -INFINITY;
      mx = fmaxf(mx, sv[j]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
    const float m_new = fmaxf(m_run, mx);  // token 0 of a page is always valid
    const float alpha = exp2f(m_run - m_new);
    float pj[4];
    float psum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pj[j] = exp2f(sv[j] - m_new);
      psum += pj[j];
    }
    l_run = l_run * alpha + psum;
    m_run = m_new;
#pragma unroll
    for (int nd = 0; nd < NTD; ++nd) {
      o[nd][0] *= alpha;
      o[nd][1] *= alpha;
    }
    const uint32_t pa[4] = {pack2<T>(pj[0], pj[1]), 0u, pack2<T>(pj[2], pj[3]), 0u};
    // O += P V, two n-tiles of 8 dims per ldmatrix.x4.trans
#pragma unroll
    for (int ndp = 0; ndp < NTD / 2; ++ndp) {
      uint32_t b[4];
      const int token = (mi & 1) * 8 + lr;
      ldmatrix_x4_trans(b, vb + tile_off(token, (2 * ndp + (mi >> 1)) * 8));
      mma_16816<T>(o[2 * ndp], pa, b[0], b[1]);
      mma_16816<T>(o[2 * ndp + 1], pa, b[2], b[3]);
    }

    __syncwarp();
    if (issued < nb_w && k + NSTAGE == issued) {
      const int kn = issued;
      if ((kn & 31) == 0) refill_pages(kn);
      const int pg = page_of(kn);
      if (lane == 0) fence_proxy_async();
      issue(s, pg);
      ++issued;
    }
  }

  if (failed) {
    if (lane == 0) atomicOr(p.status, kStatusWaitTimeout);
    for (int k = kfail; k < issued; ++k) mbar_wait_bounded(&my_bar[k % NSTAGE], (k / NSTAGE) & 1);
  }
  l_run += __shfl_xor_sync(kFull, l_run, 1);
  l_run += __shfl_xor_sync(kFull, l_run, 2);

  __syncthreads();  // all warps done with their stages: reuse shared memory for the merge
  float *mo = reinterpret_cast<float *>(smem);  // [kWarps][G][D]
  float *mm = mo + kWarps * G * D;              // [kWarps][G]
  float *ml = mm + kWarps * G;                  // [kWarps][G]
  if (gid < G) {
#pragma unroll
    for (int nd = 0; nd < NTD; ++nd) {
      mo[(warp * G + gid) * D + nd * 8 + 2 * tig] = o[nd][0];
      mo[(warp * G + gid) * D + nd * 8 + 2 * tig + 1] = o[nd][1];
    }
    if (tig == 0) {
      mm[warp * G + gid] = m_run;
      ml[warp * G + gid] = l_run;
    }
  }
  __syncthreads();
  if (__syncthreads_or(failed ? 1 : 0)) return;
  merge_warps_store<T, D, G>(p, mo, mm, ml, row, ri, kvh, part, nparts == 1);
}

// ---- host side ------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int stages_for(int head_dim) {
  static int env = [] {
    const char *e = std::getenv("MS_ATTN_STAGES");
    return e ? std::atoi(e) : 0;
  }();
  if (env == 2 || env == 3 || env == 4) return env;
  return head_dim == 128 ? 3 : 4;
}

template <typename T, int D, int G, int NSTAGE>
cudaError_t launch_tc_t(const Params &p, const CUtensorMap &km, const CUtensorMap &vm, int num_rows,
                        cudaStream_t stream) {
  auto kern = paged_attention_tc_kernel<T, D, G, NSTAGE>;
  constexpr size_t stage_bytes = size_t(kWarps) * NSTAGE * 2 * (D / 64) * kHalfBytes;
  const size_t merge = (size_t(kWarps) * G * D + 2 * kWarps * G) * sizeof(float);
  const size_t smem = 1024 + std::max(stage_bytes + kWarps * NSTAGE * sizeof(uint64_t), merge);
  static std::atomic<bool> attr_done[64];  // zero-initialised (static storage)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attr_done[dev].store(true, std::memory_order_release);  // setting twice is harmless
  }
  dim3 grid(num_rows, p.num_kv_heads, p.max_parts);
  kern<<<grid, kWarps * 32, smem, stream>>>(km, vm, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_combine<T, D, G>(p, num_rows, stream);
}

template <typename T, int D, int G>
cudaError_t launch_tc_stages(const Params &p, const CUtensorMap &km, const CUtensorMap &vm, int num_rows,
                             cudaStream_t stream) {
  switch (stages_for(D)) {
    case 2: return launch_tc_t<T, D, G, 2>(p, km, vm, num_rows, stream);
    case 4: return launch_tc_t<T, D, G, 4>(p, km, vm, num_rows, stream);
    default: return launch_tc_t<T, D, G, 3>(p, km, vm, num_rows, stream);
  }
}

template <typename T, int D>
cudaError_t launch_tc_group(const Params &p, const CUtensorMap &km, const CUtensorMap &vm, int group,
                            int num_rows, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_tc_stages<T, D, 1>(p, km, vm, num_rows, stream);
    case 2: return launch_tc_stages<T, D, 2>(p, km, vm, num_rows, stream);
    case 4: return launch_tc_stages<T, D, 4>(p, km, vm, num_rows, stream);
    case 7: return launch_tc_stages<T, D, 7>(p, km, vm, num_rows, stream);
    case 8: return launch_tc_stages<T, D, 8>(p, km, vm, num_rows, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_tc_dim(const Params &p, const CUtensorMap &km, const CUtensorMap &vm, int head_dim, int group,
                          int num_rows, cudaStream_t stream) {
  if (head_dim == 128) return launch_tc_group<T, 128>(p, km, vm, group, num_rows, stream);
  return launch_tc_group<T, 64>(p, km, vm, group, num_rows, stream);
}

}  // namespace

bool attention_tc_supported(int dtype, int head_dim, int group) {
  if (dtype != MS_DTYPE_BF16 && dtype != MS_DTYPE_F16) return false;
  if (head_dim != 64 && head_dim != 128) return false;
  if (group != 1 && group != 2 && group != 4 && group != 7 && group != 8) return false;
  return encode_fn() != nullptr;
}

cudaError_t launch_attention_tc(const Params &p, const AttnArgs &a, int group, cudaStream_t stream) {
  CUtensorMap km, vm;
  const int64_t tiles = a.pool_tiles > 0 ? a.pool_tiles : (int64_t(1) << 31) - 1;
  if (a.k_map) {
    km = *static_cast<const CUtensorMap *>(a.k_map);
  } else if (!encode_pool_tensor_map(&km, a.k_pool, a.dtype, a.head_dim, tiles)) {
    return cudaErrorInvalidValue;
  }
  if (a.v_map) {
    vm = *static_cast<const CUtensorMap *>(a.v_map);
  } else if (!encode_pool_tensor_map(&vm, a.v_pool, a.dtype, a.head_dim, tiles)) {
    return cudaErrorInvalidValue;
  }
  if (a.dtype == MS_DTYPE_BF16) return launch_tc_dim<__nv_bfloat16>(p, km, vm, a.head_dim, group, a.num_rows, stream);
  return launch_tc_dim<__half>(p, km, vm, a.head_dim, group, a.num_rows, stream);
}

}  // namespace attn

bool attention_tc_available(int dtype, int head_dim, int group) {
  return attn::attention_tc_supported(dtype, head_dim, group);
}

bool encode_pool_tensor_map(void *map_out, const void *pool, int dtype, int head_dim, int64_t pool_tiles) {
  auto fn = attn::encode_fn();
  if (!fn || !map_out || !pool || pool_tiles <= 0 || (head_dim != 64 && head_dim != 128)) return false;
  if (reinterpret_cast<uintptr_t>(pool) % 16 != 0) return false;
  // pool [tiles = pages * kv_heads][16 tokens][D] viewed as 4-D
  // {64 dims, D/64 halves, 16 tokens, tiles}, boxes of {64, 1, 16, 1}
  const cuuint64_t dims[4] = {64, cuuint64_t(head_dim / 64), 16, cuuint64_t(pool_tiles)};
  const cuuint64_t strides[3] = {128, cuuint64_t(head_dim) * 2, cuuint64_t(head_dim) * 2 * 16};
  const cuuint32_t box[4] = {64, 1, 16, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType t =
      dtype == MS_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(static_cast<CUtensorMap *>(map_out), t, 4, const_cast<void *>(pool), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace ms
