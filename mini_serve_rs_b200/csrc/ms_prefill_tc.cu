// K3p: ragged paged causal prefill attention on tensor cores (bf16 / f16).
//
// Restates the prefill branch of Attention::forward (src/backends/qwen2.rs:
// 329-345: repeat_kv, causal mask of :476-503 with the seqlen_offset columns
// of a cached prefix, softmax, P.V) without materialising the mask or
// repeating K/V: a CTA takes one tile of a sequence chunk -- TPB query tokens
// x the G query heads of one KV head, 64 rows of the m16 MMA tiles -- and
// streams the sequence's pages (keys 0 .. last query position of the tile)
// through a CTA-shared TMA ring.  Every page is used by all four warps
// (16 rows each): S = Q K^T (mma.m16n8k16), causal / length mask, online
// softmax in base 2, O += P V.  Pages beyond a warp's causal range are
// skipped by that warp.  Stale keys past the sequence's length in its last
// page are masked in S and their V fragments zeroed in registers.
#include <algorithm>
#include <atomic>
#include <array>
#include <vector>
#include <mutex>

#include "ms_attention_common.cuh"

namespace ms {
namespace attn {
namespace {

constexpr int kHalfBytes = 16 * 64 * 2;

template <typename T> __device__ __forceinline__ uint32_t pack2p(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2p<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2p<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ uint32_t tile_off_p(int token, int dim) {
  const int dh = dim >> 6, c = (dim & 63) >> 3;
  return uint32_t(dh * kHalfBytes + token * 128 + ((c ^ (token & 7)) << 4));
}

// rows of the m16 tile per query token: G rounded up to a divisor of 16
template <int G> struct RowsPerToken { static constexpr int value = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; };

struct PrefillParams {
  const void *q;
  void *out;
  const int32_t *block_tables;
  const int32_t *tiles;  // [num_tiles][4]: first packed row, rows, position of first row, table row
  unsigned *status;
  int max_blocks_per_seq;
  int num_kv_heads;
  float qscale;
};

template <typename T, int D, int G, int NSTAGE>
__global__ void __launch_bounds__(kWarps * 32)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                            PrefillParams p) {
  constexpr int RPT = RowsPerToken<G>::value;
  constexpr int TPW = 16 / RPT;  // query tokens per warp
  constexpr int NDH = D / 64;
  constexpr int TILE_BYTES = NDH * kHalfBytes;
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int KSTEPS = D / 16;
  constexpr int NTD = D / 8;

  extern __shared__ unsigned char smem_dyn[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + size_t(NSTAGE) * STAGE_BYTES);

  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int row0 = p.tiles[tile * 4 + 0], nrows = p.tiles[tile * 4 + 1];
  const int pos0 = p.tiles[tile * 4 + 2], trow = p.tiles[tile * 4 + 3];
  const int32_t *table = p.block_tables + size_t(trow) * p.max_blocks_per_seq;
  const int kv_len = pos0 + nrows;                 // keys 0 .. kv_len-1 exist for this tile
  const int npages = (kv_len + kBS - 1) / kBS;

  // this lane's two m16 rows: gid and gid + 8 of the warp's tile
  int tok_l[2], head[2], pos[2];
  bool rvalid[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int m = gid + 8 * r;
    tok_l[r] = warp * TPW + m / RPT;
    head[r] = m % RPT;
    rvalid[r] = head[r] < G && tok_l[r] < nrows;
    pos[r] = rvalid[r] ? pos0 + tok_l[r] : -1;
  }
  // highest key any row of this warp may see
  const int warp_last_tok = min(nrows - 1, warp * TPW + TPW - 1);
  const int warp_max_pos = warp_last_tok >= warp * TPW ? pos0 + warp_last_tok : -1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
    fence_proxy_async();
  }
  __syncthreads();

  auto issue = [&](int s, int page_idx) {  // thread 0 only
    const int pg = table[page_idx];
    unsigned char *st = smem + size_t(s) * STAGE_BYTES;
    const int tl = pg * p.num_kv_heads + kvh;
    mbar_expect_tx(&full[s], STAGE_BYTES);
#pragma unroll
    for (int dh = 0; dh < NDH; ++dh) {
      tma_load_4d(st + dh * kHalfBytes, &kmap, 0, dh, 0, tl, &full[s]);
      tma_load_4d(st + TILE_BYTES + dh * kHalfBytes, &vmap, 0, dh, 0, tl, &full[s]);
    }
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < min(NSTAGE, npages); ++k) issue(k, k);

  // Q fragments for rows gid (a0, a2) and gid+8 (a1, a3)
  uint32_t qa[KSTEPS][4];
  {
    const T *qb = static_cast<const T *>(p.q);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const T *qr = qb + ((size_t(row0) + (rvalid[r] ? tok_l[r] : 0)) * p.num_kv_heads * G + size_t(kvh) * G +
                          (rvalid[r] ? head[r] : 0)) * D;
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        qa[kk][r] = rvalid[r] ? *reinterpret_cast<const uint32_t *>(qr + kk * 16 + 2 * tig) : 0u;
        qa[kk][2 + r] = rvalid[r] ? *reinterpret_cast<const uint32_t *>(qr + kk * 16 + 8 + 2 * tig) : 0u;
      }
    }
  }
  float o[NTD][4];
#pragma unroll
  for (int nd = 0; nd < NTD; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int mi = lane >> 3, ri = lane & 7;

  bool failed = false;
  int kdone = 0;
  for (int k = 0; k < npages; ++k) {
    const int s = k % NSTAGE;
    const uint32_t ph = (k / NSTAGE) & 1;
    const bool ok = __all_sync(kFull, mbar_wait_bounded(&full[s], ph));  // warp-uniform
    const int key0 = k * kBS;
    if (ok && key0 <= warp_max_pos) {  // warp-uniform: some row of this warp sees this page
      unsigned char *st = smem + size_t(s) * STAGE_BYTES;
      const uint32_t kb = smem_addr(st), vb = kb + TILE_BYTES;
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        uint32_t b[4];
        ldmatrix_x4(b, kb + tile_off_p((mi >> 1) * 8 + ri, kk * 16 + (mi & 1) * 8));
        const uint32_t a[4] = {qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]};
        mma_16816<T>(sc[0], a, b[0], b[1]);
        mma_16816<T>(sc[1], a, b[2], b[3]);
      }
      // per row r: keys key0 + {2tig, 2tig+1, 8+2tig, 9+2tig}; C regs r*2 + {0,1}
      float pr[2][4];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float sv[4] = {sc[0][2 * r], sc[0][2 * r + 1], sc[1][2 * r], sc[1][2 * r + 1]};
        const int kt[4] = {key0 + 2 * tig, key0 + 2 * tig + 1, key0 + 8 + 2 * tig, key0 + 9 + 2 * tig};
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sv[j] = (kt[j] <= pos[r]) ? sv[j] * p.qscale : -INFINITY;  // causal (and length: pos < kv_len)
          mx = fmaxf(mx, sv[j]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
        const float m_new = fmaxf(m_run[r], mx);
        const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_run[r] - m_new);
        float psum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          pr[r][j] = (sv[j] == -INFINITY) ? 0.f : exp2f(sv[j] - m_new);
          psum += pr[r][j];
        }
        l_run[r] = l_run[r] * alpha + psum;
        m_run[r] = m_new;
#pragma unroll
        for (int nd = 0; nd < NTD; ++nd) {
          o[nd][2 * r] *= alpha;
          o[nd][2 * r + 1] *= alpha;
        }
      }
      const uint32_t pa[4] = {pack2p<T>(pr[0][0], pr[0][1]), pack2p<T>(pr[1][0], pr[1][1]),
                              pack2p<T>(pr[0][2], pr[0][3]), pack2p<T>(pr[1][2], pr[1][3])};
      // V fragments hold keys key0 + 2tig, +1 (b0) and key0 + 8 + 2tig, +1 (b1): zero stale keys
      const bool partial = key0 + kBS > kv_len;
      uint32_t vmask0 = 0xffffffffu, vmask1 = 0xffffffffu;
      if (partial) {
        const int k0 = key0 + 2 * tig, k1 = key0 + 8 + 2 * tig;
        vmask0 = (k0 < kv_len ? 0x0000ffffu : 0u) | (k0 + 1 < kv_len ? 0xffff0000u : 0u);
        vmask1 = (k1 < kv_len ? 0x0000ffffu : 0u) | (k1 + 1 < kv_len ? 0xffff0000u : 0u);
      }
#pragma unroll
      for (int ndp = 0; ndp < NTD / 2; ++ndp) {
        uint32_t b[4];
        ldmatrix_x4_trans(b, vb + tile_off_p((mi & 1) * 8 + ri, (2 * ndp + (mi >> 1)) * 8));
        b[0] &= vmask0;
        b[1] &= vmask1;
        b[2] &= vmask0;
        b[3] &= vmask1;
        mma_16816<T>(o[2 * ndp], pa, b[0], b[1]);
        mma_16816<T>(o[2 * ndp + 1], pa, b[2], b[3]);
      }
    }
    // every warp is done with stage s (and agrees on failure) before it is refilled
    if (__syncthreads_or(ok ? 0 : 1)) {
      failed = true;
      kdone = k;
      break;
    }
    kdone = k + 1;
    if (threadIdx.x == 0 && k + NSTAGE < npages) {
      fence_proxy_async();
      issue(s, k + NSTAGE);
    }
  }
  if (failed) {
    if (threadIdx.x == 0) {
      atomicOr(p.status, kStatusWaitTimeout);
      // drain the copies still in flight (bounded)
      for (int k = kdone; k < min(npages, kdone + NSTAGE); ++k) mbar_wait_bounded(&full[k % NSTAGE], (k / NSTAGE) & 1);
    }
  }
  if (__syncthreads_or(failed ? 1 : 0)) return;

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(kFull, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(kFull, l_run[r], 2);
  }
  T *ob = static_cast<T *>(p.out);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!rvalid[r]) continue;
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
    T *orow = ob + ((size_t(row0) + tok_l[r]) * p.num_kv_heads * G + size_t(kvh) * G + head[r]) * D;
#pragma unroll
    for (int nd = 0; nd < NTD; ++nd) {
      const float v2[2] = {o[nd][2 * r] * inv, o[nd][2 * r + 1] * inv};
      Vec2<T>::store(orow + nd * 8 + 2 * tig, v2);
    }
  }
}


template <typename T, int D, int G>
cudaError_t launch_prefill_t(const PrefillParams &p, const CUtensorMap &km, const CUtensorMap &vm, int num_tiles,
                             cudaStream_t stream) {
  constexpr int NSTAGE = 3;
  auto kern = paged_prefill_tc_kernel<T, D, G, NSTAGE>;
  const size_t smem = 1024 + size_t(NSTAGE) * 2 * (D / 64) * kHalfBytes + NSTAGE * sizeof(uint64_t);
  static std::atomic<bool> attr_done[64];  // zero-initialised (static storage)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attr_done[dev].store(true, std::memory_order_release);  // setting twice is harmless
  }
  dim3 grid(num_tiles, p.num_kv_heads);
  kern<<<grid, kWarps * 32, smem, stream>>>(km, vm, p);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t prefill_group(const PrefillParams &p, const CUtensorMap &km, const CUtensorMap &vm, int group,
                          int num_tiles, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_prefill_t<T, D, 1>(p, km, vm, num_tiles, stream);
    case 2: return launch_prefill_t<T, D, 2>(p, km, vm, num_tiles, stream);
    case 4: return launch_prefill_t<T, D, 4>(p, km, vm, num_tiles, stream);
    case 7: return launch_prefill_t<T, D, 7>(p, km, vm, num_tiles, stream);
    case 8: return launch_prefill_t<T, D, 8>(p, km, vm, num_tiles, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace
// tcgen05 build (ms_prefill_tc5.cu)
bool prefill_tc5_enabled();
int prefill_tc5_tokens_per_tile(int group);
cudaError_t launch_prefill_tc5(const void *q, void *out, const int32_t *block_tables, int max_blocks_per_seq,
                               const int32_t *tiles, int num_tiles, int num_kv_heads, int group, int head_dim,
                               float scale, unsigned *status, int dtype, const void *k_pool, const void *v_pool,
                               cudaStream_t stream);
}  // namespace attn

int prefill_tokens_per_tile(int group) {
  if (attn::prefill_tc5_enabled()) return attn::prefill_tc5_tokens_per_tile(group);
  const int rpt = group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8;
  return attn::kWarps * (16 / rpt);
}

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
  if (attn::prefill_tc5_enabled())
    return attn::launch_prefill_tc5(a.q, a.out, a.block_tables, a.max_blocks_per_seq, a.tiles, a.num_tiles,
                                    a.num_kv_heads, group, a.head_dim, a.scale, status, a.dtype, a.k_pool, a.v_pool,
                                    stream);
  CUtensorMap km, vm;
  const int64_t tiles = a.pool_tiles > 0 ? a.pool_tiles : (int64_t(1) << 31) - 1;
  if (a.k_map) km = *static_cast<const CUtensorMap *>(a.k_map);
  else if (!encode_pool_tensor_map(&km, a.k_pool, a.dtype, a.head_dim, tiles)) return cudaErrorInvalidValue;
  if (a.v_map) vm = *static_cast<const CUtensorMap *>(a.v_map);
  else if (!encode_pool_tensor_map(&vm, a.v_pool, a.dtype, a.head_dim, tiles)) return cudaErrorInvalidValue;
  attn::PrefillParams p;
  p.q = a.q;
  p.out = a.out;
  p.block_tables = a.block_tables;
  p.tiles = a.tiles;
  p.max_blocks_per_seq = a.max_blocks_per_seq;
  p.num_kv_heads = a.num_kv_heads;
  p.qscale = a.scale * attn::kLog2e;
  p.status = status;
  if (a.dtype == MS_DTYPE_BF16) {
    return a.head_dim == 128 ? attn::prefill_group<__nv_bfloat16, 128>(p, km, vm, group, a.num_tiles, stream)
                             : attn::prefill_group<__nv_bfloat16, 64>(p, km, vm, group, a.num_tiles, stream);
  }
  return a.head_dim == 128 ? attn::prefill_group<__half, 128>(p, km, vm, group, a.num_tiles, stream)
                           : attn::prefill_group<__half, 64>(p, km, vm, group, a.num_tiles, stream);
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
