// K3: split-K paged GQA attention for sm_100a.
//
// Replaces decode_attention_gqa_zero_copy (src/backends/qwen2.rs:182-203) and
// the per-sequence loop around it (qwen2.rs:722-746), and supersedes the
// reference's prototype paged_gqa_decode_tiled_kernel
// (docs/colab_cuda_kernels/mini_serve_kernels.cu:191-245).
//
// Pool layout (the prototype's, mini_serve_kernels.cu:193-195):
//   k_pool / v_pool [num_blocks, num_kv_heads, 16, head_dim]
// so the 16 x head_dim tile of one (page, kv head) is contiguous (4 KiB for
// bf16 / 128).  Work unit = one CTA per (query row, kv head, partition of
// `partition_blocks` pages).  The CTA's 4 warps take pages round-robin; each
// warp streams its pages through a private ring of shared-memory stages filled
// by TMA bulk copies (cp.async.bulk, no multicast) completing on per-stage
// mbarriers.  All query heads of the kv head are served from one K/V read.
// Scores use a transposed butterfly reduction (16*G partial dot products
// reduced across the warp in log2(32) rounds); softmax is online in base 2;
// warps merge in shared memory, partitions merge in a second kernel by
// log-sum-exp.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "ms_attention_common.cuh"

namespace ms {
namespace attn {

// ---- transposed butterfly: NVP partial values per lane -> NVP/32 totals ------
// After the call, lane L holds in v[j] the warp-wide sum of original index
// L * (NVP/32) + j.
template <int N, int OFF> struct Butterfly {
  static __device__ __forceinline__ void run(float *v, int lane) {
    const bool up = (lane & OFF) != 0;
#pragma unroll
    for (int j = 0; j < N / 2; ++j) {
      float send = up ? v[j] : v[j + N / 2];
      float keep = up ? v[j + N / 2] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, OFF);
    }
    Butterfly<N / 2, OFF / 2>::run(v, lane);
  }
};
template <int N> struct Butterfly<N, 0> {
  static __device__ __forceinline__ void run(float *, int) {}
};

template <typename T, int D> struct TileLoad {
  static constexpr int DPL = D / 32;
  static __device__ __forceinline__ void load(const T *row, int lane, float (&o)[DPL]) {
    if constexpr (DPL == 4) {
      Vec4<T>::load(row + lane * 4, o);
    } else {
      Vec2<T>::load(row + lane * 2, o);
    }
  }
};


template <typename T, int D, int G, int NSTAGE>
__global__ void __launch_bounds__(kWarps * 32) paged_attention_kernel(Params p) {
  constexpr int DPL = D / 32;
  constexpr int SUB = (G > 4) ? 8 : 16;      // tokens per scoring sub-tile
  constexpr int NSUB = kBS / SUB;
  constexpr int NV = G * SUB;
  constexpr int NVP = ((NV + 31) / 32) * 32;
  constexpr int R = NVP / 32;                // totals per lane after the butterfly
  constexpr int LPH = SUB / R;               // lanes per head
  static_assert(LPH * R == SUB && LPH * G <= 32, "lane mapping");
  constexpr int TILE = kBS * D;              // elements per (page, kv head) tile
  constexpr uint32_t TILE_BYTES = TILE * sizeof(T);

  extern __shared__ __align__(128) unsigned char smem_raw[];
  T *stages = reinterpret_cast<T *>(smem_raw);  // [kWarps][NSTAGE][2][TILE]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw + size_t(kWarps) * NSTAGE * 2 * TILE_BYTES);

  const int ri = blockIdx.x;
  const int row = p.row_index ? p.row_index[ri] : ri;
  const int kvh = blockIdx.y;
  const int part = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

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

  // this warp's pages: blk0 + warp + k * kWarps
  const int nb_w = (blk1 - blk0 - warp + kWarps - 1) / kWarps;
  T *my_stage = stages + size_t(warp) * NSTAGE * 2 * TILE;
  uint64_t *my_bar = bars + warp * NSTAGE;
  const T *kbase = static_cast<const T *>(p.k_pool);
  const T *vbase = static_cast<const T *>(p.v_pool);
  const size_t head_off = size_t(kvh) * TILE;
  const size_t page_stride = size_t(p.num_kv_heads) * TILE;

  if (lane == 0) {
    for (int s = 0; s < NSTAGE; ++s) mbar_init(&my_bar[s], 1);
    fence_barrier_init();
    fence_proxy_async();
  }
  __syncwarp();

  // page ids of this warp, 32 at a time in a register (lane k holds page k)
  int page_reg = 0;
  auto page_of = [&](int k) -> int {
    return __shfl_sync(kFull, page_reg, k & 31);
  };
  auto refill_pages = [&](int k0) {
    int k = k0 + lane;
    page_reg = (k < nb_w) ? table[blk0 + warp + k * kWarps] : 0;
  };
  auto issue = [&](int s, int page) {
    if (lane == 0) {
      T *dk = my_stage + size_t(s) * 2 * TILE;
      mbar_expect_tx(&my_bar[s], 2 * TILE_BYTES);
      bulk_g2s(dk, kbase + size_t(page) * page_stride + head_off, TILE_BYTES, &my_bar[s]);
      bulk_g2s(dk + TILE, vbase + size_t(page) * page_stride + head_off, TILE_BYTES, &my_bar[s]);
    }
  };

  // queries of this kv head, pre-scaled for base-2 softmax
  float qv[G][DPL];
  {
    const T *qrow = static_cast<const T *>(p.q) + (size_t(row) * p.num_kv_heads * G + size_t(kvh) * G) * D;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      TileLoad<T, D>::load(qrow + h * D, lane, qv[h]);
#pragma unroll
      for (int d = 0; d < DPL; ++d) qv[h][d] *= p.qscale;
    }
  }

  float m_run[G], acc[G][DPL];
  float l_lane = 0.f;
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m_run[h] = -INFINITY;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[h][d] = 0.f;
  }
  const int hl = lane / LPH;  // head of this lane's score totals (>= G: padding lane)

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
    const uint32_t parity = (k / NSTAGE) & 1;
    // the whole warp agrees before leaving, so no lane is left waiting in a shuffle
    if (!__all_sync(kFull, mbar_wait_bounded(&my_bar[s], parity, p.wait_limit))) {
      failed = true;
      kfail = k;
      break;
    }
    const T *kt = my_stage + size_t(s) * 2 * TILE;
    const T *vt = kt + TILE;
    const int blk = blk0 + warp + k * kWarps;
    const int valid = min(kBS, ctx - blk * kBS);

#pragma unroll
    for (int sub = 0; sub < NSUB; ++sub) {
      const int t0 = sub * SUB;
      if (t0 >= valid) break;  // warp-uniform: the rest of the page is padding
      float v[NVP];
#pragma unroll
      for (int i = 0; i < NVP; ++i) v[i] = 0.f;
#pragma unroll
      for (int t = 0; t < SUB; ++t) {
        if (t0 + t < valid) {
          float kk[DPL];
          TileLoad<T, D>::load(kt + (t0 + t) * D, lane, kk);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            float a = 0.f;
#pragma unroll
            for (int d = 0; d < DPL; ++d) a = fmaf(qv[h][d], kk[d], a);
            v[h * SUB + t] = a;
          }
        }
      }
      Butterfly<NVP, 16>::run(v, lane);
      // lane holds totals for index lane*R + j -> head hl, token (lane*R + j) % SUB
      float mloc = -INFINITY;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const int t = (lane * R + j) % SUB;
        if (hl >= G || t0 + t >= valid) v[j] = -INFINITY;
        mloc = fmaxf(mloc, v[j]);
      }
#pragma unroll
      for (int o = LPH / 2; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(kFull, mloc, o));
      float alpha[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float mb = __shfl_sync(kFull, mloc, h * LPH);
        const float mn = fmaxf(m_run[h], mb);
        alpha[h] = exp2f(m_run[h] - mn);
        m_run[h] = mn;
      }
      float pv[R];
      float mh = -INFINITY;
#pragma unroll
      for (int h = 0; h < G; ++h)
        if (hl == h) mh = m_run[h];
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        pv[j] = (v[j] == -INFINITY) ? 0.f : exp2f(v[j] - mh);
        psum += pv[j];
      }
      float al = 1.f;
#pragma unroll
      for (int h = 0; h < G; ++h)
        if (hl == h) al = alpha[h];
      l_lane = l_lane * al + psum;
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[h][d] *= alpha[h];
#pragma unroll
      for (int t = 0; t < SUB; ++t) {
        if (t0 + t < valid) {
          float vv[DPL];
          TileLoad<T, D>::load(vt + (t0 + t) * D, lane, vv);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const int idx = h * SUB + t;
            const float ph = __shfl_sync(kFull, pv[idx % R], idx / R);
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc[h][d] = fmaf(ph, vv[d], acc[h][d]);
          }
        }
      }
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
    // drain the copies this warp still has in flight (bounded), then leave
    for (int k = kfail; k < issued; ++k) {
      const int s = k % NSTAGE;
      mbar_wait_bounded(&my_bar[s], (k / NSTAGE) & 1);
    }
  }

  // l per head: sum over the head's LPH lanes
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) l_lane += __shfl_xor_sync(kFull, l_lane, o);

  // ---- merge the warps through shared memory (stages are free now) ----------
  __syncthreads();
  float *mo = reinterpret_cast<float *>(smem_raw);       // [kWarps][G][D]
  float *mm = mo + kWarps * G * D;                        // [kWarps][G]
  float *ml = mm + kWarps * G;                            // [kWarps][G]
#pragma unroll
  for (int h = 0; h < G; ++h) {
#pragma unroll
    for (int d = 0; d < DPL; ++d) mo[(warp * G + h) * D + lane * DPL + d] = acc[h][d];
  }
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float lh = __shfl_sync(kFull, l_lane, h * LPH);
    if (lane == 0) {
      mm[warp * G + h] = m_run[h];
      ml[warp * G + h] = lh;
    }
  }
  __syncthreads();
  int any_failed = __syncthreads_or(failed ? 1 : 0);
  if (any_failed) return;

  merge_warps_store<T, D, G>(p, mo, mm, ml, row, ri, kvh, part, nparts == 1);
}

template <typename T, int D, int G>
constexpr int default_stages() {
  return (sizeof(T) * D * kBS * 2 <= 8192) ? 3 : 2;
}

template <typename T, int D, int G>
size_t smem_bytes() {
  constexpr int NSTAGE = default_stages<T, D, G>();
  size_t stages = size_t(kWarps) * NSTAGE * 2 * kBS * D * sizeof(T) + kWarps * NSTAGE * sizeof(uint64_t);
  size_t merge = (size_t(kWarps) * G * D + 2 * kWarps * G) * sizeof(float);
  return std::max(stages, merge);
}

template <typename T, int D, int G>
cudaError_t launch_t(const Params &p, int num_rows, cudaStream_t stream) {
  constexpr int NSTAGE = default_stages<T, D, G>();
  auto kern = paged_attention_kernel<T, D, G, NSTAGE>;
  const size_t smem = smem_bytes<T, D, G>();
  static std::atomic<bool> attr_done[64];  // per device; zero-initialised (static storage)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attr_done[dev].store(true, std::memory_order_release);  // setting twice is harmless
  }
  dim3 grid(num_rows, p.num_kv_heads, p.max_parts);
  kern<<<grid, kWarps * 32, smem, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_combine<T, D, G>(p, num_rows, stream);
}

template <typename T, int D>
cudaError_t dispatch_group(const Params &p, int group, int num_rows, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_t<T, D, 1>(p, num_rows, stream);
    case 2: return launch_t<T, D, 2>(p, num_rows, stream);
    case 4: return launch_t<T, D, 4>(p, num_rows, stream);
    case 7: return launch_t<T, D, 7>(p, num_rows, stream);
    case 8: return launch_t<T, D, 8>(p, num_rows, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t dispatch_dim(const Params &p, int head_dim, int group, int num_rows, cudaStream_t stream) {
  if (head_dim == 128) return dispatch_group<T, 128>(p, group, num_rows, stream);
  if (head_dim == 64) return dispatch_group<T, 64>(p, group, num_rows, stream);
  return cudaErrorInvalidValue;
}

// Device status word of the launches made without an engine status word
// (the prototype-compatible launchers, ms_launch_* with a null status): the
// kernels OR their kStatus* bits into it; ms_kernel_status reads and clears it.
__device__ unsigned g_status_scratch;

// Test hook: >= 0 replaces the poll limit of the page-loop waits (ms_test_set_attention_wait_limit).
std::atomic<int> g_test_wait_limit{-1};

}  // namespace attn

cudaError_t standalone_status_word(unsigned **out) {
  void *sp = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&sp, attn::g_status_scratch);
  if (e == cudaSuccess) *out = static_cast<unsigned *>(sp);
  return e;
}

int choose_partition_blocks(int num_rows, int num_kv_heads, int max_ctx, long long total_blocks) {
  // Aim for >= ~16 CTAs per SM in total while keeping >= 2 pages per warp.
  // Depends on the total work only, not on the longest row: a partition
  // larger than a row is simply that row's single partition, and a graph
  // captured for a context capacity keeps the same partitioning as an eager
  // launch of the same step.
  long long work = std::max<long long>(1, total_blocks) * num_kv_heads;
  const long long target_ctas = 148LL * 16;
  long long pb = (work + target_ctas - 1) / target_ctas;
  pb = std::max<long long>(pb, 2 * attn::kWarps);
  pb = std::min<long long>(pb, 64);
  pb = ((pb + attn::kWarps - 1) / attn::kWarps) * attn::kWarps;
  (void)num_rows;
  (void)max_ctx;
  return int(pb);
}

int64_t attention_workspace_bytes(int num_rows, int num_heads, int max_ctx, int part_blocks) {
  const int max_blk = (max_ctx + attn::kBS - 1) / attn::kBS;
  const int parts = (max_blk + part_blocks - 1) / part_blocks;
  if (parts <= 1) return 0;
  // per (row, q head, part): D floats (bounded by 128) + float2
  return int64_t(num_rows) * num_heads * parts * (128 * 4 + 8) + 256;
}

cudaError_t launch_paged_attention(const AttnArgs &a, cudaStream_t stream) {
  if (a.num_rows <= 0) return cudaSuccess;
  if (a.num_heads <= 0 || a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads != 0 ||
      a.block_size != attn::kBS || a.max_ctx <= 0 || a.part_blocks <= 0)
    return cudaErrorInvalidValue;
  const int group = a.num_heads / a.num_kv_heads;
  attn::Params p;
  p.q = a.q;
  p.k_pool = a.k_pool;
  p.v_pool = a.v_pool;
  p.block_tables = a.block_tables;
  p.row_table = a.row_table;
  p.row_ctx = a.row_ctx;
  p.row_index = a.row_index;
  p.out = a.out;
  p.max_blocks_per_seq = a.max_blocks_per_seq;
  p.num_kv_heads = a.num_kv_heads;
  p.part_blocks = a.part_blocks;
  const int max_blk = (a.max_ctx + attn::kBS - 1) / attn::kBS;
  p.max_parts = (max_blk + a.part_blocks - 1) / a.part_blocks;
  if (p.max_parts > 65535) return cudaErrorInvalidValue;
  p.qscale = a.scale * attn::kLog2e;
  const int test_limit = attn::g_test_wait_limit.load(std::memory_order_relaxed);
  p.wait_limit = test_limit >= 0 ? test_limit : attn::kWaitLimit;
  p.status = a.status;
  if (p.status == nullptr) {
    cudaError_t e = standalone_status_word(&p.status);
    if (e != cudaSuccess) return e;
  }
  p.ws_o = nullptr;
  p.ws_ml = nullptr;
  if (p.max_parts > 1) {
    const size_t n_slots = size_t(a.num_rows) * a.num_kv_heads * p.max_parts;
    const size_t need = n_slots * group * (a.head_dim * sizeof(float) + sizeof(float2));
    if (a.workspace == nullptr || size_t(a.workspace_bytes) < need) return cudaErrorInvalidValue;
    p.ws_o = static_cast<float *>(a.workspace);
    p.ws_ml = reinterpret_cast<float2 *>(static_cast<char *>(a.workspace) +
                                         n_slots * group * a.head_dim * sizeof(float));
  }
  if (attn::attention_tc_supported(a.dtype, a.head_dim, group))
    return attn::launch_attention_tc(p, a, group, stream);
  switch (a.dtype) {
    case 0: return attn::dispatch_dim<float>(p, a.head_dim, group, a.num_rows, stream);
    case 1: return attn::dispatch_dim<__nv_bfloat16>(p, a.head_dim, group, a.num_rows, stream);
    case 2: return attn::dispatch_dim<__half>(p, a.head_dim, group, a.num_rows, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ms

// ---------------------------------------------------------------------------
// C ABI
using ms::AttnArgs;

extern "C" int64_t ms_attention_workspace_bytes(int32_t num_rows, int32_t num_heads, int32_t max_ctx,
                                                int32_t partition_blocks, int32_t block_size) {
  if (block_size != 16 || num_rows <= 0 || max_ctx <= 0) return 0;
  if (partition_blocks <= 0) partition_blocks = ms::choose_partition_blocks(num_rows, 8, max_ctx, 0);
  return ms::attention_workspace_bytes(num_rows, num_heads, max_ctx, partition_blocks);
}

extern "C" int ms_launch_paged_attention(const void *q, const void *k_pool, const void *v_pool,
                                         const int32_t *block_tables, int32_t max_blocks_per_seq,
                                         const int32_t *row_table, const int32_t *row_ctx,
                                         int32_t num_rows, int32_t max_ctx, void *out,
                                         int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                         int32_t block_size, float scale, int32_t partition_blocks,
                                         void *workspace, int64_t workspace_bytes, int32_t dtype,
                                         void *stream) {
  if (num_rows < 0 || max_ctx < 0) return int(cudaErrorInvalidValue);
  if (num_rows == 0) return 0;
  if (partition_blocks <= 0)
    partition_blocks = ms::choose_partition_blocks(num_rows, num_kv_heads, max_ctx,
                                                   (long long)num_rows * ((max_ctx + 15) / 16));
  AttnArgs a{};
  a.q = q;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.block_tables = block_tables;
  a.max_blocks_per_seq = max_blocks_per_seq;
  a.row_table = row_table;
  a.row_ctx = row_ctx;
  a.num_rows = num_rows;
  a.max_ctx = max_ctx;
  a.out = out;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.part_blocks = partition_blocks;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.dtype = dtype;
  a.status = nullptr;
  return int(ms::launch_paged_attention(a, static_cast<cudaStream_t>(stream)));
}

// ---- prototype-compatible launchers (mini_serve_kernels.cu:267-296) -----------
namespace {
struct ProtoWorkspace {
  void *ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_proto_mu;
ProtoWorkspace g_proto_ws[64];

int proto_attention(const void *q, const void *k_pool, const void *v_pool, const int *block_tables,
                    const int *seq_lens, void *out, int batch_size, int num_heads, int num_kv_heads,
                    int max_blocks_per_seq, float scale, int dtype) {
  // argument checks of mini_serve_kernels.cu:272-273
  if (batch_size <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return int(cudaErrorInvalidValue);
  if (max_blocks_per_seq <= 0) return int(cudaErrorInvalidValue);
  const int max_ctx = max_blocks_per_seq * 16;
  const int part = ms::choose_partition_blocks(batch_size, num_kv_heads, max_ctx,
                                               (long long)batch_size * max_blocks_per_seq / 2);
  const int64_t need = ms::attention_workspace_bytes(batch_size, num_heads, max_ctx, part);
  void *ws = nullptr;
  if (need > 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return int(cudaErrorInvalidDevice);
    std::lock_guard<std::mutex> lk(g_proto_mu);
    ProtoWorkspace &w = g_proto_ws[dev];
    if (w.bytes < size_t(need)) {
      if (w.ptr) {
        cudaError_t e = cudaStreamSynchronize(0);
        if (e != cudaSuccess) return int(e);
        cudaFree(w.ptr);
        w.ptr = nullptr;
        w.bytes = 0;
      }
      cudaError_t e = cudaMalloc(&w.ptr, size_t(need));
      if (e != cudaSuccess) return int(e);
      w.bytes = size_t(need);
    }
    ws = w.ptr;
  }
  return ms_launch_paged_attention(q, k_pool, v_pool, block_tables, max_blocks_per_seq, nullptr,
                                   seq_lens, batch_size, max_ctx, out, num_heads, num_kv_heads, 128,
                                   16, scale, part, ws, need, dtype, nullptr);
}
}  // namespace

extern "C" int launch_paged_gqa_decode_tiled_f32(const float *d_q, const float *d_k_pool,
                                                 const float *d_v_pool, const int *d_block_tables,
                                                 const int *d_seq_lens, float *d_out, int batch_size,
                                                 int num_heads, int num_kv_heads,
                                                 int max_blocks_per_seq, float scale) {
  return proto_attention(d_q, d_k_pool, d_v_pool, d_block_tables, d_seq_lens, d_out, batch_size,
                         num_heads, num_kv_heads, max_blocks_per_seq, scale, MS_DTYPE_F32);
}

extern "C" int launch_paged_gqa_decode_tiled_f16(const void *d_q, const void *d_k_pool,
                                                 const void *d_v_pool, const int *d_block_tables,
                                                 const int *d_seq_lens, void *d_out, int batch_size,
                                                 int num_heads, int num_kv_heads,
                                                 int max_blocks_per_seq, float scale) {
  return proto_attention(d_q, d_k_pool, d_v_pool, d_block_tables, d_seq_lens, d_out, batch_size,
                         num_heads, num_kv_heads, max_blocks_per_seq, scale, MS_DTYPE_F16);
}

extern "C" int launch_paged_gqa_decode_tiled_bf16(const void *d_q, const void *d_k_pool,
                                                  const void *d_v_pool, const int *d_block_tables,
                                                  const int *d_seq_lens, void *d_out, int batch_size,
                                                  int num_heads, int num_kv_heads,
                                                  int max_blocks_per_seq, float scale) {
  return proto_attention(d_q, d_k_pool, d_v_pool, d_block_tables, d_seq_lens, d_out, batch_size,
                         num_heads, num_kv_heads, max_blocks_per_seq, scale, MS_DTYPE_BF16);
}

extern "C" int ms_kernel_status(int32_t device, uint32_t *out) {
  if (!out || device < 0) return MS_E_INVALID;
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e == cudaSuccess) e = cudaSetDevice(device);
  if (e != cudaSuccess) return MS_E_DEVICE;
  unsigned v = 0, zero = 0;
  e = cudaDeviceSynchronize();  // every launch made before this call has finished
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, ms::attn::g_status_scratch, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(ms::attn::g_status_scratch, &zero, sizeof(zero));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return MS_E_DEVICE;
  *out = v;
  return MS_OK;
}

extern "C" int ms_test_set_attention_wait_limit(int32_t polls) {
  ms::attn::g_test_wait_limit.store(polls < 0 ? -1 : polls, std::memory_order_relaxed);
  return MS_OK;
}
