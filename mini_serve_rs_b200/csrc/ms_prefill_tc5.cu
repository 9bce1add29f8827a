// K3p on the 5th-generation tensor cores: ragged paged causal prefill with
// tcgen05.mma, accumulators in tensor memory (TMEM).
//
// Same contract as the mma.sync build (ms_prefill_tc.cu; the prefill branch
// of Attention::forward, src/backends/qwen2.rs:329-345, causal mask of
// :476-503 incl. the offset columns of a cached prefix), but a CTA takes 128
// query rows: TPB = 128 / RPT tokens x the G query heads of one KV head
// (RPT = G rounded up to 1, 2, 4 or 8; padding rows are masked).  Thread t
// owns row t, which is TMEM lane t, so the softmax needs no shuffles.
//
// Per group of 64 keys (4 pages of the sequence, landed by TMA in one of two
// stages, 128-byte swizzle):
//   1. thread 0 issues S = Q K^T: D/16 tcgen05.mma (M 128, N 64, K 16) with Q
//      and K read from shared memory through K-major descriptors, S in TMEM
//      columns [0, 64); tcgen05.commit -> mbarrier;
//   2. every thread tcgen05.ld's its row of S, masks (key <= its position),
//      and runs the online softmax in base 2.  The running max is only moved
//      when the tile's max exceeds it by more than 8 (then O and l are
//      rescaled: tcgen05.ld / st of the row), so P = 2^(s - m) stays <= 256;
//   3. P (rounded to the K/V type) overwrites the group's K tile -- the S MMA
//      has consumed it -- in the K-major swizzled layout, V rows of keys past
//      the sequence are zeroed, fence.proxy.async, CTA barrier;
//   4. thread 0 issues O += P V: 4 tcgen05.mma (M 128, N D, K 16) with V as an
//      MN-major operand, O in TMEM columns [64, 64 + D).
// The next group's S MMA is issued after this PV MMA by the same thread, so
// its completion implies the PV finished: the stage it used is then refilled
// two groups ahead.  At the end each thread loads its O row, divides by l and
// stores it.  Shared memory: Q (128 x D) + 2 stages of K/P and V (64 keys x D)
// = 96 KiB for D = 128, so two CTAs share an SM and overlap one CTA's softmax
// with the other's MMAs; TMEM: 256 columns per CTA (128 for D = 64).
//
// Every wait is bounded (mbarrier polls); on expiry the CTA records
// kStatusWaitTimeout, drains its copies and MMAs (bounded), frees TMEM and
// returns.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "ms_attention_common.cuh"

namespace ms {
namespace attn {
namespace {

constexpr int kRows = 128;     // query rows per CTA = TMEM lanes
constexpr int kKeys = 64;      // keys per group (4 pages)
constexpr float kRescale = 8.0f;  // move the running max only when it grows by more than 2^8

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = uint64_t((addr >> 4) & 0x3fff);
  d |= uint64_t((lbo_bytes >> 4) & 0x3fff) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3fff) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  d |= uint64_t(2) << 61;  // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: f32 accumulate, A and B of the same
// 16-bit type (bf16: format 1, f16: format 0), K-major A.
template <typename T>
__device__ __forceinline__ uint32_t umma_idesc(int M, int N, int b_mn_major) {
  constexpr uint32_t f = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | (uint32_t(b_mn_major) << 16) | (uint32_t(N >> 3) << 17) |
         (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t addr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <typename T> __device__ __forceinline__ uint32_t pack_pair(float a, float b);
template <> __device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack_pair<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

template <int G> struct RowsPerTok5 { static constexpr int value = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; };

struct Prefill5Params {
  const void *q;
  void *out;
  const int32_t *block_tables;
  const int32_t *tiles;  // [num_tiles][4]: first packed row, rows, position of first row, table row
  unsigned *status;
  int max_blocks_per_seq;
  int num_kv_heads;
  float qscale;
};

template <typename T, int D, int G>
__global__ void __launch_bounds__(kRows) paged_prefill_tc5_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                  const __grid_constant__ CUtensorMap vmap,
                                                                  Prefill5Params p) {
  constexpr int RPT = RowsPerTok5<G>::value;
  constexpr int NDH = D / 64;                          // 64-dim (128-byte) halves
  constexpr int QHALF = kRows * 128;                   // one 64-dim half of the Q tile
  constexpr int KVHALF = kKeys * 128;                  // one 64-dim half of a 64-key K or V tile
  constexpr int KV_BYTES = NDH * KVHALF;
  constexpr int KP_BYTES = KV_BYTES > kRows * 128 ? KV_BYTES : kRows * 128;  // K tile, then P (128 x 64 keys)
  constexpr int STAGE_BYTES = KP_BYTES + KV_BYTES;     // K/P tile, V tile
  constexpr int PAGE_HALF = kBS * 128;                 // one TMA box: 16 keys x 64 dims
  constexpr int TMEM_COLS = kKeys + D <= 128 ? 128 : 256;  // S, then O

  extern __shared__ unsigned char smem_dyn[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  unsigned char *sq = smem;                            // Q: NDH halves of 128 rows x 128 B
  unsigned char *stages = smem + NDH * QHALF;
  __shared__ uint64_t full[2], s_done, o_done, drain;
  __shared__ uint32_t tmem_base;
  __shared__ int failed_s;

  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5;
  const int row0 = p.tiles[tile * 4 + 0], nrows = p.tiles[tile * 4 + 1];
  const int pos0 = p.tiles[tile * 4 + 2], trow = p.tiles[tile * 4 + 3];
  const int32_t *table = p.block_tables + size_t(trow) * p.max_blocks_per_seq;
  const int kv_len = pos0 + nrows;
  const int npages = (kv_len + kBS - 1) / kBS;
  const int ngroups = (kv_len + kKeys - 1) / kKeys;

  // this thread's query row
  const int tok = t / RPT, head = t % RPT;
  const bool rvalid = head < G && tok < nrows;
  const int pos = rvalid ? pos0 + tok : -1;

  if (t == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&s_done, 1);
    mbar_init(&o_done, 1);
    mbar_init(&drain, 1);
    failed_s = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }

  auto issue = [&](int grp) {  // thread 0: the group's existing pages into stage grp & 1
    const int s = grp & 1;
    unsigned char *kst = stages + size_t(s) * STAGE_BYTES, *vst = kst + KP_BYTES;
    const int first = grp * (kKeys / kBS), n = min(kKeys / kBS, npages - first);
    mbar_expect_tx(&full[s], uint32_t(n) * 2 * NDH * PAGE_HALF);
    for (int j = 0; j < n; ++j) {
      const int tl = table[first + j] * p.num_kv_heads + kvh;
#pragma unroll
      for (int dh = 0; dh < NDH; ++dh) {
        tma_load_4d(kst + dh * KVHALF + j * PAGE_HALF, &kmap, 0, dh, 0, tl, &full[s]);
        tma_load_4d(vst + dh * KVHALF + j * PAGE_HALF, &vmap, 0, dh, 0, tl, &full[s]);
      }
    }
  };

  // Q row t -> K-major swizzled tile (zeros for padding rows)
  {
    const T *qr = static_cast<const T *>(p.q) +
                  ((size_t(row0) + (rvalid ? tok : 0)) * p.num_kv_heads * G + size_t(kvh) * G + (rvalid ? head : 0)) * D;
#pragma unroll
    for (int dh = 0; dh < NDH; ++dh)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = rvalid ? reinterpret_cast<const uint4 *>(qr + dh * 64)[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(sq + dh * QHALF + t * 128 + ((c ^ (t & 7)) << 4)) = v;
      }
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t tm_s = tmem, tm_o = tmem + kKeys;  // S columns [0, 64), O columns [64, 64 + D)
  (void)failed_s;
  const uint32_t lane_off = uint32_t(warp * 32) << 16;
  if (t == 0) {
    issue(0);
    if (ngroups > 1) issue(1);
  }

  const uint32_t id_s = umma_idesc<T>(kRows, kKeys, 0), id_o = umma_idesc<T>(kRows, D, 1);
  float m_run = -INFINITY, l_run = 0.f;
  bool failed = false;
  int issued_groups = min(2, ngroups), landed = 0;  // (thread 0) groups issued / seen landed
  for (int g = 0; g < ngroups; ++g) {
    const int s = g & 1;
    unsigned char *kst = stages + size_t(s) * STAGE_BYTES, *vst = kst + KP_BYTES;
    const int key0 = g * kKeys;
    // 1. S = Q K^T (thread 0), after the stage landed
    if (t == 0) {
      if (mbar_wait_bounded(&full[s], (g >> 1) & 1)) {
        landed = g + 1;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk & 3) * 32;  // 16 dims further within the 128-byte row
          const uint64_t a = umma_desc_sw128(smem_addr(sq + (kk >> 2) * QHALF) + off, 16, 1024);
          const uint64_t b = umma_desc_sw128(smem_addr(kst + (kk >> 2) * KVHALF) + off, 16, 1024);
          umma(tm_s, a, b, id_s, kk > 0);
        }
      } else {
        failed_s = 1;
      }
      umma_commit(&s_done);
    }
    if (!mbar_wait_bounded(&s_done, g & 1)) failed = true;
    tc_fence_after();
    if (__syncthreads_or(failed || failed_s)) {
      failed = true;
      break;
    }
    // the PV MMA of group g - 1 is complete (issued before this S): refill its stage
    if (t == 0 && g >= 1 && g + 1 < ngroups) {
      fence_proxy_async();
      issue(g + 1);
      issued_groups = g + 2;
    }
    // 2. softmax on this thread's row
    float sv[kKeys];
    {
      float a[32];
      tmem_ld32(tm_s + lane_off, a);
#pragma unroll
      for (int i = 0; i < 32; ++i) sv[i] = a[i];
      tmem_ld32(tm_s + lane_off + 32, a);
#pragma unroll
      for (int i = 0; i < 32; ++i) sv[32 + i] = a[i];
    }
    float mt = -INFINITY;
#pragma unroll
    for (int i = 0; i < kKeys; ++i) {
      sv[i] = (key0 + i <= pos) ? sv[i] * p.qscale : -INFINITY;  // causal (and length: pos < kv_len)
      mt = fmaxf(mt, sv[i]);
    }
    const bool grow = mt > m_run + kRescale || (m_run == -INFINITY && mt > -INFINITY);
    float alpha = 1.f;
    if (grow) {
      alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - mt);
      m_run = mt;
    }
    // rescale O in TMEM (warp-collective) when any row of the warp moved its max after O started
    if (g > 0 && __any_sync(kFull, grow && alpha != 1.f)) {
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        float o[32];
        tmem_ld32(tm_o + lane_off + c0, o);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= alpha;
        tmem_st32(tm_o + lane_off + c0, o);
      }
    }
    float psum = 0.f;
#pragma unroll
    for (int i = 0; i < kKeys; ++i) {
      sv[i] = (sv[i] == -INFINITY) ? 0.f : exp2f(sv[i] - m_run);
      psum += sv[i];
    }
    l_run = l_run * alpha + psum;
    // 3. P over the consumed K tile (64 keys = one 128-byte row per query row)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 w;
      w.x = pack_pair<T>(sv[8 * c + 0], sv[8 * c + 1]);
      w.y = pack_pair<T>(sv[8 * c + 2], sv[8 * c + 3]);
      w.z = pack_pair<T>(sv[8 * c + 4], sv[8 * c + 5]);
      w.w = pack_pair<T>(sv[8 * c + 6], sv[8 * c + 7]);
      *reinterpret_cast<uint4 *>(kst + t * 128 + ((c ^ (t & 7)) << 4)) = w;
    }
    // V rows of keys past the sequence (stale, or pages never loaded) -> 0
    const int vk = kv_len - key0;  // valid keys of this group
    if (vk < kKeys)
      for (int i = t; i < (kKeys - vk) * 8 * NDH; i += kRows) {
        const int dh = i / ((kKeys - vk) * 8), rem = i % ((kKeys - vk) * 8);
        *reinterpret_cast<uint4 *>(vst + dh * KVHALF + (vk + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
      }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    // 4. O += P V (thread 0)
    if (t == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kKeys / 16; ++kk) {
        const uint64_t a = umma_desc_sw128(smem_addr(kst) + kk * 32, 16, 1024);
        const uint64_t b = umma_desc_sw128(smem_addr(vst) + kk * 2048, KVHALF, 1024);
        umma(tm_o, a, b, id_o, (g > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&o_done);
    }
  }

  // drain: every MMA issued by thread 0 and every copy issued is complete
  bool ok_end = !failed;
  if (t == 0) {
    umma_commit(&drain);
    for (int g = landed; g < issued_groups; ++g)
      if (!mbar_wait_bounded(&full[g & 1], (g >> 1) & 1)) ok_end = false;
  }
  if (!mbar_wait_bounded(&drain, 0)) ok_end = false;
  tc_fence_after();
  if (__syncthreads_and(ok_end)) {
    // O row / l -> out; every thread takes part in the warp-collective TMEM loads
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    T *orow = static_cast<T *>(p.out) +
              ((size_t(row0) + (rvalid ? tok : 0)) * p.num_kv_heads * G + size_t(kvh) * G + (rvalid ? head : 0)) * D;
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 32) {
      float o[32];
      tmem_ld32(tm_o + lane_off + c0, o);
      if (rvalid) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_pair<T>(o[i] * inv, o[i + 1] * inv);
          w.y = pack_pair<T>(o[i + 2] * inv, o[i + 3] * inv);
          w.z = pack_pair<T>(o[i + 4] * inv, o[i + 5] * inv);
          w.w = pack_pair<T>(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4 *>(orow + c0 + i) = w;
        }
      }
    }
  } else if (t == 0) {
    atomicOr(p.status, kStatusWaitTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

template <typename T, int D, int G>
cudaError_t launch_t5(const Prefill5Params &p, const CUtensorMap &km, const CUtensorMap &vm, int num_tiles,
                      cudaStream_t stream) {
  auto kern = paged_prefill_tc5_kernel<T, D, G>;
  constexpr int NDH = D / 64;
  constexpr int KV_BYTES = NDH * kKeys * 128;
  constexpr int KP_BYTES = KV_BYTES > kRows * 128 ? KV_BYTES : kRows * 128;
  const size_t smem = 1024 + size_t(NDH) * kRows * 128 + 2 * size_t(KP_BYTES + KV_BYTES);
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  dim3 grid(num_tiles, p.num_kv_heads);
  kern<<<grid, kRows, smem, stream>>>(km, vm, p);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t t5_group(const Prefill5Params &p, const CUtensorMap &km, const CUtensorMap &vm, int group, int num_tiles,
                     cudaStream_t stream) {
  switch (group) {
    case 1: return launch_t5<T, D, 1>(p, km, vm, num_tiles, stream);
    case 2: return launch_t5<T, D, 2>(p, km, vm, num_tiles, stream);
    case 4: return launch_t5<T, D, 4>(p, km, vm, num_tiles, stream);
    case 7: return launch_t5<T, D, 7>(p, km, vm, num_tiles, stream);
    case 8: return launch_t5<T, D, 8>(p, km, vm, num_tiles, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

// Whether the tcgen05 build runs prefill tiles (MS_PREFILL_TC5=0 selects the
// mma.sync build); the tile size (tokens per tile) depends on it.
bool prefill_tc5_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("MS_PREFILL_TC5");
    return !(e && e[0] == '0');
  }();
  return on;
}

int prefill_tc5_tokens_per_tile(int group) {
  const int rpt = group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8;
  return kRows / rpt;
}

cudaError_t launch_prefill_tc5(const void *q, void *out, const int32_t *block_tables, int max_blocks_per_seq,
                               const int32_t *tiles, int num_tiles, int num_kv_heads, int group, int head_dim,
                               float scale, unsigned *status, int dtype, const CUtensorMap &km, const CUtensorMap &vm,
                               cudaStream_t stream) {
  Prefill5Params p;
  p.q = q;
  p.out = out;
  p.block_tables = block_tables;
  p.tiles = tiles;
  p.status = status;
  p.max_blocks_per_seq = max_blocks_per_seq;
  p.num_kv_heads = num_kv_heads;
  p.qscale = scale * kLog2e;
  if (dtype == MS_DTYPE_BF16) {
    if (head_dim == 128) return t5_group<__nv_bfloat16, 128>(p, km, vm, group, num_tiles, stream);
    if (head_dim == 64) return t5_group<__nv_bfloat16, 64>(p, km, vm, group, num_tiles, stream);
  } else if (dtype == MS_DTYPE_F16) {
    if (head_dim == 128) return t5_group<__half, 128>(p, km, vm, group, num_tiles, stream);
    if (head_dim == 64) return t5_group<__half, 64>(p, km, vm, group, num_tiles, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace attn
}  // namespace ms
