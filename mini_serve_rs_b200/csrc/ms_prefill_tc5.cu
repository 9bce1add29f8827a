// K3p on the 5th-generation tensor cores: ragged paged causal prefill with
// tcgen05.mma, accumulators in tensor memory (TMEM).
//
// The prefill branch of Attention::forward (src/backends/qwen2.rs:329-345,
// causal mask of :476-503 incl. the offset columns of a cached prefix) over
// the paged pool; ms_prefill_tc.cu plans the tiles and launches it.  A CTA takes 256
// query rows of one KV head in two halves of 128 (the TMEM lanes), TPH = 128
// / RPT tokens x the G query heads each (RPT = G rounded up to 1, 2, 4 or 8;
// padding rows are computed like the half's first row and not stored).  The
// halves share every K/V tile.  Softmax thread t owns row t % 128 of its
// half, which is its TMEM lane, so the softmax needs no shuffles.  Grid: (KV
// heads, tiles); the host lists tiles longest first.
//
// Keys go in groups of 128 (8 pages).  The CTA has three roles that meet only
// at mbarriers:
//   * warps 0-7, softmax, 4 per half: for group g, wait until S(g) is in
//     TMEM, read the row twice, 32 columns at a time (row max, then P), mask
//     causally (only groups that reach past the half's first position), and
//     run the online softmax in base 2 with the scale folded into one FMA
//     before 2^x.  The running max moves only when the group's max exceeds it
//     by more than 8 (then the warp rescales its O rows in TMEM), so
//     P = 2^(s - m) stays <= 256.  P, rounded to the K/V type, is stored over
//     S(g)'s own TMEM columns (two 16-bit values per column) and the warp
//     arrives on p_ready;
//   * warp 8, one thread, MMAs in the order S_A(0) S_B(0) | PV_A(g) S_A(g+1)
//     PV_B(g) S_B(g+1) | ...: S = Q K(g)^T (M 128, N 128, K-major Q and K from
//     shared memory), O += P(g) V(g) (A = P read from TMEM, V an MN-major
//     operand).  MMAs of one thread run in order, so S(g+1) overwrites P(g)
//     only after PV(g) read it, and one half's softmax overlaps the other
//     half's MMAs;
//   * warp 9, copies: the K and V tiles (32 KB each for D = 128) by cp.async
//     in the order the MMAs consume them, through a ring of shared-memory
//     slots freed by tcgen05.commit of the consuming MMAs; each lane arrives
//     on the slot's barrier once its copies complete.  It starts while the
//     softmax warps load Q; the MMA thread waits for Q on q_full.
// Softmax warp w owns tile rows [32 w, 32 w + 32), its TMEM lanes: it loads
// those Q rows, and stores their O rows (staged through the freed Q tile), by
// whole lines, 16 lanes x 16 bytes per 256-byte row.
// Shared memory: Q (2 x 128 x D) + 4 slots of 32 KB = 193 KiB for D = 128
// (8 slots of 16 KB for D = 64), one CTA per SM; TMEM: 512 columns (per half
// S/P 128 + O D).
//
// Every wait is bounded (mbarrier polls that also watch a CTA abort flag);
// on expiry the CTA records kStatusWaitTimeout, drains its MMAs and copies
// (bounded), frees TMEM and returns.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "ms_attention_common.cuh"

namespace ms {
namespace attn {
namespace {

constexpr int kRows = 128;     // query rows per CTA = TMEM lanes
constexpr int kKeys = 128;     // keys per group (8 pages): the S MMA is M 128 x N 128
constexpr float kRescale = 8.0f;  // move the running max only when it grows by more than 2^8
constexpr int kExp2OnFma = 3;     // of every 8 score pairs, this many take 2^x on the FMA pipe (exp2_poly2)

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

// 32 consecutive 32-bit columns of this thread's TMEM lane, without waiting
// (tcgen05.wait::ld before the registers are read).
__device__ __forceinline__ void tmem_ld32_async(uint32_t addr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

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
  const void *k_pool;  // [pool_blocks][Hkv][16][D]
  const void *v_pool;
  void *out;
  const int32_t *block_tables;
  const int32_t *tiles;  // [num_tiles][4]: first packed row, rows, position of first row, table row
  unsigned *status;
  int max_blocks_per_seq;
  int num_kv_heads;
  float qscale;
};

constexpr int kHalves = 2;  // query halves of 128 rows per CTA, sharing every K/V tile

template <int D> struct Ring5 {
  static constexpr int kHalf = kKeys * 128;                 // 128 keys x 64 dims (one 128-byte row per key)
  static constexpr int kTile = (D / 64) * kHalf;            // one K or V tile
  static constexpr int kSlots = D == 128 ? 4 : 8;
  static constexpr int kQ = (D / 64) * kRows * 128;         // one query half
  static constexpr int kSmem = 1024 + kHalves * kQ + kSlots * kTile;  // + alignment slack
};

// Bounded mbarrier wait that gives up early once another role set `abort`.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort) {
  for (int i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && *abort) return false;
  }
  return false;
}
__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst_smem)), "l"(src) : "memory");
}
// arrive on `bar` (without raising its expected count) once this thread's earlier cp.async copies completed
__device__ __forceinline__ void cp_async_arrive_on(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// max of three (sm_100 three-input max.f32)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// 2^x for two x <= 8 on the FMA and integer pipes instead of the transcendental unit
// (Cody and Waite's argument split): j = rint(x) by adding and subtracting 1.5 * 2^23,
// f = x - j in [-0.5, 0.5], 2^f by a cubic fitted here for relative error on [-0.5, 0.5]
// (7.5e-5 at most in f32 Horner form), and j added to the exponent field.  x is clamped at
// -126 so the exponent never underflows into the sign (masked scores give ~1e-38, not 0).
__device__ __forceinline__ void exp2_poly2(float &y0, float &y1, float x0, float x1) {
  constexpr float kR = 12582912.f;  // 1.5 * 2^23: adding it rounds to an integer in the low mantissa bits
  constexpr float c0 = 0.99992812f, c1 = 0.69326097f, c2 = 0.24261054f, c3 = 0.05517132f;
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float t0, t1, j0, j1, f0, f1, p0, p1;
  add2(t0, t1, x0, x1, kR, kR);
  add2(j0, j1, t0, t1, -kR, -kR);
  add2(f0, f1, x0, x1, -j0, -j1);
  fma2(p0, p1, f0, f1, c3, c3, c2, c2);
  fma2(p0, p1, p0, p1, f0, f1, c1, c1);
  fma2(p0, p1, p0, p1, f0, f1, c0, c0);
  // bits(t) = bits(1.5 * 2^23) + j, whose low 9 bits are zero: bits(t) << 23 == j << 23 (mod 2^32)
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// O (TMEM, M 128 x N) += P (TMEM, 128 x 16, two values per column) * B (shared-memory descriptor)
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void tmem_st32u(uint32_t addr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 columns of this thread's TMEM lane, without waiting: tcgen05.wait::st before another
// thread or the tensor core may read them
__device__ __forceinline__ void tmem_st16u_async(uint32_t addr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

constexpr int kThreads5 = 320;  // 2 x 4 softmax warps (one group of 4 per query half), the MMA warp, the copy warp

template <typename T, int D, int G>
__global__ void __launch_bounds__(kThreads5, 1) paged_prefill_tc5_kernel(Prefill5Params p) {
  constexpr int RPT = RowsPerTok5<G>::value;
  constexpr int TPH = kRows / RPT;     // tokens per query half
  constexpr int NDH = D / 64;          // 64-dim (128-byte) halves
  constexpr int QHALF = kRows * 128;   // one 64-dim half of a query half
  constexpr int HALF = Ring5<D>::kHalf, TILE = Ring5<D>::kTile, NSLOT = Ring5<D>::kSlots, QB = Ring5<D>::kQ;
  constexpr int PAGES = kKeys / kBS;   // pages per group
  constexpr int TMEM_COLS = 512;       // query half h: S (then P) at 256 h + [0, 128), O at 256 h + [128, 128 + D)

  extern __shared__ unsigned char smem_dyn[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  unsigned char *sq = smem;  // query half h at h * QB: NDH 64-dim halves of 128 rows x 128 B
  unsigned char *ring = smem + kHalves * QB;
  __shared__ uint64_t full[NSLOT], empty[NSLOT], s_full[kHalves], p_ready[kHalves], pv_done[kHalves], drain, q_full;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_s;
  __shared__ int mma_landed_s, issued_s;

  const int kvh = blockIdx.x, tile = blockIdx.y;  // kv heads vary fastest: a tile's heads start together
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int row0 = p.tiles[tile * 4 + 0], nrows = p.tiles[tile * 4 + 1];
  const int pos0 = p.tiles[tile * 4 + 2], trow = p.tiles[tile * 4 + 3];
  const int32_t *table = p.block_tables + size_t(trow) * p.max_blocks_per_seq;
  const int kv_len = pos0 + nrows;
  const int npages = (kv_len + kBS - 1) / kBS;
  const int ngroups = (kv_len + kKeys - 1) / kKeys;
  const int ntiles = 2 * ngroups;  // ring order K0 V0 K1 V1 ...: K(g) is tile 2g, V(g) tile 2g + 1
  // groups each query half attends to (its last token's causal range); half 1 may be empty
  int ng[kHalves];
#pragma unroll
  for (int h = 0; h < kHalves; ++h) {
    const int last = min(nrows, (h + 1) * TPH);  // tokens up to the end of half h
    ng[h] = last > h * TPH ? (pos0 + last + kKeys - 1) / kKeys : 0;
  }

  if (t == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&full[i], 32);  // the copy warp's lanes
      mbar_init(&empty[i], 1);
    }
    for (int h = 0; h < kHalves; ++h) {
      mbar_init(&s_full[h], 1);
      mbar_init(&p_ready[h], 4);  // one arrive per softmax warp of the half
      mbar_init(&pv_done[h], 1);
    }
    mbar_init(&drain, 1);
    mbar_init(&q_full, 4 * kHalves);  // one arrive per softmax warp once its Q rows are in shared memory
    abort_s = 0;
    mma_landed_s = 0;
    issued_s = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  // softmax thread t: query half qh = warp / 4, row rt = t % 128 of that half (TMEM lane rt)
  const int qh = warp >> 2, rt = t & (kRows - 1);
  const int tok = qh * TPH + rt / RPT, head = rt % RPT;
  const bool rvalid = warp < 4 * kHalves && head < G && tok < nrows;
  const int ng_q = qh == 0 ? ng[0] : ng[1];  // groups of this thread's half (softmax warps)
  // the CTA starts here: the copy warp's first K/V tiles overlap the Q load below
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  // Rows by whole lines: RPI rows of the tile per warp instruction, CPR lanes x 16 bytes each.
  // Softmax warp w owns tile rows [32 w, 32 w + 32) (its TMEM lanes), so it loads Q and
  // stores O for exactly those rows.
  constexpr int CPR = D / 8, RPI = 32 / CPR;
  if (warp < 4 * kHalves) {
    // Q rows -> K-major swizzled tile (zeros for padding rows), all loads before the stores
    const int cc = lane % CPR, sub = lane / CPR;
    uint4 qv[32 / RPI];
#pragma unroll
    for (int i = 0; i < 32 / RPI; ++i) {
      const int r = (warp & 3) * 32 + i * RPI + sub;  // row within the half
      const int tk = qh * TPH + r / RPT, hd = r % RPT;
      const T *src = static_cast<const T *>(p.q) +
                     ((size_t(row0) + tk) * p.num_kv_heads * G + size_t(kvh) * G + hd) * D + cc * 8;
      qv[i] = hd < G && tk < nrows ? __ldg(reinterpret_cast<const uint4 *>(src)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 32 / RPI; ++i) {
      const int r = (warp & 3) * 32 + i * RPI + sub, dh = cc >> 3, c = cc & 7;
      *reinterpret_cast<uint4 *>(sq + qh * QB + dh * QHALF + r * 128 + ((c ^ (r & 7)) << 4)) = qv[i];
    }
    fence_proxy_async();  // the MMAs read Q through the async proxy
    __syncwarp();
    if (lane == 0) mbar_arrive(&q_full);
  }

  float l_run = 0.f;
  if (warp < 4 * kHalves) {
    // ---- softmax: row rt of query half qh ----
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t tm_s = tmem + qh * 256, tm_o = tm_s + kKeys;
    const int pos_first = pos0 + qh * TPH;            // first position of this half
    const int pos = rvalid ? pos0 + tok : pos_first;  // padding rows copy the half's first row mask
    const float c = p.qscale;
    // the lowest half that attends to the last group zeroes its V rows past the sequence
    const bool zeroes_v = ng_q == ngroups && (qh == 0 || ng[0] < ngroups);
    float m_run = -INFINITY;
    for (int g = 0; g < ng_q; ++g) {
      if (!__all_sync(kFull, wait_or_abort(&s_full[qh], g & 1, &abort_s))) {
        abort_s = 1;
        break;
      }
      tc_fence_after();
      // S is read from TMEM twice, 32 columns at a time (the next chunk loads while one is used):
      // pass 1 takes the row max, pass 2 turns the scores into P.  Only groups that reach past
      // the half's first position take the causal mask (a CTA-uniform branch).
      const int key0 = g * kKeys;
      const bool diag = key0 + kKeys - 1 > pos_first;
      constexpr int NC = kKeys / 32;
      auto score = [&](auto masked, const uint32_t *cur, int k, int i) {
        const float v = __uint_as_float(cur[i]);
        if constexpr (decltype(masked)::value) return key0 + 32 * k + i <= pos ? v : -INFINITY;
        return v;
      };
      auto row_max = [&](auto masked) {
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        uint32_t ca[32], cb[32];
        tmem_ld32_async(tm_s + lane_off, ca);
#pragma unroll
        for (int k = 0; k < NC; ++k) {
          tmem_wait_ld();
          const uint32_t *cur = (k & 1) ? cb : ca;
          if (k + 1 < NC) tmem_ld32_async(tm_s + lane_off + 32 * (k + 1), (k & 1) ? ca : cb);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            mx[i & 3] = max3f(mx[i & 3], score(masked, cur, k, 2 * i), score(masked, cur, k, 2 * i + 1));
        }
        return fmaxf(max3f(mx[0], mx[1], mx[2]), mx[3]);
      };
      const float mt = diag ? row_max(std::true_type{}) : row_max(std::false_type{});
      const float mts = mt * c;
      const bool grow = mts > m_run + kRescale;  // m_run = -inf: any finite max
      float alpha = 1.f;
      if (grow) {
        alpha = ex2_approx(m_run - mts);
        m_run = mts;
      }
      if (g > 0 && __any_sync(kFull, grow)) {
        // O is being accumulated by PV(g - 1): wait for it, then rescale this warp's rows
        if (!__all_sync(kFull, wait_or_abort(&pv_done[qh], (g - 1) & 1, &abort_s))) {
          abort_s = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          float o[32];
          tmem_ld32(tm_o + lane_off + c0, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tm_o + lane_off + c0, o);
        }
      }
      const float negm = -m_run;
      float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // P of chunk k (16 columns of value pairs) goes to columns [16k, 16k + 16): over S chunks
      // already read, never over the chunk loading next.  Two scores per packed FMA and add.
      auto make_p = [&](auto masked) {
        uint32_t ca[32], cb[32];
        tmem_ld32_async(tm_s + lane_off, ca);
#pragma unroll
        for (int k = 0; k < NC; ++k) {
          tmem_wait_ld();
          const uint32_t *cur = (k & 1) ? cb : ca;
          if (k + 1 < NC) tmem_ld32_async(tm_s + lane_off + 32 * (k + 1), (k & 1) ? ca : cb);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x0, x1, a, b;
            ffma2(x0, x1, score(masked, cur, k, 2 * i), score(masked, cur, k, 2 * i + 1), c, negm);
            if ((i & 7) < kExp2OnFma) {  // a share of the exponentials off the transcendental unit
              exp2_poly2(a, b, x0, x1);
            } else {
              a = ex2_approx(x0);
              b = ex2_approx(x1);
            }
            fadd2(ps[2 * (i & 3)], ps[2 * (i & 3) + 1], a, b);
            pk[i] = pack_pair<T>(a, b);
          }
          tmem_st16u_async(tm_s + lane_off + 16 * k, pk);  // over S columns this thread has read
        }
        tmem_wait_st();  // once, before the p_ready arrive hands P to the tensor core
      };
      if (diag) make_p(std::true_type{});
      else make_p(std::false_type{});
      const float psum = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      l_run = l_run * alpha + psum;
      // the last group's V rows past the sequence (stale, or pages never loaded) -> 0
      const int vk = kv_len - key0;
      if (zeroes_v && g == ngroups - 1 && vk < kKeys) {
        const int iv = 2 * g + 1;
        if (!__all_sync(kFull, wait_or_abort(&full[iv % NSLOT], (iv / NSLOT) & 1, &abort_s))) {
          abort_s = 1;
          break;
        }
        unsigned char *vst = ring + (iv % NSLOT) * TILE;
        for (int i = rt; i < (kKeys - vk) * 8 * NDH; i += kRows) {
          const int dh = i / ((kKeys - vk) * 8), rem = i % ((kKeys - vk) * 8);
          *reinterpret_cast<uint4 *>(vst + dh * HALF + (vk + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[qh]);
    }
  } else if (warp == 4 * kHalves) {
    // ---- MMA issue, one thread: S_A(0) S_B(0) | PV_A(g) S_A(g+1) PV_B(g) S_B(g+1) | ... ----
    // Each half's S overwrites its P only after its PV (MMAs of a thread run in order), and
    // one half's softmax overlaps the other half's MMAs.
    if (lane == 0) {
      const uint32_t id_s = umma_idesc<T>(kRows, kKeys, 0), id_o = umma_idesc<T>(kRows, D, 1);
      int landed = 0;  // tiles [0, landed) seen complete, in ring order
      auto wait_tile = [&](int i) {
        for (; landed <= i; ++landed) {
          if (!wait_or_abort(&full[landed % NSLOT], (landed / NSLOT) & 1, &abort_s)) return false;
          fence_proxy_async();  // the copies were generic-proxy writes
        }
        tc_fence_after();
        return true;
      };
      // Descriptors are built once; an operand at byte offset o from a base is the base
      // descriptor + (o >> 4) (the 14-bit start field cannot carry: shared addresses are < 256 KiB),
      // so the MMAs below issue back to back.
      const uint64_t dq = umma_desc_sw128(smem_addr(sq), 16, 1024);         // Q, K-major
      const uint64_t dk = umma_desc_sw128(smem_addr(ring), 16, 1024);       // K tiles, K-major
      const uint64_t dv = umma_desc_sw128(smem_addr(ring), HALF, 1024);     // V tiles, MN-major
      auto issue_s = [&](int h, int g) {
        const uint64_t a0 = dq + uint64_t((h * QB) >> 4), b0 = dk + uint64_t((((2 * g) % NSLOT) * TILE) >> 4);
        const uint32_t d = tmem + h * 256;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (((kk >> 2) * QHALF + (kk & 3) * 32) >> 4), offk = (((kk >> 2) * HALF + (kk & 3) * 32) >> 4);
          umma(d, a0 + off, b0 + offk, id_s, kk > 0);
        }
        umma_commit(&s_full[h]);
      };
      auto issue_pv = [&](int h, int g) {
        const uint64_t b0 = dv + uint64_t((((2 * g + 1) % NSLOT) * TILE) >> 4);
        const uint32_t d = tmem + h * 256 + kKeys, a = tmem + h * 256;
        const uint32_t acc0 = g > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) umma_ts(d, a + kk * 8, b0 + uint64_t((kk * 2048) >> 4), id_o, kk > 0 ? 1u : acc0);
        umma_commit(&pv_done[h]);
      };
      bool ok = wait_or_abort(&q_full, 0, &abort_s) && wait_tile(0);
      if (ok) {
#pragma unroll
        for (int h = 0; h < kHalves; ++h)
          if (ng[h] > 0) issue_s(h, 0);
        umma_commit(&empty[0]);
      }
      for (int g = 0; g < ngroups && ok; ++g) {
        // V(g) and K(g + 1) were copied long before P(g) is ready (their slots were freed by
        // MMAs of groups g - 2 and g - 1): take both, with the proxy fence for the copies, here
        // rather than between p_ready and the MMAs
        if (!wait_tile(min(2 * g + 2, ntiles - 1))) {
          ok = false;
          break;
        }
#pragma unroll
        for (int h = 0; h < kHalves && ok; ++h) {
          if (g < ng[h]) {
            if (!wait_or_abort(&p_ready[h], g & 1, &abort_s)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(h, g);
          }
          if (g + 1 < ng[h]) issue_s(h, g + 1);
        }
        if (!ok) break;
        umma_commit(&empty[(2 * g + 1) % NSLOT]);                      // V(g): its PVs are issued
        if (g + 1 < ngroups) umma_commit(&empty[(2 * g + 2) % NSLOT]);  // K(g+1): its S MMAs are issued
      }
      if (!ok) abort_s = 1;
      mma_landed_s = landed;
    }
  } else {
    // ---- copies: tiles in ring order, 16 bytes per lane per instruction ----
    // Lane l holds page id (32 w + l) of the current window w of each stream
    // (K and V visit the groups in order), and the next window is loaded as
    // soon as the current one is taken, so no tile waits on a table read.
    // A page of one kv head is 16 rows of D elements, contiguous in the pool;
    // lane l always copies 16-byte column l % CPR of rows l / CPR, l / CPR +
    // RPI, ... into the swizzled operand layout.  After a tile's copies each
    // lane arms an arrive on the slot's full barrier that fires when they
    // complete (cp.async.mbarrier.arrive.noinc); the MMA thread makes them
    // visible to the tensor core (fence.proxy.async) after its wait.
    constexpr int CPR = D / 8, RPI = 32 / CPR, IPP = kBS / RPI;  // chunks per row, rows per instruction, per page
    const int cc = lane % CPR, dh = cc >> 3, ch = cc & 7, r0 = lane / CPR;
    auto table_at = [&](int i) { return i < npages ? table[i] : 0; };
    int kw = 0, vw = 0;
    int kcur = table_at(lane), vcur = kcur, knxt = table_at(32 + lane), vnxt = knxt;
    int issued = 0;
    for (int i = 0; i < ntiles; ++i) {
      const int slot = i % NSLOT;
      if (i >= NSLOT && !__all_sync(kFull, wait_or_abort(&empty[slot], ((i / NSLOT) - 1) & 1, &abort_s))) {
        abort_s = 1;
        break;
      }
      const bool is_v = i & 1;
      const int grp = i >> 1;
      const int first = grp * PAGES, n = min(PAGES, npages - first);
      const int w = first >> 5;
      int &cw = is_v ? vw : kw, &cur = is_v ? vcur : kcur, &nxt = is_v ? vnxt : knxt;
      if (w != cw) {  // groups advance one at a time, so w == cw + 1
        cur = nxt;
        cw = w;
        nxt = table_at(32 * (w + 1) + lane);
      }
      const T *pool = static_cast<const T *>(is_v ? p.v_pool : p.k_pool);
      unsigned char *dst = ring + slot * TILE + dh * HALF;
#pragma unroll
      for (int j = 0; j < PAGES; ++j) {
        const int pid = __shfl_sync(kFull, cur, (first & 31) + j);
        if (j < n) {
          const T *src = pool + (size_t(pid) * p.num_kv_heads + kvh) * (kBS * D) + cc * 8;
#pragma unroll
          for (int k = 0; k < IPP; ++k) {
            const int r = r0 + k * RPI;  // row within the page
            const int kr = j * kBS + r;  // key row within the tile
            cp_async16(dst + kr * 128 + ((ch ^ (kr & 7)) << 4), src + r * D);
          }
        }
      }
      cp_async_arrive_on(&full[slot]);
      issued = i + 1;
    }
    cp_async_wait_all();
    if (lane == 0) issued_s = issued;
  }

  // join: every role has left its loop; then drain MMAs and copies in flight
  __syncthreads();
  bool ok_end = !abort_s;
  if (warp == 4 * kHalves && lane == 0) {
    umma_commit(&drain);
    if (!mbar_wait_bounded(&drain, 0)) ok_end = false;
  } else if (warp == 4 * kHalves + 1 && lane == 0) {
    // the copies are complete (cp.async.wait_all); their barrier arrives must land before the CTA exits
    for (int i = mma_landed_s; i < issued_s; ++i)
      if (!mbar_wait_bounded(&full[i % NSLOT], (i / NSLOT) & 1)) ok_end = false;
  }
  tc_fence_before();
  const bool all_ok = __syncthreads_and(ok_end);
  tc_fence_after();
  if (all_ok) {
    if (warp < 4 * kHalves && ng_q > 0) {
      // O row / l -> shared memory (the Q tile is free once the MMAs drained): tile row
      // R = 32 warp + lane, D * 2 bytes, 16-byte chunk c at c ^ (R & 7); then this warp's 32
      // rows -> out by whole lines.  Every thread of the half takes part in the warp-collective
      // TMEM loads.
      const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
      const uint32_t tm_o = tmem + qh * 256 + kKeys;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      unsigned char *stage = sq + size_t(warp * 32) * (D * 2);
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        float o[32];
        tmem_ld32(tm_o + lane_off + c0, o);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_pair<T>(o[i] * inv, o[i + 1] * inv);
          w.y = pack_pair<T>(o[i + 2] * inv, o[i + 3] * inv);
          w.z = pack_pair<T>(o[i + 4] * inv, o[i + 5] * inv);
          w.w = pack_pair<T>(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4 *>(stage + lane * (D * 2) + ((((c0 + i) >> 3) ^ (lane & 7)) << 4)) = w;
        }
      }
      __syncwarp();
      const int cc = lane % CPR, sub = lane / CPR;
#pragma unroll
      for (int i = 0; i < 32 / RPI; ++i) {
        const int r = i * RPI + sub;                  // row within this warp's 32
        const int rh = (warp & 3) * 32 + r;           // row within the half
        const int tk = qh * TPH + rh / RPT, hd = rh % RPT;
        if (hd < G && tk < nrows) {
          const uint4 v = *reinterpret_cast<const uint4 *>(stage + r * (D * 2) + ((cc ^ (r & 7)) << 4));
          *reinterpret_cast<uint4 *>(static_cast<T *>(p.out) +
                                     ((size_t(row0) + tk) * p.num_kv_heads * G + size_t(kvh) * G + hd) * D + cc * 8) = v;
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
cudaError_t launch_t5(const Prefill5Params &p, int num_tiles, cudaStream_t stream) {
  auto kern = paged_prefill_tc5_kernel<T, D, G>;
  const size_t smem = Ring5<D>::kSmem;
  static std::atomic<bool> attr_done[64];  // zero-initialised (static storage)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    attr_done[dev].store(true, std::memory_order_release);  // setting twice is harmless
  }
  if (num_tiles > 65535) return cudaErrorInvalidValue;
  dim3 grid(p.num_kv_heads, num_tiles);
  kern<<<grid, kThreads5, smem, stream>>>(p);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t t5_group(const Prefill5Params &p, int group, int num_tiles, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_t5<T, D, 1>(p, num_tiles, stream);
    case 2: return launch_t5<T, D, 2>(p, num_tiles, stream);
    case 4: return launch_t5<T, D, 4>(p, num_tiles, stream);
    case 7: return launch_t5<T, D, 7>(p, num_tiles, stream);
    case 8: return launch_t5<T, D, 8>(p, num_tiles, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int prefill_tc5_tokens_per_tile(int group) {
  const int rpt = group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8;
  return kHalves * kRows / rpt;
}

cudaError_t launch_prefill_tc5(const void *q, void *out, const int32_t *block_tables, int max_blocks_per_seq,
                               const int32_t *tiles, int num_tiles, int num_kv_heads, int group, int head_dim,
                               float scale, unsigned *status, int dtype, const void *k_pool, const void *v_pool,
                               cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool)) & 15) return cudaErrorInvalidValue;
  Prefill5Params p;
  p.q = q;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.out = out;
  p.block_tables = block_tables;
  p.tiles = tiles;
  p.status = status;
  p.max_blocks_per_seq = max_blocks_per_seq;
  p.num_kv_heads = num_kv_heads;
  p.qscale = scale * kLog2e;
  if (dtype == MS_DTYPE_BF16) {
    if (head_dim == 128) return t5_group<__nv_bfloat16, 128>(p, group, num_tiles, stream);
    if (head_dim == 64) return t5_group<__nv_bfloat16, 64>(p, group, num_tiles, stream);
  } else if (dtype == MS_DTYPE_F16) {
    if (head_dim == 128) return t5_group<__half, 128>(p, group, num_tiles, stream);
    if (head_dim == 64) return t5_group<__half, 64>(p, group, num_tiles, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace attn
}  // namespace ms
