// K6b: on-device temperature / top-p sampling (sample_token with temperature
// > 0, src/backends/candle.rs:737-763).
//
// The reference moves each row's logits to the host and runs
// candle_transformers::generation::LogitsProcessor (candle-transformers 0.11.0,
// Cargo.lock:390-391): scaled = logits * (1 / temperature) in f32, softmax,
// and for 0 < top_p < 1 the nucleus cut of sample_topp -- probabilities sorted
// descending (ties in index order), a token is zeroed once the running sum of
// the tokens before it reaches top_p -- then a draw from the remaining weights.
// Temperatures below 1e-7 select argmax (LogitsProcessor::new).
//
// A cluster of kCluster CTAs works on one row, in passes over its logits,
// z = x * inv_t:
//   1. the max m of z and an exponential race over all tokens: token i scores
//      z_i - log(E_i) with E_i = -log(U_i) ~ Exp(1), and the largest score
//      picks i with probability exp(z_i) / sum(exp(z)).  U_i comes from
//      SplitMix64 (Steele, Lea, Flood, "Fast splittable pseudorandom number
//      generators", OOPSLA 2014) over (seed, token index), so a (seed, logits)
//      pair always yields the same token.  Without a nucleus this is the draw;
//   2. nucleus rows: token weights are w = trunc(e * 2^40), e = exp(z - m)
//      (exact integer masses, so sums do not depend on their order).  The
//      kept set is the shortest prefix of the ranking (e descending, index
//      ascending) whose mass reaches ceil(top_p * W).  The race winner over
//      a superset of it is the winner over it whenever it is itself kept, so
//      each candidate costs one pass: its ranked-before mass against the
//      target, plus the race over the tokens ranked above it (the next
//      candidate when it is rejected); after the first, which also sums W,
//      only tokens ranked above the candidate compute anything.  Each check
//      succeeds with probability at least top_p;
//   3. after 8 rejections a 4-pass radix select over the bits of e (u64 mass
//      histograms in shared memory) finds the edge key v*: tokens above v*
//      are kept, and of the tokens equal to v* the first c in index order,
//      c = ceil((target - mass above) / w*); then the race over the kept set.
// The reference seeds its generator from the wall clock, so parity is the
// sampled distribution (and, against the CPU restatement of this kernel, the
// exact token for a given seed).
//
// Layout: CTA c of a row's cluster takes the contiguous slice [c S, c S + S)
// of the row (S = ceil(V / kCluster) rounded up to 4 tokens) and, when the
// slice fits, keeps it in shared memory for every pass, so the row crosses
// HBM once: kChunks bulk copies (cp.async.bulk, one mbarrier each) stream it
// in and pass 1 starts on the first piece.  Each reduction (max, race winner,
// masses, radix histograms, tie counts) is a CTA reduction, then an exchange
// through distributed shared memory: every CTA publishes its share, a
// cluster barrier, and every CTA combines all shares itself, so all CTAs of
// a row take the same branches.  Max, the (score, index) argmax and integer
// sums do not depend on the order of combination, so the token drawn does
// not depend on how the row is split.  A copy that never lands (a bounded
// wait that runs out) sets kStatusWaitTimeout and leaves the row's argmax.
// A launch without top-p values has no nucleus row, so pass 1 is its only
// pass: it runs one CTA per row over global memory, with nothing to stage.
#include <cooperative_groups.h>

#include <atomic>
#include <cstdint>

#include "ms_attention_common.cuh"
#include "ms_common.cuh"
#include "ms_internal.h"

namespace ms {
namespace {
namespace cg = cooperative_groups;

constexpr int kCluster = 8;      // CTAs per row (the portable cluster size)
constexpr int kThreads = 256;         // cluster launches: 2 CTAs per SM with a 76 KB slice (V = 151936)
constexpr int kThreadsOnePass = 512;  // one CTA per row (no nucleus row in the launch)
constexpr int kChunks = 4;               // bulk copies per staged slice
constexpr int kMaxStaged = 48 * 1024;    // tokens of a slice kept in shared memory (192 KB)
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

// SplitMix64 state of token i: seed + (i + 1) * golden.
__device__ __forceinline__ uint64_t splitmix_state(uint64_t seed, int i) { return seed + (uint64_t(i) + 1) * kGolden; }

// Uniform in (0, 1): the top 24 bits of the SplitMix64 output, centred.
// Only bits 40-63 are used, and the mix's last step (z ^= z >> 31) leaves
// them as they are, so it is skipped.  (k + 0.5) * 2^-24 is one FMA: scaling
// by a power of two commutes with rounding to nearest, so k * 2^-24 + 2^-25
// rounds to the same float as (float(k) + 0.5f) * 2^-24.
__device__ __forceinline__ float uniform_open(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return fmaf(float(uint32_t(z >> 40)), 1.0f / 16777216.0f, 1.0f / 33554432.0f);
}

// z = x * (1 / T) rounded on its own (never fused into a later add), so
// every pass computes bit-identical z and e = exp(z - m) for a token.
__device__ __forceinline__ float scaled(float x, float inv_t) { return __fmul_rn(x, inv_t); }
__device__ __forceinline__ float weight_e(float z, float m) { return expf(__fsub_rn(z, m)); }

// trunc(e * 2^40) for 0 <= e <= 1 from the bits of e: e = mant * 2^(exp - 150)
// with the implicit bit, so e * 2^40 = mant * 2^(exp - 110) (exact; integer
// ALU work instead of a float -> u64 conversion).  Zero for e < 2^-40.
__device__ __forceinline__ uint64_t weight_of(float e) {
  const uint32_t b = __float_as_uint(e);
  const int ex = int(b >> 23);  // sign is 0 for e > 0
  if (!(e > 0.f) || ex == 0 || ex > 127) return 0ull;  // zero, NaN, subnormal (< 2^-126), above 1
  const uint64_t mant = (b & 0x7fffffu) | 0x800000u;
  const int sh = ex - 110;
  return sh >= 0 ? mant << sh : (sh > -24 ? mant >> (-sh) : 0ull);
}

// Calls f(src[k], i0 + k) for every k < n owned by this thread: two 16-byte
// loads in flight per iteration when `vec` (src 16-byte aligned, n a multiple
// of 4), scalar otherwise.
template <int NT, typename F>
__device__ __forceinline__ void for_range(const float *src, int i0, int n, bool vec, F &&f) {
  if (vec) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    const int n4 = n >> 2;
    for (int q = threadIdx.x; q < n4; q += 2 * NT) {
      const bool hb = q + NT < n4;
      const float4 u = s4[q];
      const float4 w = hb ? s4[q + NT] : make_float4(0.f, 0.f, 0.f, 0.f);
      const int i = i0 + 4 * q;
      f(u.x, i); f(u.y, i + 1); f(u.z, i + 2); f(u.w, i + 3);
      if (hb) {
        const int j = i + 4 * NT;
        f(w.x, j); f(w.y, j + 1); f(w.z, j + 2); f(w.w, j + 3);
      }
    }
  } else {
    for (int k = threadIdx.x; k < n; k += NT) f(src[k], i0 + k);
  }
}

// Race score of token i: z_i - log(E_i), E_i = -log(U_i) ~ Exp(1).  The
// largest score over a set picks i with probability exp(z_i) / sum(exp(z)).
// The inner log is the accurate logf (u near 1 needs it: E is then tiny);
// E >= 6e-8, so the fast __logf (3 ulp) serves the outer one.
__device__ __forceinline__ float race_score(float z, uint64_t state) {
  return __fsub_rn(z, __logf(-logf(uniform_open(state))));
}

struct Best {
  float score;
  int idx;
};
__device__ __forceinline__ void take(Best &b, float s, int i) {
  if (s > b.score || (s == b.score && i < b.idx)) { b.score = s; b.idx = i; }
}

template <int NT>
__device__ float block_max(float v, float *red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < NT / 32 ? red[lane] : -INFINITY;
  t = warp_max(t);
  __syncthreads();
  return t;
}

template <int NT>
__device__ uint64_t block_sum_u64(uint64_t v, uint64_t *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  uint64_t t = lane < NT / 32 ? red[lane] : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
  __syncthreads();
  return t;
}

// Exclusive prefix over threads (thread order) of a per-thread count.
template <int NT>
__device__ int block_exclusive_count(int v, int *red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < NT / 32 ? red[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(kFull, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < NT / 32) red[lane] = wi - w;
  }
  __syncthreads();
  const int r = red[warp] + incl - v;
  __syncthreads();
  return r;
}

// Block argmax of (score, index), ties to the lowest index; every thread
// returns the result.
template <int NT>
__device__ Best block_best(Best b, float *redf, int *redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) take(b, __shfl_xor_sync(kFull, b.score, o), __shfl_xor_sync(kFull, b.idx, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { redf[warp] = b.score; redi[warp] = b.idx; }
  __syncthreads();
  Best r{-INFINITY, 0x7fffffff};
  if (lane < NT / 32) { r.score = redf[lane]; r.idx = redi[lane]; }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) take(r, __shfl_xor_sync(kFull, r.score, o), __shfl_xor_sync(kFull, r.idx, o));
  __syncthreads();
  return r;
}

// One CTA's share of a cluster reduction.
struct Share {
  float m;
  float score;
  int idx;
  unsigned flags;
  uint64_t a, b;
};

// The shares of all CTAs of the cluster, combined.
struct Combined {
  float m;
  Best best;
  unsigned flags;
  uint64_t a, b;
  uint64_t a_below;  // a summed over the CTAs of lower rank
};

// Publishes this CTA's share (thread 0 writes it to slot `k & 1`) and returns
// the combination of every CTA's share; all threads of all CTAs get the same
// result.  Slots alternate: the slot written by reduction k + 2 was last read
// before its readers arrived at the cluster barrier of reduction k + 1.
template <int C>
__device__ Combined cluster_combine(const Share &mine, Share *slots, int &k) {
  cg::cluster_group cl = cg::this_cluster();
  Share *slot = slots + (k & 1);
  ++k;
  if (threadIdx.x == 0) *slot = mine;
  cl.sync();  // barrier.cluster arrive (release) + wait (acquire)
  const unsigned me = cl.block_rank();
  Combined r{-INFINITY, Best{-INFINITY, 0x7fffffff}, 0u, 0ull, 0ull, 0ull};
#pragma unroll
  for (unsigned c = 0; c < unsigned(C); ++c) {
    const Share v = *cl.map_shared_rank(slot, c);
    r.m = fmaxf(r.m, v.m);
    take(r.best, v.score, v.idx);
    r.flags |= v.flags;
    r.a += v.a;
    r.b += v.b;
    if (c < me) r.a_below += v.a;
  }
  return r;
}

// C CTAs per row: kCluster with the row staged in shared memory (kStaged) or
// read from global memory in every pass; 1 (unstaged) for launches that the
// host knows have no nucleus row, where pass 1 is the only pass.
template <bool kStaged, int C, int NT>
__global__ void __cluster_dims__(C, 1, 1) __launch_bounds__(NT, 2)
    sample_kernel(SampleArgs a, int slice) {
  extern __shared__ __align__(16) float sm[];  // the staged slice: token lo + k at sm[k]
  __shared__ uint64_t hist[2][256];            // radix pass p uses hist[p & 1]
  __shared__ uint64_t tot[256];                // the cluster's histogram
  __shared__ uint64_t red64[NT / 32];
  __shared__ float redf[NT / 32];
  __shared__ int redi[NT / 32];
  __shared__ Share slots[2];
  __shared__ uint64_t chunk_full[kChunks];
  __shared__ uint64_t sel_above;
  __shared__ int sel_bin;

  cg::cluster_group cl = cg::this_cluster();
  const int rank = int(cl.block_rank());
  const int row = blockIdx.x / C;
  const double temp = double(a.temperature[row]);
  if (!(temp >= 1e-7)) return;  // argmax (LogitsProcessor::new maps these to ArgMax); every CTA of the row leaves here
  const int V = a.vocab;
  const float *x = a.logits + size_t(row) * V;
  const int lo = min(V, rank * slice), n = min(V, lo + slice) - lo;
  const bool vec = (V & 3) == 0 && aligned16(x);  // then lo, the chunks and n are multiples of 4 tokens
  const float *src = kStaged ? sm : x + lo;       // passes after the first read the slice here
  const bool svec = kStaged ? (n & 3) == 0 : vec;
  const float inv_t = float(1.0 / temp);
  uint64_t seed = 0;
  if (a.seeds) seed = a.seeds[row];
  else if (a.seed_lo) seed = (uint64_t(a.seed_hi[row]) << 32) | a.seed_lo[row];
  int red = 0;  // cluster reductions so far
  // leave with `tok` (>= 0) as the row's token; the barrier keeps this CTA's
  // shared memory alive until every CTA of the row has read its last share
  auto leave = [&](int tok) {
    if (tok >= 0 && rank == 0 && threadIdx.x == 0) {
      a.out[row] = tok;
      if (a.row_slot && a.slot_last) a.slot_last[a.row_slot[row]] = tok;
    }
    cl.sync();
  };

  // 1. max of the scaled logits and the race over every token: token i
  //    scores z_i - log(E_i).  A token whose weight underflows (e < 2^-40)
  //    cannot win against the top token (its score is below m - 11, the top
  //    token's above m - 3), so the race needs no weights.
  float m = -INFINITY;
  Best best{-INFINITY, 0x7fffffff};
  auto race_all = [&](float xv, int i) {
    const float z = scaled(xv, inv_t);
    m = fmaxf(m, z);
    take(best, race_score(z, splitmix_state(seed, i)), i);
  };
  unsigned flags = 0;
  const int per = ((n + kChunks - 1) / kChunks + 3) & ~3;  // tokens per bulk copy
  if constexpr (kStaged) {
    if (vec) {
      if (threadIdx.x == 0) {
        for (int c = 0; c < kChunks; ++c) attn::mbar_init(&chunk_full[c], 1);
        attn::fence_barrier_init();
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int c = 0; c < kChunks; ++c) {
          const int c0 = min(n, c * per), c1 = min(n, c0 + per);
          if (c1 > c0) {
            attn::mbar_expect_tx(&chunk_full[c], uint32_t(c1 - c0) * 4u);
            attn::bulk_g2s(sm + c0, x + lo + c0, uint32_t(c1 - c0) * 4u, &chunk_full[c]);
          } else {
            attn::mbar_arrive(&chunk_full[c]);
          }
        }
      }
      for (int c = 0; c < kChunks; ++c) {
        const int c0 = min(n, c * per), c1 = min(n, c0 + per);
        if (!attn::mbar_wait_bounded(&chunk_full[c], 0)) {
          flags |= kStatusWaitTimeout;
          continue;
        }
        for_range<NT>(sm + c0, lo + c0, c1 - c0, true, race_all);
      }
    } else {
      for (int k = threadIdx.x; k < n; k += NT) {
        const float v = x[lo + k];
        sm[k] = v;  // read by other threads after the block reductions below
        race_all(v, lo + k);
      }
    }
  } else {
    for_range<NT>(x + lo, lo, n, vec, race_all);
  }
  m = block_max<NT>(m, redf);
  best = block_best<NT>(best, redf, redi);
  flags = __syncthreads_or(flags) ? kStatusWaitTimeout : 0u;
  {
    const Combined r = cluster_combine<C>(Share{m, best.score, best.idx, flags, 0ull, 0ull}, slots, red);
    if (r.flags) {
      // a slice copy did not land in time: wait for this CTA's copies once more
      // (bounded), report, and leave the row's argmax in place
      if (kStaged && vec && threadIdx.x == 0)
        for (int c = 0; c < kChunks; ++c) attn::mbar_wait_bounded(&chunk_full[c], 0);
      if (rank == 0 && threadIdx.x == 0 && a.status) atomicOr(a.status, r.flags);
      leave(-1);
      return;
    }
    m = r.m;
    best = r.best;
  }
  if (!(m > -INFINITY) || !(m < INFINITY) || best.idx == 0x7fffffff) {  // all -inf / NaN: keep argmax
    leave(-1);
    return;
  }
  const double top_p = a.top_p ? double(a.top_p[row]) : 1.0;
  if (!(top_p > 0.0 && top_p < 1.0)) {
    leave(best.idx);
    return;
  }

  // 2. nucleus: the kept set is a prefix of the ranking (e descending, index
  //    ascending).  If the race winner over a set that contains the kept set
  //    is itself kept, it is the winner over the kept set; otherwise the kept
  //    set lies inside the tokens ranked above it, so race again there.  Each
  //    check is one pass: the mass ranked before candidate j against
  //    ceil(top_p * W), and the next candidate.  The first check also sums W
  //    (e for every token); later ones compute e only where it can rank
  //    before j: e = exp(z - m) is monotone in z, so that needs z >= z_j less
  //    a margin wider than the span of z that rounds to the same e.
  uint64_t target = 0;
  int j = best.idx;
  for (int iter = 0; iter < 8; ++iter) {
    const float zj = scaled(x[j], inv_t);
    const float ej = weight_e(zj, m);
    const float zlo = iter == 0 ? -INFINITY : zj - 1e-6f * (1.0f + fabsf(zj - m));
    uint64_t w_all = 0, w_before = 0;
    Best next{-INFINITY, 0x7fffffff};
    for_range<NT>(src, lo, n, svec, [&](float xv, int i) {
      const float z = scaled(xv, inv_t);
      if (z < zlo) return;
      const float e = weight_e(z, m);
      const uint64_t w = weight_of(e);
      w_all += w;
      if (i != j && (e > ej || (e == ej && i < j))) {
        w_before += w;
        take(next, race_score(z, splitmix_state(seed, i)), i);
      }
    });
    const uint64_t wa = iter == 0 ? block_sum_u64<NT>(w_all, red64) : 0ull;
    const uint64_t wb = block_sum_u64<NT>(w_before, red64);
    next = block_best<NT>(next, redf, redi);
    const Combined r = cluster_combine<C>(Share{-INFINITY, next.score, next.idx, 0u, wa, wb}, slots, red);
    if (iter == 0) target = uint64_t(ceil(top_p * double(r.a)));
    if (weight_of(ej) > 0 && r.b < target) {
      leave(j);
      return;
    }
    if (r.best.idx == 0x7fffffff) break;  // cannot happen: the top token is always kept
    j = r.best.idx;
  }

  // 3. fallback after 8 rejected candidates (rare unless top_p is small):
  //    the nucleus edge by a 4-pass radix select over the bits of e, then the
  //    race over the kept tokens.
  uint32_t edge = 0;           // key of the last kept probability value
  long long keep_ties = -1;    // tokens equal to edge kept (-1: all of them)
  {
    uint64_t above = 0;  // mass strictly above the selected key range
    uint32_t prefix = 0, pmask = 0;
    for (int shift = 24, hp = 0; shift >= 0; shift -= 8, ++hp) {
      uint64_t *h = hist[hp & 1];
      for (int b = threadIdx.x; b < 256; b += NT) h[b] = 0;
      __syncthreads();
      // warp-aggregated: lanes that hit the same bin add their weights with
      // two 32-bit reductions (w <= 2^40 splits into 21 + 20 bits), and one
      // lane per bin issues the shared-memory atomic
      for (int base = 0; base < n; base += NT) {
        const int k = base + threadIdx.x;
        unsigned bin = 0xffffu;
        uint64_t w = 0;
        if (k < n) {
          const float e = weight_e(scaled(src[k], inv_t), m);
          const uint32_t key = __float_as_uint(e);
          if ((key & pmask) == prefix) {
            w = weight_of(e);
            if (w) bin = (key >> shift) & 255u;
          }
        }
        if (bin == 0xffffu) w = 0;
        const unsigned peers = __match_any_sync(kFull, bin);
        const uint32_t hs = __reduce_add_sync(peers, uint32_t(w >> 20));
        const uint32_t ls = __reduce_add_sync(peers, uint32_t(w & 0xfffffu));
        if (bin != 0xffffu && int(threadIdx.x & 31) == __ffs(peers) - 1)
          atomicAdd(reinterpret_cast<unsigned long long *>(&h[bin]), (uint64_t(hs) << 20) + ls);
      }
      // every CTA's histogram is complete; h[p & 1] is next cleared two passes
      // later, after the barrier of the next pass (so after all reads below)
      cl.sync();
      for (int b = threadIdx.x; b < 256; b += NT) {
        uint64_t sum = 0;
#pragma unroll
        for (int c = 0; c < C; ++c) sum += cl.map_shared_rank(h, c)[b];
        tot[b] = sum;
      }
      __syncthreads();
      if (threadIdx.x < 32) {  // scan the 256 bins from the top: lane l holds bins 255-8l .. 248-8l
        const int lane = threadIdx.x;
        uint64_t loc[8], sum = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) { loc[k] = tot[255 - 8 * lane - k]; sum += loc[k]; }
        uint64_t incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint64_t v = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += v;
        }
        const unsigned cross = __ballot_sync(kFull, above + incl >= target);
        const int L = cross ? __ffs(cross) - 1 : 31;
        if (lane == L) {
          uint64_t cum = above + (incl - sum);
          int sel = 255 - 8 * lane - 7;
          for (int k = 0; k < 8; ++k) {
            if (cum + loc[k] >= target && loc[k] > 0) { sel = 255 - 8 * lane - k; break; }
            cum += loc[k];
          }
          sel_bin = sel;
          sel_above = cum;
        }
      }
      __syncthreads();
      prefix |= uint32_t(sel_bin) << shift;
      pmask |= 255u << shift;
      above = sel_above;
      if (shift == 0) {
        const uint64_t w_edge = weight_of(__uint_as_float(prefix));
        if (w_edge > 0) {
          const long long n_ties = (long long)(tot[sel_bin] / w_edge);
          const uint64_t need = target > above ? target - above : 1;
          const long long c = (long long)((need + w_edge - 1) / w_edge);
          keep_ties = c >= n_ties ? -1 : c;
        }
      }
      __syncthreads();
    }
    edge = prefix;
  }
  best = Best{-INFINITY, 0x7fffffff};
  if (keep_ties < 0) {
    for_range<NT>(src, lo, n, svec, [&](float xv, int i) {
      const float z = scaled(xv, inv_t);
      const float e = weight_e(z, m);
      if (__float_as_uint(e) < edge || weight_of(e) == 0) return;
      take(best, race_score(z, splitmix_state(seed, i)), i);
    });
  } else {
    // ties at the edge are kept in index order: contiguous chunks per thread,
    // the CTAs' slices in rank order
    const int cper = (n + NT - 1) / NT;
    const int k0 = min(n, int(threadIdx.x) * cper), k1 = min(n, k0 + cper);
    int ties = 0;
    for (int k = k0; k < k1; ++k) ties += __float_as_uint(weight_e(scaled(src[k], inv_t), m)) == edge;
    const int before_cta = block_exclusive_count<NT>(ties, redi);
    const uint64_t cta_ties = block_sum_u64<NT>(uint64_t(ties), red64);
    const Combined r = cluster_combine<C>(Share{-INFINITY, -INFINITY, 0x7fffffff, 0u, cta_ties, 0ull}, slots, red);
    long long tie_rank = (long long)r.a_below + before_cta;
    for (int k = k0; k < k1; ++k) {
      const float z = scaled(src[k], inv_t);
      const uint32_t key = __float_as_uint(weight_e(z, m));
      if (key < edge) continue;
      if (key == edge && tie_rank++ >= keep_ties) continue;
      take(best, race_score(z, splitmix_state(seed, lo + k)), lo + k);
    }
  }
  best = block_best<NT>(best, redf, redi);
  const Combined r = cluster_combine<C>(Share{-INFINITY, best.score, best.idx, 0u, 0ull, 0ull}, slots, red);
  leave(r.best.idx != 0x7fffffff ? r.best.idx : -1);
}

// Shared memory opt-in for the staged kernel, once per device.
std::atomic<uint64_t> g_sample_attr_done{0};

}  // namespace

cudaError_t launch_sample(const SampleArgs &a, cudaStream_t st) {
  if (a.rows == 0) return cudaSuccess;
  if (a.rows < 0 || a.vocab <= 0 || !a.logits || !a.temperature || !a.out) return cudaErrorInvalidValue;
  if (a.rows > (1 << 27)) return cudaErrorInvalidValue;
  SampleArgs b = a;
  if (!b.status) {
    cudaError_t e = standalone_status_word(&b.status);
    if (e != cudaSuccess) return e;
  }
  if (!a.top_p) {  // no nucleus row: one CTA per row, one pass over the logits in global memory
    sample_kernel<false, 1, kThreadsOnePass><<<unsigned(a.rows), kThreadsOnePass, 0, st>>>(b, (a.vocab + 3) & ~3);
    return cudaGetLastError();
  }
  const int slice = ((a.vocab + kCluster - 1) / kCluster + 3) & ~3;
  const dim3 grid(unsigned(a.rows) * kCluster);
  if (slice <= kMaxStaged) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (!(g_sample_attr_done.load() & bit)) {
      e = cudaFuncSetAttribute(sample_kernel<true, kCluster, kThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kMaxStaged * int(sizeof(float)));
      if (e != cudaSuccess) return e;
      g_sample_attr_done.fetch_or(bit);
    }
    sample_kernel<true, kCluster, kThreads><<<grid, kThreads, size_t(slice) * sizeof(float), st>>>(b, slice);
  } else {
    sample_kernel<false, kCluster, kThreads><<<grid, kThreads, 0, st>>>(b, slice);
  }
  return cudaGetLastError();
}

}  // namespace ms

extern "C" int ms_launch_sample(const float *logits, int32_t rows, int32_t vocab, const float *temperature,
                                const float *top_p, const uint64_t *seeds, int32_t *out, void *stream) {
  ms::SampleArgs a{};
  a.logits = logits;
  a.rows = rows;
  a.vocab = vocab;
  a.temperature = temperature;
  a.top_p = top_p;
  a.seeds = seeds;
  a.out = out;
  return int(ms::launch_sample(a, static_cast<cudaStream_t>(stream)));
}
