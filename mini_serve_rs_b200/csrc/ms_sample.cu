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
// Here one CTA per row works in passes over the row's logits (L2-resident
// after the first), z = x * inv_t:
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
#include <cstdint>

#include "ms_common.cuh"
#include "ms_internal.h"

namespace ms {
namespace {

constexpr int kThreads = 512;  // 2 CTAs (rows) per SM: a 256-row batch is one wave
constexpr int kWarpsPerCta = kThreads / 32;
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

__device__ __forceinline__ uint64_t splitmix64_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// SplitMix64 state of token i: seed + (i + 1) * golden (advanced by
// kThreads * golden per strided iteration).
__device__ __forceinline__ uint64_t splitmix_state(uint64_t seed, int i) { return seed + (uint64_t(i) + 1) * kGolden; }

// Uniform in (0, 1): the top 24 bits of the SplitMix64 output, centred.
__device__ __forceinline__ float uniform_open(uint64_t state) {
  const uint64_t z = splitmix64_mix(state);
  return (float(uint32_t(z >> 40)) + 0.5f) * (1.0f / 16777216.0f);
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

// Calls f(x[i], i) for every i < V owned by this thread: two 16-byte loads
// in flight per iteration when the row is 16-byte aligned, scalar otherwise.
template <typename F>
__device__ __forceinline__ void for_row(const float *x, int V, F &&f) {
  if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    const int n4 = V >> 2;
    for (int q = threadIdx.x; q < n4; q += 2 * kThreads) {
      const bool hb = q + kThreads < n4;
      const float4 a = x4[q];
      const float4 b = hb ? x4[q + kThreads] : make_float4(0.f, 0.f, 0.f, 0.f);
      f(a.x, 4 * q); f(a.y, 4 * q + 1); f(a.z, 4 * q + 2); f(a.w, 4 * q + 3);
      if (hb) {
        const int qb = 4 * (q + kThreads);
        f(b.x, qb); f(b.y, qb + 1); f(b.z, qb + 2); f(b.w, qb + 3);
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += kThreads) f(x[i], i);
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

__device__ float block_max(float v, float *red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kWarpsPerCta ? red[lane] : -INFINITY;
  t = warp_max(t);
  __syncthreads();
  return t;
}

__device__ uint64_t block_sum_u64(uint64_t v, uint64_t *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  uint64_t t = lane < kWarpsPerCta ? red[lane] : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
  __syncthreads();
  return t;
}

// Exclusive prefix over threads (thread order) of a per-thread count.
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
    const int w = lane < kWarpsPerCta ? red[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(kFull, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < kWarpsPerCta) red[lane] = wi - w;
  }
  __syncthreads();
  const int r = red[warp] + incl - v;
  __syncthreads();
  return r;
}

// Block argmax of (score, index), ties to the lowest index; every thread
// returns the result.
__device__ Best block_best(Best b, float *redf, int *redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) take(b, __shfl_xor_sync(kFull, b.score, o), __shfl_xor_sync(kFull, b.idx, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { redf[warp] = b.score; redi[warp] = b.idx; }
  __syncthreads();
  Best r{-INFINITY, 0x7fffffff};
  if (lane < kWarpsPerCta) { r.score = redf[lane]; r.idx = redi[lane]; }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) take(r, __shfl_xor_sync(kFull, r.score, o), __shfl_xor_sync(kFull, r.idx, o));
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  __shared__ uint64_t hist[256];
  __shared__ uint64_t red64[kWarpsPerCta];
  __shared__ float redf[kWarpsPerCta];
  __shared__ int redi[kWarpsPerCta];
  __shared__ uint64_t sel_above;
  __shared__ int sel_bin;

  const int row = blockIdx.x;
  const double temp = double(a.temperature[row]);
  if (!(temp >= 1e-7)) return;  // argmax (LogitsProcessor::new maps these to ArgMax)
  const int V = a.vocab;
  const float *x = a.logits + size_t(row) * V;
  const float inv_t = float(1.0 / temp);
  uint64_t seed = 0;
  if (a.seeds) seed = a.seeds[row];
  else if (a.seed_lo) seed = (uint64_t(a.seed_hi[row]) << 32) | a.seed_lo[row];
  auto finish = [&](int tok) {
    if (threadIdx.x == 0) {
      a.out[row] = tok;
      if (a.row_slot && a.slot_last) a.slot_last[a.row_slot[row]] = tok;
    }
  };

  // 1. max of the scaled logits and the race over every token: token i
  //    scores z_i - log(E_i).  A token whose weight underflows (e < 2^-40)
  //    cannot win against the top token (its score is below m - 11, the top
  //    token's above m - 3), so the race needs no weights.
  float m = -INFINITY;
  Best best{-INFINITY, 0x7fffffff};
  for_row(x, V, [&](float xv, int i) {
    const float z = scaled(xv, inv_t);
    m = fmaxf(m, z);
    take(best, race_score(z, splitmix_state(seed, i)), i);
  });
  m = block_max(m, redf);
  best = block_best(best, redf, redi);
  if (!(m > -INFINITY) || !(m < INFINITY) || best.idx == 0x7fffffff) return;  // all -inf / NaN: keep argmax
  const double top_p = a.top_p ? double(a.top_p[row]) : 1.0;
  if (!(top_p > 0.0 && top_p < 1.0)) {
    finish(best.idx);
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
    for_row(x, V, [&](float xv, int i) {
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
    if (iter == 0) target = uint64_t(ceil(top_p * double(block_sum_u64(w_all, red64))));
    w_before = block_sum_u64(w_before, red64);
    next = block_best(next, redf, redi);
    if (weight_of(ej) > 0 && w_before < target) {
      finish(j);
      return;
    }
    if (next.idx == 0x7fffffff) break;  // cannot happen: the top token is always kept
    j = next.idx;
  }

  // 3. fallback after 8 rejected candidates (rare unless top_p is small):
  //    the nucleus edge by a 4-pass radix select over the bits of e, then the
  //    race over the kept tokens.
  uint32_t edge = 0;           // key of the last kept probability value
  long long keep_ties = -1;    // tokens equal to edge kept (-1: all of them)
  {
    uint64_t above = 0;  // mass strictly above the selected key range
    uint32_t prefix = 0, pmask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += kThreads) hist[b] = 0;
      __syncthreads();
      // warp-aggregated: lanes that hit the same bin add their weights with
      // two 32-bit reductions (w <= 2^40 splits into 21 + 20 bits), and one
      // lane per bin issues the shared-memory atomic
      for (int base = 0; base < V; base += kThreads) {
        const int i = base + threadIdx.x;
        unsigned bin = 0xffffu;
        uint64_t w = 0;
        if (i < V) {
          const float e = weight_e(scaled(x[i], inv_t), m);
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
          atomicAdd(reinterpret_cast<unsigned long long *>(&hist[bin]), (uint64_t(hs) << 20) + ls);
      }
      __syncthreads();
      if (threadIdx.x < 32) {  // scan the 256 bins from the top: lane l holds bins 255-8l .. 248-8l
        const int lane = threadIdx.x;
        uint64_t loc[8], s = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) { loc[k] = hist[255 - 8 * lane - k]; s += loc[k]; }
        uint64_t incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint64_t n = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += n;
        }
        const unsigned cross = __ballot_sync(kFull, above + incl >= target);
        const int L = cross ? __ffs(cross) - 1 : 31;
        if (lane == L) {
          uint64_t cum = above + (incl - s);
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
          const long long n_ties = (long long)(hist[sel_bin] / w_edge);
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
    for_row(x, V, [&](float xv, int i) {
      const float z = scaled(xv, inv_t);
      const float e = weight_e(z, m);
      if (__float_as_uint(e) < edge || weight_of(e) == 0) return;
      take(best, race_score(z, splitmix_state(seed, i)), i);
    });
  } else {
    // ties at the edge are kept in index order: contiguous chunks per thread
    const int per = (V + kThreads - 1) / kThreads;
    const int i0 = min(V, int(threadIdx.x) * per), i1 = min(V, i0 + per);
    int ties = 0;
    for (int i = i0; i < i1; ++i) ties += __float_as_uint(weight_e(scaled(x[i], inv_t), m)) == edge;
    int rank = block_exclusive_count(ties, redi);
    for (int i = i0; i < i1; ++i) {
      const float z = scaled(x[i], inv_t);
      const uint32_t key = __float_as_uint(weight_e(z, m));
      if (key < edge) continue;
      if (key == edge && rank++ >= keep_ties) continue;
      take(best, race_score(z, splitmix_state(seed, i)), i);
    }
  }
  best = block_best(best, redf, redi);
  if (best.idx != 0x7fffffff) finish(best.idx);
}

}  // namespace

cudaError_t launch_sample(const SampleArgs &a, cudaStream_t st) {
  if (a.rows == 0) return cudaSuccess;
  if (a.rows < 0 || a.vocab <= 0 || !a.logits || !a.temperature || !a.out) return cudaErrorInvalidValue;
  sample_kernel<<<a.rows, kThreads, 0, st>>>(a);
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
