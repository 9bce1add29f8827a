// K5 + K2: fused (bias) + per-head QK RMSNorm + rotate-half RoPE + paged KV append.
//
// Restates, per packed token, Attention::forward up to the cache append
// (src/backends/qwen2.rs:287-313): projections arrive as one fused
// [T, (Hq + 2 Hkv) * D] GEMM output; bias (qwen2.rs:234-248) and QK-norm
// (qwen2.rs:297-304, the RmsNorm of :68-75 over head_dim) are applied before
// RoPE (apply_rope, :132-142, with the cos/sin tables of :91-108, kept in f32
// for every model dtype); the rotated K and the V rows are written straight
// into their paged-pool slot (the append of :349-361, now into 16-token pages
// addressed by slot_mapping), the rotated q into a dense [T, Hq, D] buffer
// for K3.  All arithmetic is f32 and each stored value is rounded once, so a
// 16-bit output is within half a unit in its last place of the f32
// reference's value from the same inputs (f32 mode divides by the norm as the
// reference does; 16-bit outputs multiply by its reciprocal).
//
// Two builds: qk_norm_rope_append_vec_kernel (16-byte aligned operands, the
// engine's case) moves 16-byte vectors, several per thread; the general
// qk_norm_rope_append_kernel runs one warp per (token, head), lane l holding
// dims [l*D/32, (l+1)*D/32), so the rotate-half partner of each dim sits in
// lane l ^ 16.
#include <type_traits>

#include <algorithm>
#include <atomic>

#include "ms_attention_common.cuh"

namespace ms {
namespace {

// x / norm * w: the reference's division in f32 mode, the reciprocal for 16-bit outputs.
template <typename T>
__device__ __forceinline__ float qk_scale(float x, float norm, float rn, float w) {
  if constexpr (std::is_same<T, float>::value) return (x / norm) * w;
  return x * rn * w;
}

template <typename T, int D>
__global__ void qk_norm_rope_append_kernel(const T *__restrict__ qkv, const T *__restrict__ bias,
                                           const T *__restrict__ qn, const T *__restrict__ kn,
                                           const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                                           const int32_t *__restrict__ positions,
                                           const int64_t *__restrict__ slot_mapping, T *__restrict__ q_out,
                                           T *__restrict__ k_pool, T *__restrict__ v_pool, int num_tokens,
                                           int hq, int hkv, int block_size, float eps) {
  constexpr int DPL = D / 32;
  constexpr int HALF = D / 2;
  const int heads = hq + 2 * hkv;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= (long long)num_tokens * heads) return;
  const int lane = threadIdx.x & 31;
  const int t = int(gw / heads);
  const int h = int(gw % heads);
  const int d0 = lane * DPL;

  float x[DPL];
  const T *src = qkv + (size_t(t) * heads + h) * D + d0;
  if constexpr (DPL == 4) Vec4<T>::load(src, x); else Vec2<T>::load(src, x);
  if (bias) {
    float b[DPL];
    const T *bs = bias + size_t(h) * D + d0;
    if constexpr (DPL == 4) Vec4<T>::load(bs, b); else Vec2<T>::load(bs, b);
#pragma unroll
    for (int i = 0; i < DPL; ++i) x[i] += b[i];
  }

  if (h >= hq + hkv) {  // V head: straight into the pool
    const int vh = h - hq - hkv;
    const int64_t slot = slot_mapping[t];
    const int64_t blk = slot / block_size, off = slot % block_size;
    T *dst = v_pool + ((size_t(blk) * hkv + vh) * block_size + off) * D + d0;
    if constexpr (DPL == 4) Vec4<T>::store(dst, x); else Vec2<T>::store(dst, x);
    return;
  }

  const bool is_q = h < hq;
  const T *nw = is_q ? qn : kn;
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    const float norm = sqrtf(ss / float(D) + eps);
    const float rn = 1.0f / norm;
    float w[DPL];
    if constexpr (DPL == 4) Vec4<T>::load(nw + d0, w); else Vec2<T>::load(nw + d0, w);
#pragma unroll
    for (int i = 0; i < DPL; ++i) x[i] = qk_scale<T>(x[i], norm, rn, w[i]);
  }

  // rotate-half RoPE
  const int pos = positions[t];
  const int j0 = d0 % HALF;
  float c[DPL], s[DPL];
  const float *cp = cos_t + size_t(pos) * HALF + j0;
  const float *sp = sin_t + size_t(pos) * HALF + j0;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    c[i] = cp[i];
    s[i] = sp[i];
  }
  float partner[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) partner[i] = __shfl_xor_sync(kFull, x[i], 16);
  const bool lower = lane < 16;
  float y[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) y[i] = fmaf(x[i], c[i], (lower ? -partner[i] : partner[i]) * s[i]);

  if (is_q) {
    T *dst = q_out + (size_t(t) * hq + h) * D + d0;
    if constexpr (DPL == 4) Vec4<T>::store(dst, y); else Vec2<T>::store(dst, y);
  } else {
    const int kh = h - hq;
    const int64_t slot = slot_mapping[t];
    const int64_t blk = slot / block_size, off = slot % block_size;
    T *dst = k_pool + ((size_t(blk) * hkv + kh) * block_size + off) * D + d0;
    if constexpr (DPL == 4) Vec4<T>::store(dst, y); else Vec2<T>::store(dst, y);
  }
}

// Staged K5 (16-byte aligned operands, power-of-two page size, every pair
// item of a token in one CTA of 256 threads).  The CTA is persistent over
// tokens blockIdx.x, blockIdx.x + gridDim.x, ...: one thread streams each
// token's whole projection row (heads x D values, 8 KB for Qwen3-0.6B) and its
// two RoPE table rows (f32 cos / sin at the token's position) into a ring of
// kStages shared-memory slots with bulk copies (cp.async.bulk) completing on
// one mbarrier per slot, kStages tokens ahead of the threads that use them, so
// each SM keeps tens of KB of loads in flight with few registers.  The
// tokens' positions and slots are read into shared memory once at the start.
//
// A thread holds one "pair item" of a head: dims [d, d + N) and their
// rotate-half partners [d + D/2, d + D/2 + N), so RoPE needs no exchange
// between threads; PPH = D / 2N consecutive threads hold a head and reduce its
// QK-norm sum with PPH-wide shuffles; q, k and v heads fall in separate warps.
// The norm weights (and bias) of a thread's head are loaded once.  A slot is
// refilled only after the CTA barrier that follows its last read.  Every wait
// is bounded: on expiry the CTA records kStatusWaitTimeout, waits (bounded)
// for the copies it issued and returns.
constexpr int kStages = 4;
constexpr int kMaxTokPerCta = 64;

template <typename T, int D>
__global__ void __launch_bounds__(256) qk_norm_rope_append_staged_kernel(
    const T *__restrict__ qkv, const T *__restrict__ bias, const T *__restrict__ qn, const T *__restrict__ kn,
    const float *__restrict__ cos_t, const float *__restrict__ sin_t, const int32_t *__restrict__ positions,
    const int64_t *__restrict__ slot_mapping, T *__restrict__ q_out, T *__restrict__ k_pool,
    T *__restrict__ v_pool, int num_tokens, int hq, int hkv, int bs_shift, float eps, unsigned *status) {
  using R = Raw16<T>;
  constexpr int N = R::N;
  constexpr int HALF = D / 2;
  constexpr int PPH = HALF / N;  // threads per head
  constexpr uint32_t kTab = HALF * sizeof(float);
  const int heads = hq + 2 * hkv;
  const uint32_t row_bytes = uint32_t(heads) * D * sizeof(T);
  extern __shared__ __align__(128) unsigned char smem5[];
  unsigned char *rows = smem5;                                           // [kStages][row_bytes]
  float *tabs = reinterpret_cast<float *>(smem5 + kStages * row_bytes);  // [kStages][cos | sin][HALF]
  __shared__ uint64_t full[kStages];
  __shared__ int pos_s[kMaxTokPerCta];
  __shared__ int64_t slot_s[kMaxTokPerCta];

  const int n_my = blockIdx.x < num_tokens ? (num_tokens - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int item = threadIdx.x;
  const bool live = item < heads * PPH;
  const int h = live ? item / PPH : 0;
  const int d0 = (item % PPH) * N;
  const bool is_v = h >= hq + hkv;
  const bool is_q = h < hq;
  const T *nw = is_v ? nullptr : (is_q ? qn : kn);

  for (int i = threadIdx.x; i < n_my; i += blockDim.x) {
    const int t = blockIdx.x + i * gridDim.x;
    pos_s[i] = __ldg(positions + t);
    slot_s[i] = __ldg(slot_mapping + t);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) attn::mbar_init(&full[s], 1);
    attn::fence_barrier_init();
  }
  float bl[N], bh[N], wl[N], wh[N];
  if (bias && live) {
    R::unpack(__ldg(reinterpret_cast<const uint4 *>(bias + size_t(h) * D + d0)), bl);
    R::unpack(__ldg(reinterpret_cast<const uint4 *>(bias + size_t(h) * D + d0 + HALF)), bh);
  }
  if (nw && live) {
    R::unpack(__ldg(reinterpret_cast<const uint4 *>(nw + d0)), wl);
    R::unpack(__ldg(reinterpret_cast<const uint4 *>(nw + d0 + HALF)), wh);
  }
  __syncthreads();

  auto issue = [&](int i) {  // thread 0: token i of this CTA into slot i % kStages
    const int s = i % kStages;
    const int t = blockIdx.x + i * gridDim.x;
    const size_t pos = size_t(pos_s[i]);
    attn::mbar_expect_tx(&full[s], row_bytes + 2 * kTab);
    attn::bulk_g2s(rows + size_t(s) * row_bytes, qkv + size_t(t) * heads * D, row_bytes, &full[s]);
    attn::bulk_g2s(tabs + s * 2 * HALF, cos_t + pos * HALF, kTab, &full[s]);
    attn::bulk_g2s(tabs + s * 2 * HALF + HALF, sin_t + pos * HALF, kTab, &full[s]);
  };
  int issued = 0;
  if (threadIdx.x == 0)
    for (; issued < min(kStages, n_my); ++issued) issue(issued);

  for (int i = 0; i < n_my; ++i) {
    const int s = i % kStages;
    const bool ok = attn::mbar_wait_bounded(&full[s], (i / kStages) & 1);
    if (__syncthreads_or(!ok)) {  // give up: record it, let the copies in flight land, leave
      if (threadIdx.x == 0) {
        if (status) atomicOr(status, kStatusWaitTimeout);
        for (int j = i; j < issued; ++j) attn::mbar_wait_bounded(&full[j % kStages], (j / kStages) & 1);
      }
      return;
    }
    const int t = blockIdx.x + i * gridDim.x;
    const unsigned char *row = rows + size_t(s) * row_bytes + (size_t(h) * D + d0) * sizeof(T);
    if (live) {
      const uint4 xl = *reinterpret_cast<const uint4 *>(row);
      const uint4 xh = *reinterpret_cast<const uint4 *>(row + HALF * sizeof(T));
      float fl[N], fh[N];
      R::unpack(xl, fl);
      R::unpack(xh, fh);
      if (bias) {
#pragma unroll
        for (int k = 0; k < N; ++k) {
          fl[k] += bl[k];
          fh[k] += bh[k];
        }
      }
      const int64_t slot = slot_s[i];
      const int64_t blk = slot >> bs_shift;
      const int off = int(slot & ((int64_t(1) << bs_shift) - 1));
      if (is_v) {  // V: into the pool
        T *dst = v_pool + ((size_t(blk) * hkv + (h - hq - hkv)) * (size_t(1) << bs_shift) + off) * D + d0;
        reinterpret_cast<uint4 *>(dst)[0] = bias ? R::pack(fl) : xl;
        reinterpret_cast<uint4 *>(dst + HALF)[0] = bias ? R::pack(fh) : xh;
      } else {
        if (nw) {
          float ss = 0.f;
#pragma unroll
          for (int k = 0; k < N; ++k) ss = fmaf(fh[k], fh[k], fmaf(fl[k], fl[k], ss));
#pragma unroll
          for (int o = PPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(__activemask(), ss, o);
          const float norm = sqrtf(ss / float(D) + eps);
          const float rn = 1.0f / norm;
#pragma unroll
          for (int k = 0; k < N; ++k) {
            fl[k] = qk_scale<T>(fl[k], norm, rn, wl[k]);
            fh[k] = qk_scale<T>(fh[k], norm, rn, wh[k]);
          }
        }
        const float *cs = tabs + s * 2 * HALF + d0;
        const float *sn = cs + HALF;
        float yl[N], yh[N];
#pragma unroll
        for (int k = 0; k < N; ++k) {
          const float c = cs[k], sv = sn[k];
          yl[k] = fmaf(fl[k], c, -fh[k] * sv);  // lo' = lo cos - hi sin
          yh[k] = fmaf(fh[k], c, fl[k] * sv);   // hi' = hi cos + lo sin
        }
        T *dst = is_q ? q_out + (size_t(t) * hq + h) * D + d0
                      : k_pool + ((size_t(blk) * hkv + (h - hq)) * (size_t(1) << bs_shift) + off) * D + d0;
        reinterpret_cast<uint4 *>(dst)[0] = R::pack(yl);
        reinterpret_cast<uint4 *>(dst + HALF)[0] = R::pack(yh);
      }
    }
    __syncthreads();  // slot s has been read by every thread
    if (threadIdx.x == 0 && issued < n_my) {
      attn::fence_proxy_async();  // the generic-proxy reads of the slot before its async refill
      issue(issued++);
    }
  }
}

template <typename T, int D>
cudaError_t launch_staged(const void *qkv, const void *bias, const void *qn, const void *kn, const void *cs,
                          const void *sn, const int32_t *positions, const int64_t *slots, void *q_out,
                          void *k_pool, void *v_pool, int T_, int hq, int hkv, int bs_shift, float eps,
                          unsigned *status, cudaStream_t st) {
  auto kern = qk_norm_rope_append_staged_kernel<T, D>;
  const int row_bytes = (hq + 2 * hkv) * D * int(sizeof(T));
  const int smem = kStages * (row_bytes + 2 * (D / 2) * int(sizeof(float)));
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  // per device: the shared-memory attribute set so far and the resident CTAs it allows
  static std::atomic<int> smem_set[64], resident[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (smem > smem_set[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int n_sm = 0, per = 0;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, 256, smem);
    resident[dev].store(std::max(1, per) * std::max(1, n_sm), std::memory_order_relaxed);
    smem_set[dev].store(smem, std::memory_order_release);  // setting twice is harmless
  }
  // one resident wave of persistent CTAs, each holding at most kMaxTokPerCta tokens
  int grid = resident[dev].load(std::memory_order_relaxed);
  grid = std::max(grid, (T_ + kMaxTokPerCta - 1) / kMaxTokPerCta);
  grid = std::min(grid, T_);
  if (status == nullptr) {
    e = standalone_status_word(&status);
    if (e != cudaSuccess) return e;
  }
  kern<<<grid, 256, smem, st>>>((const T *)qkv, (const T *)bias, (const T *)qn, (const T *)kn, (const float *)cs,
                                (const float *)sn, positions, slots, (T *)q_out, (T *)k_pool, (T *)v_pool, T_, hq,
                                hkv, bs_shift, eps, status);
  return cudaGetLastError();
}

inline bool host_aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
cudaError_t launch_typed(const void *qkv, const void *bias, const void *qn, const void *kn, const void *cs,
                         const void *sn, const int32_t *positions, const int64_t *slots, void *q_out,
                         void *k_pool, void *v_pool, int T_, int hq, int hkv, int D, int bs, float eps,
                         unsigned *status, cudaStream_t st) {
  int bs_shift = 0;
  while ((1 << bs_shift) < bs) ++bs_shift;
  // the staged build: 16-bit types, one CTA of 256 threads holds every pair item of a token
  const bool staged = !std::is_same<T, float>::value && (D == 128 || D == 64) && (1 << bs_shift) == bs &&
                      (hq + 2 * hkv) * (D / 2 / Raw16<T>::N) <= 256 && host_aligned16(qkv) &&
                      (!bias || host_aligned16(bias)) && (!qn || host_aligned16(qn)) && (!kn || host_aligned16(kn)) &&
                      host_aligned16(cs) && host_aligned16(sn) && host_aligned16(q_out) && host_aligned16(k_pool) &&
                      host_aligned16(v_pool);
  if (staged) {
    if (D == 128)
      return launch_staged<T, 128>(qkv, bias, qn, kn, cs, sn, positions, slots, q_out, k_pool, v_pool, T_, hq, hkv,
                                   bs_shift, eps, status, st);
    return launch_staged<T, 64>(qkv, bias, qn, kn, cs, sn, positions, slots, q_out, k_pool, v_pool, T_, hq, hkv,
                                bs_shift, eps, status, st);
  }
  const long long warps = (long long)T_ * (hq + 2 * hkv);
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  if (D == 128) {
    qk_norm_rope_append_kernel<T, 128><<<blocks, threads, 0, st>>>(
        (const T *)qkv, (const T *)bias, (const T *)qn, (const T *)kn, (const float *)cs, (const float *)sn,
        positions, slots, (T *)q_out, (T *)k_pool, (T *)v_pool, T_, hq, hkv, bs, eps);
  } else if (D == 64) {
    qk_norm_rope_append_kernel<T, 64><<<blocks, threads, 0, st>>>(
        (const T *)qkv, (const T *)bias, (const T *)qn, (const T *)kn, (const float *)cs, (const float *)sn,
        positions, slots, (T *)q_out, (T *)k_pool, (T *)v_pool, T_, hq, hkv, bs, eps);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qk_norm_rope_append(const void *qkv, const void *bias, const void *q_norm_w,
                                       const void *k_norm_w, const void *cos_table, const void *sin_table,
                                       const int32_t *positions, const int64_t *slot_mapping, void *q_out,
                                       void *k_pool, void *v_pool, int num_tokens, int num_heads,
                                       int num_kv_heads, int head_dim, int block_size, float eps, int dtype,
                                       cudaStream_t st, unsigned *status) {
  if (num_tokens == 0) return cudaSuccess;
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || block_size <= 0) return cudaErrorInvalidValue;
  switch (dtype) {
    case MS_DTYPE_F32:
      return launch_typed<float>(qkv, bias, q_norm_w, k_norm_w, cos_table, sin_table, positions, slot_mapping,
                                 q_out, k_pool, v_pool, num_tokens, num_heads, num_kv_heads, head_dim,
                                 block_size, eps, status, st);
    case MS_DTYPE_BF16:
      return launch_typed<__nv_bfloat16>(qkv, bias, q_norm_w, k_norm_w, cos_table, sin_table, positions,
                                         slot_mapping, q_out, k_pool, v_pool, num_tokens, num_heads,
                                         num_kv_heads, head_dim, block_size, eps, status, st);
    case MS_DTYPE_F16:
      return launch_typed<__half>(qkv, bias, q_norm_w, k_norm_w, cos_table, sin_table, positions, slot_mapping,
                                  q_out, k_pool, v_pool, num_tokens, num_heads, num_kv_heads, head_dim,
                                  block_size, eps, status, st);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace ms

extern "C" int ms_launch_qk_norm_rope_append(const void *qkv, const void *bias, const void *q_norm_w,
                                             const void *k_norm_w, const void *cos_table, const void *sin_table,
                                             const int32_t *positions, const int64_t *slot_mapping, void *q_out,
                                             void *k_pool, void *v_pool, int32_t num_tokens, int32_t num_heads,
                                             int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                             float eps, int32_t dtype, void *stream) {
  return int(ms::launch_qk_norm_rope_append(qkv, bias, q_norm_w, k_norm_w, cos_table, sin_table, positions,
                                            slot_mapping, q_out, k_pool, v_pool, num_tokens, num_heads,
                                            num_kv_heads, head_dim, block_size, eps, dtype,
                                            static_cast<cudaStream_t>(stream), nullptr));
}
