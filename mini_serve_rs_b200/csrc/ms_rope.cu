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

#include "ms_common.cuh"
#include "ms_internal.h"

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

// Vectorised K5 (16-byte aligned operands, power-of-two page size).  A thread
// holds one "pair item" of a head: dims [d, d + N) and their rotate-half
// partners [d + D/2, d + D/2 + N), so RoPE needs no exchange between threads
// and one set of cos/sin entries serves both halves; PPH = D / 2N consecutive
// threads hold a head and reduce its QK-norm sum with PPH-wide shuffles.  A
// row of threads (blockDim.x, a multiple of 32) covers every pair item of one
// token, so a warp never spans two tokens and q, k and v heads fall in
// separate warps; the CTA's TOKY rows take TOKY tokens, and each thread takes
// KT tokens TOKY apart, issuing all its loads before any math.  The norm
// weights (and bias) of a thread's head are loaded once.  16-bit math runs on
// packed f32x2 instructions.
template <typename T, int D, int KT>
__global__ void __launch_bounds__(256) qk_norm_rope_append_vec_kernel(
    const T *__restrict__ qkv, const T *__restrict__ bias, const T *__restrict__ qn, const T *__restrict__ kn,
    const float *__restrict__ cos_t, const float *__restrict__ sin_t, const int32_t *__restrict__ positions,
    const int64_t *__restrict__ slot_mapping, T *__restrict__ q_out, T *__restrict__ k_pool,
    T *__restrict__ v_pool, int num_tokens, int hq, int hkv, int bs_shift, float eps) {
  using R = Raw16<T>;
  constexpr int N = R::N;
  constexpr int HALF = D / 2;
  constexpr int PPH = HALF / N;  // threads per head
  constexpr bool kF32 = std::is_same<T, float>::value;
  const int heads = hq + 2 * hkv;
  const int item = threadIdx.x;
  const bool live = item < heads * PPH;
  const int h = live ? item / PPH : 0;
  const int d0 = (item % PPH) * N;
  const bool is_v = h >= hq + hkv;
  const bool is_q = h < hq;
  const T *nw = is_v ? nullptr : (is_q ? qn : kn);

  // tokens of this thread
  int tok[KT];
#pragma unroll
  for (int k = 0; k < KT; ++k) tok[k] = (blockIdx.x * KT + k) * blockDim.y + threadIdx.y;
  uint4 xl[KT], xh[KT];
#pragma unroll
  for (int k = 0; k < KT; ++k) {
    const bool ok = live && tok[k] < num_tokens;
    const uint4 *src = reinterpret_cast<const uint4 *>(qkv + (size_t(ok ? tok[k] : 0) * heads + h) * D + d0);
    xl[k] = ok ? __ldg(src) : make_uint4(0, 0, 0, 0);
    xh[k] = ok ? __ldg(src + HALF / N) : make_uint4(0, 0, 0, 0);
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

#pragma unroll
  for (int k = 0; k < KT; ++k) {
    if (tok[k] >= num_tokens) break;  // uniform over the row, so over each warp
    const int t = tok[k];
    float fl[N], fh[N];
    R::unpack(xl[k], fl);
    R::unpack(xh[k], fh);
    if (bias) {
#pragma unroll
      for (int i = 0; i < N; i += 2) {
        add2(fl[i], fl[i + 1], fl[i], fl[i + 1], bl[i], bl[i + 1]);
        add2(fh[i], fh[i + 1], fh[i], fh[i + 1], bh[i], bh[i + 1]);
      }
    }
    const int64_t slot = __ldg(slot_mapping + t);
    const int64_t blk = slot >> bs_shift;
    const int off = int(slot & ((int64_t(1) << bs_shift) - 1));
    if (is_v) {  // V: into the pool (warp-uniform branch)
      if (live) {
        T *dst = v_pool + ((size_t(blk) * hkv + (h - hq - hkv)) * (size_t(1) << bs_shift) + off) * D + d0;
        reinterpret_cast<uint4 *>(dst)[0] = bias ? R::pack(fl) : xl[k];
        reinterpret_cast<uint4 *>(dst + HALF)[0] = bias ? R::pack(fh) : xh[k];
      }
      continue;
    }
    if (nw) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < N; i += 2) {
        fma2(s0, s1, fl[i], fl[i + 1], fl[i], fl[i + 1], s0, s1);
        fma2(s0, s1, fh[i], fh[i + 1], fh[i], fh[i + 1], s0, s1);
      }
      float ss = s0 + s1;
#pragma unroll
      for (int o = PPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
      const float norm = sqrtf(ss / float(D) + eps);
      if constexpr (kF32) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
          fl[i] = (fl[i] / norm) * wl[i];
          fh[i] = (fh[i] / norm) * wh[i];
        }
      } else {
        const float rn = 1.0f / norm;
#pragma unroll
        for (int i = 0; i < N; i += 2) {
          float a0, a1, b0, b1;
          mul2(a0, a1, wl[i], wl[i + 1], rn, rn);
          mul2(b0, b1, wh[i], wh[i + 1], rn, rn);
          mul2(fl[i], fl[i + 1], fl[i], fl[i + 1], a0, a1);
          mul2(fh[i], fh[i + 1], fh[i], fh[i + 1], b0, b1);
        }
      }
    }
    // rotate-half RoPE: lo' = lo cos - hi sin, hi' = hi cos + lo sin
    float cf[N], sf[N];
    {
      const float4 *cp = reinterpret_cast<const float4 *>(cos_t + size_t(__ldg(positions + t)) * HALF + d0);
      const float4 *sp = reinterpret_cast<const float4 *>(sin_t + size_t(__ldg(positions + t)) * HALF + d0);
#pragma unroll
      for (int q = 0; q < N / 4; ++q) {
        const float4 c4 = __ldg(cp + q), s4 = __ldg(sp + q);
        cf[4 * q] = c4.x; cf[4 * q + 1] = c4.y; cf[4 * q + 2] = c4.z; cf[4 * q + 3] = c4.w;
        sf[4 * q] = s4.x; sf[4 * q + 1] = s4.y; sf[4 * q + 2] = s4.z; sf[4 * q + 3] = s4.w;
      }
    }
    float yl[N], yh[N];
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      float u0, u1, v0, v1;
      mul2(u0, u1, fh[i], fh[i + 1], sf[i], sf[i + 1]);    // hi sin
      mul2(v0, v1, fl[i], fl[i + 1], sf[i], sf[i + 1]);    // lo sin
      fma2(yl[i], yl[i + 1], fl[i], fl[i + 1], cf[i], cf[i + 1], -u0, -u1);
      fma2(yh[i], yh[i + 1], fh[i], fh[i + 1], cf[i], cf[i + 1], v0, v1);
    }
    if (!live) continue;
    T *dst = is_q ? q_out + (size_t(t) * hq + h) * D + d0
                  : k_pool + ((size_t(blk) * hkv + (h - hq)) * (size_t(1) << bs_shift) + off) * D + d0;
    reinterpret_cast<uint4 *>(dst)[0] = R::pack(yl);
    reinterpret_cast<uint4 *>(dst + HALF)[0] = R::pack(yh);
  }
}

template <typename T, int D>
cudaError_t launch_vec(const void *qkv, const void *bias, const void *qn, const void *kn, const void *cs,
                       const void *sn, const int32_t *positions, const int64_t *slots, void *q_out, void *k_pool,
                       void *v_pool, int T_, int hq, int hkv, int bs_shift, float eps, cudaStream_t st) {
  constexpr int KT = 2;
  const int items = (hq + 2 * hkv) * (D / 2 / Raw16<T>::N);
  const int bx = (items + 31) / 32 * 32;
  if (bx > 256) return cudaErrorInvalidValue;
  const int by = std::max(1, 256 / bx);
  const int tokens_per_cta = by * KT;
  const dim3 block(bx, by), grid((T_ + tokens_per_cta - 1) / tokens_per_cta);
  qk_norm_rope_append_vec_kernel<T, D, KT><<<grid, block, 0, st>>>(
      (const T *)qkv, (const T *)bias, (const T *)qn, (const T *)kn, (const float *)cs, (const float *)sn, positions,
      slots, (T *)q_out, (T *)k_pool, (T *)v_pool, T_, hq, hkv, bs_shift, eps);
  return cudaGetLastError();
}

inline bool host_aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
cudaError_t launch_typed(const void *qkv, const void *bias, const void *qn, const void *kn, const void *cs,
                         const void *sn, const int32_t *positions, const int64_t *slots, void *q_out,
                         void *k_pool, void *v_pool, int T_, int hq, int hkv, int D, int bs, float eps,
                         cudaStream_t st) {
  int bs_shift = 0;
  while ((1 << bs_shift) < bs) ++bs_shift;
  // the vector build: one row of at most 256 threads holds every pair item of a token
  const bool vec = (D == 128 || D == 64) && (1 << bs_shift) == bs && (hq + 2 * hkv) * (D / 2 / Raw16<T>::N) <= 256 &&
                   host_aligned16(qkv) && (!bias || host_aligned16(bias)) &&
                   (!qn || host_aligned16(qn)) && (!kn || host_aligned16(kn)) && host_aligned16(cs) &&
                   host_aligned16(sn) && host_aligned16(q_out) && host_aligned16(k_pool) && host_aligned16(v_pool);
  if (vec) {
    if (D == 128)
      return launch_vec<T, 128>(qkv, bias, qn, kn, cs, sn, positions, slots, q_out, k_pool, v_pool, T_, hq, hkv,
                                bs_shift, eps, st);
    return launch_vec<T, 64>(qkv, bias, qn, kn, cs, sn, positions, slots, q_out, k_pool, v_pool, T_, hq, hkv,
                             bs_shift, eps, st);
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
                                       cudaStream_t st) {
  if (num_tokens == 0) return cudaSuccess;
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || block_size <= 0) return cudaErrorInvalidValue;
  switch (dtype) {
    case MS_DTYPE_F32:
      return launch_typed<float>(qkv, bias, q_norm_w, k_norm_w, cos_table, sin_table, positions, slot_mapping,
                                 q_out, k_pool, v_pool, num_tokens, num_heads, num_kv_heads, head_dim,
                                 block_size, eps, st);
    case MS_DTYPE_BF16:
      return launch_typed<__nv_bfloat16>(qkv, bias, q_norm_w, k_norm_w, cos_table, sin_table, positions,
                                         slot_mapping, q_out, k_pool, v_pool, num_tokens, num_heads,
                                         num_kv_heads, head_dim, block_size, eps, st);
    case MS_DTYPE_F16:
      return launch_typed<__half>(qkv, bias, q_norm_w, k_norm_w, cos_table, sin_table, positions, slot_mapping,
                                  q_out, k_pool, v_pool, num_tokens, num_heads, num_kv_heads, head_dim,
                                  block_size, eps, st);
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
                                            static_cast<cudaStream_t>(stream)));
}
