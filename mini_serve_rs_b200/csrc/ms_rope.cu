// K5 + K2: fused (bias) + per-head QK RMSNorm + rotate-half RoPE + paged KV append.
//
// Restates, per packed token, Attention::forward up to the cache append
// (src/backends/qwen2.rs:287-313): projections arrive as one fused
// [T, (Hq + 2 Hkv) * D] GEMM output; bias (qwen2.rs:234-248) and QK-norm
// (qwen2.rs:297-304, the RmsNorm of :68-75 over head_dim) are applied before
// RoPE (apply_rope, :132-142, with cos/sin tables of :91-108 stored in the
// model dtype); the rotated K and the V rows are written straight into their
// paged-pool slot (the append of :349-361, now into 16-token pages addressed
// by slot_mapping), the rotated q into a dense [T, Hq, D] buffer for K3.
// Every product and sum is rounded to the model dtype where Candle rounds.
//
// One warp per (token, head); lane l holds dims [l*D/32, (l+1)*D/32), so the
// rotate-half partner of each dim sits in lane l ^ 16.
#include "ms_common.cuh"
#include "ms_internal.h"

namespace ms {
namespace {

template <typename T, int D>
__global__ void qk_norm_rope_append_kernel(const T *__restrict__ qkv, const T *__restrict__ bias,
                                           const T *__restrict__ qn, const T *__restrict__ kn,
                                           const T *__restrict__ cos_t, const T *__restrict__ sin_t,
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
    for (int i = 0; i < DPL; ++i) x[i] = round_to<T>(x[i] + b[i]);
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
    float w[DPL];
    if constexpr (DPL == 4) Vec4<T>::load(nw + d0, w); else Vec2<T>::load(nw + d0, w);
#pragma unroll
    for (int i = 0; i < DPL; ++i) x[i] = round_to<T>(round_to<T>(x[i] / norm) * w[i]);
  }

  // rotate-half RoPE
  const int pos = positions[t];
  const int j0 = d0 % HALF;
  float c[DPL], s[DPL];
  const T *cp = cos_t + size_t(pos) * HALF + j0;
  const T *sp = sin_t + size_t(pos) * HALF + j0;
  if constexpr (DPL == 4) { Vec4<T>::load(cp, c); Vec4<T>::load(sp, s); }
  else { Vec2<T>::load(cp, c); Vec2<T>::load(sp, s); }
  float partner[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) partner[i] = __shfl_xor_sync(kFull, x[i], 16);
  const bool lower = lane < 16;
  float y[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const float rot = lower ? -partner[i] : partner[i];
    const float a = round_to<T>(x[i] * c[i]);
    const float b = round_to<T>(rot * s[i]);
    y[i] = round_to<T>(a + b);
  }

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

template <typename T>
cudaError_t launch_typed(const void *qkv, const void *bias, const void *qn, const void *kn, const void *cs,
                         const void *sn, const int32_t *positions, const int64_t *slots, void *q_out,
                         void *k_pool, void *v_pool, int T_, int hq, int hkv, int D, int bs, float eps,
                         cudaStream_t st) {
  const long long warps = (long long)T_ * (hq + 2 * hkv);
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  if (D == 128) {
    qk_norm_rope_append_kernel<T, 128><<<blocks, threads, 0, st>>>(
        (const T *)qkv, (const T *)bias, (const T *)qn, (const T *)kn, (const T *)cs, (const T *)sn, positions,
        slots, (T *)q_out, (T *)k_pool, (T *)v_pool, T_, hq, hkv, bs, eps);
  } else if (D == 64) {
    qk_norm_rope_append_kernel<T, 64><<<blocks, threads, 0, st>>>(
        (const T *)qkv, (const T *)bias, (const T *)qn, (const T *)kn, (const T *)cs, (const T *)sn, positions,
        slots, (T *)q_out, (T *)k_pool, (T *)v_pool, T_, hq, hkv, bs, eps);
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
