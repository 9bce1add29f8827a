// K4 fused residual-add + RMSNorm, K6 glue (SiLU-mul, argmax), dtype conversion.
//
// K4 restates RmsNorm::forward (src/backends/qwen2.rs:68-75) fused with the
// residual adds of DecoderLayer::forward (qwen2.rs:420-427) and of the batched
// decode (qwen2.rs:751-756).  All arithmetic is f32 and every stored value is
// rounded once: the residual output is the rounded sum, and the norm is taken
// from the unrounded f32 sum, y = round(s * (1 / sqrt(mean(s^2) + eps)) * w),
// so a 16-bit output is within half a unit in its last place of the f32
// reference's value computed from the same inputs.  In f32 mode the division
// is the reference's x / norm.  One CTA (or one warp) per row, 16-byte
// vector loads, warp-shuffle (+ shared-memory) reduce.
#include <algorithm>
#include <atomic>
#include <type_traits>

#include "ms_common.cuh"
#include "ms_internal.h"

namespace ms {
namespace {

inline bool host_aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T> struct V16;  // 16 bytes of T
template <> struct V16<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const float *p, float (&o)[4]) { Vec4<float>::load(p, o); }
  static __device__ __forceinline__ void store(float *p, const float (&o)[4]) { Vec4<float>::store(p, o); }
};
template <typename T> struct V16Half {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const T *p, float (&o)[8]) {
    float a[4], b[4];
    Vec4<T>::load(p, a);
    Vec4<T>::load(p + 4, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) { o[i] = a[i]; o[4 + i] = b[i]; }
  }
  static __device__ __forceinline__ void store(T *p, const float (&o)[8]) {
    float a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) { a[i] = o[i]; b[i] = o[4 + i]; }
    Vec4<T>::store(p, a);
    Vec4<T>::store(p + 4, b);
  }
};
template <> struct V16<__nv_bfloat16> : V16Half<__nv_bfloat16> {};
template <> struct V16<__half> : V16Half<__half> {};

__device__ __forceinline__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// x / norm * w with one rounding at the store: f32 keeps the reference's
// division; 16-bit outputs multiply by the row's reciprocal norm (its error is
// far below the output's rounding).
template <typename T>
__device__ __forceinline__ float norm_weight(float x, float norm, float rn, float w) {
  if constexpr (std::is_same<T, float>::value) return (x / norm) * w;
  return x * rn * w;
}

template <typename T>
__global__ void add_rmsnorm_kernel(const T *__restrict__ x, const T *__restrict__ r,
                                   const int32_t *__restrict__ row_index, const T *__restrict__ w,
                                   T *__restrict__ resid_out, T *__restrict__ norm_out, int hidden,
                                   float eps) {
  constexpr int N = V16<T>::N;
  __shared__ float red[32];
  const int row = blockIdx.x;
  const size_t src = row_index ? size_t(row_index[row]) : size_t(row);
  const int c = threadIdx.x;  // chunk of N elements
  const bool active = c * N < hidden;
  float s[N];
  float sq = 0.f;
  if (active) {
    V16<T>::load(x + src * hidden + c * N, s);
    if (r) {
      float rr[N];
      V16<T>::load(r + src * hidden + c * N, rr);
#pragma unroll
      for (int i = 0; i < N; ++i) s[i] += rr[i];
    }
    if (resid_out) V16<T>::store(resid_out + size_t(row) * hidden + c * N, s);  // rounds once
#pragma unroll
    for (int i = 0; i < N; ++i) sq = fmaf(s[i], s[i], sq);
  }
  const float total = block_sum(sq, red);
  const float norm = sqrtf(total / float(hidden) + eps);
  const float rn = 1.0f / norm;
  if (active) {
    float ww[N], y[N];
    V16<T>::load(w + c * N, ww);
#pragma unroll
    for (int i = 0; i < N; ++i) y[i] = norm_weight<T>(s[i], norm, rn, ww[i]);
    V16<T>::store(norm_out + size_t(row) * hidden + c * N, y);
  }
}

// Warp-per-row K4 (the path for 16-byte aligned rows of up to 8 x 32 chunks,
// i.e. hidden <= 2048 in 16-bit types; wider rows use add_rmsnorm_kernel): a
// warp reduces its row with shuffles only.  The grid holds a few CTAs of 4
// warps per SM and each warp walks rows warps-apart, loading its next row
// (x, r: CPL 16-byte chunks per lane each) before it works on the current
// one, so every SM keeps reads in flight while it writes: reads and writes of
// different rows overlap instead of running as one read wave then one write
// wave.  The f32 sums stay in registers between the reduction and the output.
template <typename T, int CPL>
__global__ void __launch_bounds__(128) add_rmsnorm_warp_kernel(const T *__restrict__ x, const T *__restrict__ r,
                                                               const int32_t *__restrict__ row_index,
                                                               const T *__restrict__ w, T *__restrict__ resid_out,
                                                               T *__restrict__ norm_out, int rows, int hidden,
                                                               float eps) {
  using R = Raw16<T>;
  constexpr int N = R::N;
  const int lane = threadIdx.x & 31;
  const int chunks = hidden / N;
  const int stride = gridDim.x * 4;
  int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  uint4 nx[CPL], nr[CPL];  // the next row's x and r
  auto fetch = [&](int rw) {
    const size_t src = row_index ? size_t(__ldg(row_index + rw)) : size_t(rw);
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + src * hidden);
    const uint4 *rr = r ? reinterpret_cast<const uint4 *>(r + src * hidden) : nullptr;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = lane + 32 * k;
      if (c < chunks) {
        nx[k] = __ldg(xr + c);
        if (rr) nr[k] = __ldg(rr + c);
      }
    }
  };
  if (row < rows) fetch(row);
  const uint4 *wr = reinterpret_cast<const uint4 *>(w);
  while (row < rows) {  // warp-uniform
    float f[CPL][N];  // the f32 sums
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = lane + 32 * k;
      if (c < chunks) {
        R::unpack(nx[k], f[k]);
        if (r) {
          float b[N];
          R::unpack(nr[k], b);
#pragma unroll
          for (int i = 0; i < N; ++i) f[k][i] += b[i];
          if (resid_out) reinterpret_cast<uint4 *>(resid_out + size_t(row) * hidden)[c] = R::pack(f[k]);
        } else if (resid_out) {
          reinterpret_cast<uint4 *>(resid_out + size_t(row) * hidden)[c] = nx[k];
        }
#pragma unroll
        for (int i = 0; i < N; ++i) sq = fmaf(f[k][i], f[k][i], sq);
      }
    }
    // the current row is in registers: fetch the next one while this one is reduced and written
    const int next = row + stride;
    if (next < rows) fetch(next);
    sq = warp_sum(sq);
    const float norm = sqrtf(sq / float(hidden) + eps);
    const float rn = 1.0f / norm;
    uint4 *out = reinterpret_cast<uint4 *>(norm_out + size_t(row) * hidden);
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = lane + 32 * k;
      if (c < chunks) {
        float ww[N], y[N];
        R::unpack(__ldg(wr + c), ww);
#pragma unroll
        for (int i = 0; i < N; ++i) y[i] = norm_weight<T>(f[k][i], norm, rn, ww[i]);
        out[c] = R::pack(y);
      }
    }
    row = next;
  }
}

template <typename T>
cudaError_t launch_add_rmsnorm_warp(const void *x, const void *r, const int32_t *row_index, const void *w,
                                    void *resid_out, void *norm_out, int rows, int hidden, float eps,
                                    cudaStream_t st) {
  const int per_lane = (hidden / Raw16<T>::N + 31) / 32;
  auto go = [&](auto kern) {
    // as many CTAs of 4 warps as are resident at once (one wave); rows beyond it are walked by the same warps
    static std::atomic<int> resident{0};
    int n = resident.load(std::memory_order_relaxed);
    if (n == 0) {
      int dev = 0, sms = 0, per_sm = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, 0);
      n = std::max(1, per_sm * sms);
      resident.store(n, std::memory_order_relaxed);
    }
    const dim3 grid(std::min((rows + 3) / 4, n));
    kern<<<grid, 128, 0, st>>>((const T *)x, (const T *)r, row_index, (const T *)w, (T *)resid_out, (T *)norm_out,
                               rows, hidden, eps);
    return cudaGetLastError();
  };
  if (per_lane <= 1) return go(add_rmsnorm_warp_kernel<T, 1>);
  if (per_lane <= 2) return go(add_rmsnorm_warp_kernel<T, 2>);
  if (per_lane <= 4) return go(add_rmsnorm_warp_kernel<T, 4>);
  return go(add_rmsnorm_warp_kernel<T, 8>);
}

// act = silu(gate) * up (qwen2.rs:169-174) in f32, rounded once; gate_up =
// [gate | up] per row.
template <typename T>
__global__ void silu_mul_kernel(const T *__restrict__ gu, T *__restrict__ out, int rows, int inter) {
  constexpr int N = V16<T>::N;
  const int chunks = inter / N;
  const long long total = (long long)rows * chunks;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / chunks;
    const int c = int(i % chunks);
    float g[N], u[N], y[N];
    V16<T>::load(gu + row * 2 * inter + c * N, g);
    V16<T>::load(gu + row * 2 * inter + inter + c * N, u);
#pragma unroll
    for (int k = 0; k < N; ++k) y[k] = g[k] / (1.0f + expf(-g[k])) * u[k];  // one rounding, at the store
    V16<T>::store(out + row * inter + c * N, y);
  }
}

// Row-wise argmax of f32 logits; ties resolve to the lowest index.
__global__ void argmax_kernel(const float *__restrict__ logits, int vocab, int32_t *__restrict__ out,
                              const int32_t *__restrict__ row_slot, int32_t *__restrict__ slot_last) {
  const int row = blockIdx.x;
  const float *l = logits + size_t(row) * vocab;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  if ((vocab & 3) == 0) {
    const int n4 = vocab >> 2;
    const float4 *l4 = reinterpret_cast<const float4 *>(l);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = l4[i];
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (vv[k] > best) { best = vv[k]; bi = 4 * i + k; }
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += blockDim.x)
      if (l[i] > best) { best = l[i]; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(kFull, best, o);
    const int oi = __shfl_xor_sync(kFull, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sb[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(kFull, best, o);
      const int oi = __shfl_xor_sync(kFull, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) {
      if (bi == 0x7fffffff) bi = 0;  // all NaN / -inf
      out[row] = bi;
      if (row_slot && slot_last) slot_last[row_slot[row]] = bi;
    }
  }
}

template <typename S, typename D>
__global__ void convert_kernel(const S *__restrict__ src, D *__restrict__ dst, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = Elem<D>::from_f(Elem<S>::to_f(src[i]));
}

template <typename S>
cudaError_t convert_from(const S *src, void *dst, int dst_dtype, int64_t n, cudaStream_t st) {
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n + threads - 1) / threads, 148 * 32);
  switch (dst_dtype) {
    case MS_DTYPE_F32: convert_kernel<S, float><<<blocks, threads, 0, st>>>(src, (float *)dst, n); break;
    case MS_DTYPE_BF16: convert_kernel<S, __nv_bfloat16><<<blocks, threads, 0, st>>>(src, (__nv_bfloat16 *)dst, n); break;
    case MS_DTYPE_F16: convert_kernel<S, __half><<<blocks, threads, 0, st>>>(src, (__half *)dst, n); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_add_rmsnorm(const void *x, const void *r, const int32_t *row_index, const void *w,
                               void *resid_out, void *norm_out, int rows, int hidden, float eps,
                               int dtype, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  if (rows < 0 || hidden <= 0) return cudaErrorInvalidValue;
  const int n = dtype == MS_DTYPE_F32 ? 4 : 8;
  if (hidden % n != 0 || hidden / n > 1024) return cudaErrorInvalidValue;
  const bool vec16 = (hidden * (dtype == MS_DTYPE_F32 ? 4 : 2)) % 16 == 0 && hidden / n <= 8 * 32 && host_aligned16(x) &&
                     (!r || host_aligned16(r)) && host_aligned16(w) && (!resid_out || host_aligned16(resid_out)) &&
                     host_aligned16(norm_out);
  if (vec16) {
    switch (dtype) {
      case MS_DTYPE_F32: return launch_add_rmsnorm_warp<float>(x, r, row_index, w, resid_out, norm_out, rows, hidden, eps, st);
      case MS_DTYPE_BF16: return launch_add_rmsnorm_warp<__nv_bfloat16>(x, r, row_index, w, resid_out, norm_out, rows, hidden, eps, st);
      case MS_DTYPE_F16: return launch_add_rmsnorm_warp<__half>(x, r, row_index, w, resid_out, norm_out, rows, hidden, eps, st);
      default: return cudaErrorInvalidValue;
    }
  }
  const int threads = ((hidden / n + 31) / 32) * 32;
  switch (dtype) {
    case MS_DTYPE_F32:
      add_rmsnorm_kernel<float><<<rows, threads, 0, st>>>((const float *)x, (const float *)r, row_index,
                                                          (const float *)w, (float *)resid_out,
                                                          (float *)norm_out, hidden, eps);
      break;
    case MS_DTYPE_BF16:
      add_rmsnorm_kernel<__nv_bfloat16><<<rows, threads, 0, st>>>(
          (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)r, row_index, (const __nv_bfloat16 *)w,
          (__nv_bfloat16 *)resid_out, (__nv_bfloat16 *)norm_out, hidden, eps);
      break;
    case MS_DTYPE_F16:
      add_rmsnorm_kernel<__half><<<rows, threads, 0, st>>>((const __half *)x, (const __half *)r, row_index,
                                                           (const __half *)w, (__half *)resid_out,
                                                           (__half *)norm_out, hidden, eps);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void *gu, void *out, int rows, int inter, int dtype, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const int n = dtype == MS_DTYPE_F32 ? 4 : 8;
  if (rows < 0 || inter % n != 0) return cudaErrorInvalidValue;
  const long long total = (long long)rows * (inter / n);
  const int threads = 256;
  const long long blocks = std::min<long long>((total + threads - 1) / threads, 148LL * 16);
  switch (dtype) {
    case MS_DTYPE_F32: silu_mul_kernel<float><<<blocks, threads, 0, st>>>((const float *)gu, (float *)out, rows, inter); break;
    case MS_DTYPE_BF16: silu_mul_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>((const __nv_bfloat16 *)gu, (__nv_bfloat16 *)out, rows, inter); break;
    case MS_DTYPE_F16: silu_mul_kernel<__half><<<blocks, threads, 0, st>>>((const __half *)gu, (__half *)out, rows, inter); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float *logits, int rows, int vocab, int32_t *out, const int32_t *row_slot,
                          int32_t *slot_last_token, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  if (rows < 0 || vocab <= 0) return cudaErrorInvalidValue;
  argmax_kernel<<<rows, 1024, 0, st>>>(logits, vocab, out, row_slot, slot_last_token);
  return cudaGetLastError();
}

cudaError_t launch_convert(const void *src, int src_dtype, void *dst, int dst_dtype, int64_t n,
                           cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  switch (src_dtype) {
    case MS_DTYPE_F32: return convert_from<float>((const float *)src, dst, dst_dtype, n, st);
    case MS_DTYPE_BF16: return convert_from<__nv_bfloat16>((const __nv_bfloat16 *)src, dst, dst_dtype, n, st);
    case MS_DTYPE_F16: return convert_from<__half>((const __half *)src, dst, dst_dtype, n, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ms

// ---- C ABI --------------------------------------------------------------------
extern "C" int ms_launch_add_rmsnorm(const void *x, const void *r, const int32_t *row_index, const void *w,
                                     void *resid_out, void *norm_out, int32_t rows, int32_t hidden,
                                     float eps, int32_t dtype, void *stream) {
  return int(ms::launch_add_rmsnorm(x, r, row_index, w, resid_out, norm_out, rows, hidden, eps, dtype,
                                    static_cast<cudaStream_t>(stream)));
}

extern "C" int ms_launch_silu_mul(const void *gate_up, void *out, int32_t rows, int32_t inter,
                                  int32_t dtype, void *stream) {
  return int(ms::launch_silu_mul(gate_up, out, rows, inter, dtype, static_cast<cudaStream_t>(stream)));
}

extern "C" int ms_launch_argmax(const float *logits, int32_t rows, int32_t vocab, int32_t *out,
                                void *stream) {
  return int(ms::launch_argmax(logits, rows, vocab, out, nullptr, nullptr, static_cast<cudaStream_t>(stream)));
}

// prototype-compatible RMSNorm (mini_serve_kernels.cu:247-265): same checks,
// default stream, cudaError_t as int.  The f16 prototype rounds x*inv_rms to
// f16 before the weight multiply (.cu:183-184), as this kernel does.
extern "C" int launch_rmsnorm_f32(const float *d_x, const float *d_w, float *d_out, int num_rows,
                                  int hidden_size, float eps) {
  if (num_rows <= 0 || hidden_size <= 0) return int(cudaErrorInvalidValue);
  return int(ms::launch_add_rmsnorm(d_x, nullptr, nullptr, d_w, nullptr, d_out, num_rows, hidden_size,
                                    eps, MS_DTYPE_F32, 0));
}

extern "C" int launch_rmsnorm_f16(const void *d_x, const void *d_w, void *d_out, int num_rows,
                                  int hidden_size, float eps) {
  if (num_rows <= 0 || hidden_size <= 0) return int(cudaErrorInvalidValue);
  return int(ms::launch_add_rmsnorm(d_x, nullptr, nullptr, d_w, nullptr, d_out, num_rows, hidden_size,
                                    eps, MS_DTYPE_F16, 0));
}

extern "C" int launch_rmsnorm_bf16(const void *d_x, const void *d_w, void *d_out, int num_rows,
                                   int hidden_size, float eps) {
  if (num_rows <= 0 || hidden_size <= 0) return int(cudaErrorInvalidValue);
  return int(ms::launch_add_rmsnorm(d_x, nullptr, nullptr, d_w, nullptr, d_out, num_rows, hidden_size,
                                    eps, MS_DTYPE_BF16, 0));
}
