// Pieces shared by the K3 paged-attention kernels (SIMT f32 build and the
// tensor-core 16-bit build): launch parameters, PTX wrappers for mbarriers,
// bulk / tensor TMA copies, ldmatrix and mma.sync, the cross-warp merge
// epilogue and the partition combine kernel.
#pragma once

#include <cuda.h>

#include "ms_common.cuh"
#include "ms_internal.h"

namespace ms {
namespace attn {

constexpr int kBS = 16;              // tokens per KV page (kv_cache.rs block_size)
constexpr int kWarps = 4;            // warps per CTA
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kWaitLimit = 1 << 22;  // bounded mbarrier polling

struct Params {
  const void *q;
  const void *k_pool;
  const void *v_pool;
  const int32_t *block_tables;
  const int32_t *row_table;
  const int32_t *row_ctx;
  const int32_t *row_index;  // launch row -> packed row (null: identity)
  void *out;
  float *ws_o;    // [launch rows][Hkv][max_parts][G][D]
  float2 *ws_ml;  // [rows][Hkv][max_parts][G]
  unsigned *status;
  int max_blocks_per_seq;
  int num_kv_heads;
  int part_blocks;  // pages per partition
  int max_parts;
  float qscale;    // softmax scale * log2(e)
  int wait_limit;  // polls before a wait in the page loop gives up (the drain after it uses kWaitLimit)
};

// ---- PTX wrappers ------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// 1-D bulk copy global -> shared (no multicast), completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// 4-D tiled tensor copy global -> shared (no multicast), completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Polls with an iteration limit; returns false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int limit = kWaitLimit) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D = A(16x16, row) * B(16x8, col) + D with f32 accumulators.
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma_16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                  uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- epilogue: merge the CTA's warps, write the output or the partition ---------
// mo [kWarps][G][D] (unnormalised O, relative to the warp's running max),
// mm / ml [kWarps][G] (running max in base 2, running sum) are in shared
// memory and visible to the whole CTA when this is called.
template <typename T, int D, int G>
__device__ __forceinline__ void merge_warps_store(const Params &p, const float *mo, const float *mm,
                                                  const float *ml, int row, int ri, int kvh, int part,
                                                  bool single) {
  for (int i = threadIdx.x; i < G * D; i += kWarps * 32) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mm[w * G + h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = mm[w * G + h];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      L += f * ml[w * G + h];
      O += f * mo[(w * G + h) * D + d];
    }
    const size_t qh = size_t(row) * p.num_kv_heads * G + size_t(kvh) * G + h;
    if (single) {
      static_cast<T *>(p.out)[qh * D + d] = Elem<T>::from_f(L > 0.f ? O / L : 0.f);
    } else {
      const size_t slot = (size_t(ri) * p.num_kv_heads + kvh) * p.max_parts + part;
      p.ws_o[(slot * G + h) * D + d] = O;
      if (d == 0) p.ws_ml[slot * G + h] = make_float2(M, L);
    }
  }
}

// Merge the partitions of rows that needed more than one (log-sum-exp).
template <typename T, int D, int G>
__global__ void combine_kernel(Params p) {
  const int ri = blockIdx.x;
  const int row = p.row_index ? p.row_index[ri] : ri;
  const int kvh = blockIdx.y;
  const int ctx = p.row_ctx[row];
  const int nblk = max(0, (ctx + kBS - 1) / kBS);
  const int nparts = min(p.max_parts, (nblk + p.part_blocks - 1) / p.part_blocks);
  if (nparts <= 1) return;
  const size_t base = (size_t(ri) * p.num_kv_heads + kvh) * p.max_parts;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
    for (int s = 0; s < nparts; ++s) M = fmaxf(M, p.ws_ml[(base + s) * G + h].x);
    float L = 0.f, O = 0.f;
    for (int s = 0; s < nparts; ++s) {
      const float2 ml = p.ws_ml[(base + s) * G + h];
      const float f = (ml.x == -INFINITY) ? 0.f : exp2f(ml.x - M);
      L += f * ml.y;
      O += f * p.ws_o[((base + s) * G + h) * D + d];
    }
    const size_t qh = size_t(row) * p.num_kv_heads * G + size_t(kvh) * G + h;
    static_cast<T *>(p.out)[qh * D + d] = Elem<T>::from_f(L > 0.f ? O / L : 0.f);
  }
}

// Launch the partition combine if any row can have more than one partition.
template <typename T, int D, int G>
cudaError_t launch_combine(const Params &p, int num_rows, cudaStream_t stream) {
  if (p.max_parts <= 1) return cudaSuccess;
  dim3 g2(num_rows, p.num_kv_heads);
  combine_kernel<T, D, G><<<g2, (G * D < 1024 ? G * D : 1024), 0, stream>>>(p);
  return cudaGetLastError();
}

// Tensor-core (mma.sync) build for 16-bit K/V; maps may be null (encoded per call).
cudaError_t launch_attention_tc(const Params &p, const AttnArgs &a, int group, cudaStream_t stream);
bool attention_tc_supported(int dtype, int head_dim, int group);

}  // namespace attn
}  // namespace ms
