// Tensor parallelism: the all-reduce after o_proj / down_proj fused with the
// residual add + RMSNorm that follows it, over NVLink peer memory.
//
// The reference has no tensor parallelism.  The 7B configuration shards the
// model by KV head: o_proj and down_proj are row-sharded, so each rank's GEMM
// produces a partial sum of the layer output, which must be summed over ranks
// before the residual add and the next RMSNorm (DecoderLayer::forward,
// src/backends/qwen2.rs:414-428).  Instead of an NCCL all-reduce followed by
// K4, each rank's GEMM writes its partial sum into a buffer the other ranks
// have mapped (CUDA IPC), and one kernel per rank:
//   1. start barrier, per CTA: CTA b stores the call's epoch into slot
//      [b][my rank] of every rank's signal array (st.release.sys), then waits
//      (ld.acquire.sys, bounded by a 20 s global-timer limit) until every
//      rank's CTA b has done the same.  A rank's CTA b runs only after that
//      rank's GEMM finished, so all partial sums are complete;
//   2. one CTA per row: sum the row over ranks in rank order 0..tp-1 in f32
//      (every rank computes the same bits), add the residual in f32, store
//      that sum rounded once as the new residual, and RMSNorm it from the f32
//      sum as K4 does -- the rows read over NVLink once per rank.
// Two partial-sum buffers alternate (o_proj, down_proj, o_proj, ...).  A
// rank overwrites a buffer only after its next call's barrier, which every
// rank passes only after finishing the previous call: the one that read it.
// A wait that runs out records kStatusWaitTimeout, skips the row work and
// returns; the host turns the status into MS_E_DEVICE and quarantines.
#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <vector>

#include "ms_common.cuh"
#include "ms_engine.h"

namespace ms {
namespace {

constexpr int kMaxTp = 8;
constexpr int kMaxCtas = 256;
constexpr uint64_t kWaitNs = 20ull * 1000 * 1000 * 1000;

struct ArArgs {
  const void *bufs[kMaxTp];  // each rank's partial sums [rows_total, hidden] (own rank: local)
  uint32_t *sig[kMaxTp];     // each rank's signal array [kMaxCtas][kMaxTp]
  int tp, rank;
  uint32_t epoch;
  const void *residual;
  const int32_t *row_index;  // null: row i reads row i
  const void *w;
  void *resid_out;           // null: not written (final norm)
  void *norm_out;
  int rows, hidden;
  float eps;
  unsigned *status;
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One CTA per row (rows strided by the grid), one 16-byte chunk per thread
// (hidden / chunk <= 1024, which engine creation checks): every load of a
// row -- the TP remote partial sums and the residual -- is issued before any
// arithmetic, so a row costs one NVLink round trip, not one per chunk.
template <typename T, int TP>
__global__ void __launch_bounds__(1024) ar_add_rmsnorm_kernel(ArArgs a) {
  using R = Raw16<T>;
  constexpr int N = R::N;
  __shared__ float red[32];
  const int b = blockIdx.x;

  // 1. start barrier with every rank's CTA b
  bool ok = true;
  if (threadIdx.x < TP) {
    st_release_sys(a.sig[threadIdx.x] + b * kMaxTp + a.rank, a.epoch);
    const uint32_t *f = a.sig[a.rank] + b * kMaxTp + threadIdx.x;
    const uint64_t t0 = global_ns();
    while (int32_t(ld_acquire_sys(f) - a.epoch) < 0) {
      if (global_ns() - t0 > kWaitNs) {
        ok = false;
        atomicOr(a.status, kStatusWaitTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  if (!__syncthreads_and(ok)) return;

  // 2. rows: sum over ranks in rank order, residual add, RMSNorm
  const int c = threadIdx.x;
  const bool active = c < a.hidden / N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  for (int i = b; i < a.rows; i += gridDim.x) {
    const size_t src = a.row_index ? size_t(a.row_index[i]) : size_t(i);
    uint4 v[TP], rv = make_uint4(0, 0, 0, 0);
    float sf[N];
    float sq = 0.f;
    if (active) {
#pragma unroll
      for (int r = 0; r < TP; ++r)
        v[r] = __ldcg(reinterpret_cast<const uint4 *>(static_cast<const T *>(a.bufs[r]) + src * a.hidden) + c);
      rv = reinterpret_cast<const uint4 *>(static_cast<const T *>(a.residual) + src * a.hidden)[c];
      float acc[N], f[N], rr[N];
#pragma unroll
      for (int e = 0; e < N; ++e) acc[e] = 0.f;
#pragma unroll
      for (int r = 0; r < TP; ++r) {
        R::unpack(v[r], f);
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] += f[e];
      }
      R::unpack(rv, rr);
#pragma unroll
      for (int e = 0; e < N; ++e) {
        sf[e] = acc[e] + rr[e];  // f32; rounded once where it is stored
        sq = fmaf(sf[e], sf[e], sq);
      }
      if (a.resid_out) reinterpret_cast<uint4 *>(static_cast<T *>(a.resid_out) + size_t(i) * a.hidden)[c] = R::pack(sf);
    }
    // block sum of squares
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    float tot = lane < nw ? red[lane] : 0.f;
    tot = warp_sum(tot);
    __syncthreads();  // red is reused by the next row
    if (active) {
      const float norm = sqrtf(tot / float(a.hidden) + a.eps);
      const float rn = 1.0f / norm;
      float ww[N], y[N];
      R::unpack(reinterpret_cast<const uint4 *>(a.w)[c], ww);
#pragma unroll
      for (int e = 0; e < N; ++e)
        y[e] = std::is_same<T, float>::value ? (sf[e] / norm) * ww[e] : sf[e] * rn * ww[e];
      reinterpret_cast<uint4 *>(static_cast<T *>(a.norm_out) + size_t(i) * a.hidden)[c] = R::pack(y);
    }
  }
}

}  // namespace

// Allocates and exchanges the peer-mapped buffers.  Every rank calls it at
// engine creation (it runs NCCL collectives); all ranks end up using the fused
// path only if all of them set it up (a MIN over ranks), else all use NCCL.
int tp_fused_setup(Engine *eng) {
  eng->ar_fused = false;
  if (eng->tp <= 1) return MS_OK;
  const char *env = std::getenv("MS_TP_FUSED");
  int32_t want = !(env && std::strcmp(env, "0") == 0) && (eng->tp == 2 || eng->tp == 4 || eng->tp == 8) &&
                 eng->H % (16 / int(eng->esize)) == 0 && eng->H / (16 / int(eng->esize)) <= 1024;
  const size_t part = (size_t(eng->opts.max_tokens_per_step) * eng->H * eng->esize + 255) & ~size_t(255);
  const size_t sig_bytes = size_t(kMaxCtas) * kMaxTp * sizeof(uint32_t);
  cudaIpcMemHandle_t mine{};
  if (want) {
    if (cudaMalloc(&eng->ar_sym, 2 * part + sig_bytes) != cudaSuccess ||
        cudaMemset(static_cast<char *>(eng->ar_sym) + 2 * part, 0, sig_bytes) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine, eng->ar_sym) != cudaSuccess) {
      cudaGetLastError();
      want = 0;
    }
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return eng->fail(MS_E_DEVICE, "tp setup: device sync");
  // exchange handles (all ranks take part even when they opt out)
  void *d_x = nullptr;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  if (cudaMalloc(&d_x, hb * eng->tp + 256) != cudaSuccess) return eng->fail(MS_E_DEVICE, "tp setup: cudaMalloc");
  std::vector<char> host(hb * eng->tp + 256, 0);
  std::memcpy(host.data() + hb * eng->rank, &mine, hb);
  int32_t *d_ok = reinterpret_cast<int32_t *>(static_cast<char *>(d_x) + hb * eng->tp);
  std::memcpy(host.data() + hb * eng->tp, &want, sizeof(want));
  cudaMemcpy(d_x, host.data(), host.size(), cudaMemcpyHostToDevice);
  if (nccl_allgather_bytes(d_x, hb, eng->rank, eng->comm, eng->stream) != 0 ||
      nccl_allreduce_min_i32(d_ok, eng->comm, eng->stream) != 0 || cudaStreamSynchronize(eng->stream) != cudaSuccess) {
    cudaFree(d_x);
    return eng->fail(MS_E_DEVICE, "tp setup: handle exchange failed");
  }
  cudaMemcpy(host.data(), d_x, host.size(), cudaMemcpyDeviceToHost);
  cudaFree(d_x);
  int32_t all_ok = 0;
  std::memcpy(&all_ok, host.data() + hb * eng->tp, sizeof(all_ok));
  // open the peers' buffers; every rank must succeed, or every rank falls back
  int32_t opened = all_ok;
  for (int r = 0; r < eng->tp && opened; ++r) {
    char *base = nullptr;
    if (r == eng->rank) {
      base = static_cast<char *>(eng->ar_sym);
    } else {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, host.data() + hb * r, hb);
      void *p = nullptr;
      if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        opened = 0;
        break;
      }
      eng->ar_peer_maps.push_back(p);
      base = static_cast<char *>(p);
    }
    eng->ar_buf[0][r] = base;
    eng->ar_buf[1][r] = base + part;
    eng->ar_sig[r] = reinterpret_cast<uint32_t *>(base + 2 * part);
  }
  {
    int32_t *d_o = nullptr;
    if (cudaMalloc(&d_o, sizeof(int32_t)) != cudaSuccess) return eng->fail(MS_E_DEVICE, "tp setup: cudaMalloc");
    cudaMemcpy(d_o, &opened, sizeof(opened), cudaMemcpyHostToDevice);
    if (nccl_allreduce_min_i32(d_o, eng->comm, eng->stream) != 0 || cudaStreamSynchronize(eng->stream) != cudaSuccess) {
      cudaFree(d_o);
      return eng->fail(MS_E_DEVICE, "tp setup: agreement failed");
    }
    cudaMemcpy(&opened, d_o, sizeof(opened), cudaMemcpyDeviceToHost);
    cudaFree(d_o);
  }
  eng->ar_fused = opened != 0;
  eng->ar_capable = eng->ar_fused;
  if (!eng->ar_fused) tp_fused_teardown(eng);
  return MS_OK;
}

void tp_fused_teardown(Engine *eng) {
  for (void *p : eng->ar_peer_maps) cudaIpcCloseMemHandle(p);
  eng->ar_peer_maps.clear();
  if (eng->ar_sym) cudaFree(eng->ar_sym);
  eng->ar_sym = nullptr;
  eng->ar_fused = false;
  eng->ar_capable = false;
}

cudaError_t launch_ar_add_rmsnorm(Engine *eng, int which, const void *residual, const int32_t *row_index,
                                  const void *w, void *resid_out, void *norm_out, int rows, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  ArArgs a{};
  for (int r = 0; r < eng->tp; ++r) {
    a.bufs[r] = eng->ar_buf[which][r];
    a.sig[r] = eng->ar_sig[r];
  }
  a.tp = eng->tp;
  a.rank = eng->rank;
  a.epoch = ++eng->ar_epoch;
  a.residual = residual;
  a.row_index = row_index;
  a.w = w;
  a.resid_out = resid_out;
  a.norm_out = norm_out;
  a.rows = rows;
  a.hidden = eng->H;
  a.eps = float(eng->cfg.rms_norm_eps);
  a.status = eng->d_status;
  const int grid = std::min(kMaxCtas, rows);
  const int chunks = eng->H / (16 / int(eng->esize));
  if (chunks > 1024) return cudaErrorInvalidValue;
  const int threads = std::max(32, (chunks + 31) / 32 * 32);
  auto go = [&](auto kern) {
    kern<<<grid, threads, 0, st>>>(a);
    return cudaGetLastError();
  };
  const bool f32 = eng->dtype == MS_DTYPE_F32;
  switch (eng->tp) {
    case 2: return f32 ? go(ar_add_rmsnorm_kernel<float, 2>) : go(ar_add_rmsnorm_kernel<__nv_bfloat16, 2>);
    case 4: return f32 ? go(ar_add_rmsnorm_kernel<float, 4>) : go(ar_add_rmsnorm_kernel<__nv_bfloat16, 4>);
    case 8: return f32 ? go(ar_add_rmsnorm_kernel<float, 8>) : go(ar_add_rmsnorm_kernel<__nv_bfloat16, 8>);
    default: break;
  }
  return cudaErrorInvalidValue;
}

}  // namespace ms
