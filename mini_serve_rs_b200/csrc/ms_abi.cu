// extern "C" surface of include/ms_engine.h for the engine-level entry points.
// Every entry point catches C++ exceptions and turns them into status codes.
#include <cstring>
#include <algorithm>
#include <exception>
#include <new>
#include <string>

#include "ms_engine.h"

using ms::Engine;

namespace {
thread_local std::string g_create_error;

template <typename F>
int guarded(Engine *eng, F &&f) {
  try {
    return f();
  } catch (const std::bad_alloc &) {
    if (eng) eng->err = "host out of memory";
    return MS_E_PRESSURE;
  } catch (const std::exception &e) {
    if (eng) eng->err = e.what();
    return MS_E_INVALID;
  } catch (...) {
    if (eng) eng->err = "unknown C++ exception";
    return MS_E_INVALID;
  }
}
}  // namespace

struct ms_engine : Engine {};

extern "C" int ms_engine_create(const ms_model_cfg *cfg, const ms_engine_opts *opts, ms_engine **out) {
  if (!cfg || !opts || !out) return MS_E_INVALID;
  *out = nullptr;
  ms_engine *e = new (std::nothrow) ms_engine();
  if (!e) return MS_E_PRESSURE;
  int rc;
  try {
    rc = ms::create_impl(cfg, opts, e);
  } catch (const std::exception &ex) {
    rc = MS_E_INVALID;
    e->err = ex.what();
  }
  if (rc != MS_OK) {
    g_create_error = e->err;
    ms::destroy_impl(e);
    delete e;
    return rc == MS_E_INVALID || rc == MS_E_PRESSURE ? rc : MS_E_DEVICE;
  }
  *out = e;
  return MS_OK;
}

extern "C" int ms_engine_destroy(ms_engine *eng) {
  if (!eng) return MS_OK;
  ms::destroy_impl(eng);
  delete eng;
  return MS_OK;
}

extern "C" int ms_engine_load_weight(ms_engine *eng, const char *name, const void *data, int64_t numel,
                                     int32_t src_dtype, int32_t src_on_device) {
  if (!eng) return MS_E_INVALID;
  return guarded(eng, [&] { return ms::load_weight_impl(eng, name, data, numel, src_dtype, src_on_device); });
}

extern "C" int ms_engine_finalize(ms_engine *eng) {
  if (!eng) return MS_E_INVALID;
  return guarded(eng, [&] { return ms::finalize_impl(eng); });
}

extern "C" int ms_engine_memory(const ms_engine *eng, int64_t *weights_bytes, int64_t *pool_bytes,
                                int64_t *workspace_bytes) {
  if (!eng) return MS_E_INVALID;
  if (weights_bytes) *weights_bytes = int64_t(eng->wbytes);
  if (pool_bytes) *pool_bytes = int64_t(eng->pool_bytes);
  if (workspace_bytes) *workspace_bytes = int64_t(eng->sbytes + eng->in_cap * 4);
  return MS_OK;
}

extern "C" int ms_seq_admit(ms_engine *eng, uint64_t seq_id, const uint32_t *prompt, int32_t prompt_len,
                            const int32_t *block_ids, int32_t num_blocks, int32_t num_cached) {
  if (!eng) return MS_E_INVALID;
  return guarded(eng, [&] {
    return ms::seq_admit_impl(eng, seq_id, prompt, prompt_len, block_ids, num_blocks, num_cached);
  });
}

extern "C" int ms_seq_append_block(ms_engine *eng, uint64_t seq_id, int32_t block_id) {
  if (!eng) return MS_E_INVALID;
  return guarded(eng, [&] { return ms::seq_append_block_impl(eng, seq_id, block_id); });
}

extern "C" int ms_seq_release(ms_engine *eng, uint64_t seq_id) {
  if (!eng) return MS_E_INVALID;
  return guarded(eng, [&] { return ms::seq_release_impl(eng, seq_id); });
}

extern "C" int ms_seq_cached_tokens(const ms_engine *eng, uint64_t seq_id, int32_t *out) {
  if (!eng || !out) return MS_E_INVALID;
  auto it = eng->seqs.find(seq_id);
  if (it == eng->seqs.end()) return MS_E_NOT_FOUND;
  *out = it->second.cached;
  return MS_OK;
}

extern "C" int ms_step_launch(ms_engine *eng, const ms_step_desc *desc) {
  if (!eng) return MS_E_INVALID;
  return guarded(eng, [&] { return ms::step_launch_impl(eng, desc); });
}

extern "C" int ms_step_wait(ms_engine *eng, uint32_t *out_tokens, uint8_t *out_flags) {
  if (!eng) return MS_E_INVALID;
  return guarded(eng, [&] { return ms::step_wait_impl(eng, out_tokens, out_flags); });
}

extern "C" int ms_step(ms_engine *eng, const ms_step_desc *desc, uint32_t *out_tokens, uint8_t *out_flags) {
  if (!eng) return MS_E_INVALID;
  int rc = ms_step_launch(eng, desc);
  if (rc != MS_OK) return rc;
  return ms_step_wait(eng, out_tokens, out_flags);
}

extern "C" int ms_engine_stream(const ms_engine *eng, void **stream_out) {
  if (!eng || !stream_out) return MS_E_INVALID;
  *stream_out = eng->stream;
  return MS_OK;
}

extern "C" int ms_is_healthy(const ms_engine *eng) { return eng && eng->healthy ? 1 : 0; }

extern "C" int ms_mark_unhealthy(ms_engine *eng) {
  if (!eng) return MS_E_INVALID;
  eng->quarantine();
  return MS_OK;
}

extern "C" int ms_inject_fault(ms_engine *eng, int32_t code) {
  if (!eng) return MS_E_INVALID;
  eng->inject = code ? 1 : 0;
  return MS_OK;
}

extern "C" int ms_last_error(const ms_engine *eng, char *buf, int32_t len) {
  if (!buf || len <= 0) return MS_E_INVALID;
  const std::string &m = eng ? eng->err : g_create_error;
  const size_t n = std::min<size_t>(m.size(), size_t(len - 1));
  std::memcpy(buf, m.data(), n);
  buf[n] = 0;
  return MS_OK;
}

extern "C" int ms_debug_dump_tables(ms_engine *eng, int32_t *num_tokens, int32_t *cu_seqlens, int32_t *positions,
                                    int64_t *slot_mapping, int32_t *block_tables) {
  if (!eng) return MS_E_INVALID;
  if (eng->pending) return eng->fail(MS_E_INVALID, "step in flight");
  cudaError_t e = cudaSetDevice(eng->dev);
  const int S = eng->last_nseq, T = eng->last_T;
  if (num_tokens) *num_tokens = T;
  if (S == 0) return MS_OK;
  if (e == cudaSuccess) e = cudaStreamSynchronize(eng->stream);
  if (e == cudaSuccess && cu_seqlens)
    e = cudaMemcpy(cu_seqlens, eng->d_cu, size_t(S + 1) * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && positions) e = cudaMemcpy(positions, eng->d_pos, size_t(T) * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && slot_mapping)
    e = cudaMemcpy(slot_mapping, eng->d_slots, size_t(T) * 8, cudaMemcpyDeviceToHost);
  const int mb = eng->opts.max_blocks_per_seq;
  for (int i = 0; e == cudaSuccess && block_tables && i < S; ++i)
    e = cudaMemcpy(block_tables + size_t(i) * mb, eng->d_block_tables + size_t(eng->last_slots[i]) * mb,
                   size_t(mb) * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, cudaGetErrorString(e));
  return MS_OK;
}

extern "C" int ms_debug_logits(ms_engine *eng, float *out, int64_t count) {
  if (!eng || !out) return MS_E_INVALID;
  if (eng->pending) return eng->fail(MS_E_INVALID, "step in flight");
  const int64_t n = int64_t(eng->last_nseq) * eng->V;
  if (count < n) return eng->fail(MS_E_INVALID, "output buffer too small");
  cudaError_t e = cudaSetDevice(eng->dev);
  if (e == cudaSuccess) e = cudaStreamSynchronize(eng->stream);
  if (e == cudaSuccess) e = cudaMemcpy(out, eng->logits, size_t(n) * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, cudaGetErrorString(e));
  return MS_OK;
}

extern "C" int ms_debug_pool_ptr(ms_engine *eng, int32_t layer, int32_t which, void **ptr) {
  if (!eng || !ptr || layer < 0 || layer >= eng->L || (which != 0 && which != 1)) return MS_E_INVALID;
  *ptr = static_cast<char *>(eng->pool) + (size_t(2 * layer) + which) * eng->layer_pool_elems * eng->esize;
  return MS_OK;
}

extern "C" int ms_engine_set_profiling(ms_engine *eng, int32_t on) {
  if (!eng) return MS_E_INVALID;
  eng->profiling = on != 0;
  return MS_OK;
}

extern "C" int ms_engine_tp_fused(const ms_engine *eng, int32_t *fused) {
  if (!eng || !fused) return MS_E_INVALID;
  *fused = eng->ar_fused ? 1 : 0;
  return MS_OK;
}

extern "C" int ms_engine_set_tp_fused(ms_engine *eng, int32_t on) {
  if (!eng) return MS_E_INVALID;
  if (eng->pending) return eng->fail(MS_E_INVALID, "ms_engine_set_tp_fused between launch and wait");
  if (on && !eng->ar_capable) return eng->fail(MS_E_INVALID, "fused all-reduce not set up on this engine");
  eng->ar_fused = on != 0;
  return MS_OK;
}

extern "C" int ms_engine_set_graphs(ms_engine *eng, int32_t on) {
  if (!eng) return MS_E_INVALID;
  if (eng->pending) return eng->fail(MS_E_INVALID, "ms_engine_set_graphs between launch and wait");
  eng->graphs_enabled = on != 0;
  if (!eng->graphs_enabled) {
    cudaSetDevice(eng->dev);
    cudaStreamSynchronize(eng->stream);
    eng->drop_graphs();
  }
  return MS_OK;
}

extern "C" int ms_engine_graph_stats(const ms_engine *eng, int64_t *captures, int64_t *replays, int32_t *cached) {
  if (!eng) return MS_E_INVALID;
  if (captures) *captures = eng->graph_captures;
  if (replays) *replays = eng->graph_replays;
  if (cached) *cached = int32_t(eng->graphs.size());
  return MS_OK;
}

extern "C" int ms_engine_profile(ms_engine *eng, int64_t *kernel_launches, int64_t *attn_launches,
                                 double *attn_ms_total, double *attn_bytes_total) {
  if (!eng) return MS_E_INVALID;
  if (kernel_launches) *kernel_launches = eng->kernel_launches;
  double ms = 0.0;
  if (eng->prof_used) {
    cudaError_t e = cudaSetDevice(eng->dev);
    if (e == cudaSuccess) e = cudaStreamSynchronize(eng->stream);
    for (size_t i = 0; e == cudaSuccess && i + 1 < eng->prof_used; i += 2) {
      float t = 0.f;
      e = cudaEventElapsedTime(&t, eng->prof_ev[i], eng->prof_ev[i + 1]);
      ms += t;
    }
    if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, cudaGetErrorString(e));
  }
  if (attn_launches) *attn_launches = int64_t(eng->prof_used / 2);
  if (attn_ms_total) *attn_ms_total = ms;
  if (attn_bytes_total) *attn_bytes_total = eng->prof_bytes;
  eng->prof_used = 0;
  eng->prof_bytes = 0.0;
  return MS_OK;
}

extern "C" int ms_engine_profile_allreduce(ms_engine *eng, int64_t *calls, double *ms_total) {
  if (!eng) return MS_E_INVALID;
  double ms = 0.0;
  if (eng->prof_ar_used) {
    cudaError_t e = cudaSetDevice(eng->dev);
    if (e == cudaSuccess) e = cudaStreamSynchronize(eng->stream);
    for (size_t i = 0; e == cudaSuccess && i + 1 < eng->prof_ar_used; i += 2) {
      float t = 0.f;
      e = cudaEventElapsedTime(&t, eng->prof_ar_ev[i], eng->prof_ar_ev[i + 1]);
      ms += t;
    }
    if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, cudaGetErrorString(e));
  }
  if (calls) *calls = int64_t(eng->prof_ar_used / 2);
  if (ms_total) *ms_total = ms;
  eng->prof_ar_used = 0;
  return MS_OK;
}

extern "C" int ms_debug_stop_after_layer(ms_engine *eng, int32_t layer) {
  if (!eng || layer < -1 || layer >= eng->L) return MS_E_INVALID;
  if (eng->pending) return eng->fail(MS_E_INVALID, "ms_debug_stop_after_layer between launch and wait");
  if (layer >= 0 && eng->ar_fused) return eng->fail(MS_E_INVALID, "not available with the fused TP all-reduce");
  eng->debug_stop_layer = layer;
  return MS_OK;
}

extern "C" int ms_debug_buffer(ms_engine *eng, const char *name, void *out, int64_t bytes) {
  if (!eng || !name || !out) return MS_E_INVALID;
  if (eng->pending) return eng->fail(MS_E_INVALID, "step in flight");
  const std::string n(name);
  const size_t T = size_t(eng->last_T), S = size_t(eng->last_nseq), es = eng->esize;
  const void *src = nullptr;
  size_t sz = 0;
  if (n == "x_resid") { src = eng->x_resid; sz = T * eng->H * es; }
  else if (n == "x_norm") { src = eng->x_norm; sz = T * eng->H * es; }
  else if (n == "x_tmp") { src = eng->x_tmp; sz = T * eng->H * es; }
  else if (n == "qkv") { src = eng->qkv; sz = T * eng->qkv_dim * es; }
  else if (n == "q") { src = eng->qbuf; sz = T * eng->hq * eng->D * es; }
  else if (n == "attn") { src = eng->attn; sz = T * eng->hq * eng->D * es; }
  else if (n == "gu") { src = eng->gu; sz = T * 2 * eng->I * es; }
  else if (n == "act") { src = eng->act; sz = T * eng->I * es; }
  else if (n == "last_norm") { src = eng->last_norm; sz = S * eng->H * es; }
  else if (n == "row_ctx") { src = eng->d_row_ctx; sz = T * 4; }
  else if (n == "row_table") { src = eng->d_row_table; sz = T * 4; }
  else if (n == "positions") { src = eng->d_pos; sz = T * 4; }
  else return eng->fail(MS_E_INVALID, "unknown buffer " + n);
  if (int64_t(sz) > bytes) return eng->fail(MS_E_INVALID, "output buffer too small");
  cudaError_t e = cudaSetDevice(eng->dev);
  if (e == cudaSuccess) e = cudaStreamSynchronize(eng->stream);
  if (e == cudaSuccess) e = cudaMemcpy(out, src, sz, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, cudaGetErrorString(e));
  return MS_OK;
}
