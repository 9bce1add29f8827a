// Engine: weights, paged KV pool, sequence bookkeeping and the forward step.
//
// Host side of the replacement of CandleBackend (src/backends/candle.rs) and
// of ModelForCausalLM (src/backends/qwen2.rs:583-764).  Device work of one
// step (all on the engine's stream):
//   K1 pack -> K4 (embedding gather + norm) -> per layer
//   [cuBLAS QKV -> K5/K2 -> K3 (+combine) -> cuBLAS O -> K4 -> cuBLAS gate|up
//    -> K6 SiLU-mul -> cuBLAS down -> K4] -> cuBLAS lm_head (last tokens) ->
//   K6 argmax.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <cstdlib>
#include <string>

#include "ms_engine.h"

namespace ms {

#define MS_CUDA_TRY(expr)                                                                    \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    if (_e != cudaSuccess)                                                                   \
      return eng->fail(MS_E_DEVICE, std::string(#expr) + ": " + cudaGetErrorString(_e));     \
  } while (0)

#define MS_BLAS_TRY(expr)                                                                    \
  do {                                                                                       \
    cublasStatus_t _s = (expr);                                                              \
    if (_s != CUBLAS_STATUS_SUCCESS)                                                         \
      return eng->fail(MS_E_DEVICE, std::string(#expr) + ": cublas status " + std::to_string(int(_s))); \
  } while (0)

static size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

static size_t dtype_size(int dt) { return dt == MS_DTYPE_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------
// creation

int create_impl(const ms_model_cfg *cfg, const ms_engine_opts *opts, Engine *eng) {
  eng->cfg = *cfg;
  eng->opts = *opts;
  if (opts->tp_size < 1 || opts->tp_rank < 0 || opts->tp_rank >= opts->tp_size)
    return eng->fail(MS_E_INVALID, "tp_rank must lie in [0, tp_size)");
  if (opts->tp_size > 1) {
    if (!opts->nccl_comm) return eng->fail(MS_E_INVALID, "tp_size > 1 needs an NCCL communicator");
    if (!nccl_available()) return eng->fail(MS_E_DEVICE, "NCCL is not loadable in this process");
    if (cfg->num_kv_heads % opts->tp_size || cfg->num_heads % opts->tp_size ||
        cfg->intermediate_size % opts->tp_size)
      return eng->fail(MS_E_INVALID, "heads, kv heads and intermediate size must divide by tp_size");
  }
  if (cfg->head_dim != 128 && cfg->head_dim != 64) return eng->fail(MS_E_INVALID, "head_dim must be 64 or 128");
  if (cfg->num_heads <= 0 || cfg->num_kv_heads <= 0 || cfg->num_heads % cfg->num_kv_heads)
    return eng->fail(MS_E_INVALID, "num_heads must be a multiple of num_kv_heads");
  const int g = cfg->num_heads / cfg->num_kv_heads;
  if (g != 1 && g != 2 && g != 4 && g != 7 && g != 8) return eng->fail(MS_E_INVALID, "unsupported GQA group size");
  if (cfg->dtype != MS_DTYPE_BF16 && cfg->dtype != MS_DTYPE_F32) return eng->fail(MS_E_INVALID, "dtype must be bf16 or f32");
  if (opts->block_size != 16) return eng->fail(MS_E_INVALID, "block_size must be 16");
  if (opts->pool_blocks <= 0 || opts->max_seqs <= 0 || opts->max_tokens_per_step <= 0 ||
      opts->max_blocks_per_seq <= 0)
    return eng->fail(MS_E_INVALID, "pool_blocks, max_seqs, max_tokens_per_step and max_blocks_per_seq must be positive");
  const int vec = cfg->dtype == MS_DTYPE_F32 ? 4 : 8;
  if (cfg->hidden_size % vec || (cfg->intermediate_size / opts->tp_size) % vec || cfg->hidden_size / vec > 1024)
    return eng->fail(MS_E_INVALID, "hidden/intermediate sizes must be multiples of 8 (bf16) or 4 (f32)");
  if (opts->max_seqs > 16384) return eng->fail(MS_E_INVALID, "max_seqs must be <= 16384");

  eng->dev = opts->device;
  eng->dtype = cfg->dtype;
  eng->esize = dtype_size(cfg->dtype);
  eng->tp = opts->tp_size;
  eng->rank = opts->tp_rank;
  eng->comm = opts->nccl_comm;
  eng->D = cfg->head_dim;
  eng->hq = cfg->num_heads / eng->tp;
  eng->hkv = cfg->num_kv_heads / eng->tp;
  eng->H = cfg->hidden_size;
  eng->I = cfg->intermediate_size / eng->tp;
  eng->V = cfg->vocab_size;
  eng->L = cfg->num_layers;
  eng->qkv_dim = (eng->hq + 2 * eng->hkv) * eng->D;

  MS_CUDA_TRY(cudaSetDevice(eng->dev));
  MS_CUDA_TRY(cudaStreamCreateWithFlags(&eng->stream, cudaStreamNonBlocking));
  MS_CUDA_TRY(cudaEventCreateWithFlags(&eng->done_ev, cudaEventDisableTiming));
  MS_BLAS_TRY(cublasCreate(&eng->blas));
  MS_BLAS_TRY(cublasSetStream(eng->blas, eng->stream));
  // no TF32 and no reduced-precision reductions: f32 mode must match the CPU path
  MS_BLAS_TRY(cublasSetMathMode(eng->blas, CUBLAS_DEFAULT_MATH));
  const size_t blas_ws = 32u << 20;
  MS_CUDA_TRY(cudaMalloc(&eng->blas_ws, blas_ws));
  MS_BLAS_TRY(cublasSetWorkspace(eng->blas, eng->blas_ws, blas_ws));

  // ---- weights ----
  const size_t es = eng->esize;
  const size_t H = eng->H, I = eng->I, V = eng->V, D = eng->D;
  size_t off = 0;
  auto take = [&](size_t elems) { size_t o = off; off += align256(elems * es); return o; };
  const size_t o_embed = take(V * H);
  const size_t o_lm = cfg->tie_word_embeddings ? o_embed : take(V * H);
  const size_t o_norm = take(H);
  struct LOff { size_t ln1, ln2, qkv, bqkv, qn, kn, o, gu, down; };
  std::vector<LOff> lo(eng->L);
  for (int l = 0; l < eng->L; ++l) {
    lo[l].ln1 = take(H);
    lo[l].ln2 = take(H);
    lo[l].qkv = take(size_t(eng->qkv_dim) * H);
    lo[l].bqkv = cfg->attn_bias ? take(eng->qkv_dim) : SIZE_MAX;
    lo[l].qn = cfg->qk_norm ? take(D) : SIZE_MAX;
    lo[l].kn = cfg->qk_norm ? take(D) : SIZE_MAX;
    lo[l].o = take(H * eng->hq * D);
    lo[l].gu = take(2 * I * H);
    lo[l].down = take(H * I);
  }
  eng->wbytes = off;
  MS_CUDA_TRY(cudaMalloc(&eng->wbuf, eng->wbytes));
  char *wb = static_cast<char *>(eng->wbuf);
  eng->embed = wb + o_embed;
  eng->lm_head = wb + o_lm;
  eng->final_norm = wb + o_norm;
  eng->layers.resize(eng->L);
  for (int l = 0; l < eng->L; ++l) {
    LayerW &w = eng->layers[l];
    w.ln1 = wb + lo[l].ln1;
    w.ln2 = wb + lo[l].ln2;
    w.w_qkv = wb + lo[l].qkv;
    w.b_qkv = lo[l].bqkv == SIZE_MAX ? nullptr : wb + lo[l].bqkv;
    w.q_norm = lo[l].qn == SIZE_MAX ? nullptr : wb + lo[l].qn;
    w.k_norm = lo[l].kn == SIZE_MAX ? nullptr : wb + lo[l].kn;
    w.w_o = wb + lo[l].o;
    w.w_gu = wb + lo[l].gu;
    w.w_down = wb + lo[l].down;
  }
  eng->required.push_back("model.embed_tokens.weight");
  eng->required.push_back("model.norm.weight");
  if (!cfg->tie_word_embeddings) eng->required.push_back("lm_head.weight");
  for (int l = 0; l < eng->L; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    for (const char *s : {"input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                          "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                          "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"})
      eng->required.push_back(p + s);
    if (cfg->attn_bias)
      for (const char *s : {"self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias"})
        eng->required.push_back(p + s);
    if (cfg->qk_norm)
      for (const char *s : {"self_attn.q_norm.weight", "self_attn.k_norm.weight"}) eng->required.push_back(p + s);
  }

  // ---- RoPE tables (qwen2.rs:91-108): inv_freq = 1f32 / theta.powf(i/dim) as f32,
  // freqs = t * inv_freq in f32, sin/cos in f32 (kept in f32 for every model dtype) ----
  eng->rope_len = cfg->max_position_embeddings;
  if (eng->rope_len <= 0) return eng->fail(MS_E_INVALID, "max_position_embeddings must be positive");
  {
    const int half = int(D) / 2;
    std::vector<float> inv(half);
    for (int i = 0; i < half; ++i)
      inv[i] = 1.0f / float(std::pow(cfg->rope_theta, double(2 * i) / double(D)));
    const size_t n = size_t(eng->rope_len) * half;
    std::vector<float> c(n), s(n);
    for (int t = 0; t < eng->rope_len; ++t)
      for (int i = 0; i < half; ++i) {
        const float f = float(t) * inv[i];
        c[size_t(t) * half + i] = std::cos(f);
        s[size_t(t) * half + i] = std::sin(f);
      }
    // f32 tables in every mode (K5 computes in f32 and rounds each output once)
    MS_CUDA_TRY(cudaMalloc(&eng->cos_t, n * 4));
    MS_CUDA_TRY(cudaMalloc(&eng->sin_t, n * 4));
    MS_CUDA_TRY(cudaMemcpy(eng->cos_t, c.data(), n * 4, cudaMemcpyHostToDevice));
    MS_CUDA_TRY(cudaMemcpy(eng->sin_t, s.data(), n * 4, cudaMemcpyHostToDevice));
  }

  // ---- paged KV pool ----
  eng->layer_pool_elems = size_t(opts->pool_blocks) * eng->hkv * 16 * D;
  eng->pool_bytes = eng->layer_pool_elems * 2 * eng->L * es;
  MS_CUDA_TRY(cudaMalloc(&eng->pool, eng->pool_bytes));

  // ---- tensor maps for the tensor-core attention kernels ----
  eng->use_tc = attention_tc_available(eng->dtype, eng->D, eng->hq / eng->hkv);
  if (eng->use_tc) {
    eng->kmaps.resize(eng->L);
    eng->vmaps.resize(eng->L);
    const int64_t tiles = opts->pool_blocks * eng->hkv;
    for (int l = 0; l < eng->L; ++l) {
      char *kp = static_cast<char *>(eng->pool) + size_t(2 * l) * eng->layer_pool_elems * es;
      char *vp = kp + eng->layer_pool_elems * es;
      if (!encode_pool_tensor_map(&eng->kmaps[l], kp, eng->dtype, eng->D, tiles) ||
          !encode_pool_tensor_map(&eng->vmaps[l], vp, eng->dtype, eng->D, tiles))
        return eng->fail(MS_E_DEVICE, "cuTensorMapEncodeTiled failed for the KV pool");
    }
  }

  // ---- per-slot state ----
  MS_CUDA_TRY(cudaMalloc(&eng->d_block_tables, size_t(opts->max_seqs) * opts->max_blocks_per_seq * 4));
  MS_CUDA_TRY(cudaMemset(eng->d_block_tables, 0, size_t(opts->max_seqs) * opts->max_blocks_per_seq * 4));
  MS_CUDA_TRY(cudaMalloc(&eng->d_slot_last, size_t(opts->max_seqs) * 4));
  MS_CUDA_TRY(cudaMemset(eng->d_slot_last, 0, size_t(opts->max_seqs) * 4));
  MS_CUDA_TRY(cudaMalloc(&eng->d_status, 4));
  MS_CUDA_TRY(cudaMemset(eng->d_status, 0, 4));
  for (int i = opts->max_seqs - 1; i >= 0; --i) eng->free_slots.push_back(i);

  // ---- step buffers ----
  const size_t T = opts->max_tokens_per_step, S = opts->max_seqs;
  size_t so = 0;
  auto stake = [&](size_t bytes) { size_t o = so; so += align256(bytes); return o; };
  const size_t o_cu = stake((S + 1) * 4), o_pos = stake(T * 4), o_rt = stake(T * 4), o_rc = stake(T * 4);
  const size_t o_li = stake(S * 4), o_next = stake(S * 4), o_slots = stake(T * 8);
  const size_t o_resid = stake(T * H * es), o_norm2 = stake(T * H * es), o_tmp = stake(T * H * es);
  const size_t o_qkv = stake(T * size_t(eng->qkv_dim) * es), o_q = stake(T * eng->hq * D * es);
  const size_t o_attn = stake(T * eng->hq * D * es), o_gu = stake(T * 2 * I * es), o_act = stake(T * I * es);
  const size_t o_last = stake(S * H * es), o_logits = stake(S * V * 4);
  eng->attn_ws_bytes = 256u << 20;
  const size_t o_ws = stake(eng->attn_ws_bytes);
  eng->sbytes = so;
  MS_CUDA_TRY(cudaMalloc(&eng->sbuf, eng->sbytes));
  char *sb = static_cast<char *>(eng->sbuf);
  eng->d_cu = reinterpret_cast<int32_t *>(sb + o_cu);
  eng->d_pos = reinterpret_cast<int32_t *>(sb + o_pos);
  eng->d_row_table = reinterpret_cast<int32_t *>(sb + o_rt);
  eng->d_row_ctx = reinterpret_cast<int32_t *>(sb + o_rc);
  eng->d_last_index = reinterpret_cast<int32_t *>(sb + o_li);
  eng->d_next = reinterpret_cast<int32_t *>(sb + o_next);
  eng->d_slots = reinterpret_cast<int64_t *>(sb + o_slots);
  eng->x_resid = sb + o_resid;
  eng->x_norm = sb + o_norm2;
  eng->x_tmp = sb + o_tmp;
  eng->qkv = sb + o_qkv;
  eng->qbuf = sb + o_q;
  eng->attn = sb + o_attn;
  eng->gu = sb + o_gu;
  eng->act = sb + o_act;
  eng->last_norm = sb + o_last;
  eng->logits = reinterpret_cast<float *>(sb + o_logits);
  eng->attn_ws = sb + o_ws;

  MS_CUDA_TRY(cudaMallocHost(&eng->h_next, S * 4));
  MS_CUDA_TRY(cudaMallocHost(&eng->h_status, 4));
  // fixed staging of graph-replayed steps (the captured copy reads these pointers)
  MS_CUDA_TRY(cudaMallocHost(&eng->h_gin, graph_in_elems(opts->max_seqs) * 4));
  MS_CUDA_TRY(cudaMalloc(&eng->d_gin, graph_in_elems(opts->max_seqs) * 4));
  {
    const char *e = std::getenv("MS_CUDA_GRAPHS");
    eng->graphs_enabled = !(e && std::string(e) == "0");
  }
  // the memsets and table uploads above ran on the legacy stream; the engine
  // stream is non-blocking, so finish them before any step can be enqueued
  MS_CUDA_TRY(cudaDeviceSynchronize());
  if (eng->tp > 1) {
    const int rc = tp_fused_setup(eng);
    if (rc != MS_OK) return rc;
  }
  return MS_OK;
}

void destroy_impl(Engine *eng) {
  if (!eng) return;
  cudaSetDevice(eng->dev);
  if (eng->stream) cudaStreamSynchronize(eng->stream);
  eng->drop_graphs();
  tp_fused_teardown(eng);
  if (eng->blas) cublasDestroy(eng->blas);
  for (void *p : {eng->blas_ws, eng->wbuf, eng->cos_t, eng->sin_t, eng->pool, (void *)eng->d_block_tables,
                  (void *)eng->d_slot_last, (void *)eng->d_status, eng->sbuf, (void *)eng->d_in, (void *)eng->d_gin})
    if (p) cudaFree(p);
  for (void *p : {(void *)eng->h_in, (void *)eng->h_next, (void *)eng->h_status, (void *)eng->h_gin})
    if (p) cudaFreeHost(p);
  for (cudaEvent_t e : eng->prof_ev) cudaEventDestroy(e);
  for (cudaEvent_t e : eng->prof_ar_ev) cudaEventDestroy(e);
  if (eng->done_ev) cudaEventDestroy(eng->done_ev);
  if (eng->stream) cudaStreamDestroy(eng->stream);
}

}  // namespace ms
