// Engine forward: the device work of one packed step, enqueued on the engine
// stream.  Order of operations per layer follows DecoderLayer::forward
// (src/backends/qwen2.rs:414-428) and the batched decode of qwen2.rs:663-757;
// the final norm and lm_head run on each sequence's last packed row only
// (qwen2.rs:620-626, 759-763).
#include <algorithm>
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

namespace {

cudaDataType_t cuda_type(int dt) { return dt == MS_DTYPE_F32 ? CUDA_R_32F : CUDA_R_16BF; }

// Y[T, out] = X[T, in] * W[out, in]^T (candle_nn::Linear, no bias): a
// column-major GEMM Y^T = W^T(op T) * X^T with f32 accumulation.
cublasStatus_t linear(Engine *eng, const void *W, const void *X, void *Y, int out, int T, int in,
                      bool f32_out = false) {
  const float one = 1.f, zero = 0.f;
  const cudaDataType_t t = cuda_type(eng->dtype);
  return cublasGemmEx(eng->blas, CUBLAS_OP_T, CUBLAS_OP_N, out, T, in, &one, W, t, in, X, t, in, &zero, Y,
                      f32_out ? CUDA_R_32F : t, out, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
}

}  // namespace

namespace {
// Records the next profiling event of a log on the engine stream (created on
// first use).
cudaError_t prof_mark(Engine *eng, std::vector<cudaEvent_t> &log, size_t &used) {
  if (used == log.size()) {
    cudaEvent_t e;
    cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) return err;
    log.push_back(e);
  }
  return cudaEventRecord(log[used++], eng->stream);
}
cudaError_t prof_mark(Engine *eng) { return prof_mark(eng, eng->prof_ev, eng->prof_used); }
// Brackets a tensor-parallel all-reduce section when profiling.
cudaError_t prof_ar_mark(Engine *eng) {
  if (!eng->profiling || eng->tp <= 1) return cudaSuccess;
  return prof_mark(eng, eng->prof_ar_ev, eng->prof_ar_used);
}
}  // namespace

int decode_partition(const Engine *eng, const StepPlan &plan, int max_ctx) {
  if (plan.n_dec <= 0) return 1;
  int part = choose_partition_blocks(plan.n_dec, eng->hkv, max_ctx, plan.blocks_dec);
  while (attention_workspace_bytes(plan.n_dec, eng->hq, max_ctx, part) > int64_t(eng->attn_ws_bytes)) part *= 2;
  return part;
}

int enqueue_forward(Engine *eng, const StepPlan &plan) {
  const int S = plan.S, T = plan.T, dc = plan.delta_cap;
  cudaStream_t st = eng->stream;
  const int dt = eng->dtype;
  const float eps = float(eng->cfg.rms_norm_eps);
  const size_t es = eng->esize;

  // the step description, then a clean status word
  MS_CUDA_TRY(cudaMemcpyAsync(plan.d_desc, plan.h_desc, plan.desc_elems * 4, cudaMemcpyHostToDevice, st));
  MS_CUDA_TRY(cudaMemsetAsync(eng->d_status, 0, sizeof(unsigned), st));

  // ---- K1: pack ----
  int32_t *d = plan.d_desc + plan.hdr;
  PackArgs pa{};
  pa.seq_row = d;
  pa.seq_ntok = d + S;
  pa.seq_start = d + 2 * S;
  pa.num_seqs = S;
  pa.tokens = d + 3 * S;
  int32_t *samp = pa.tokens + T;  // [temp S][top_p S][seed_lo S][seed_hi S] when plan.sample
  pa.delta_row = samp + (plan.sample ? 4 * S : 0);
  pa.delta_idx = pa.delta_row + dc;
  pa.delta_block = pa.delta_idx + dc;
  pa.num_deltas = dc;
  pa.num_deltas_dev = plan.graph ? plan.d_desc : nullptr;
  pa.block_tables = eng->d_block_tables;
  pa.max_blocks_per_seq = eng->opts.max_blocks_per_seq;
  pa.block_size = eng->opts.block_size;
  pa.cu_seqlens = eng->d_cu;
  pa.positions = eng->d_pos;
  pa.slot_mapping = eng->d_slots;
  pa.row_table = eng->d_row_table;
  pa.row_ctx = eng->d_row_ctx;
  pa.last_index = eng->d_last_index;
  pa.slot_last_tok = eng->d_slot_last;
  pa.tokens_from_device = 1;
  pa.status = eng->d_status;
  pa.pool_blocks = eng->opts.pool_blocks;
  MS_CUDA_TRY(launch_pack(pa, st));
  const int32_t *tokens = pa.tokens;

  const int32_t *dec_rows = plan.split ? pa.delta_block + dc : nullptr;
  const int32_t *tiles = plan.split ? pa.delta_block + dc + plan.n_dec : nullptr;
  const int part = plan.part;
  const int64_t pool_tiles = eng->opts.pool_blocks * eng->hkv;

  // ---- layer 0 input: embedding gather + input norm (K4 without residual) ----
  MS_CUDA_TRY(launch_add_rmsnorm(eng->embed, nullptr, tokens, eng->layers[0].ln1, eng->x_resid, eng->x_norm, T,
                                 eng->H, eps, dt, st));
  const size_t pool_layer_bytes = eng->layer_pool_elems * es;
  for (int l = 0; l < eng->L; ++l) {
    const LayerW &w = eng->layers[l];
    char *kp = static_cast<char *>(eng->pool) + size_t(2 * l) * pool_layer_bytes;
    char *vp = kp + pool_layer_bytes;
    // QKV projection, then bias / QK-norm / RoPE / paged append
    MS_BLAS_TRY(linear(eng, w.w_qkv, eng->x_norm, eng->qkv, eng->qkv_dim, T, eng->H));
    MS_CUDA_TRY(launch_qk_norm_rope_append(eng->qkv, w.b_qkv, w.q_norm, w.k_norm, eng->cos_t, eng->sin_t, eng->d_pos,
                                           eng->d_slots, eng->qbuf, kp, vp, T, eng->hq, eng->hkv, eng->D,
                                           eng->opts.block_size, eps, dt, st, eng->d_status));
    // paged attention: one-token rows through split-K decode, prompt chunks through prefill tiles
    if (plan.n_dec > 0) {
      AttnArgs a{};
      a.q = eng->qbuf;
      a.k_pool = kp;
      a.v_pool = vp;
      a.block_tables = eng->d_block_tables;
      a.max_blocks_per_seq = eng->opts.max_blocks_per_seq;
      a.row_table = eng->d_row_table;
      a.row_ctx = eng->d_row_ctx;
      a.row_index = dec_rows;
      a.num_rows = plan.n_dec;
      a.max_ctx = plan.max_ctx_launch;
      a.out = eng->attn;
      a.num_heads = eng->hq;
      a.num_kv_heads = eng->hkv;
      a.head_dim = eng->D;
      a.block_size = eng->opts.block_size;
      a.scale = 1.0f / std::sqrt(float(eng->D));
      a.part_blocks = part;
      a.workspace = eng->attn_ws;
      a.workspace_bytes = int64_t(eng->attn_ws_bytes);
      a.dtype = dt;
      a.status = eng->d_status;
      if (eng->use_tc) {
        a.k_map = &eng->kmaps[l];
        a.v_map = &eng->vmaps[l];
        a.pool_tiles = pool_tiles;
      }
      if (eng->profiling) MS_CUDA_TRY(prof_mark(eng));
      MS_CUDA_TRY(launch_paged_attention(a, st));
      if (eng->profiling) {
        MS_CUDA_TRY(prof_mark(eng));
        // K and V rows read, q in, out written, one table entry per page, one ctx per row
        eng->prof_bytes += plan.ctx_dec * eng->hkv * eng->D * 2.0 * es + 2.0 * plan.n_dec * eng->hq * eng->D * es +
                           double(plan.blocks_dec) * 4.0 + 4.0 * plan.n_dec;
      }
    }
    if (plan.n_tiles > 0) {
      PrefillArgs pf{};
      pf.q = eng->qbuf;
      pf.k_pool = kp;
      pf.v_pool = vp;
      pf.block_tables = eng->d_block_tables;
      pf.max_blocks_per_seq = eng->opts.max_blocks_per_seq;
      pf.tiles = tiles;
      pf.num_tiles = plan.n_tiles;
      pf.out = eng->attn;
      pf.num_heads = eng->hq;
      pf.num_kv_heads = eng->hkv;
      pf.head_dim = eng->D;
      pf.block_size = eng->opts.block_size;
      pf.scale = 1.0f / std::sqrt(float(eng->D));
      pf.dtype = dt;
      pf.status = eng->d_status;
      MS_CUDA_TRY(launch_paged_prefill(pf, st));
    }
    // o_proj, residual add + post-attention norm
    if (eng->ar_fused) {  // partial sums into the peer-mapped buffer, then sum + add + norm in one kernel
      MS_BLAS_TRY(linear(eng, w.w_o, eng->attn, eng->ar_buf[0][eng->rank], eng->H, T, eng->hq * eng->D));
      MS_CUDA_TRY(prof_ar_mark(eng));
      MS_CUDA_TRY(launch_ar_add_rmsnorm(eng, 0, eng->x_resid, nullptr, w.ln2, eng->x_resid, eng->x_norm, T, st));
      MS_CUDA_TRY(prof_ar_mark(eng));
    } else {
      MS_BLAS_TRY(linear(eng, w.w_o, eng->attn, eng->x_tmp, eng->H, T, eng->hq * eng->D));
      MS_CUDA_TRY(prof_ar_mark(eng));
      if (eng->tp > 1 && nccl_allreduce_sum(eng->x_tmp, size_t(T) * eng->H, dt, eng->comm, st) != 0)
        return eng->fail(MS_E_DEVICE, "NCCL all-reduce after o_proj failed");
      MS_CUDA_TRY(launch_add_rmsnorm(eng->x_tmp, eng->x_resid, nullptr, w.ln2, eng->x_resid, eng->x_norm, T,
                                     eng->H, eps, dt, st));
      MS_CUDA_TRY(prof_ar_mark(eng));
    }
    // MLP
    MS_BLAS_TRY(linear(eng, w.w_gu, eng->x_norm, eng->gu, 2 * eng->I, T, eng->H));
    MS_CUDA_TRY(launch_silu_mul(eng->gu, eng->act, T, eng->I, dt, st));
    if (eng->ar_fused) {
      MS_BLAS_TRY(linear(eng, w.w_down, eng->act, eng->ar_buf[1][eng->rank], eng->H, T, eng->I));
      MS_CUDA_TRY(prof_ar_mark(eng));
      if (l + 1 < eng->L)
        MS_CUDA_TRY(launch_ar_add_rmsnorm(eng, 1, eng->x_resid, nullptr, eng->layers[l + 1].ln1, eng->x_resid,
                                          eng->x_norm, T, st));
      else  // final norm on each sequence's last row only
        MS_CUDA_TRY(launch_ar_add_rmsnorm(eng, 1, eng->x_resid, eng->d_last_index, eng->final_norm, nullptr,
                                          eng->last_norm, S, st));
      MS_CUDA_TRY(prof_ar_mark(eng));
      continue;
    }
    MS_BLAS_TRY(linear(eng, w.w_down, eng->act, eng->x_tmp, eng->H, T, eng->I));
    if (l == eng->debug_stop_layer) break;
    MS_CUDA_TRY(prof_ar_mark(eng));
    if (eng->tp > 1 && nccl_allreduce_sum(eng->x_tmp, size_t(T) * eng->H, dt, eng->comm, st) != 0)
      return eng->fail(MS_E_DEVICE, "NCCL all-reduce after down_proj failed");
    if (l + 1 < eng->L) {
      MS_CUDA_TRY(launch_add_rmsnorm(eng->x_tmp, eng->x_resid, nullptr, eng->layers[l + 1].ln1, eng->x_resid,
                                     eng->x_norm, T, eng->H, eps, dt, st));
    } else {
      // last layer: residual add + final norm on each sequence's last row only
      MS_CUDA_TRY(launch_add_rmsnorm(eng->x_tmp, eng->x_resid, eng->d_last_index, eng->final_norm, nullptr,
                                     eng->last_norm, S, eng->H, eps, dt, st));
    }
    MS_CUDA_TRY(prof_ar_mark(eng));
  }
  if (eng->debug_stop_layer >= 0 && eng->debug_stop_layer < eng->L && !eng->ar_fused) {
    // debugging stop: no lm_head or sampling; the step still returns (stale) tokens and the status
    eng->last_launches = 0;
    MS_CUDA_TRY(cudaMemcpyAsync(eng->h_next, eng->d_next, size_t(S) * 4, cudaMemcpyDeviceToHost, st));
    MS_CUDA_TRY(cudaMemcpyAsync(eng->h_status, eng->d_status, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    return MS_OK;
  }
  // lm_head in f32 output, greedy argmax, tokens back to the host
  MS_BLAS_TRY(linear(eng, eng->lm_head, eng->last_norm, eng->logits, eng->V, S, eng->H, true));
  MS_CUDA_TRY(launch_argmax(eng->logits, S, eng->V, eng->d_next, pa.seq_row, eng->d_slot_last, st));
  if (plan.sample) {  // rows with temperature >= 1e-7 replace their argmax by a draw
    SampleArgs sa;
    sa.logits = eng->logits;
    sa.rows = S;
    sa.vocab = eng->V;
    sa.temperature = reinterpret_cast<const float *>(samp);
    sa.top_p = plan.nucleus ? reinterpret_cast<const float *>(samp + S) : nullptr;  // null: one pass suffices
    sa.seed_lo = reinterpret_cast<const uint32_t *>(samp + 2 * S);
    sa.seed_hi = reinterpret_cast<const uint32_t *>(samp + 3 * S);
    sa.out = eng->d_next;
    sa.row_slot = pa.seq_row;
    sa.slot_last = eng->d_slot_last;
    sa.status = eng->d_status;
    MS_CUDA_TRY(launch_sample(sa, st));
  }
  {
    const int max_blk = (plan.max_ctx_launch + 15) / 16;
    const int parts = plan.n_dec > 0 ? (max_blk + part - 1) / part : 0;
    const int attn_launches = (plan.n_dec > 0 ? 1 + (parts > 1 ? 1 : 0) : 0) + (plan.n_tiles > 0 ? 1 : 0);
    eng->last_launches = 3 + (plan.sample ? 1 : 0) + int64_t(eng->L) * (4 + attn_launches);
    eng->kernel_launches += eng->last_launches;
  }
  MS_CUDA_TRY(cudaMemcpyAsync(eng->h_next, eng->d_next, size_t(S) * 4, cudaMemcpyDeviceToHost, st));
  MS_CUDA_TRY(cudaMemcpyAsync(eng->h_status, eng->d_status, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  return MS_OK;
}

}  // namespace ms
