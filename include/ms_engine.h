/*
 * ms_engine.h -- C ABI of the B200 (sm_100a) continuous-batching forward step
 * for Qwen2 / Qwen3 decoder models.
 *
 * This library replaces the execution backend of RLSE:
 *   src/backends/candle.rs:377-698   CandleBackend::step_batch
 *   src/backends/qwen2.rs:620-764    ModelForCausalLM::{forward, step_decode_batch}
 * behind the reference's backend contract (src/backends/traits.rs:15-50,
 * trait ModelBackend).  The scheduler (src/scheduler/scheduler.rs) and the
 * logical block manager (src/cache/kv_cache.rs) stay on the caller side: their
 * logical block ids are the physical page ids of this library's paged KV pool.
 *
 * Conventions
 *  - Every function returns int: MS_OK (0) or an MS_E_* code.  The message of
 *    the last failure is available from ms_last_error().
 *  - Error mapping onto src/core/errors.rs:8-17 (EngineError):
 *      MS_E_PRESSURE     -> CachePressure       (recoverable capacity rejection)
 *      MS_E_INVALID      -> BackendError        (caller broke the contract)
 *      MS_E_DEVICE       -> BackendError        (CUDA/cuBLAS failure; engine quarantined)
 *      MS_E_INJECTED     -> BackendError        (host-injected fault; engine quarantined)
 *      MS_E_QUARANTINED  -> NoHealthyWorkers    (engine already quarantined)
 *      MS_E_TOKEN_LIMIT  -> TokenLimitExceeded
 *  - An engine is bound to one CUDA device and one stream.  It is not
 *    reentrant: the caller serialises calls, as the reference's
 *    `active_models` mutex does (src/backends/candle.rs:385).
 *  - Host arrays passed in are borrowed for the duration of the call only.
 *  - Kernel-level launchers (ms_launch_*, launch_*) take caller-owned device
 *    pointers, are asynchronous, and return a cudaError_t value as int.
 */
#ifndef MS_ENGINE_H
#define MS_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MS_ABI_VERSION 1

/* status codes */
#define MS_OK 0
#define MS_E_INVALID 1
#define MS_E_PRESSURE 2
#define MS_E_DEVICE 3
#define MS_E_INJECTED 4
#define MS_E_QUARANTINED 5
#define MS_E_TOKEN_LIMIT 6
#define MS_E_NOT_FOUND 7

/* element types */
#define MS_DTYPE_F32 0
#define MS_DTYPE_BF16 1
#define MS_DTYPE_F16 2

/* ms_step_desc.flags */
#define MS_STEP_TOKENS_FROM_DEVICE 1u /* decode inputs = tokens this engine produced last step */
#define MS_STEP_KEEP_LOGITS 2u        /* keep the step's f32 logits for ms_debug_logits */

/* ms_step out_flags bits */
#define MS_FLAG_PREFILLED 1u /* this step ran the sequence's prefill */
#define MS_FLAG_NO_TOKEN 2u  /* no token this step: the prompt is still being prefilled in chunks */

/* Model configuration.  Mirrors the fields of qwen2.rs:9-54 (Config) that the
 * forward step reads.  qk_norm / attn_bias / tie_word_embeddings are decided
 * in the reference by the presence of tensors (qwen2.rs:231-260, 592-596);
 * here the caller states them. */
typedef struct ms_model_cfg {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t num_layers;
  int32_t num_heads;    /* query heads */
  int32_t num_kv_heads; /* key/value heads */
  int32_t head_dim;     /* 64 or 128 */
  int32_t max_position_embeddings;
  double rope_theta;
  double rms_norm_eps;
  int32_t qk_norm;             /* 1: per-head RMSNorm on q and k (Qwen3) */
  int32_t attn_bias;           /* 1: q/k/v projections carry a bias (Qwen2) */
  int32_t tie_word_embeddings; /* 1: lm_head shares model.embed_tokens.weight */
  int32_t dtype;               /* MS_DTYPE_BF16 (default serving) or MS_DTYPE_F32 (parity mode) */
} ms_model_cfg;

/* Engine sizing.  pool_blocks is the number of physical KV pages per layer;
 * page ids handed in through ms_seq_admit / ms_seq_append_block must lie in
 * [0, pool_blocks).  block_size must be 16 (kv_cache.rs, main.rs:26). */
typedef struct ms_engine_opts {
  int32_t device;
  int32_t tp_rank;  /* tensor-parallel rank (0 when tp_size == 1) */
  int32_t tp_size;  /* 1, 2 or 4; shards by KV head */
  void *nccl_comm;  /* ncclComm_t when tp_size > 1, else NULL */
  int64_t pool_blocks;
  int32_t block_size;
  int32_t max_seqs;            /* concurrent sequences (sequence slots) */
  int32_t max_tokens_per_step; /* packed tokens per ms_step */
  int32_t max_blocks_per_seq;  /* block-table row length */
} ms_engine_opts;

typedef struct ms_engine ms_engine;

/* One continuous-batching iteration, the argument of
 * ModelBackend::step_batch (traits.rs:196-199).  seq_ids lists the active
 * sequences in the scheduler's order.  A sequence that has not been prefilled
 * runs its prompt (minus the tokens already cached, see ms_seq_admit); every
 * other sequence decodes one token: input_tokens[i] (the last output token,
 * candle.rs:622) at position positions[i] (= prompt + outputs - 1,
 * candle.rs:624-628).  positions may be NULL; when given it is checked
 * against the engine's own count.  Prefill entries of input_tokens and
 * positions are ignored. */
typedef struct ms_step_desc {
  int32_t num_seqs;
  const uint64_t *seq_ids;
  const uint32_t *input_tokens; /* may be NULL with MS_STEP_TOKENS_FROM_DEVICE */
  const int32_t *positions;     /* may be NULL */
  uint32_t flags;
  /* Sampling, per sequence (sample_token, candle.rs:737-763).  All three may
   * be NULL: greedy argmax for every sequence.  temperature[i] < 1e-7 (or
   * NULL) is greedy; otherwise the token is drawn from softmax(logits /
   * temperature[i]), cut to the top-p nucleus when 0 < top_p[i] < 1 (top_p
   * NULL: no cut), with the random stream seeded by seeds[i] (NULL: 0).
   * Zero-initialised descriptors from older callers stay greedy. */
  const float *temperature;
  const float *top_p;
  const uint64_t *seeds;
  /* Chunked prefill: at most token_budget packed tokens this step (0: no
   * limit).  Decode rows come first (one token each, never deferred); the
   * rest of the budget goes to unfinished prompts in list order, each taking
   * as many of its remaining prompt tokens as fit.  A prompt that does not
   * finish gets MS_FLAG_NO_TOKEN (its out_tokens entry is 0) and continues
   * from where it stopped in the next step; its block table only has to
   * cover the tokens scheduled so far. */
  int32_t token_budget;
} ms_step_desc;

/* ---- engine lifetime --------------------------------------------------- */

/* Replaces CandleBackend::load_hf (candle.rs:40-227) minus file IO: allocates
 * weights, the paged KV pool and step workspaces on opts->device. */
int ms_engine_create(const ms_model_cfg *cfg, const ms_engine_opts *opts, ms_engine **out);
int ms_engine_destroy(ms_engine *eng);

/* Load one tensor by its Hugging Face name (the names VarBuilder resolves in
 * qwen2.rs, e.g. "model.layers.3.self_attn.q_proj.weight").  src_dtype is an
 * MS_DTYPE_*; src_on_device != 0 means `data` is a device pointer on the
 * engine's device.  Under tensor parallelism the caller passes the full
 * tensor and the engine keeps its shard. */
int ms_engine_load_weight(ms_engine *eng, const char *name, const void *data, int64_t numel,
                          int32_t src_dtype, int32_t src_on_device);
/* Checks that every tensor was loaded; the engine accepts steps afterwards. */
int ms_engine_finalize(ms_engine *eng);

/* Bytes of device memory the engine holds (weights + pool + workspaces). */
int ms_engine_memory(const ms_engine *eng, int64_t *weights_bytes, int64_t *pool_bytes,
                     int64_t *workspace_bytes);

/* ---- tensor parallelism (no counterpart in the reference) ---------------
 * One engine per GPU; tp_size engines form one model replica, sharded by KV
 * head (q/k/v rows and o_proj columns per KV-head group, gate/up rows and
 * down columns per intermediate slice).  The partial o_proj and down_proj
 * outputs are summed with an NCCL all-reduce on the engine stream.  These
 * helpers create the communicator with the NCCL already loaded in the process
 * (or libnccl.so.2): rank 0 makes the id, every rank passes the same bytes. */
int ms_nccl_get_unique_id(uint8_t *out, int32_t len);
int ms_nccl_comm_init(void **comm_out, int32_t nranks, const uint8_t *unique_id, int32_t rank,
                      int32_t device);
int ms_nccl_comm_destroy(void *comm);

/* ---- sequence lifetime (scheduler deltas) ------------------------------ */

/* Admit a sequence (scheduler.rs:347-369): its prompt tokens and the logical
 * KV blocks KVCache::allocate returned (kv_cache.rs:61-84).  num_cached
 * prompt tokens already have their K/V in those blocks (a shared prefix);
 * when num_cached == prompt length the last prompt token is replayed, as the
 * reference does on an exact prefix hit without logits (candle.rs:447-455). */
int ms_seq_admit(ms_engine *eng, uint64_t seq_id, const uint32_t *prompt, int32_t prompt_len,
                 const int32_t *block_ids, int32_t num_blocks, int32_t num_cached);
/* KVCache::allocate_block result pushed onto seq.kv_blocks (scheduler.rs:422-449). */
int ms_seq_append_block(ms_engine *eng, uint64_t seq_id, int32_t block_id);
/* ModelBackend::cancel_sequence (traits.rs:200, candle.rs:700-704): drops all
 * per-request state.  Idempotent: an unknown id returns MS_OK. */
int ms_seq_release(ms_engine *eng, uint64_t seq_id);
/* Number of tokens whose K/V the engine holds for seq_id. */
int ms_seq_cached_tokens(const ms_engine *eng, uint64_t seq_id, int32_t *out);

/* ---- paged prefix cache (kv_cache.rs:14-145 + prefix_cache.rs:57-345) ---
 * A host-side page manager the scheduler uses in place of KVCache.  A cached
 * 16-token chunk is the pool page holding its K/V, so a prefix hit shares
 * pages (reference counts) instead of copying snapshots; chain keys are the
 * reference's SHA-256 chain (prefix_cache.rs:103-124).  Flow per request:
 * ms_pages_admit -> ms_seq_admit(eng, id, prompt, blocks, n, cached) ->
 * steps (ms_pages_allocate_block + ms_seq_append_block as it grows) ->
 * ms_pages_publish once its prompt is prefilled -> ms_seq_release +
 * ms_pages_release.  Thread-safe (one mutex); one manager per pool. */
typedef struct ms_pages ms_pages;
typedef struct ms_pages_stats {
  int64_t total_blocks;
  int64_t free_blocks;       /* on the free stack */
  int64_t cached_chunks;     /* prefix-cache entries (one page each) */
  int64_t cache_only_blocks; /* cached pages no sequence holds (evictable) */
  int64_t hits, misses, tokens_saved; /* record_reuse, prefix_cache.rs:359-367 */
  int64_t evictions;         /* cached chunks evicted */
  int64_t rejections;        /* admissions / block requests refused (CachePressure) */
  int64_t reserved_blocks;   /* worst-case pages held by reservations */
  int64_t peak_reserved_blocks;
  int64_t reservation_rejections; /* ms_pages_reserve refused (CachePressure) */
} ms_pages_stats;
/* max_chunks = 0 disables the prefix cache: block ids are then exactly
 * KVCache's (LIFO stack popping 0, 1, 2, ... first). */
int ms_pages_create(int64_t total_blocks, int32_t block_size, int32_t max_chunks, ms_pages **out);
int ms_pages_destroy(ms_pages *pm);
/* Scheduler admission (scheduler.rs:347-369): pages for max(prompt_len, 1)
 * tokens, the leading ones shared from the prefix cache (at most
 * (prompt_len - 1) / block_size chunks, so the last prompt token is always
 * computed), the rest fresh.  cached_tokens_out = shared chunks * block_size,
 * the num_cached of ms_seq_admit.  All or nothing; MS_E_PRESSURE when the free
 * pages, after evicting unused cached chunks, do not suffice. */
int ms_pages_admit(ms_pages *pm, uint64_t seq_id, const uint32_t *prompt, int32_t prompt_len,
                   int32_t *blocks_out, int32_t capacity, int32_t *num_blocks_out, int32_t *cached_tokens_out);
/* KVCache::allocate_block (kv_cache.rs:86-99). */
int ms_pages_allocate_block(ms_pages *pm, uint64_t seq_id, int32_t *block_out);
/* KVCache::release (kv_cache.rs:101-111): drops the sequence's references. */
int ms_pages_release(ms_pages *pm, uint64_t seq_id, int32_t *released_out);
/* After the sequence's prompt is prefilled (insert_kv, candle.rs:552-573):
 * its full prompt chunks not yet cached enter the cache as its own pages. */
int ms_pages_publish(ms_pages *pm, uint64_t seq_id, const uint32_t *prompt, int32_t prompt_len,
                     int32_t *published_out);
/* PrefixCache::lookup (prefix_cache.rs:126-157): leading cached tokens. */
int ms_pages_lookup(ms_pages *pm, const uint32_t *prompt, int32_t prompt_len, int32_t *matched_tokens);
/* reserve_sequence's memory budget (candle.rs:349-375, tensor_memory.rs:72-111,
 * prefix_cache.rs:229-244) with the page pool as the budget: a request is
 * charged its worst case, ceil((prompt_len + max_tokens) / block_size) pages.
 * Reservations plus the pages only the prefix cache holds must fit the pool;
 * least recently used cache-only pages are evicted to make room, and when
 * that is not enough the call returns MS_E_PRESSURE (CachePressure) and
 * charges nothing (the entries evicted on the way stay evicted, as in the
 * reference).  Idempotent per seq_id (a second call returns MS_OK without
 * a new charge); prompt_len or max_tokens <= 0 is MS_E_TOKEN_LIMIT.
 * ms_pages_release also ends the sequence's reservation.  While every
 * admitted sequence holds a reservation, its page requests never fail. */
int ms_pages_reserve(ms_pages *pm, uint64_t seq_id, int64_t prompt_len, int64_t max_tokens);
int ms_pages_stats_get(ms_pages *pm, ms_pages_stats *out);
/* The chain keys (32 bytes each) of the full chunks of tokens; returns their
 * count, -1 on bad arguments or capacity (in keys) too small. */
int ms_prefix_chunk_hashes(const uint32_t *tokens, int32_t num_tokens, int32_t chunk_size, uint8_t *out,
                           int32_t capacity);

/* ---- the hot path ------------------------------------------------------ */

/* step_batch: one token per sequence into out_tokens[num_seqs] (greedy
 * argmax of f32 logits, candle.rs:737-751), MS_FLAG_* bits into out_flags
 * (may be NULL).  Synchronous: returns after the tokens reached the host. */
int ms_step(ms_engine *eng, const ms_step_desc *desc, uint32_t *out_tokens, uint8_t *out_flags);

/* ms_step split in two.  ms_step_launch validates, uploads the step's inputs
 * and enqueues all device work on the engine stream; ms_step_wait copies the
 * tokens back and synchronises.  Exactly one wait follows each launch. */
int ms_step_launch(ms_engine *eng, const ms_step_desc *desc);
int ms_step_wait(ms_engine *eng, uint32_t *out_tokens, uint8_t *out_flags);

/* The engine's CUDA stream (cudaStream_t) for callers that time or order work. */
int ms_engine_stream(const ms_engine *eng, void **stream_out);

/* ---- instrumentation (no counterpart in the reference) ------------------
 * kernel_launches counts this library's own kernel launches since creation.
 * With profiling on, CUDA events bracket every paged-attention launch (and
 * its partition merge) on the engine stream; ms_engine_profile synchronises,
 * returns the number of bracketed launches, their summed duration and their
 * summed algorithmic bytes (K and V rows read + q/out + table entries), then
 * clears the event log. */
int ms_engine_set_profiling(ms_engine *eng, int32_t on);
int ms_engine_profile(ms_engine *eng, int64_t *kernel_launches, int64_t *attn_launches,
                      double *attn_ms_total, double *attn_bytes_total);
/* Under tensor parallelism with profiling on, CUDA events also bracket each
 * all-reduce section after o_proj and down_proj (the fused peer-memory
 * all-reduce + residual add + RMSNorm kernel, or NCCL all-reduce + K4):
 * returns how many sections were bracketed and their summed duration, then
 * clears that log. */
int ms_engine_profile_allreduce(ms_engine *eng, int64_t *calls, double *ms_total);

/* ---- CUDA graphs of decode steps (no counterpart in the reference) -------
 * Steps with one token per sequence, at most num_seqs new block-table
 * entries and tp_size 1 are replayed from captured CUDA graphs keyed by
 * (num_seqs, attention partition size, context capacity): the first step of
 * a key runs eagerly, the second is captured, later ones replay (the step
 * description goes through a fixed-layout staging buffer).  Results are
 * identical to eager steps.  On by default; the environment variable
 * MS_CUDA_GRAPHS=0 or ms_engine_set_graphs(eng, 0) turns it off (which also
 * drops the cached graphs).  Not used while profiling is on. */
int ms_engine_set_graphs(ms_engine *eng, int32_t on);
int ms_engine_graph_stats(const ms_engine *eng, int64_t *captures, int64_t *replays, int32_t *cached);

/* Tensor parallelism: *fused = 1 when the all-reduces after o_proj and
 * down_proj run as one peer-memory kernel fused with the residual add and
 * RMSNorm (NVLink, CUDA IPC mappings set up at creation), 0 when they go
 * through NCCL (tp_size 1, MS_TP_FUSED=0, or a rank that could not map its
 * peers -- all ranks then agree on NCCL).  No reference counterpart. */
int ms_engine_tp_fused(const ms_engine *eng, int32_t *fused);
/* Selects the all-reduce path of later steps: on = 1 the fused peer-memory
 * kernel (only where creation set it up, else MS_E_INVALID), on = 0 NCCL
 * all-reduce + K4.  Every rank of the tensor-parallel group must switch
 * between the same two steps.  No reference counterpart. */
int ms_engine_set_tp_fused(ms_engine *eng, int32_t on);

/* ---- health (traits.rs:175-180, candle.rs:324-335) --------------------- */
int ms_is_healthy(const ms_engine *eng);
int ms_mark_unhealthy(ms_engine *eng);
/* Host-side fault injection for tests: the next ms_step fails with
 * MS_E_INJECTED and quarantines the engine.  No device fault is involved. */
int ms_inject_fault(ms_engine *eng, int32_t code);
/* Copy the message of the last failure (NUL-terminated, truncated to len). */
int ms_last_error(const ms_engine *eng, char *buf, int32_t len);

/* ---- debugging / parity ------------------------------------------------ */

/* Packed metadata of the last step as the on-GPU packer wrote it:
 * cu_seqlens[num_seqs+1], positions[T], slot_mapping[T],
 * block_tables[num_seqs * max_blocks_per_seq] (rows in step order).
 * Any pointer may be NULL.  *num_tokens receives T. */
int ms_debug_dump_tables(ms_engine *eng, int32_t *num_tokens, int32_t *cu_seqlens,
                         int32_t *positions, int64_t *slot_mapping, int32_t *block_tables);
/* f32 logits of the last step run with MS_STEP_KEEP_LOGITS: [num_seqs, vocab]. */
int ms_debug_logits(ms_engine *eng, float *out, int64_t count);
/* Copy an activation buffer of the last step to host memory, for parity
 * checks of a single layer: "x_resid" / "x_norm" / "x_tmp" [T, H],
 * "qkv" [T, (Hq + 2 Hkv) * D], "q" and "attn" [T, Hq * D], "gu" [T, 2I],
 * "act" [T, I], "last_norm" [num_seqs, H] (model dtype), "row_ctx" /
 * "row_table" / "positions" [T] (int32).  Fails if `bytes` is too small. */
int ms_debug_buffer(ms_engine *eng, const char *name, void *out, int64_t bytes);
/* Debugging, for per-layer parity checks: layer >= 0 makes later steps stop
 * after that layer's MLP down projection (no residual add after it, no final
 * norm, lm_head or sampling), so ms_debug_buffer returns that layer's "attn"
 * (attention output), "x_resid" (residual after attention), "x_norm"
 * (post-attention RMSNorm) and "x_tmp" (MLP output); -1 turns it off.  Such a
 * step leaves its sequences' later layers without K/V: release them after.
 * Eager steps only; not with the fused TP all-reduce. */
int ms_debug_stop_after_layer(ms_engine *eng, int32_t layer);
/* Device address of layer `layer`'s K (which = 0) or V (which = 1) page pool,
 * laid out [pool_blocks, num_kv_heads_local, block_size, head_dim]. */
int ms_debug_pool_ptr(ms_engine *eng, int32_t layer, int32_t which, void **ptr);

/* ---- kernel-level operators (device pointers, asynchronous) ------------ */

/* K1: ragged batch packer.  From per-sequence (table row, token count, first
 * position) and block-table deltas, writes cu_seqlens[nseq+1],
 * positions[T], slot_mapping[T] (block_table[row][pos/bs]*bs + pos%bs),
 * row_table[T] and row_ctx[T] = pos + 1.  Replaces the host tensor building
 * of candle.rs:603-630 and qwen2.rs:649-655. */
int ms_launch_pack(const int32_t *seq_row, const int32_t *seq_ntok, const int32_t *seq_start,
                   int32_t num_seqs, const int32_t *delta_row, const int32_t *delta_idx,
                   const int32_t *delta_block, int32_t num_deltas, int32_t *block_tables,
                   int32_t max_blocks_per_seq, int32_t block_size, int32_t *cu_seqlens,
                   int32_t *positions, int64_t *slot_mapping, int32_t *row_table,
                   int32_t *row_ctx, void *stream);

/* K4: fused residual add + RMSNorm (qwen2.rs:68-75 with the adds of
 * qwen2.rs:420-427).  With s = x + r in f32 (r may be NULL: s = x):
 * resid_out = s and norm_out = s / sqrt(mean(s^2) + eps) * w, each computed
 * in f32 and rounded once to the dtype.  row_index (may be NULL) gathers
 * input rows; outputs are compact.  resid_out may be NULL. */
int ms_launch_add_rmsnorm(const void *x, const void *r, const int32_t *row_index,
                          const void *w, void *resid_out, void *norm_out, int32_t rows,
                          int32_t hidden, float eps, int32_t dtype, void *stream);

/* K5 + K2: per-head q/k RMSNorm (optional), rotate-half RoPE at positions[t]
 * with the cos/sin tables (f32 [max_pos, D/2] for every dtype), q written to
 * q_out [T, Hq, D]; k and v written into the paged pools at slot_mapping[t]
 * (qwen2.rs:287-313).  qkv is [T, (Hq + 2 Hkv) * D]; bias (may be NULL) is
 * added first.  Arithmetic is f32; each output is rounded once. */
int ms_launch_qk_norm_rope_append(const void *qkv, const void *bias, const void *q_norm_w,
                                  const void *k_norm_w, const void *cos_table,
                                  const void *sin_table, const int32_t *positions,
                                  const int64_t *slot_mapping, void *q_out, void *k_pool,
                                  void *v_pool, int32_t num_tokens, int32_t num_heads,
                                  int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                  float eps, int32_t dtype, void *stream);

/* K3: split-K paged GQA attention, one query row per entry
 * (decode_attention_gqa_zero_copy, qwen2.rs:182-203, batched over rows).
 * Row t attends to tokens [0, row_ctx[t]) of block-table row row_table[t]
 * (row_table may be NULL: row t uses table row t).  q [T, Hq, D], out
 * [T, Hq, D].  Blocks of `partition_blocks` pages are processed by separate
 * CTAs and merged by log-sum-exp; `workspace` must hold
 * ms_attention_workspace_bytes(...) bytes when more than one partition is
 * needed.  Pass partition_blocks = 0 to let the launcher choose. */
int64_t ms_attention_workspace_bytes(int32_t num_rows, int32_t num_heads, int32_t max_ctx,
                                     int32_t partition_blocks, int32_t block_size);
int ms_launch_paged_attention(const void *q, const void *k_pool, const void *v_pool,
                              const int32_t *block_tables, int32_t max_blocks_per_seq,
                              const int32_t *row_table, const int32_t *row_ctx,
                              int32_t num_rows, int32_t max_ctx, void *out, int32_t num_heads,
                              int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                              float scale, int32_t partition_blocks, void *workspace,
                              int64_t workspace_bytes, int32_t dtype, void *stream);

/* K3p: ragged causal prefill attention over the paged pool, bf16 / f16 on
 * tensor cores (the prefill branch of qwen2.rs:329-345 with the causal mask
 * of :476-503, including the offset columns of a cached prefix).  A tile is
 * up to ms_prefill_tiles' tile size of consecutive tokens of one sequence:
 * tiles[num_tiles][4] (device) = first packed row, rows, position of the
 * first row, block-table row.  Row t attends to keys 0..position(t) of its
 * table row; q / out as for ms_launch_paged_attention. */
int ms_launch_paged_prefill(const void *q, const void *k_pool, const void *v_pool,
                            const int32_t *block_tables, int32_t max_blocks_per_seq,
                            const int32_t *tiles, int32_t num_tiles, void *out, int32_t num_heads,
                            int32_t num_kv_heads, int32_t head_dim, int32_t block_size, float scale,
                            int32_t dtype, void *stream);
/* Host helper: cut per-sequence prompt chunks (first packed row, tokens,
 * first position, block-table row) into prefill tiles.  Returns the number
 * of tiles written to tiles_out, or -1 if capacity (in tiles) is too small. */
int ms_prefill_tiles(const int32_t *seq_row0, const int32_t *seq_ntok, const int32_t *seq_start,
                     const int32_t *seq_table_row, int32_t num_seqs, int32_t num_heads,
                     int32_t num_kv_heads, int32_t *tiles_out, int32_t capacity);

/* Status of the kernels launched without an engine on `device`: the
 * prototype-compatible launchers below, ms_launch_sample, and
 * ms_launch_paged_attention / ms_launch_paged_prefill (which use it when their
 * own status word is NULL).
 * Synchronises the device, returns the OR of the kernels' status bits since
 * the last call (1 = a bounded wait ran out and the kernel returned without
 * writing its output, 2 = an index out of range) and clears them.  No
 * counterpart in the reference, whose kernels do not wait on barriers. */
int ms_kernel_status(int32_t device, uint32_t *status_out);
/* Test hook: polls >= 0 limits every page-loop wait of the decode-attention
 * kernels launched afterwards to that many polls -- 0 makes the first wait
 * give up at once -- and polls < 0 restores the default of 4M polls.  A test
 * can so make a wait run out while every copy the kernel started still lands
 * (the drain after a failed wait keeps the default limit). */
int ms_test_set_attention_wait_limit(int32_t polls);

/* K6b on-device sampling over f32 logits [rows, vocab]: for each row with
 * temperature[row] >= 1e-7 the token is drawn as candle-transformers'
 * LogitsProcessor draws it (softmax of logits / temperature, top-p nucleus
 * when 0 < top_p[row] < 1, ties at the nucleus edge kept in index order) from
 * a counter-based stream seeded by seeds[row]; rows below 1e-7 are left as
 * they are in out (run ms_launch_argmax first).  top_p and seeds may be NULL.
 * Each row runs on a cluster of 8 CTAs; a staging copy that does not land in
 * time leaves the row's out untouched and sets bit 1 of the status word that
 * ms_kernel_status returns. */
int ms_launch_sample(const float *logits, int32_t rows, int32_t vocab, const float *temperature,
                     const float *top_p, const uint64_t *seeds, int32_t *out, void *stream);

/* K6 glue. */
int ms_launch_silu_mul(const void *gate_up, void *out, int32_t rows, int32_t inter,
                       int32_t dtype, void *stream);
int ms_launch_argmax(const float *logits, int32_t rows, int32_t vocab, int32_t *out,
                     void *stream);

/* ---- prototype-compatible launchers ------------------------------------
 * Same signatures and argument checks as the reference's prototype C ABI
 * (docs/colab_cuda_kernels/mini_serve_kernels.cu:247-296): default stream,
 * asynchronous, cudaError_t as int, block size 16, head_dim 128.  They run
 * this library's kernels.  The return value covers the launch only; a
 * failure inside the kernel (a bounded wait that ran out) sets a bit of the
 * device's status word, which ms_kernel_status returns. */
int launch_rmsnorm_f32(const float *d_x, const float *d_w, float *d_out, int num_rows,
                       int hidden_size, float eps);
int launch_rmsnorm_f16(const void *d_x, const void *d_w, void *d_out, int num_rows,
                       int hidden_size, float eps);
int launch_rmsnorm_bf16(const void *d_x, const void *d_w, void *d_out, int num_rows,
                        int hidden_size, float eps);
int launch_paged_gqa_decode_tiled_f32(const float *d_q, const float *d_k_pool,
                                      const float *d_v_pool, const int *d_block_tables,
                                      const int *d_seq_lens, float *d_out, int batch_size,
                                      int num_heads, int num_kv_heads, int max_blocks_per_seq,
                                      float scale);
int launch_paged_gqa_decode_tiled_f16(const void *d_q, const void *d_k_pool,
                                      const void *d_v_pool, const int *d_block_tables,
                                      const int *d_seq_lens, void *d_out, int batch_size,
                                      int num_heads, int num_kv_heads, int max_blocks_per_seq,
                                      float scale);
int launch_paged_gqa_decode_tiled_bf16(const void *d_q, const void *d_k_pool,
                                       const void *d_v_pool, const int *d_block_tables,
                                       const int *d_seq_lens, void *d_out, int batch_size,
                                       int num_heads, int num_kv_heads, int max_blocks_per_seq,
                                       float scale);

/* No counterpart in the reference.  Same arguments, checks and result as
 * launch_paged_gqa_decode_tiled_bf16, for callers that must not allocate
 * device memory (their allocator already owns the HBM budget, or they cannot
 * afford the device-wide synchronisation of cudaMalloc/cudaFree on the hot
 * path): it calls no allocation routine and keeps its split-K scratch in a
 * fixed 16 MiB buffer inside the library, which every GPU that loads the
 * library holds until exit.  A call whose scratch would exceed 16 MiB
 * (batch_size * num_heads * partitions * 520 bytes) returns
 * cudaErrorMemoryAllocation without launching anything.  The CUDA runtime
 * reserves the 16 MiB on a device when it loads the buffer's module there --
 * under CUDA's default lazy module loading, at the first call on that device
 * -- so make one call per device before the caller's allocator claims its
 * HBM, and before any stream capture.  Calls share the buffer: calls that may
 * overlap on the GPU race and must be serialised by the caller.  A bounded
 * wait that ran out inside the kernel is reported by ms_kernel_status. */
int launch_paged_gqa_decode_tiled_bf16_noalloc(const void *d_q, const void *d_k_pool,
                                               const void *d_v_pool, const int *d_block_tables,
                                               const int *d_seq_lens, void *d_out, int batch_size,
                                               int num_heads, int num_kv_heads,
                                               int max_blocks_per_seq, float scale);

#ifdef __cplusplus
}
#endif

#endif /* MS_ENGINE_H */
