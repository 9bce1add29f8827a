// Engine step: one continuous-batching iteration (ModelBackend::step_batch,
// src/backends/traits.rs:196-199; CandleBackend::step_batch,
// src/backends/candle.rs:377-698).
//
// The reference runs every new sequence's prefill alone and then one batched
// decode; here all of them go into one packed ragged batch: prefill rows
// carry their whole (uncached) prompt, decode rows one token at
// prompt + outputs - 1 (candle.rs:622-628).  Each sequence gets its greedy
// token from the f32 logits of its last packed row (candle.rs:737-751).
#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <string>
#include <thread>

#include "ms_engine.h"

namespace ms {

#define MS_CUDA_TRY(expr)                                                                    \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    if (_e != cudaSuccess)                                                                   \
      return eng->fail(MS_E_DEVICE, std::string(#expr) + ": " + cudaGetErrorString(_e));     \
  } while (0)

namespace {

struct RowPlan {
  Seq *seq;
  int ntok, start;
  bool prefill;
  bool partial = false;  // a prompt chunk that does not reach the prompt's end
  int orig = 0;          // index in the step description
};

int grow_staging(Engine *eng, size_t elems) {
  if (elems <= eng->in_cap) return MS_OK;
  size_t cap = std::max<size_t>(elems, eng->in_cap * 2);
  cap = std::max<size_t>(cap, 1 << 16);
  if (eng->h_in) cudaFreeHost(eng->h_in);
  if (eng->d_in) cudaFree(eng->d_in);
  eng->h_in = nullptr;
  eng->d_in = nullptr;
  eng->in_cap = 0;
  MS_CUDA_TRY(cudaMallocHost(&eng->h_in, cap * 4));
  MS_CUDA_TRY(cudaMalloc(&eng->d_in, cap * 4));
  eng->in_cap = cap;
  return MS_OK;
}

}  // namespace


int step_launch_impl(Engine *eng, const ms_step_desc *desc) {
  if (!eng->healthy) {
    eng->err = "Backend quarantined; restart required";
    return MS_E_QUARANTINED;
  }
  if (!eng->finalized) return eng->fail(MS_E_INVALID, "engine not finalized (weights missing)");
  if (eng->pending) return eng->fail(MS_E_INVALID, "ms_step_launch called twice without ms_step_wait");
  if (!desc) return eng->fail(MS_E_INVALID, "null step description");
  if (eng->inject) {
    eng->inject = 0;
    return eng->fail(MS_E_INJECTED, "injected fault");
  }
  const int S_in = desc->num_seqs;
  if (S_in < 0 || S_in > eng->opts.max_seqs) return eng->fail(MS_E_INVALID, "num_seqs out of range");
  if (desc->token_budget < 0) return eng->fail(MS_E_INVALID, "negative token_budget");
  if (S_in == 0) {  // candle.rs:381-383: an empty batch is a no-op
    eng->pending = true;
    eng->last_nseq = 0;
    eng->last_in = 0;
    eng->last_T = 0;
    return MS_OK;
  }
  if (!desc->seq_ids) return eng->fail(MS_E_INVALID, "null seq_ids");
  eng->last_ids.assign(desc->seq_ids, desc->seq_ids + S_in);
  const bool from_dev = (desc->flags & MS_STEP_TOKENS_FROM_DEVICE) != 0;

  // ---- plan (validate everything before touching state) ----
  std::vector<RowPlan> all(S_in);
  std::unordered_map<uint64_t, int> seen;
  int n_decode = 0;
  for (int i = 0; i < S_in; ++i) {
    const uint64_t id = desc->seq_ids[i];
    auto it = eng->seqs.find(id);
    if (it == eng->seqs.end()) return eng->fail(MS_E_NOT_FOUND, "unknown sequence id " + std::to_string(id));
    if (!seen.emplace(id, i).second) return eng->fail(MS_E_INVALID, "sequence listed twice in one step");
    Seq &s = it->second;
    RowPlan &r = all[i];
    r.seq = &s;
    r.orig = i;
    r.prefill = !s.prefilled;
    const int plen = int(s.prompt.size());
    if (r.prefill) {
      if (s.cached >= plen) {  // exact cached prefix: replay the last prompt token (candle.rs:447-455)
        r.start = plen - 1;
        r.ntok = 1;
      } else {
        r.start = s.cached;
        r.ntok = plen - s.cached;
      }
    } else {
      ++n_decode;
      r.start = s.cached;
      r.ntok = 1;
      if (desc->positions && desc->positions[i] != s.cached)
        return eng->fail(MS_E_INVALID, "decode position " + std::to_string(desc->positions[i]) +
                                           " does not match the engine's " + std::to_string(s.cached));
      if (!from_dev) {
        if (!desc->input_tokens) return eng->fail(MS_E_INVALID, "null input_tokens");
        if (desc->input_tokens[i] >= uint32_t(eng->V)) return eng->fail(MS_E_INVALID, "input token outside the vocabulary");
      }
    }
  }
  // chunked prefill: decode rows first, then prompt tokens in list order
  if (desc->token_budget > 0) {
    long long left = (long long)desc->token_budget - n_decode;
    for (RowPlan &r : all) {
      if (!r.prefill) continue;
      const int take = int(std::max(0LL, std::min<long long>(r.ntok, left)));
      left -= take;
      r.partial = take < r.ntok;
      r.ntok = take;
    }
  }
  std::vector<RowPlan> plan;
  std::vector<int> map(S_in, -1);
  plan.reserve(S_in);
  for (int i = 0; i < S_in; ++i)
    if (all[i].ntok > 0) {
      map[i] = int(plan.size());
      plan.push_back(all[i]);
    }
  const int S = int(plan.size());
  int T = 0, nd = 0, max_ctx = 0;
  long long total_blocks = 0;
  double total_ctx = 0.0;  // sum over packed rows of the keys each row attends to
  for (RowPlan &r : plan) {
    const Seq &s = *r.seq;
    const int end = r.start + r.ntok;
    if (end > eng->rope_len) return eng->fail(MS_E_TOKEN_LIMIT, "position beyond max_position_embeddings");
    if (int64_t(end) > int64_t(s.blocks.size()) * eng->opts.block_size)
      return eng->fail(MS_E_INVALID, "block table too short for position " + std::to_string(end - 1));
    T += r.ntok;
    nd += int(s.blocks.size()) - s.synced;
    max_ctx = std::max(max_ctx, end);
    for (int j = 0; j < r.ntok; ++j) {
      total_ctx += double(r.start + j + 1);
      total_blocks += (r.start + j + 1 + 15) / 16;
    }
  }
  if (T > eng->opts.max_tokens_per_step)
    return eng->fail(MS_E_PRESSURE, "step needs " + std::to_string(T) + " tokens, engine holds " +
                                        std::to_string(eng->opts.max_tokens_per_step));
  eng->last_in = S_in;
  eng->last_map = map;
  eng->last_out_flags.assign(S_in, uint8_t(MS_FLAG_NO_TOKEN));
  if (S == 0) {  // every listed prompt deferred by a zero budget
    eng->pending = true;
    eng->last_nseq = 0;
    eng->last_T = 0;
    return MS_OK;
  }

  // ---- attention work split: decode rows (one token) and prefill tiles ----
  StepPlan sp;
  sp.S = S;
  sp.T = T;
  sp.nd = nd;
  sp.split = eng->use_tc;
  std::vector<int32_t> dec_rows, tiles;
  if (sp.split) {
    std::vector<int32_t> prow0, pntok, pstart, ptrow;
    int row0 = 0;
    for (int i = 0; i < S; ++i) {
      const RowPlan &r = plan[i];
      const int end = r.start + r.ntok;
      if (r.ntok == 1) {
        dec_rows.push_back(row0);
        sp.max_ctx_dec = std::max(sp.max_ctx_dec, end);
        sp.blocks_dec += (end + 15) / 16;
        sp.ctx_dec += double(end);
      } else {
        prow0.push_back(row0);
        pntok.push_back(r.ntok);
        pstart.push_back(r.start);
        ptrow.push_back(r.seq->slot);
      }
      row0 += r.ntok;
    }
    sp.n_dec = int(dec_rows.size());
    if (!prow0.empty()) {
      const int group = eng->hq / eng->hkv;
      const int cap = T;  // a tile holds at least one token
      tiles.resize(size_t(4) * cap);
      sp.n_tiles = build_prefill_tiles(prow0.data(), pntok.data(), pstart.data(), ptrow.data(), int(prow0.size()),
                                       group, tiles.data(), cap);
      if (sp.n_tiles < 0) return eng->fail(MS_E_INVALID, "prefill tile list overflow");
    }
  } else {
    sp.n_dec = T;
    sp.max_ctx_dec = max_ctx;
    sp.blocks_dec = total_blocks;
    sp.ctx_dec = total_ctx;
  }

  // ---- decode attention launch shape ----
  sp.part = decode_partition(eng, sp, sp.max_ctx_dec);
  sp.max_ctx_launch = sp.max_ctx_dec;

  // ---- replay a captured graph for pure-decode steps ----
  // Eligible: one token per sequence (so the decode rows are the packed rows
  // and there are no prefill tiles), at most S block-table deltas, no
  // collectives, no per-launch profiling events.
  const bool graph_ok = eng->graphs_enabled && eng->tp == 1 && !eng->profiling && eng->debug_stop_layer < 0 &&
                        T == S && nd <= S &&
                        (!sp.split || (sp.n_dec == S && sp.n_tiles == 0));
  Engine::StepGraph *g = nullptr;
  bool capture = false;
  if (graph_ok) {
    for (auto &c : eng->graphs)
      if (c.S == S && c.part == sp.part && c.max_ctx_cap >= sp.max_ctx_dec) g = &c;
    if (!g) {
      // first step of a (batch, partition) key runs eagerly (one-time launch
      // attributes, library heuristics); the next one is captured
      int &warm = eng->graph_warm[int64_t(S) << 32 | uint32_t(sp.part)];
      if (warm++ > 0) {
        const int max_blk = (sp.max_ctx_dec + 15) / 16;
        const int cap_ctx = ((max_blk + sp.part - 1) / sp.part + 1) * sp.part * 16;  // one spare partition
        if (attention_workspace_bytes(S, eng->hq, cap_ctx, sp.part) <= int64_t(eng->attn_ws_bytes)) {
          capture = true;
          if (eng->graphs.size() >= 16) {  // evict the least recently used
            auto lru = std::min_element(eng->graphs.begin(), eng->graphs.end(),
                                        [](const Engine::StepGraph &x, const Engine::StepGraph &y) {
                                          return x.last_use < y.last_use;
                                        });
            cudaGraphExecDestroy(lru->exec);
            eng->graphs.erase(lru);
          }
          eng->graphs.emplace_back();
          g = &eng->graphs.back();
          g->S = S;
          g->part = sp.part;
          g->max_ctx_cap = cap_ctx;
        }
      }
    }
  }

  // ---- stage the step description: one pinned buffer, one upload ----
  // (a graph always carries the sampling block: all-greedy rows exit at once)
  bool want_sample = false;
  if (desc->temperature)
    for (int i = 0; i < S && !want_sample; ++i) want_sample = double(desc->temperature[plan[i].orig]) >= 1e-7;
  int32_t *h;
  if (g) {
    sp.graph = true;
    sp.sample = true;
    sp.nucleus = true;  // the captured launch serves whatever top-p a replay brings
    sp.hdr = 4;
    sp.delta_cap = S;
    sp.max_ctx_launch = g->max_ctx_cap;
    sp.h_desc = eng->h_gin;
    sp.d_desc = eng->d_gin;
    sp.desc_elems = 4 + size_t(11) * S;
    h = eng->h_gin;
    h[0] = nd;
    h[1] = h[2] = h[3] = 0;
    h += 4;
  } else {
    sp.sample = want_sample;
    sp.delta_cap = nd;
    const size_t need = size_t(3) * S + T + (sp.sample ? size_t(4) * S : 0) + size_t(3) * nd +
                        (sp.split ? size_t(sp.n_dec) + 4 * size_t(sp.n_tiles) : 0);
    int rc = grow_staging(eng, need);
    if (rc != MS_OK) return rc;
    sp.h_desc = eng->h_in;
    sp.d_desc = eng->d_in;
    sp.desc_elems = need;
    h = eng->h_in;
  }
  const int dc = sp.delta_cap;
  int32_t *h_row = h, *h_ntok = h + S, *h_start = h + 2 * S, *h_tok = h + 3 * S;
  int32_t *h_samp = h_tok + T;
  int32_t *h_drow = h_samp + (sp.sample ? 4 * S : 0), *h_didx = h_drow + dc, *h_dblk = h_didx + dc;
  if (sp.sample) {
    float *temp = reinterpret_cast<float *>(h_samp), *topp = reinterpret_cast<float *>(h_samp + S);
    uint32_t *slo = reinterpret_cast<uint32_t *>(h_samp + 2 * S), *shi = reinterpret_cast<uint32_t *>(h_samp + 3 * S);
    for (int i = 0; i < S; ++i) {
      const int o = plan[i].orig;
      temp[i] = desc->temperature ? desc->temperature[o] : 0.f;
      topp[i] = desc->top_p ? desc->top_p[o] : 1.f;
      if (double(temp[i]) >= 1e-7 && topp[i] > 0.f && topp[i] < 1.f) sp.nucleus = true;
      const uint64_t sd = desc->seeds ? desc->seeds[o] : 0ull;
      slo[i] = uint32_t(sd);
      shi[i] = uint32_t(sd >> 32);
    }
  }
  int t = 0, d = 0;
  for (int i = 0; i < S; ++i) {
    const RowPlan &r = plan[i];
    Seq &s = *r.seq;
    h_row[i] = s.slot;
    h_ntok[i] = r.ntok;
    h_start[i] = r.start;
    if (r.prefill) {
      for (int j = 0; j < r.ntok; ++j) h_tok[t++] = int32_t(s.prompt[r.start + j]);
    } else {
      h_tok[t++] = from_dev ? -1 : int32_t(desc->input_tokens[r.orig]);
    }
    for (int b = s.synced; b < int(s.blocks.size()); ++b, ++d) {
      h_drow[d] = s.slot;
      h_didx[d] = b;
      h_dblk[d] = s.blocks[b];
    }
  }
  if (sp.split && !sp.graph) {
    int32_t *h_dec = h_dblk + dc;
    std::copy(dec_rows.begin(), dec_rows.end(), h_dec);
    std::copy(tiles.begin(), tiles.begin() + 4 * size_t(sp.n_tiles), h_dec + sp.n_dec);
  }
  if (sp.graph) sp.split = false;  // decode rows are the packed rows: identity row list
  MS_CUDA_TRY(cudaSetDevice(eng->dev));
  if (g && !capture) {
    MS_CUDA_TRY(cudaGraphLaunch(g->exec, eng->stream));
    eng->kernel_launches += g->launches;
    ++eng->graph_replays;
  } else if (capture) {
    MS_CUDA_TRY(cudaStreamBeginCapture(eng->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_forward(eng, sp);
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(eng->stream, &graph);
    if (rc != MS_OK) {
      if (graph) cudaGraphDestroy(graph);
      eng->graphs.pop_back();
      return rc;
    }
    cudaError_t ie = ce;
    if (ie == cudaSuccess) ie = cudaGraphInstantiate(&g->exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
      eng->graphs.pop_back();
      return eng->fail(MS_E_DEVICE, std::string("graph capture: ") + cudaGetErrorString(ie));
    }
    g->launches = eng->last_launches;
    ++eng->graph_captures;
    MS_CUDA_TRY(cudaGraphLaunch(g->exec, eng->stream));
  } else {
    int rc = enqueue_forward(eng, sp);
    if (rc != MS_OK) return rc;
  }
  if (g) g->last_use = ++eng->graph_clock;
  MS_CUDA_TRY(cudaEventRecord(eng->done_ev, eng->stream));

  // ---- commit host state ----
  eng->last_slots.resize(S);
  eng->last_flags.assign(S, 0);
  for (int i = 0; i < S; ++i) {
    RowPlan &r = plan[i];
    eng->last_slots[i] = r.seq->slot;
    if (r.partial) eng->last_flags[i] = MS_FLAG_NO_TOKEN;
    else if (r.prefill) eng->last_flags[i] = MS_FLAG_PREFILLED;
    eng->last_out_flags[r.orig] = eng->last_flags[i];
    r.seq->cached = r.start + r.ntok;
    if (!r.partial) r.seq->prefilled = true;
    r.seq->synced = int(r.seq->blocks.size());
  }
  eng->last_nseq = S;
  eng->last_T = T;
  eng->last_max_ctx = max_ctx;
  eng->pending = true;
  return MS_OK;
}

int step_wait_impl(Engine *eng, uint32_t *out_tokens, uint8_t *out_flags) {
  if (!eng->pending) return eng->fail(MS_E_INVALID, "ms_step_wait without a launched step");
  eng->pending = false;
  const int S = eng->last_nseq, S_in = eng->last_in;
  if (S == 0) {
    for (int i = 0; i < S_in; ++i) {
      if (out_tokens) out_tokens[i] = 0;
      if (out_flags) out_flags[i] = MS_FLAG_NO_TOKEN;
    }
    return MS_OK;
  }
  if (eng->tp > 1) {
    // Host watchdog for the collectives: a peer that died or hangs would
    // otherwise block the step forever.  Poll the step's completion and the
    // communicator's asynchronous error; past the deadline abort the
    // communicator and quarantine the engine.
    static const double timeout_s = [] {
      const char *e = std::getenv("MS_STEP_TIMEOUT_S");
      return e ? std::atof(e) : 120.0;
    }();
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      const cudaError_t q = cudaEventQuery(eng->done_ev);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return eng->fail(MS_E_DEVICE, std::string("step: ") + cudaGetErrorString(q));
      const int ae = nccl_async_error(eng->comm);
      const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if ((ae != 0 && ae != 7 /* ncclInProgress */) || el > timeout_s) {
        nccl_abort(eng->comm);
        return eng->fail(MS_E_DEVICE, ae != 0 ? "NCCL asynchronous error " + std::to_string(ae)
                                              : std::string("step exceeded the collective timeout"));
      }
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }
  MS_CUDA_TRY(cudaEventSynchronize(eng->done_ev));
  if (*eng->h_status != 0)
    return eng->fail(MS_E_DEVICE, "device status word " + std::to_string(*eng->h_status) +
                                      " (1 = bounded wait gave up, 2 = index out of range)");
  for (int i = 0; i < S_in; ++i) {
    const int p = eng->last_map[i];
    const uint8_t f = eng->last_out_flags[i];
    if (out_tokens) out_tokens[i] = (p < 0 || (f & MS_FLAG_NO_TOKEN)) ? 0u : uint32_t(eng->h_next[p]);
    if (out_flags) out_flags[i] = f;
  }
  return MS_OK;
}

}  // namespace ms
