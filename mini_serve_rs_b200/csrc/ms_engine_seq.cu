// Engine sequence lifetime: the scheduler's admit / append / release deltas.
//
// ms_seq_admit mirrors what the reference does when a request first reaches
// the backend (src/scheduler/scheduler.rs:347-369 allocation, then
// src/backends/candle.rs:405-418 model state); ms_seq_append_block mirrors the
// one-ahead growth push (scheduler.rs:422-449); ms_seq_release mirrors
// ModelBackend::cancel_sequence (candle.rs:700-704).  Block ids are the
// scheduler's logical ids (kv_cache.rs) used directly as page ids.
#include <string>

#include "ms_engine.h"

namespace ms {

int seq_admit_impl(Engine *eng, uint64_t id, const uint32_t *prompt, int prompt_len, const int32_t *blocks,
                   int nblocks, int num_cached) {
  if (!eng->healthy) {
    eng->err = "Backend quarantined; restart required";
    return MS_E_QUARANTINED;
  }
  if (eng->pending) return eng->fail(MS_E_INVALID, "sequence change while a step is in flight");
  if (eng->seqs.count(id)) return eng->fail(MS_E_INVALID, "sequence id already admitted");
  if (prompt_len <= 0 || !prompt) return eng->fail(MS_E_TOKEN_LIMIT, "prompt must hold at least one token");
  if (prompt_len > eng->rope_len)
    return eng->fail(MS_E_TOKEN_LIMIT, "Request exceeds model context or has zero tokens");
  if (nblocks < 0 || (nblocks > 0 && !blocks)) return eng->fail(MS_E_INVALID, "bad block list");
  if (nblocks > eng->opts.max_blocks_per_seq) return eng->fail(MS_E_PRESSURE, "block table row full");
  if (num_cached < 0 || num_cached > prompt_len) return eng->fail(MS_E_INVALID, "num_cached out of range");
  if (int64_t(num_cached) > int64_t(nblocks) * eng->opts.block_size)
    return eng->fail(MS_E_INVALID, "cached tokens exceed the given blocks");
  for (int i = 0; i < nblocks; ++i)
    if (blocks[i] < 0 || blocks[i] >= eng->opts.pool_blocks)
      return eng->fail(MS_E_INVALID, "block id " + std::to_string(blocks[i]) + " outside the pool");
  for (int i = 0; i < prompt_len; ++i)
    if (prompt[i] >= uint32_t(eng->V)) return eng->fail(MS_E_INVALID, "prompt token outside the vocabulary");
  if (eng->free_slots.empty()) return eng->fail(MS_E_PRESSURE, "no free sequence slot");
  Seq s;
  s.slot = eng->free_slots.back();
  eng->free_slots.pop_back();
  s.prompt.assign(prompt, prompt + prompt_len);
  s.blocks.assign(blocks, blocks + nblocks);
  s.synced = 0;
  s.cached = num_cached;
  s.prefilled = false;
  eng->seqs.emplace(id, std::move(s));
  return MS_OK;
}

int seq_append_block_impl(Engine *eng, uint64_t id, int32_t block) {
  if (!eng->healthy) {
    eng->err = "Backend quarantined; restart required";
    return MS_E_QUARANTINED;
  }
  if (eng->pending) return eng->fail(MS_E_INVALID, "sequence change while a step is in flight");
  auto it = eng->seqs.find(id);
  if (it == eng->seqs.end()) return eng->fail(MS_E_NOT_FOUND, "unknown sequence id");
  if (block < 0 || block >= eng->opts.pool_blocks) return eng->fail(MS_E_INVALID, "block id outside the pool");
  if (int(it->second.blocks.size()) >= eng->opts.max_blocks_per_seq)
    return eng->fail(MS_E_PRESSURE, "block table row full");
  it->second.blocks.push_back(block);
  return MS_OK;
}

int seq_release_impl(Engine *eng, uint64_t id) {
  if (eng->pending) return eng->fail(MS_E_INVALID, "sequence change while a step is in flight");
  auto it = eng->seqs.find(id);
  if (it == eng->seqs.end()) return MS_OK;  // idempotent, like cancel_sequence
  eng->free_slots.push_back(it->second.slot);
  eng->seqs.erase(it);
  return MS_OK;
}

}  // namespace ms
