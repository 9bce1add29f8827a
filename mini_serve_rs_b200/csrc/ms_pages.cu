// Paged prefix cache: the reference's logical block manager
// (src/cache/kv_cache.rs:14-145) and its prefix cache
// (src/cache/prefix_cache.rs:57-345) as one host-side page manager.
//
// The reference stores, for each cached 16-token chunk, an owned copy of the
// whole prefix's K/V (every layer, all tokens up to the chunk end) plus the
// last logits, charged to a byte budget (tensor_memory.rs:72-111), and a hit
// copies that snapshot into the request's contiguous cache
// (candle.rs:436-574).  Here a chunk is exactly one page of the paged pool
// (chunk size == block size == 16), so a cached chunk IS the page that holds
// its K/V for every layer: a hit shares the pages (reference counts, no
// copy), and the pool itself is the memory budget.
//
// * Chain keys follow PrefixCache::compute_chunk_hashes (prefix_cache.rs:
//   103-124): key_i = SHA-256(hex(key_{i-1}) || tokens of chunk i as u32 LE),
//   hex in lower case; only full chunks get keys.
// * admit (Scheduler allocate, scheduler.rs:347-369, + lookup_kv): the prompt's
//   leading cached chunks are shared, capped so that at least the last prompt
//   token is computed (the reference's exact-hit replay, candle.rs:447-455);
//   fresh pages cover the rest of max(prompt_len, 1) tokens, popped from the
//   LIFO free stack (kv_cache.rs:23-35, 61-84).  All or nothing: when the
//   stack runs short, least recently used cached chunks that no sequence
//   holds are evicted (reserve_memory, prefix_cache.rs:227-243); if that is
//   not enough the request gets CachePressure and nothing changes.
// * publish (insert_kv after a prefill, candle.rs:552-573): the sequence's
//   full prompt chunks enter the cache as its own pages (the cache takes a
//   reference).  These pages are never written again: later tokens of the
//   sequence go to later pages.
// * Eviction removes the least recently used chunk that has no cached child,
//   so a cached chain never loses an inner link (a page holds only its own
//   16 tokens, unlike the reference's full-prefix snapshots); the cap of
//   max_chunks entries (prefix_cache.rs:319-321) evicts the same way.
// * release (kv_cache.rs:101-111) drops the sequence's references and pushes
//   pages nobody holds back in allocation order.
// With max_chunks = 0 it hands out exactly the block ids KVCache hands out.
#include <algorithm>
#include <array>
#include <cstdint>
#include <cstring>
#include <list>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "ms_internal.h"

namespace ms {
namespace {

// ---- SHA-256 (FIPS 180-4) ------------------------------------------------------
constexpr uint32_t kK[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

class Sha256 {
 public:
  void update(const uint8_t *p, size_t n) {
    len_ += n;
    while (n) {
      const size_t take = std::min(n, size_t(64) - fill_);
      std::memcpy(buf_ + fill_, p, take);
      fill_ += take;
      p += take;
      n -= take;
      if (fill_ == 64) {
        block(buf_);
        fill_ = 0;
      }
    }
  }
  std::array<uint8_t, 32> finish() {
    const uint64_t bits = len_ * 8;
    const uint8_t pad = 0x80;
    update(&pad, 1);
    const uint8_t zero = 0;
    while (fill_ != 56) update(&zero, 1);
    uint8_t lb[8];
    for (int i = 0; i < 8; ++i) lb[i] = uint8_t(bits >> (56 - 8 * i));
    update(lb, 8);
    std::array<uint8_t, 32> out;
    for (int i = 0; i < 8; ++i)
      for (int b = 0; b < 4; ++b) out[4 * i + b] = uint8_t(h_[i] >> (24 - 8 * b));
    return out;
  }

 private:
  void block(const uint8_t *p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t(p[4 * i]) << 24) | (uint32_t(p[4 * i + 1]) << 16) | (uint32_t(p[4 * i + 2]) << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + kK[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d; h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
  }
  uint32_t h_[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  uint8_t buf_[64];
  size_t fill_ = 0;
  uint64_t len_ = 0;
};

using Key = std::array<uint8_t, 32>;
struct KeyHash {
  size_t operator()(const Key &k) const {
    size_t v;
    std::memcpy(&v, k.data(), sizeof(v));
    return v;
  }
};

// Chain keys of the full chunks of tokens[0..n) (prefix_cache.rs:103-124).
std::vector<Key> chain_keys(const uint32_t *tokens, int n, int chunk) {
  static const char *hexd = "0123456789abcdef";
  std::vector<Key> keys;
  const int nchunks = chunk > 0 ? n / chunk : 0;
  keys.reserve(nchunks);
  for (int i = 0; i < nchunks; ++i) {
    Sha256 s;
    if (i > 0) {
      char hex[64];
      for (int b = 0; b < 32; ++b) {
        hex[2 * b] = hexd[keys.back()[b] >> 4];
        hex[2 * b + 1] = hexd[keys.back()[b] & 15];
      }
      s.update(reinterpret_cast<const uint8_t *>(hex), 64);
    }
    for (int t = 0; t < chunk; ++t) {
      const uint32_t v = tokens[i * chunk + t];
      const uint8_t le[4] = {uint8_t(v), uint8_t(v >> 8), uint8_t(v >> 16), uint8_t(v >> 24)};
      s.update(le, 4);
    }
    keys.push_back(s.finish());
  }
  return keys;
}

}  // namespace

struct PageManager {
  int64_t total = 0;
  int bs = 16;
  int max_chunks = 0;
  std::mutex mu;
  std::vector<int32_t> free_stack;  // pop from the back: 0, 1, 2, ... initially
  std::vector<int32_t> refs;        // holders per page (sequences + the cache)
  std::unordered_map<uint64_t, std::vector<int32_t>> alloc;
  struct Chunk {
    int32_t page;
    bool has_parent;
    Key parent;
    int children;
    std::list<Key>::iterator lru;
  };
  std::unordered_map<Key, Chunk, KeyHash> chunks;
  std::list<Key> lru;  // front: least recently used
  std::unordered_map<uint64_t, int64_t> reservations;  // seq -> worst-case pages
  int64_t reserved = 0;
  ms_pages_stats st{};

  int64_t blocks_needed(int64_t tokens) const { return tokens == 0 ? 1 : (tokens + bs - 1) / bs; }

  void touch(Chunk &c) { lru.splice(lru.end(), lru, c.lru); }

  void unref(int32_t page) {
    if (--refs[page] == 0) free_stack.push_back(page);
  }

  // Evicts the least recently used chunk without a cached child; with
  // need_free, only a chunk whose page nobody else holds (so a page is freed).
  bool evict_one(bool need_free) {
    for (auto it = lru.begin(); it != lru.end(); ++it) {
      auto c = chunks.find(*it);
      if (c->second.children > 0) continue;
      if (need_free && refs[c->second.page] != 1) continue;
      if (c->second.has_parent) {
        auto p = chunks.find(c->second.parent);
        if (p != chunks.end()) --p->second.children;
      }
      unref(c->second.page);
      lru.erase(it);
      chunks.erase(c);
      ++st.evictions;
      return true;
    }
    return false;
  }

  int64_t cache_only() const {
    int64_t n = 0;
    for (const auto &kv : chunks) n += refs[kv.second.page] == 1;
    return n;
  }

  bool make_free(int64_t n) {
    while (int64_t(free_stack.size()) < n)
      if (!evict_one(true)) return false;
    return true;
  }

  // Leading cached chunks of the prompt (refreshes them), at most cap.
  int matched_chunks(const std::vector<Key> &keys, int cap, std::vector<int32_t> *pages) {
    int k = 0;
    for (; k < int(keys.size()) && k < cap; ++k) {
      auto c = chunks.find(keys[k]);
      if (c == chunks.end()) break;
      touch(c->second);
      if (pages) pages->push_back(c->second.page);
    }
    return k;
  }
};

}  // namespace ms

struct ms_pages : ms::PageManager {};

extern "C" int ms_prefix_chunk_hashes(const uint32_t *tokens, int32_t num_tokens, int32_t chunk_size,
                                      uint8_t *out, int32_t capacity) {
  if ((!tokens && num_tokens > 0) || num_tokens < 0 || chunk_size <= 0) return -1;
  const auto keys = ms::chain_keys(tokens, num_tokens, chunk_size);
  if (int32_t(keys.size()) > capacity) return -1;
  for (size_t i = 0; i < keys.size(); ++i) std::memcpy(out + 32 * i, keys[i].data(), 32);
  return int32_t(keys.size());
}

extern "C" int ms_pages_create(int64_t total_blocks, int32_t block_size, int32_t max_chunks, ms_pages **out) {
  if (!out || total_blocks <= 0 || total_blocks > INT32_MAX || block_size <= 0 || max_chunks < 0) return MS_E_INVALID;
  auto *pm = new (std::nothrow) ms_pages();
  if (!pm) return MS_E_DEVICE;
  pm->total = total_blocks;
  pm->bs = block_size;
  pm->max_chunks = max_chunks;
  pm->refs.assign(size_t(total_blocks), 0);
  pm->free_stack.reserve(size_t(total_blocks));
  for (int64_t i = total_blocks - 1; i >= 0; --i) pm->free_stack.push_back(int32_t(i));
  pm->st.total_blocks = total_blocks;
  *out = pm;
  return MS_OK;
}

extern "C" int ms_pages_destroy(ms_pages *pm) {
  delete pm;
  return MS_OK;
}

extern "C" int ms_pages_admit(ms_pages *pm, uint64_t seq_id, const uint32_t *prompt, int32_t prompt_len,
                              int32_t *blocks_out, int32_t capacity, int32_t *num_blocks_out,
                              int32_t *cached_tokens_out) {
  if (!pm || prompt_len < 0 || (prompt_len > 0 && !prompt) || !blocks_out || !num_blocks_out) return MS_E_INVALID;
  std::lock_guard<std::mutex> lk(pm->mu);
  if (pm->alloc.count(seq_id)) return MS_E_INVALID;
  const int64_t need = pm->blocks_needed(prompt_len > 0 ? prompt_len : 1);
  if (need > capacity) return MS_E_INVALID;
  std::vector<int32_t> pages;
  int k = 0;
  if (pm->max_chunks > 0 && prompt_len > 1) {
    const auto keys = ms::chain_keys(prompt, prompt_len, pm->bs);
    k = pm->matched_chunks(keys, (prompt_len - 1) / pm->bs, &pages);
  }
  for (int32_t p : pages) ++pm->refs[p];  // hold them while evicting for the rest
  const int64_t fresh = need - k;
  if (!pm->make_free(fresh)) {
    for (int32_t p : pages) pm->unref(p);
    ++pm->st.rejections;
    return MS_E_PRESSURE;
  }
  for (int64_t i = 0; i < fresh; ++i) {
    const int32_t p = pm->free_stack.back();
    pm->free_stack.pop_back();
    pm->refs[p] = 1;
    pages.push_back(p);
  }
  // record_reuse (prefix_cache.rs:359-367): a hit skips k full chunks
  if (pm->max_chunks > 0) {
    if (k > 0) {
      ++pm->st.hits;
      pm->st.tokens_saved += int64_t(k) * pm->bs;
    } else {
      ++pm->st.misses;
    }
  }
  std::memcpy(blocks_out, pages.data(), pages.size() * sizeof(int32_t));
  *num_blocks_out = int32_t(pages.size());
  if (cached_tokens_out) *cached_tokens_out = k * pm->bs;
  pm->alloc.emplace(seq_id, std::move(pages));
  return MS_OK;
}

extern "C" int ms_pages_allocate_block(ms_pages *pm, uint64_t seq_id, int32_t *block_out) {
  if (!pm || !block_out) return MS_E_INVALID;
  std::lock_guard<std::mutex> lk(pm->mu);
  auto it = pm->alloc.find(seq_id);
  if (it == pm->alloc.end()) return MS_E_NOT_FOUND;
  if (!pm->make_free(1)) {
    ++pm->st.rejections;
    return MS_E_PRESSURE;
  }
  const int32_t p = pm->free_stack.back();
  pm->free_stack.pop_back();
  pm->refs[p] = 1;
  it->second.push_back(p);
  *block_out = p;
  return MS_OK;
}

extern "C" int ms_pages_reserve(ms_pages *pm, uint64_t seq_id, int64_t prompt_len, int64_t max_tokens) {
  if (!pm) return MS_E_INVALID;
  std::lock_guard<std::mutex> lk(pm->mu);
  if (pm->reservations.count(seq_id)) return MS_OK;
  if (prompt_len <= 0 || max_tokens <= 0 || prompt_len > INT32_MAX || max_tokens > INT32_MAX) return MS_E_TOKEN_LIMIT;
  const int64_t need = (prompt_len + max_tokens + pm->bs - 1) / pm->bs;
  // prefix_cache.rs:229-244: evict cached entries until the charge fits
  int64_t only = pm->cache_only();
  while (pm->reserved + need + only > pm->total) {
    if (!pm->evict_one(true)) {
      ++pm->st.reservation_rejections;
      return MS_E_PRESSURE;
    }
    --only;
  }
  pm->reservations.emplace(seq_id, need);
  pm->reserved += need;
  pm->st.peak_reserved_blocks = std::max(pm->st.peak_reserved_blocks, pm->reserved);
  return MS_OK;
}

extern "C" int ms_pages_release(ms_pages *pm, uint64_t seq_id, int32_t *released_out) {
  if (!pm) return MS_E_INVALID;
  std::lock_guard<std::mutex> lk(pm->mu);
  auto rv = pm->reservations.find(seq_id);
  if (rv != pm->reservations.end()) {
    pm->reserved -= rv->second;
    pm->reservations.erase(rv);
  }
  auto it = pm->alloc.find(seq_id);
  int32_t n = 0;
  if (it != pm->alloc.end()) {
    for (int32_t p : it->second) pm->unref(p);
    n = int32_t(it->second.size());
    pm->alloc.erase(it);
  }
  if (released_out) *released_out = n;
  return MS_OK;
}

extern "C" int ms_pages_publish(ms_pages *pm, uint64_t seq_id, const uint32_t *prompt, int32_t prompt_len,
                                int32_t *published_out) {
  if (!pm || prompt_len < 0 || (prompt_len > 0 && !prompt)) return MS_E_INVALID;
  std::lock_guard<std::mutex> lk(pm->mu);
  auto it = pm->alloc.find(seq_id);
  if (it == pm->alloc.end()) return MS_E_NOT_FOUND;
  int32_t added = 0;
  if (pm->max_chunks > 0) {
    const auto keys = ms::chain_keys(prompt, prompt_len, pm->bs);
    const auto &pages = it->second;
    for (size_t i = 0; i < keys.size() && i < pages.size(); ++i) {
      auto c = pm->chunks.find(keys[i]);
      if (c != pm->chunks.end()) {  // already cached (possibly the page this sequence shares)
        pm->touch(c->second);
        continue;
      }
      while (int(pm->chunks.size()) >= pm->max_chunks)
        if (!pm->evict_one(false)) break;
      if (int(pm->chunks.size()) >= pm->max_chunks) break;
      if (i > 0 && !pm->chunks.count(keys[i - 1])) break;  // parent evicted to make room: chain ends
      ms::PageManager::Chunk ch;
      ch.page = pages[i];
      ch.has_parent = i > 0;
      if (i > 0) {
        ch.parent = keys[i - 1];
        ++pm->chunks[keys[i - 1]].children;
      }
      ch.children = 0;
      pm->lru.push_back(keys[i]);
      ch.lru = std::prev(pm->lru.end());
      pm->chunks.emplace(keys[i], ch);
      ++pm->refs[pages[i]];
      ++added;
    }
  }
  if (published_out) *published_out = added;
  return MS_OK;
}

extern "C" int ms_pages_lookup(ms_pages *pm, const uint32_t *prompt, int32_t prompt_len, int32_t *matched_tokens) {
  if (!pm || prompt_len < 0 || (prompt_len > 0 && !prompt) || !matched_tokens) return MS_E_INVALID;
  std::lock_guard<std::mutex> lk(pm->mu);
  const auto keys = ms::chain_keys(prompt, prompt_len, pm->bs);
  *matched_tokens = pm->matched_chunks(keys, int(keys.size()), nullptr) * pm->bs;
  return MS_OK;
}

extern "C" int ms_pages_stats_get(ms_pages *pm, ms_pages_stats *out) {
  if (!pm || !out) return MS_E_INVALID;
  std::lock_guard<std::mutex> lk(pm->mu);
  ms_pages_stats s = pm->st;
  s.free_blocks = int64_t(pm->free_stack.size());
  s.cached_chunks = int64_t(pm->chunks.size());
  int64_t only = 0;
  for (const auto &kv : pm->chunks) only += pm->refs[kv.second.page] == 1;
  s.cache_only_blocks = only;
  s.reserved_blocks = pm->reserved;
  *out = s;
  return MS_OK;
}
