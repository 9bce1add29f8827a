"""Restatement of the paged prefix cache (test infrastructure only).

`chunk_hashes` restates PrefixCache::compute_chunk_hashes
(src/cache/prefix_cache.rs:103-124) with hashlib: key_i = SHA-256 of the hex
string of key_{i-1} (absent for i = 0) followed by the chunk's tokens as u32
little-endian, rendered as lower-case hex (`hex::encode`).

`PagesRef` restates the page manager of ms_pages.cu.  It combines
KVCache (kv_cache.rs:14-145: LIFO free stack popping 0, 1, 2, ... first,
release pushing a request's blocks back in allocation order) with the
prefix cache's LRU policy (prefix_cache.rs:126-157 lookup refresh,
213-243 eviction under pressure, 319-321 the max_chunks cap).  Chunks are
pages.  It follows the same rules step by step, so a trace of admissions,
growth, publication and release yields the same block ids and counters.

`reserve` restates the admission budget (CandleBackend::reserve_sequence,
candle.rs:349-375, charging through PrefixCache::reserve_memory,
prefix_cache.rs:229-244, against TensorMemoryBudget::try_reserve,
tensor_memory.rs:72-88) with the pool as the budget: a request costs
ceil((prompt + max_tokens) / block_size) pages; reservations plus cache-only
pages must fit the pool, evicting the oldest evictable entries first; a repeat
reservation of the same id is free (candle.rs:361-363).
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict
from typing import Dict, List, Optional, Tuple

from oracle.kv_cache_ref import CachePressure


def chunk_hashes(tokens, chunk_size: int = 16) -> List[str]:
    out: List[str] = []
    prev = ""
    for i in range(len(tokens) // chunk_size):
        h = hashlib.sha256()
        if prev:
            h.update(prev.encode())
        for t in tokens[i * chunk_size:(i + 1) * chunk_size]:
            h.update(int(t).to_bytes(4, "little"))
        prev = h.hexdigest()
        out.append(prev)
    return out


class PagesRef:
    def __init__(self, total_blocks: int, block_size: int = 16, max_chunks: int = 512):
        self.total = total_blocks
        self.bs = block_size
        self.max_chunks = max_chunks
        self.free: List[int] = list(range(total_blocks - 1, -1, -1))
        self.refs = [0] * total_blocks
        self.alloc: Dict[int, List[int]] = {}
        # key -> [page, parent key or None, children]; order = LRU (first = oldest)
        self.chunks: "OrderedDict[str, list]" = OrderedDict()
        self.hits = self.misses = self.tokens_saved = self.evictions = self.rejections = 0
        self.reservations: Dict[int, int] = {}
        self.peak_reserved = self.reservation_rejections = 0

    def blocks_needed(self, tokens: int) -> int:
        return 1 if tokens == 0 else -(-tokens // self.bs)

    def _unref(self, p: int):
        self.refs[p] -= 1
        if self.refs[p] == 0:
            self.free.append(p)

    def _evict_one(self, need_free: bool) -> bool:
        for key, (page, parent, children) in self.chunks.items():
            if children > 0 or (need_free and self.refs[page] != 1):
                continue
            if parent is not None and parent in self.chunks:
                self.chunks[parent][2] -= 1
            self._unref(page)
            del self.chunks[key]
            self.evictions += 1
            return True
        return False

    def _make_free(self, n: int) -> bool:
        while len(self.free) < n:
            if not self._evict_one(True):
                return False
        return True

    def _matched(self, keys: List[str], cap: int) -> List[int]:
        pages = []
        for k in keys[:cap]:
            if k not in self.chunks:
                break
            self.chunks.move_to_end(k)
            pages.append(self.chunks[k][0])
        return pages

    def admit(self, seq: int, prompt) -> Tuple[List[int], int]:
        if seq in self.alloc:
            raise ValueError("sequence already admitted")
        n = len(prompt)
        need = self.blocks_needed(max(n, 1))
        pages: List[int] = []
        if self.max_chunks > 0 and n > 1:
            pages = self._matched(chunk_hashes(prompt, self.bs), (n - 1) // self.bs)
        k = len(pages)
        for p in pages:
            self.refs[p] += 1
        if not self._make_free(need - k):
            for p in pages:
                self._unref(p)
            self.rejections += 1
            raise CachePressure("prefix-cache pages in use; pool exhausted")
        for _ in range(need - k):
            p = self.free.pop()
            self.refs[p] = 1
            pages.append(p)
        if self.max_chunks > 0:
            if k:
                self.hits += 1
                self.tokens_saved += k * self.bs
            else:
                self.misses += 1
        self.alloc[seq] = list(pages)
        return pages, k * self.bs

    def allocate_block(self, seq: int) -> int:
        if seq not in self.alloc:
            raise KeyError(seq)
        if not self._make_free(1):
            self.rejections += 1
            raise CachePressure("KV cache pressure: no free blocks remaining for incremental allocation")
        p = self.free.pop()
        self.refs[p] = 1
        self.alloc[seq].append(p)
        return p

    def _cache_only(self) -> int:
        return sum(1 for v in self.chunks.values() if self.refs[v[0]] == 1)

    def reserve(self, seq: int, prompt_len: int, max_tokens: int):
        if seq in self.reservations:
            return
        if prompt_len <= 0 or max_tokens <= 0:
            raise ValueError("Request exceeds model context or has zero tokens")
        need = -(-(prompt_len + max_tokens) // self.bs)
        while sum(self.reservations.values()) + need + self._cache_only() > self.total:
            if not self._evict_one(True):
                self.reservation_rejections += 1
                raise CachePressure("Tensor memory budget exhausted")
        self.reservations[seq] = need
        self.peak_reserved = max(self.peak_reserved, sum(self.reservations.values()))

    def release(self, seq: int) -> int:
        self.reservations.pop(seq, None)
        pages = self.alloc.pop(seq, None)
        if pages is None:
            return 0
        for p in pages:
            self._unref(p)
        return len(pages)

    def publish(self, seq: int, prompt) -> int:
        if seq not in self.alloc:
            raise KeyError(seq)
        if self.max_chunks <= 0:
            return 0
        keys = chunk_hashes(prompt, self.bs)
        pages = self.alloc[seq]
        added = 0
        for i, key in enumerate(keys[:len(pages)]):
            if key in self.chunks:
                self.chunks.move_to_end(key)
                continue
            while len(self.chunks) >= self.max_chunks:
                if not self._evict_one(False):
                    break
            if len(self.chunks) >= self.max_chunks:
                break
            if i > 0 and keys[i - 1] not in self.chunks:
                break
            parent: Optional[str] = keys[i - 1] if i > 0 else None
            if parent is not None:
                self.chunks[parent][2] += 1
            self.chunks[key] = [pages[i], parent, 0]
            self.refs[pages[i]] += 1
            added += 1
        return added

    def lookup(self, prompt) -> int:
        keys = chunk_hashes(prompt, self.bs)
        return len(self._matched(keys, len(keys))) * self.bs

    def stats(self) -> dict:
        return {"total_blocks": self.total, "free_blocks": len(self.free), "cached_chunks": len(self.chunks),
                "cache_only_blocks": sum(1 for v in self.chunks.values() if self.refs[v[0]] == 1),
                "hits": self.hits, "misses": self.misses, "tokens_saved": self.tokens_saved,
                "evictions": self.evictions, "rejections": self.rejections,
                "reserved_blocks": sum(self.reservations.values()), "peak_reserved_blocks": self.peak_reserved,
                "reservation_rejections": self.reservation_rejections}
