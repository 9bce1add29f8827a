"""Restatement of the logical KV block manager (test infrastructure only).

Follows ``src/cache/kv_cache.rs:14-145``: a LIFO free stack initialised so
that pop() yields 0, 1, 2, ...; release pushes a request's blocks back in
allocation order.
"""
from __future__ import annotations

from typing import Dict, List


class CachePressure(Exception):
    """EngineError::CachePressure (src/core/errors.rs:10)."""


class KVCacheRef:
    def __init__(self, total_blocks: int, block_size: int = 16):
        # kv_cache.rs:23-35
        self.total_blocks = total_blocks
        self.block_size = block_size
        self.free_blocks: List[int] = list(range(total_blocks - 1, -1, -1))
        self.allocations: Dict[str, List[int]] = {}

    def free_count(self) -> int:
        return len(self.free_blocks)

    def allocated_count(self) -> int:
        return self.total_blocks - len(self.free_blocks)

    def blocks_needed(self, tokens: int) -> int:
        # kv_cache.rs:53-59
        return 1 if tokens == 0 else -(-tokens // self.block_size)

    def allocate(self, request_id: str, num_tokens: int) -> List[int]:
        # kv_cache.rs:61-84 (replaces any previous allocation under that id)
        needed = self.blocks_needed(num_tokens)
        if needed > len(self.free_blocks):
            raise CachePressure(
                f"Requested {needed} blocks ({num_tokens} tokens), but only "
                f"{len(self.free_blocks)} free blocks remain")
        blocks = [self.free_blocks.pop() for _ in range(needed)]
        self.allocations[request_id] = list(blocks)
        return blocks

    def allocate_block(self, request_id: str) -> int:
        # kv_cache.rs:86-99
        if not self.free_blocks:
            raise CachePressure("KV cache pressure: no free blocks remaining for incremental allocation")
        b = self.free_blocks.pop()
        self.allocations.setdefault(request_id, []).append(b)
        return b

    def release(self, request_id: str) -> int:
        # kv_cache.rs:101-111
        blocks = self.allocations.pop(request_id, None)
        if blocks is None:
            return 0
        self.free_blocks.extend(blocks)
        return len(blocks)

    def stats(self) -> dict:
        # kv_cache.rs:113-144
        free = len(self.free_blocks)
        allocated = self.total_blocks - free
        util = allocated / self.total_blocks if self.total_blocks else 0.0
        fs = set(self.free_blocks)
        runs = sum(1 for i in range(self.total_blocks) if i in fs and (i == 0 or (i - 1) not in fs))
        frag = (runs - 1.0) / free if free > 0 and runs > 1 else 0.0
        return {"total_blocks": self.total_blocks, "allocated_blocks": allocated,
                "free_blocks": free, "utilization": round(util * 1000) / 1000,
                "fragmentation": round(min(frag, 1.0) * 1000) / 1000}
