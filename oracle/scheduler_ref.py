"""Restatement of the continuous-batching iteration (test infrastructure only).

Follows ``src/scheduler/scheduler.rs:298-559`` for the parts that decide
which sequences run in a step, in what order, and with which logical KV
blocks: admission (``:312-382``, ``cache.allocate(id, max(prompt, 1))``),
cancellation sweep (``:401-415``), one-ahead block growth (``:422-449``),
``step_batch`` (``:456``), demux (``:472-518``) and eviction with
``swap_remove`` (``:520-559``).  Streaming, stop strings, telemetry and
drain logic are out of scope.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Set

from .kv_cache_ref import CachePressure, KVCacheRef
from .qwen_ref import RefSequence


@dataclass
class Request:
    request_id: str
    prompt_tokens: List[int]
    max_tokens: int


@dataclass
class StepRecord:
    """What one step_batch call saw: order, prefill flags and block tables."""

    request_ids: List[str]
    prefill: List[bool]
    kv_blocks: List[List[int]]
    prompt_lens: List[int]
    num_outputs: List[int]
    tokens: List[int] = field(default_factory=list)


def swap_remove(xs: list, i: int):
    """Rust Vec::swap_remove."""
    item = xs[i]
    last = xs.pop()
    if i < len(xs):
        xs[i] = last
    return item


class SchedulerRef:
    def __init__(self, cache: KVCacheRef, step_batch: Callable[[List[RefSequence]], List[int]],
                 cancel: Callable[[str], None] = lambda rid: None, max_batch_size: int = 8,
                 eos_ids: Set[int] = frozenset()):
        self.cache = cache
        self.step_batch = step_batch
        self.cancel = cancel
        self.max_batch_size = max_batch_size
        self.eos = set(eos_ids)
        self.queue: Deque[Request] = deque()
        self.active: List[RefSequence] = []
        self.finished: Dict[str, List[int]] = {}
        self.errors: Dict[str, str] = {}
        self.cancelled: Set[str] = set()
        self.records: List[StepRecord] = []

    def submit(self, req: Request):
        self.queue.append(req)

    def iteration(self) -> Optional[StepRecord]:
        # admission (scheduler.rs:312-382)
        while len(self.active) < self.max_batch_size and self.queue:
            item = self.queue.popleft()
            try:
                blocks = self.cache.allocate(item.request_id, max(len(item.prompt_tokens), 1))
            except CachePressure as e:
                self.cancel(item.request_id)
                self.errors[item.request_id] = str(e)
                continue
            self.active.append(RefSequence(item.request_id, list(item.prompt_tokens),
                                           item.max_tokens, kv_blocks=blocks))
        if not self.active:
            return None
        # cancellation sweep (scheduler.rs:401-415)
        i = 0
        while i < len(self.active):
            if self.active[i].request_id in self.cancelled:
                c = swap_remove(self.active, i)
                self.cancel(c.request_id)
                self.cache.release(c.request_id)
            else:
                i += 1
        if not self.active:
            return None
        # one-ahead growth (scheduler.rs:422-449)
        i = 0
        while i < len(self.active):
            s = self.active[i]
            next_len = len(s.prompt_tokens) + len(s.output_tokens) + 1
            if self.cache.blocks_needed(next_len) > len(s.kv_blocks):
                try:
                    s.kv_blocks.append(self.cache.allocate_block(s.request_id))
                    i += 1
                except CachePressure as e:
                    f = swap_remove(self.active, i)
                    self.errors[f.request_id] = str(e)
                    self.cancel(f.request_id)
                    self.cache.release(f.request_id)
            else:
                i += 1
        if not self.active:
            return None
        rec = StepRecord([s.request_id for s in self.active],
                         [not s.is_prefilled for s in self.active],
                         [list(s.kv_blocks) for s in self.active],
                         [len(s.prompt_tokens) for s in self.active],
                         [len(s.output_tokens) for s in self.active])
        toks = self.step_batch(self.active)
        rec.tokens = list(toks)
        self.records.append(rec)
        # demux (scheduler.rs:472-518)
        done = []
        for s, t in zip(self.active, toks):
            s.is_prefilled = True
            s.output_tokens.append(int(t))
            hit_max = len(s.output_tokens) >= s.max_tokens
            done.append(int(t) in self.eos or hit_max)
        fin = {s.request_id for s, d in zip(self.active, done) if d}
        # eviction (scheduler.rs:520-559)
        j = 0
        while j < len(self.active):
            if self.active[j].request_id in fin:
                f = swap_remove(self.active, j)
                self.finished[f.request_id] = list(f.output_tokens)
                self.cancel(f.request_id)
                self.cache.release(f.request_id)
            else:
                j += 1
        return rec

    def run(self, max_iters: int = 100000) -> Dict[str, List[int]]:
        for _ in range(max_iters):
            if self.iteration() is None and not self.queue:
                break
        return self.finished
