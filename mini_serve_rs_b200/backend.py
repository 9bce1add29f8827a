"""CudaBackend: the reference's backend contract over libms_engine.

Mirrors ``trait ModelBackend`` (src/backends/traits.rs:15-50) as
CandleBackend implements it (src/backends/candle.rs:304-705), with the
forward step running in the sm_100a engine:

* ``reserve_sequence`` -- idempotent per id (candle.rs:349-375): the request's
  worst-case KV pages, ceil((prompt + max_tokens) / 16), are charged against
  the engine's page pool (the B200 path's tensor-memory budget, see
  ``Pages.reserve``); ``CachePressure`` when they do not fit.
* ``step_batch`` -- one token per sequence in input order; sequences not yet
  prefilled get their prompt run and ``is_prefilled`` set (candle.rs:431-433);
  the others decode their last output token.  Block ids come from the
  caller's ``kv_blocks`` (the scheduler's logical KVCache ids); new ones are
  forwarded to the engine as deltas.  A ``BackendError`` quarantines the
  backend and clears all state (candle.rs:689-696).
* ``cancel_sequence`` -- idempotent release (candle.rs:700-704).

Tokenisation, EOS text handling and detokenisation stay with the caller, as
in the reference's Rust shim design; ``eos_ids`` marks EOS tokens.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Set

import numpy as np

from .engine import BackendError, Engine, NoHealthyWorkers, Pages, TokenLimitExceeded


@dataclass
class StepToken:
    """src/backends/traits.rs:6-13 (text is produced by the caller's tokenizer)."""

    token_id: int
    text: str
    is_eos: bool


class CudaBackend:
    def __init__(self, engine: Engine, name: str = "ms-b200", eos_ids: Sequence[int] = (),
                 budget: Pages = None):
        """budget: the reservation ledger; by default one over the engine's
        whole page pool (no prefix cache)."""
        self.engine = engine
        self._name = name
        self.eos: Set[int] = set(int(e) for e in eos_ids)
        self.budget = budget if budget is not None else Pages(int(engine.opts.pool_blocks),
                                                              int(engine.opts.block_size), max_chunks=0)
        self._ids: Dict[str, int] = {}      # request id -> engine sequence id (from its reservation on)
        self._admitted: Set[str] = set()    # requests the engine holds
        self._pushed: Dict[str, int] = {}   # blocks already handed to the engine
        self._reserved: Set[str] = set()
        self._next = 1
        self._healthy = True

    # ---- ModelBackend ------------------------------------------------------------
    def name(self) -> str:
        return self._name

    def is_healthy(self) -> bool:
        return self._healthy and self.engine.is_healthy()

    def mark_unhealthy(self):
        self._healthy = False
        self.engine.mark_unhealthy()
        for sid in self._ids.values():
            self.budget.release(sid)
        self._ids.clear()
        self._admitted.clear()
        self._pushed.clear()
        self._reserved.clear()

    def context_length(self) -> int:
        return int(self.engine.cfg.max_position_embeddings)

    def reserve_sequence(self, request_id: str, prompt_tokens: int, max_tokens: int):
        if not self.is_healthy():
            raise NoHealthyWorkers("Backend quarantined; restart required")
        if request_id in self._reserved:
            return
        if prompt_tokens == 0 or max_tokens == 0 or prompt_tokens + max_tokens > self.context_length():
            raise TokenLimitExceeded("Request exceeds model context or has zero tokens")
        sid = self._ids.get(request_id)
        if sid is None:
            sid = self._next
            self._next += 1
        self.budget.reserve(sid, prompt_tokens, max_tokens)  # CachePressure: nothing is kept
        self._ids[request_id] = sid
        self._reserved.add(request_id)

    def cancel_sequence(self, request_id: str):
        sid = self._ids.pop(request_id, None)
        self._pushed.pop(request_id, None)
        self._reserved.discard(request_id)
        admitted = request_id in self._admitted
        self._admitted.discard(request_id)
        if sid is not None:
            self.budget.release(sid)
            if admitted and self.engine.is_healthy():
                self.engine.release(sid)

    def step_batch(self, sequences: List) -> List[int]:
        """sequences: objects with request_id, prompt_tokens, output_tokens,
        is_prefilled, kv_blocks, max_tokens.  Returns token ids in order."""
        if not sequences:
            return []
        if not self.is_healthy():
            raise NoHealthyWorkers("Backend quarantined; restart required")
        try:
            return self._step(sequences)
        except BackendError:
            self.mark_unhealthy()
            raise

    # ---- internals ---------------------------------------------------------------
    def _step(self, sequences: List) -> List[int]:
        eng = self.engine
        ids = np.zeros(len(sequences), np.uint64)
        toks = np.zeros(len(sequences), np.uint32)
        pos = np.zeros(len(sequences), np.int32)
        for i, s in enumerate(sequences):
            rid = s.request_id
            self.reserve_sequence(rid, len(s.prompt_tokens), s.max_tokens)
            if rid not in self._admitted:
                sid = self._ids[rid]
                eng.admit(sid, s.prompt_tokens, s.kv_blocks, 0)
                self._admitted.add(rid)
                self._pushed[rid] = len(s.kv_blocks)
            else:
                for b in s.kv_blocks[self._pushed[rid]:]:
                    eng.append_block(self._ids[rid], b)
                self._pushed[rid] = len(s.kv_blocks)
            ids[i] = self._ids[rid]
            if s.is_prefilled:
                toks[i] = s.output_tokens[-1] if s.output_tokens else 1
                pos[i] = len(s.prompt_tokens) + len(s.output_tokens) - 1 if s.output_tokens else 0
        out, _ = eng.step(ids, toks, pos)
        result = [int(t) for t in out]
        for s, t in zip(sequences, result):
            s.is_prefilled = True
            if t in self.eos or len(s.output_tokens) + 1 >= s.max_tokens:
                # candle.rs:678-685: finished sequences drop their state
                self.cancel_sequence(s.request_id)
        return result
