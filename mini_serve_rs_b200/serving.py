"""Continuous-batching serving loop over the engine and the page manager.

The caller side of the hot path, as the reference's Scheduler runs it
(src/scheduler/scheduler.rs):
* FIFO admission while there is room (:312-382).  With reserve=True each
  request first reserves its worst-case pages (reserve_sequence); one whose
  reservation or pages do not fit stays queued until running requests free
  room (with nothing running, a reservation that cannot fit fails the
  request).
* One ragged ms_step per iteration over every active request (:422-449).
* Block growth before a step (:430-431).
* Release when a request finishes (:555) or fails (:446).
It also uses the B200 path's additions: pages from Pages (prefix-cache page
sharing), prompts prefilled in chunks under a per-step token budget, and
decode tokens fed back on the device.  Time is wall-clock; TTFT and
per-request decode rate follow examples/bench.rs:85-108.
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional

from . import engine as E
from .router import LatencyWindow, ReplicaMetrics


@dataclass
class Request:
    rid: int
    prompt: List[int]
    max_tokens: int
    arrival: float = 0.0          # seconds from the start of the trace
    temperature: float = 0.0
    top_p: float = 1.0
    seed: int = 0
    # filled in while serving
    blocks: List[int] = field(default_factory=list)
    cached: int = 0
    prefilled: bool = False
    out: List[int] = field(default_factory=list)
    admitted_at: Optional[float] = None
    first_token_at: Optional[float] = None
    last_token_at: Optional[float] = None
    done_at: Optional[float] = None
    error: Optional[str] = None


class ServingLoop:
    def __init__(self, eng: E.Engine, pages: E.Pages, max_active: int = 256, token_budget: int = 2048,
                 block_size: int = 16, reserve: bool = False):
        """reserve: admit a request only once its worst-case pages (prompt +
        max_tokens) are reserved (reserve_sequence's budget, scheduler.rs:325-343);
        off, pages are taken as the request grows and a pool that runs dry
        fails the growing request (scheduler.rs:430-446)."""
        self.eng = eng
        self.pages = pages
        self.reserve = reserve
        self.max_active = max_active
        self.token_budget = token_budget
        self.bs = block_size
        self.queue: Deque[Request] = deque()
        self.active: List[Request] = []
        self.finished: List[Request] = []
        self.steps = 0
        self.engine_s = 0.0  # wall time inside the engine's step call (launch + device work + wait)
        self.host_s = 0.0    # wall time of the rest of step(): admission, page growth, bookkeeping
        self.latency = LatencyWindow()  # scheduler.rs:543-550, read by the router

    def submit(self, r: Request):
        self.queue.append(r)

    def _admit(self, now: float):
        while self.queue and self.queue[0].arrival <= now and len(self.active) < self.max_active:
            r = self.queue[0]
            # reserve_sequence before the first forward (scheduler.rs:325-343): the request's
            # worst-case pages; while they do not fit it waits for running requests to finish,
            # and fails (as the reference's admission does) when nothing is running
            if self.reserve:
                try:
                    self.pages.reserve(r.rid, len(r.prompt), r.max_tokens)
                except E.EngineError as e:
                    if isinstance(e, E.CachePressure) and self.active:
                        break
                    self.queue.popleft()
                    r.error = str(e)
                    r.done_at = now
                    self.finished.append(r)
                    continue
            try:
                r.blocks, r.cached = self.pages.admit(r.rid, r.prompt)
            except E.CachePressure:
                break
            try:
                self.eng.admit(r.rid, r.prompt, r.blocks, num_cached=r.cached)
            except E.EngineError as e:
                self.pages.release(r.rid)
                self.queue.popleft()
                r.error = str(e)
                self.finished.append(r)
                continue
            r.admitted_at = now
            self.queue.popleft()
            self.active.append(r)

    def _finish(self, r: Request, now: float, error: Optional[str] = None):
        self.eng.release(r.rid)
        self.pages.release(r.rid)
        r.done_at = now
        r.error = error
        if error is None:
            self.latency.add((now - r.arrival) * 1000.0)
        self.finished.append(r)

    def metrics(self) -> ReplicaMetrics:
        """What the router reads (scheduler.rs:128-135): waiting requests that
        have arrived, active requests, mean latency of the last 64 finished."""
        now = self.clock()
        waiting = sum(1 for r in self.queue if r.arrival <= now)
        return ReplicaMetrics(queue_depth=waiting, active_count=len(self.active),
                              avg_latency_ms=self.latency.avg_ms(), healthy=self.eng.is_healthy())

    def _grow(self, now: float):
        failed = []
        for r in self.active:
            if r.prefilled:
                # the cache holds the prompt and every generated token but the last (the next
                # input): no engine call per decoding request per step
                reach = len(r.prompt) + len(r.out)
            else:
                c = self.eng.cached_tokens(r.rid)
                rem = len(r.prompt) - c
                reach = c + (min(rem, self.token_budget) if self.token_budget else rem)
            try:
                while len(r.blocks) * self.bs < reach:
                    b = self.pages.allocate_block(r.rid)
                    r.blocks.append(b)
                    self.eng.append_block(r.rid, b)
            except E.CachePressure as e:
                failed.append((r, str(e)))
        for r, msg in failed:  # scheduler.rs:430-446: the request fails
            self.active.remove(r)
            self._finish(r, now, msg)

    def step(self, now: float) -> bool:
        """One iteration at trace time `now`; False when there was nothing to run."""
        t_in = time.perf_counter()
        self._admit(now)
        if not self.active:
            return False
        self._grow(now)
        if not self.active:
            return False
        ids = [r.rid for r in self.active]
        temps = [r.temperature for r in self.active]
        need_sampling = any(t >= 1e-7 for t in temps)
        t_eng = time.perf_counter()
        toks, flags = self.eng.step(
            ids, flags=E.MS_STEP_TOKENS_FROM_DEVICE, token_budget=self.token_budget,
            temperature=temps if need_sampling else None,
            top_p=[r.top_p for r in self.active] if need_sampling else None,
            seeds=[(r.seed << 20) + len(r.out) for r in self.active] if need_sampling else None)
        t_out = time.perf_counter()
        self.engine_s += t_out - t_eng
        self.steps += 1
        t = self.clock()
        done = []
        for r, tok, f in zip(self.active, toks, flags):
            if f & E.MS_FLAG_NO_TOKEN:
                continue
            if f & E.MS_FLAG_PREFILLED:
                r.prefilled = True
                r.first_token_at = t
                self.pages.publish(r.rid, r.prompt)
            r.out.append(int(tok))
            r.last_token_at = t
            if len(r.out) >= r.max_tokens:
                done.append(r)
        for r in done:
            self.active.remove(r)
            self._finish(r, t)
        self.host_s += (t_eng - t_in) + (time.perf_counter() - t_out)
        return True

    # trace clock: seconds since run() started
    def clock(self) -> float:
        return time.perf_counter() - self._t0

    def run(self, requests: List[Request], timeout_s: float = 600.0) -> float:
        """Serve a trace in real time; returns the elapsed seconds."""
        for r in sorted(requests, key=lambda r: r.arrival):
            self.submit(r)
        self._t0 = time.perf_counter()
        while self.queue or self.active:
            now = self.clock()
            if now > timeout_s:
                raise TimeoutError("trace did not finish")
            if not self.step(now):
                nxt = self.queue[0].arrival if self.queue else now
                time.sleep(max(0.0, min(nxt - now, 0.01)))
        return self.clock()

    def run_routed(self, link, requests: Dict[int, Request], timeout_s: float = 600.0) -> float:
        """Serve the requests a Dispatcher routes to this replica (`link` is
        its ReplicaLink; `requests` maps request id -> Request, with arrival
        times on the dispatcher's clock).  The metrics go out after every step
        and while idle.  Returns the elapsed seconds on the shared clock."""
        t0_wall = link.start_time()
        # clock() = wall-clock seconds since the dispatcher's t0, on this process's perf counter
        self._t0 = time.perf_counter() - (time.time() - t0_wall)
        last = None
        while True:
            for rid in link.poll():
                self.submit(requests[rid])
            now = self.clock()
            if now > timeout_s:
                raise TimeoutError("trace did not finish")
            ran = self.step(now)
            m = self.metrics()
            key = (m.queue_depth, m.active_count, m.avg_latency_ms, m.healthy, link.got)
            if key != last:  # only changes go to the store
                link.publish(m)
                last = key
            if ran:
                continue
            if not self.queue and not self.active and link.finished():
                late = link.poll()  # assigned between the last poll and the done mark
                if not late:
                    break
                for rid in late:
                    self.submit(requests[rid])
                continue
            time.sleep(0.001)
        return self.clock()


def summarize(reqs: List[Request], elapsed: float) -> Dict[str, float]:
    """Aggregate tokens/s and TTFT percentiles (examples/bench.rs:85-108, 189)."""
    ok = [r for r in reqs if r.error is None]
    tokens = sum(len(r.out) for r in ok)
    ttft = sorted((r.first_token_at - r.arrival) * 1000.0 for r in ok if r.first_token_at is not None)
    dec = [(len(r.out) - 1) / (r.last_token_at - r.first_token_at) for r in ok
           if len(r.out) > 1 and r.last_token_at > r.first_token_at]

    def pct(v, q):
        return v[min(len(v) - 1, int(q * len(v)))] if v else float("nan")

    return {"requests": len(reqs), "failed": len(reqs) - len(ok), "tokens": tokens, "elapsed_s": elapsed,
            "aggregate_tokens_per_s": tokens / elapsed if elapsed > 0 else 0.0,
            "ttft_ms_p50": pct(ttft, 0.5), "ttft_ms_p90": pct(ttft, 0.9), "ttft_ms_p99": pct(ttft, 0.99),
            "ttft_ms_all": ttft,
            "per_request_decode_tokens_per_s_median": pct(sorted(dec), 0.5)}
