"""Restatement of the reference's latency-aware router (test infrastructure:
only tests/ may import this module).

* WorkerHandle::score, src/routing/router.rs:23-30:
  (queue_depth + active_count + 1.0) * avg_latency_ms.max(1.0)
* Router::choose_worker, router.rs:46-52: workers filtered by
  Scheduler::has_capacity (scheduler.rs:577-579: is_healthy() &&
  queue_depth() < max_waiting_requests), then Iterator::min_by on
  f64::total_cmp, which returns the first of equal minima.
* Scheduler::avg_latency_ms, scheduler.rs:114-122: 0.0 for an empty window,
  else (sum_ms / len * 10.0).round() / 10.0 over the VecDeque that keeps the
  last 64 finished requests' durations (scheduler.rs:543-550).
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

# (queue_depth, active_count, avg_latency_ms, healthy, max_waiting)
Metrics = Tuple[int, int, float, bool, int]


def score(queue: int, active: int, latency_ms: float) -> float:
    return (float(queue) + float(active) + 1.0) * max(latency_ms, 1.0)


def choose_worker(workers: Sequence[Metrics]) -> Optional[int]:
    """Index chosen by choose_worker, None for NoHealthyWorkers."""
    best: Optional[int] = None
    for i, (q, a, lat, healthy, max_waiting) in enumerate(workers):
        if not (healthy and q < max_waiting):
            continue
        if best is None or score(q, a, lat) < score(*workers[best][:3]):
            best = i
    return best


def rust_round(x: float) -> float:
    """f64::round: half away from zero (Python's round() is half to even)."""
    return math.copysign(math.floor(abs(x) + 0.5), x)


def avg_latency_ms(finished_ms: List[float]) -> float:
    window = finished_ms[-64:]
    if not window:
        return 0.0
    return rust_round(sum(window) / len(window) * 10.0) / 10.0
