"""Latency-aware routing of requests over data-parallel replicas.

The reference's Router (src/routing/router.rs) sends each request to the
worker with the lowest score among those with capacity:

* score = (queue_depth + active_count + 1) x max(avg_latency_ms, 1)
  (router.rs:23-30);
* capacity = healthy and queue_depth < max_waiting_requests
  (scheduler.rs:577-579; default 256, constants.rs);
* the first such worker wins a tie (router.rs:46-52, Iterator::min_by);
* avg_latency_ms = mean over the last 64 finished requests of the time from
  enqueue to finish, rounded to 0.1 ms, 0 before the first one
  (scheduler.rs:114-122, 543-550).

The reference reads each worker's metrics from atomics in one process.  Here
each replica is its own process (one per GPU), so every replica publishes its
metrics into a key-value store (torch.distributed's TCPStore) once per serving
step, and one dispatcher thread on rank 0 routes every request at its arrival
time.  A metric record can lag its replica by one step; the dispatcher adds the
requests it has sent that the replica has not yet reported receiving to that
replica's queue depth, so its own assignments are never missed.
"""
from __future__ import annotations

import json
import math
import threading
import time
from collections import deque
from dataclasses import dataclass
from typing import Deque, Dict, List, Optional, Sequence

MAX_WAITING_REQUESTS = 256   # src/core/constants.rs DEFAULT_MAX_WAITING_REQUESTS
LATENCY_WINDOW = 64          # scheduler.rs:546-549


class NoHealthyWorkers(RuntimeError):
    """router.rs:51: no replica is healthy with room in its queue."""


@dataclass
class ReplicaMetrics:
    queue_depth: int = 0
    active_count: int = 0
    avg_latency_ms: float = 0.0
    healthy: bool = True
    max_waiting: int = MAX_WAITING_REQUESTS
    received: int = 0   # assignments this replica has taken from the store

    def has_capacity(self) -> bool:
        return self.healthy and self.queue_depth < self.max_waiting

    def score(self) -> float:
        return (self.queue_depth + self.active_count + 1.0) * max(self.avg_latency_ms, 1.0)


def choose(metrics: Sequence[ReplicaMetrics]) -> int:
    """Index of the replica the request goes to: the lowest score among
    replicas with capacity, the first one on a tie."""
    best, best_score = -1, 0.0
    for i, m in enumerate(metrics):
        if not m.has_capacity():
            continue
        s = m.score()
        if best < 0 or s < best_score:
            best, best_score = i, s
    if best < 0:
        raise NoHealthyWorkers("No ready execution paths")
    return best


class LatencyWindow:
    """Enqueue-to-finish latencies of the last 64 finished requests."""

    def __init__(self, size: int = LATENCY_WINDOW):
        self.v: Deque[float] = deque(maxlen=size)

    def add(self, ms: float):
        self.v.append(ms)

    def avg_ms(self) -> float:
        if not self.v:
            return 0.0
        # f64::round rounds half away from zero (latencies are >= 0)
        return math.floor(sum(self.v) / len(self.v) * 10.0 + 0.5) / 10.0


# ---- the store protocol -----------------------------------------------------
# keys (all under the store the caller passes, e.g. a PrefixStore):
#   m/<r>     replica r's metrics, JSON
#   n/<r>     number of requests assigned to replica r (a counter)
#   a/<r>/<k> the k-th request id assigned to replica r
#   t0        the trace's start time (wall clock, seconds), set by rank 0
#   done      set when every request of the trace has been assigned


class ReplicaLink:
    """One replica's side: publishes its metrics and takes its assignments."""

    def __init__(self, store, rank: int):
        self.store = store
        self.rank = rank
        self.got = 0

    def publish(self, m: ReplicaMetrics):
        m.received = self.got
        self.store.set(f"m/{self.rank}", json.dumps(m.__dict__))

    def poll(self) -> List[int]:
        """Request ids assigned since the last poll, in assignment order."""
        n = int(self.store.add(f"n/{self.rank}", 0))
        out = []
        while self.got < n:
            out.append(int(self.store.get(f"a/{self.rank}/{self.got}")))
            self.got += 1
        return out

    def finished(self) -> bool:
        """True once the dispatcher has assigned the whole trace."""
        return self.store.check(["done"])

    def start_time(self, timeout_s: float = 60.0) -> float:
        end = time.time() + timeout_s
        while not self.store.check(["t0"]):
            if time.time() > end:
                raise TimeoutError("dispatcher did not publish the start time")
            time.sleep(0.001)
        return float(self.store.get("t0"))


class Dispatcher:
    """Routes a trace over `world` replicas at the requests' arrival times
    (seconds after t0).  `choices[k]` is the replica of the k-th request in
    arrival order and `snapshots[k]` the metrics that decided it."""

    def __init__(self, store, world: int, arrivals: Sequence, keep_snapshots: bool = False):
        self.store = store
        self.world = world
        self.reqs = sorted(arrivals, key=lambda r: r.arrival)
        self.sent = [0] * world
        self.choices: List[int] = []
        self.snapshots: Optional[List[List[ReplicaMetrics]]] = [] if keep_snapshots else None
        self.failed: List[int] = []
        self.error: Optional[BaseException] = None
        self.thread: Optional[threading.Thread] = None
        self.t0 = 0.0

    def metrics(self) -> List[ReplicaMetrics]:
        out = []
        for r in range(self.world):
            m = ReplicaMetrics()
            if self.store.check([f"m/{r}"]):
                m = ReplicaMetrics(**json.loads(self.store.get(f"m/{r}")))
            # assignments the replica has not reported yet are waiting in its queue
            m.queue_depth += self.sent[r] - m.received
            out.append(m)
        return out

    def assign(self, rid: int, replica: int):
        self.store.set(f"a/{replica}/{self.sent[replica]}", str(rid))
        self.sent[replica] += 1
        self.store.add(f"n/{replica}", 1)

    def route(self, rid: int) -> int:
        ms = self.metrics()
        try:
            i = choose(ms)
        except NoHealthyWorkers:
            self.failed.append(rid)
            return -1
        if self.snapshots is not None:
            self.snapshots.append(ms)
        self.choices.append(i)
        self.assign(rid, i)
        return i

    def run(self, t0: Optional[float] = None):
        try:
            self.t0 = time.time() if t0 is None else t0
            self.store.set("t0", repr(self.t0))
            for r in self.reqs:
                delay = self.t0 + r.arrival - time.time()
                if delay > 0:
                    time.sleep(delay)
                self.route(r.rid)
        except BaseException as e:  # surfaced by join()
            self.error = e
        finally:
            self.store.set("done", "1")

    def start(self, t0: Optional[float] = None) -> "Dispatcher":
        self.thread = threading.Thread(target=self.run, args=(t0,), daemon=True)
        self.thread.start()
        return self

    def join(self, timeout: Optional[float] = None):
        if self.thread:
            self.thread.join(timeout)
        if self.error:
            raise self.error


def store_client(host: str, port: int, timeout_s: float = 120.0):
    """A new client connection to the TCPStore at host:port (the dispatcher
    thread and the replica each use their own)."""
    from datetime import timedelta

    import torch.distributed as dist
    return dist.TCPStore(host, port, is_master=False, timeout=timedelta(seconds=timeout_s),
                         wait_for_workers=False)


def router_stores(rank: int, world: int, host: str = "127.0.0.1"):
    """A fresh TCPStore for one routed run, hosted by rank 0 on a free port
    (the port reaches the other ranks through torch.distributed's default
    process group).  Returns (the master store on rank 0 else None, this
    replica's client, on rank 0 a second client for the dispatcher thread
    else None).  Keep the master alive until every rank is done with it."""
    import socket
    from datetime import timedelta

    import torch.distributed as dist
    master, port = None, 0
    if rank == 0:
        with socket.socket() as sk:
            sk.bind((host, 0))
            port = sk.getsockname()[1]
        master = dist.TCPStore(host, port, is_master=True, timeout=timedelta(seconds=120), wait_for_workers=False)
    if world > 1:
        ports = [None] * world
        dist.all_gather_object(ports, port)
        port = ports[0]
    mine = master if rank == 0 else store_client(host, port)
    disp = store_client(host, port) if rank == 0 else None
    return master, mine, disp


def summarize_routing(choices: Sequence[int], world: int) -> Dict[str, object]:
    counts = [0] * world
    for c in choices:
        counts[c] += 1
    return {"policy": "router.rs score (queue + active + 1) x max(avg_latency_ms, 1), lowest with capacity",
            "requests_per_replica": counts}
