"""The latency-aware router (mini_serve_rs_b200/router.py) against the
restatement of src/routing/router.rs (oracle/router_ref.py), on the CPU.

* choose / score / capacity and the latency window on random and edge-case
  metrics;
* a routed trace over three `gloo` ranks: rank 0 hosts the store and runs the
  dispatcher thread, every rank runs a scripted replica (deterministic service
  ticks, metrics published after each tick) -- every routing decision must be
  the one router.rs makes on the metrics the dispatcher read, and every
  request must be served exactly once.
"""
import random
import socket
import time

import pytest
import torch.multiprocessing as mp

from mini_serve_rs_b200.router import (Dispatcher, LatencyWindow, NoHealthyWorkers, ReplicaLink, ReplicaMetrics,
                                       choose, router_stores)
from oracle import router_ref


def _as_tuple(m: ReplicaMetrics):
    return (m.queue_depth, m.active_count, m.avg_latency_ms, m.healthy, m.max_waiting)


def test_choose_matches_router_rs_on_random_metrics():
    rng = random.Random(5)
    for _ in range(5000):
        n = rng.randint(1, 8)
        ms = []
        for _ in range(n):
            ms.append(ReplicaMetrics(queue_depth=rng.choice([0, 1, 2, 5, 255, 256, 300]),
                                     active_count=rng.randint(0, 6),
                                     avg_latency_ms=rng.choice([0.0, 0.4, 1.0, 2.5, 10.0, 37.3]),
                                     healthy=rng.random() > 0.15, max_waiting=256))
        want = router_ref.choose_worker([_as_tuple(m) for m in ms])
        if want is None:
            with pytest.raises(NoHealthyWorkers):
                choose(ms)
        else:
            assert choose(ms) == want


def test_ties_go_to_the_first_worker_and_latency_floor_is_one_ms():
    ms = [ReplicaMetrics(1, 1, 0.2), ReplicaMetrics(0, 2, 0.9), ReplicaMetrics(2, 0, 1.0)]
    assert choose(ms) == 0  # all three score 3.0
    ms = [ReplicaMetrics(0, 0, 4.0), ReplicaMetrics(3, 0, 0.0)]  # 4.0 vs 4.0 -> first
    assert choose(ms) == 0
    ms = [ReplicaMetrics(256, 0, 1.0), ReplicaMetrics(10, 10, 50.0)]  # first is full
    assert choose(ms) == 1


def test_latency_window_matches_scheduler_rs():
    rng = random.Random(9)
    w = LatencyWindow()
    done = []
    assert w.avg_ms() == router_ref.avg_latency_ms(done) == 0.0
    for _ in range(300):
        v = rng.choice([0.05, 0.15, 0.25, 1.25, 3.35, rng.uniform(0, 500)])
        w.add(v)
        done.append(v)
        assert w.avg_ms() == router_ref.avg_latency_ms(done)


class _Req:
    def __init__(self, rid, arrival):
        self.rid, self.arrival = rid, arrival


def _trace():
    rng = random.Random(17)
    t, out = 0.0, []
    for rid in range(1, 61):
        t += rng.choice([0.0, 0.004, 0.012, 0.03])
        out.append(_Req(rid, t))
    return out


def _service_ticks(rid: int, rank: int) -> int:
    # replica 0 serves more slowly, so its latency and queue grow
    return 2 + (rid % 5) + (3 if rank == 0 else 0)


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        master, store, dstore = router_stores(rank, world)
        disp = Dispatcher(dstore, world, _trace(), keep_snapshots=True) if rank == 0 else None
        dist.barrier()
        if disp:
            disp.start(t0=time.time() + 0.1)
        link = ReplicaLink(store, rank)
        t0 = link.start_time()
        queue, active, served, lat = [], [], [], LatencyWindow()
        arrival = {r.rid: r.arrival for r in _trace()}
        while True:
            for rid in link.poll():
                queue.append(rid)
            # one scripted tick: admit up to 2, advance every active request
            while queue and len(active) < 2:
                rid = queue.pop(0)
                active.append([rid, _service_ticks(rid, rank)])
            for a in active:
                a[1] -= 1
            for a in [a for a in active if a[1] <= 0]:
                active.remove(a)
                served.append(a[0])
                lat.add((time.time() - t0 - arrival[a[0]]) * 1000.0)
            link.publish(ReplicaMetrics(queue_depth=len(queue), active_count=len(active), avg_latency_ms=lat.avg_ms()))
            if not queue and not active and link.finished():
                late = link.poll()  # assigned between the last poll and the done mark
                if not late:
                    break
                queue.extend(late)
            time.sleep(0.003)
        result = {"served": served}
        if disp:
            disp.join(30)
            result["choices"] = disp.choices
            result["snapshots"] = [[_as_tuple(m) for m in snap] for snap in disp.snapshots]
        dist.barrier()
        q.put((rank, result, None))
        del store, dstore, master
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, repr(e)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_routed_trace_over_gloo_ranks_follows_router_rs():
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, res, err = q.get(timeout=120)
        assert err is None, (rank, err)
        results[rank] = res
    for p in procs:
        p.join(timeout=30)
    choices, snaps = results[0]["choices"], results[0]["snapshots"]
    assert len(choices) == len(_trace())
    for c, snap in zip(choices, snaps):
        assert c == router_ref.choose_worker(snap), (c, snap)
    served = sorted(r for res in results.values() for r in res["served"])
    assert served == [r.rid for r in _trace()]
    for rank in range(world):  # each replica served what it was sent
        assert sorted(results[rank]["served"]) == sorted(r.rid for r, c in zip(
            sorted(_trace(), key=lambda r: r.arrival), choices) if c == rank)
    # the slow replica's growing score moves work to the others: not round-robin
    counts = [choices.count(r) for r in range(world)]
    assert counts[0] < counts[1] and counts[0] < counts[2], counts
