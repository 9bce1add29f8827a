"""reserve_sequence's memory budget on the page pool (ms_pages_reserve and
CudaBackend.reserve_sequence), on the CPU, mirroring the reference's
tests/test_tensor_memory.rs and its CachePressure admission tests:

* reservations never exceed the pool, also under 16 concurrent threads;
* a reservation is idempotent per id and ends with release (cancel);
* admission evicts cache-only prefix pages, but cannot reclaim pages that a
  live sequence still shares;
* CudaBackend raises CachePressure / TokenLimitExceeded / NoHealthyWorkers as
  CandleBackend::reserve_sequence does (candle.rs:349-375).
"""
import threading
from types import SimpleNamespace

import pytest

from mini_serve_rs_b200 import engine as E
from mini_serve_rs_b200.backend import CudaBackend


def test_reservations_stay_within_the_pool_and_are_idempotent():
    pm = E.Pages(8, 16, max_chunks=0)
    pm.reserve(1, 20, 12)    # 2 pages
    pm.reserve(2, 60, 4)     # 4 pages
    pm.reserve(3, 16, 16)    # 2 pages: the pool is fully reserved
    assert pm.stats()["reserved_blocks"] == 8
    pm.reserve(1, 500, 500)  # idempotent: no new charge
    assert pm.stats()["reserved_blocks"] == 8
    with pytest.raises(E.CachePressure):
        pm.reserve(4, 1, 1)
    st = pm.stats()
    assert st["reserved_blocks"] == 8 and st["reservation_rejections"] == 1
    pm.release(2)            # cancel ends the reservation
    pm.reserve(4, 1, 1)
    assert pm.stats()["reserved_blocks"] == 5
    assert pm.stats()["peak_reserved_blocks"] == 8
    for bad in ((5, 0, 4), (6, 4, 0)):
        with pytest.raises(E.TokenLimitExceeded):
            pm.reserve(*bad)
    pm.close()


def test_concurrent_reservations_stay_within_budget():
    # tensor_memory.rs test: 16 threads each ask for a quarter of the budget
    pm = E.Pages(100, 16, max_chunks=0)
    ok = []
    bar = threading.Barrier(16)

    def worker(i):
        bar.wait()
        try:
            pm.reserve(100 + i, 16 * 20, 16 * 5)  # 25 pages
            ok.append(i)
        except E.CachePressure:
            pass

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(16)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert len(ok) == 4
    assert pm.stats()["reserved_blocks"] == 100
    for i in ok:
        pm.release(100 + i)
    assert pm.stats()["reserved_blocks"] == 0
    pm.close()


def test_admission_evicts_cache_only_pages_but_not_shared_ones():
    pm = E.Pages(6, 16, max_chunks=8)
    prompt = list(range(40))           # 2 full chunks + 8 tokens
    pm.reserve(1, len(prompt), 8)      # 3 pages
    blocks, cached = pm.admit(1, prompt)
    assert len(blocks) == 3 and cached == 0
    assert pm.publish(1, prompt) == 2  # its 2 full chunks enter the cache
    pm.release(1)                      # now 2 cache-only pages
    st = pm.stats()
    assert st["cache_only_blocks"] == 2 and st["reserved_blocks"] == 0
    # 5 pages + 2 cache-only > 6: one cached page is evicted to make room
    pm.reserve(2, 64, 16)
    st = pm.stats()
    assert st["evictions"] == 1 and st["cache_only_blocks"] == 1 and st["reserved_blocks"] == 5
    pm.release(2)
    # a live sequence shares the remaining cached chunk: it cannot be reclaimed
    pm.reserve(3, 20, 4)               # 2 pages
    blocks, cached = pm.admit(3, prompt[:20])
    assert cached == 16
    with pytest.raises(E.CachePressure):
        pm.reserve(4, 16 * 4, 16)      # 5 pages + 2 reserved > 6
    assert pm.stats()["evictions"] == 1 and pm.stats()["reservation_rejections"] == 1
    pm.release(3)                      # the chunk is cache-only again: now it can go
    pm.reserve(4, 16 * 5, 16)          # 6 pages: the whole pool
    assert pm.stats()["evictions"] == 2 and pm.stats()["cache_only_blocks"] == 0
    pm.close()


class _FakeEngine:
    """What CudaBackend's admission path reads from an engine (no GPU)."""

    def __init__(self, pool_blocks, ctx=4096):
        self.opts = SimpleNamespace(pool_blocks=pool_blocks, block_size=16)
        self.cfg = SimpleNamespace(max_position_embeddings=ctx)
        self.healthy = True
        self.released = []

    def is_healthy(self):
        return self.healthy

    def mark_unhealthy(self):
        self.healthy = False

    def release(self, sid):
        self.released.append(sid)


def test_backend_reserve_sequence_semantics():
    eng = _FakeEngine(pool_blocks=10)
    be = CudaBackend(eng)
    be.reserve_sequence("a", 100, 28)      # 8 pages
    be.reserve_sequence("a", 100, 28)      # idempotent
    with pytest.raises(E.CachePressure):
        be.reserve_sequence("b", 30, 10)   # 3 pages > 2 left
    be.reserve_sequence("c", 16, 16)       # 2 pages
    with pytest.raises(E.TokenLimitExceeded):
        be.reserve_sequence("d", 0, 10)
    with pytest.raises(E.TokenLimitExceeded):
        be.reserve_sequence("e", 4000, 100)  # beyond the context length
    be.cancel_sequence("a")
    be.cancel_sequence("a")                # idempotent
    be.reserve_sequence("b", 30, 10)       # fits after the cancel
    assert be.budget.stats()["reserved_blocks"] == 5
    assert eng.released == []              # nothing was admitted to the engine
    be.mark_unhealthy()
    assert be.budget.stats()["reserved_blocks"] == 0
    with pytest.raises(E.NoHealthyWorkers):
        be.reserve_sequence("f", 10, 10)
