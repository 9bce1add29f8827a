"""The paged prefix cache (ms_pages_*, host code, no GPU) against its
restatements: chain keys equal the reference's SHA-256 chain
(prefix_cache.rs:103-124) computed with hashlib; with the cache off the block
ids equal KVCache's (kv_cache.rs); with it on, a random serving trace gives
the restated manager's block ids, cached-token counts and counters at every
step; and the reference's own prefix-cache tests (tests/test_prefix_cache.rs)
hold in page form.
"""
import numpy as np
import pytest

from mini_serve_rs_b200 import engine as E
from oracle.kv_cache_ref import CachePressure as RefPressure
from oracle.kv_cache_ref import KVCacheRef
from oracle.prefix_pages_ref import PagesRef, chunk_hashes


def test_chain_keys_match_hashlib_restatement():
    rng = np.random.default_rng(0)
    for n in (0, 15, 16, 17, 48, 100, 513):
        toks = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32).tolist()
        assert E.chunk_hashes(toks) == chunk_hashes(toks)
    toks = list(range(32))  # tests/test_prefix_cache.rs:4-9
    keys = E.chunk_hashes(toks)
    assert len(keys) == 2 and keys[0] != keys[1]
    assert E.chunk_hashes(list(range(16)), 8) == chunk_hashes(list(range(16)), 8)


def test_cache_off_hands_out_kvcache_block_ids():
    rng = np.random.default_rng(1)
    pg, ref = E.Pages(64, 16, max_chunks=0), KVCacheRef(64, 16)
    live = []
    for step in range(400):
        op = rng.integers(0, 3)
        if op == 0:
            sid = step + 1
            n = int(rng.integers(0, 80))
            try:
                want = ref.allocate(str(sid), max(n, 1))
            except RefPressure:
                with pytest.raises(E.CachePressure):
                    pg.admit(sid, list(range(n)))
                continue
            got, cached = pg.admit(sid, list(range(n)))
            assert got == want and cached == 0
            live.append(sid)
        elif op == 1 and live:
            sid = live[int(rng.integers(0, len(live)))]
            try:
                want = ref.allocate_block(str(sid))
            except RefPressure:
                with pytest.raises(E.CachePressure):
                    pg.allocate_block(sid)
                continue
            assert pg.allocate_block(sid) == want
        elif op == 2 and live:
            sid = live.pop(int(rng.integers(0, len(live))))
            assert pg.release(sid) == ref.release(str(sid))
    assert pg.stats()["free_blocks"] == ref.free_count()


def test_random_trace_matches_restated_manager():
    rng = np.random.default_rng(2)
    prefixes = [rng.integers(0, 50000, int(rng.integers(16, 90))).tolist() for _ in range(4)]
    pg, ref = E.Pages(96, 16, max_chunks=24), PagesRef(96, 16, max_chunks=24)
    live = {}
    for step in range(1500):
        op = int(rng.integers(0, 6))
        if op == 5:  # a reservation (for a sequence admitted now, later or never)
            sid = step + int(rng.integers(0, 3))
            plen, mt = int(rng.integers(1, 200)), int(rng.integers(1, 200))
            try:
                ref.reserve(sid, plen, mt)
            except RefPressure:
                with pytest.raises(E.CachePressure):
                    pg.reserve(sid, plen, mt)
            else:
                pg.reserve(sid, plen, mt)
        elif op <= 1:
            sid = step + 1
            base = prefixes[int(rng.integers(0, len(prefixes)))] if rng.random() < 0.8 else []
            prompt = base[:int(rng.integers(0, len(base) + 1))] + rng.integers(0, 50000, int(rng.integers(0, 40))).tolist()
            try:
                want = ref.admit(sid, prompt)
            except RefPressure:
                with pytest.raises(E.CachePressure):
                    pg.admit(sid, prompt)
                continue
            assert pg.admit(sid, prompt) == want, step
            live[sid] = prompt
        elif op == 2 and live:
            sid = list(live)[int(rng.integers(0, len(live)))]
            try:
                want = ref.allocate_block(sid)
            except RefPressure:
                with pytest.raises(E.CachePressure):
                    pg.allocate_block(sid)
                continue
            assert pg.allocate_block(sid) == want, step
        elif op == 3 and live:
            sid = list(live)[int(rng.integers(0, len(live)))]
            assert pg.publish(sid, live[sid]) == ref.publish(sid, live[sid]), step
        elif op == 4 and live:
            sid = list(live)[int(rng.integers(0, len(live)))]
            del live[sid]
            assert pg.release(sid) == ref.release(sid), step
        if step % 50 == 0:
            probe = prefixes[step % len(prefixes)]
            assert pg.lookup(probe) == ref.lookup(probe), step
        assert pg.stats() == ref.stats(), step
    st = pg.stats()
    assert st["hits"] > 50 and st["evictions"] > 0 and st["rejections"] > 0, st
    assert st["peak_reserved_blocks"] > 0 and st["reservation_rejections"] > 0, st


def test_reference_prefix_cache_tests_in_page_form():
    # tests/test_prefix_cache.rs:12-32: 48 cached tokens match 48
    pg = E.Pages(100, 16, max_chunks=100)
    prompt = list(range(48))
    assert pg.lookup(prompt) == 0
    pg.admit(1, prompt)
    assert pg.publish(1, prompt) == 3
    assert pg.lookup(prompt) == 48
    # a new request with the same prompt shares all but the last chunk: its
    # last prompt token is always computed (the exact-hit replay)
    blocks, cached = pg.admit(2, prompt)
    assert cached == 32 and blocks[:2] == [0, 1] and blocks[2] not in (0, 1, 2)
    blocks, cached = pg.admit(3, prompt + [7])
    assert cached == 48 and blocks[:3] == [0, 1, 2]
    # tests/test_prefix_cache.rs:34-53: with room for 2 chunks, caching seq_b evicts seq_a
    pg = E.Pages(100, 16, max_chunks=2)
    seq_a, seq_b = list(range(32)), list(range(100, 132))
    pg.admit(1, seq_a)
    pg.publish(1, seq_a)
    assert pg.lookup(seq_a) == 32
    pg.admit(2, seq_b)
    pg.publish(2, seq_b)
    assert pg.lookup(seq_b) == 32
    assert pg.lookup(seq_a) == 0


def test_pressure_spares_pages_in_use_and_changes_nothing():
    pg = E.Pages(4, 16, max_chunks=8)
    a = list(range(64))
    pg.admit(1, a)           # 4 pages, all of the pool
    pg.publish(1, a)         # chunks cached, still held by seq 1
    before = pg.stats()
    with pytest.raises(E.CachePressure):
        pg.admit(2, list(range(100, 116)))
    after = pg.stats()
    assert after["free_blocks"] == before["free_blocks"] == 0
    assert after["cached_chunks"] == 4 and after["rejections"] == 1
    pg.release(1)            # pages now held only by the cache
    assert pg.stats()["cache_only_blocks"] == 4
    blocks, cached = pg.admit(2, list(range(100, 116)))  # evicts the least recently used leaf
    assert len(blocks) == 1 and cached == 0
    assert pg.stats()["cached_chunks"] == 3 and pg.lookup(a) == 48
