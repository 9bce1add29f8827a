"""Host-side restatements: the logical block manager against the reference's
own known answers (tests/test_kv_cache.rs), the packer's integer formulas, and
the scheduler's block-growth invariants.  No GPU."""
import numpy as np
import pytest

from oracle.kv_cache_ref import CachePressure, KVCacheRef
from oracle.packer_ref import pack, step_inputs
from oracle.scheduler_ref import Request, SchedulerRef, swap_remove


def test_kv_cache_allocate_and_release():
    # tests/test_kv_cache.rs:4-23
    c = KVCacheRef(100, 16)
    assert c.free_count() == 100 and c.allocated_count() == 0
    blocks = c.allocate("req-1", 32)
    assert len(blocks) == 2 and c.free_count() == 98 and c.allocated_count() == 2
    assert blocks == [0, 1]  # pop order 0, 1, 2, ... (kv_cache.rs:25)
    assert c.release("req-1") == 2 and c.free_count() == 100


def test_kv_cache_pressure_message():
    # tests/test_kv_cache.rs:26-38
    c = KVCacheRef(4, 16)
    with pytest.raises(CachePressure, match="Requested 5 blocks"):
        c.allocate("req-over", 80)


def test_kv_cache_fragmentation_stats():
    # tests/test_kv_cache.rs:40-52
    c = KVCacheRef(10, 16)
    assert c.allocate("req-1", 16) == [0]
    assert c.allocate("req-2", 16) == [1]
    assert c.allocate("req-3", 16) == [2]
    c.release("req-2")
    s = c.stats()
    assert s["total_blocks"] == 10 and s["free_blocks"] == 8 and s["utilization"] > 0


def test_kv_cache_lifo_reuse_and_blocks_needed():
    c = KVCacheRef(8, 16)
    assert c.blocks_needed(0) == 1 and c.blocks_needed(16) == 1 and c.blocks_needed(17) == 2
    a = c.allocate("a", 40)  # 3 blocks: 0,1,2
    c.allocate_block("a")  # 3
    c.release("a")  # pushes 0,1,2,3 -> next pops are 3,2,1,0
    assert a == [0, 1, 2]
    assert c.allocate("b", 20) == [3, 2]


def test_packer_slot_formula_and_boundaries():
    seqs = [(1, 0, [5]), (1, 15, [7]), (1, 16, [7, 9]), (3, 14, [2, 4]), (17, 0, [11, 12])]
    p = pack(seqs)
    assert p["cu_seqlens"].tolist() == [0, 1, 2, 3, 6, 23]
    assert p["positions"][:6].tolist() == [0, 15, 16, 14, 15, 16]
    assert p["slot_mapping"][:6].tolist() == [80, 127, 144, 46, 47, 64]
    assert p["slot_mapping"][6:].tolist() == [11 * 16 + i for i in range(16)] + [192]
    assert p["row_ctx"][:3].tolist() == [1, 16, 17]
    with pytest.raises(ValueError):
        pack([(1, 16, [3])])


def test_step_inputs_follow_the_reference():
    assert step_inputs(10, [], False) == (10, 0)
    assert step_inputs(10, [4], True) == (1, 10)
    assert step_inputs(10, [4, 5, 6], True) == (1, 12)
    assert step_inputs(32, [], False, cached=16) == (16, 16)
    assert step_inputs(32, [], False, cached=32) == (1, 31)


def test_swap_remove_matches_rust():
    xs = [1, 2, 3, 4]
    assert swap_remove(xs, 1) == 2 and xs == [1, 4, 3]
    assert swap_remove(xs, 2) == 3 and xs == [1, 4]


def test_scheduler_grows_one_block_ahead_and_orders_like_the_reference():
    seen = []

    def step(seqs):
        for s in seqs:
            # the table always covers the token being written plus one
            n = len(s.prompt_tokens) + len(s.output_tokens) + 1
            assert len(s.kv_blocks) * 16 >= n - 1
        seen.append([s.request_id for s in seqs])
        return [1] * len(seqs)

    sched = SchedulerRef(KVCacheRef(64, 16), step, max_batch_size=2)
    sched.submit(Request("a", list(range(15)), 3))
    sched.submit(Request("b", list(range(16)), 1))
    sched.submit(Request("c", list(range(3)), 2))
    out = sched.run()
    assert out == {"a": [1, 1, 1], "b": [1], "c": [1, 1]}
    # b finishes after step 1 and is swap-removed; c is admitted at the tail
    assert seen[0] == ["a", "b"] and seen[1] == ["a", "c"]
    assert sched.cache.free_count() == 64
