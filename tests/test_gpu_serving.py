"""The continuous-batching loop (serving.ServingLoop) end to end: queueing
behind a full batch, prompts shared through the prefix cache, prefill in
chunks under a token budget, growth and release of pages.  In f32 mode every
request must produce the tokens it produces when served alone with whole
prompt prefill and no cache, and every page must return to the pool (the
cache keeping only its own)."""
import numpy as np
import pytest

from mini_serve_rs_b200 import engine as E
from mini_serve_rs_b200.serving import Request, ServingLoop, summarize
from oracle.qwen_ref import random_weights
from tests.golden.golden_cases import MODEL_CASES
from tests.gpu_util import need_gpu

pytestmark = pytest.mark.gpu


def _trace(cfg, n=16):
    rng = np.random.default_rng(31)
    shared = rng.integers(0, cfg.vocab_size, 40).tolist()
    reqs = []
    for i in range(n):
        own = rng.integers(0, cfg.vocab_size, int(rng.integers(3, 60))).tolist()
        prompt = shared + own if i % 3 == 0 else own
        reqs.append(Request(rid=i + 1, prompt=prompt, max_tokens=int(rng.integers(4, 14))))
    return reqs


def _serve(cfg, w, reqs, max_active, budget, max_chunks, reserve=False, pool=160):
    eng = E.Engine(cfg, pool_blocks=pool, max_seqs=8, max_tokens_per_step=512, max_blocks_per_seq=16,
                   dtype=E.MS_DTYPE_F32)
    eng.load_weights(w)
    pages = E.Pages(pool, 16, max_chunks=max_chunks)
    loop = ServingLoop(eng, pages, max_active=max_active, token_budget=budget, reserve=reserve)
    elapsed = loop.run(reqs, timeout_s=120.0)
    st = pages.stats()
    eng.close()
    return {r.rid: r.out for r in loop.finished}, summarize(loop.finished, elapsed), st, loop.steps


def test_serving_loop_matches_requests_served_alone():
    need_gpu()
    case = MODEL_CASES[1]
    cfg = case["cfg"]
    w = random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
    got, summ, st, steps = _serve(cfg, w, _trace(cfg), max_active=6, budget=40, max_chunks=32)
    want, _, _, _ = _serve(cfg, w, _trace(cfg), max_active=1, budget=0, max_chunks=0)
    assert summ["failed"] == 0 and len(got) == 16
    bad = [rid for rid in want if got[rid] != want[rid]]
    assert len(bad) <= 1, bad
    assert st["hits"] >= 3, st  # requests 4, 7, 10, 13, 16 reuse the shared prefix pages
    assert st["free_blocks"] + st["cache_only_blocks"] == st["total_blocks"], st


def test_serving_loop_with_reservations_waits_for_room_and_matches():
    """reserve=True: each request reserves its worst-case pages before
    admission (reserve_sequence); with a pool of 24 pages that cover about
    four requests' worst cases, requests wait in the queue for reservations to
    free, none fails, the tokens equal those served alone, and every
    reservation is returned."""
    need_gpu()
    case = MODEL_CASES[1]
    cfg = case["cfg"]
    w = random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
    got, summ, st, _ = _serve(cfg, w, _trace(cfg), max_active=6, budget=40, max_chunks=32, reserve=True, pool=24)
    want, _, _, _ = _serve(cfg, w, _trace(cfg), max_active=1, budget=0, max_chunks=0)
    assert summ["failed"] == 0 and len(got) == 16
    bad = [rid for rid in want if got[rid] != want[rid]]
    assert len(bad) <= 1, bad
    assert st["reservation_rejections"] > 0, st  # some requests had to wait for reservations
    assert st["peak_reserved_blocks"] <= 24 and st["reserved_blocks"] == 0, st
