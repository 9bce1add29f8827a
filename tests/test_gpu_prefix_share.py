"""Prefix-cache page sharing through the engine.

Requests get their pages from the page manager (ms_pages_*).  Requests whose
prompts share a published prefix are admitted with those pages and
num_cached, so the engine prefills only their suffix and attends over the
shared pages.  Their logits and greedy tokens must equal a run that prefills
every prompt in full on private pages (the reference's result for a prefix
hit equals a full prefill, candle.rs:1196-1293: < 1e-4), and the request
that owns the shared pages must be undisturbed.
"""
import numpy as np
import pytest

from mini_serve_rs_b200 import engine as E
from oracle.qwen_ref import random_weights
from tests.golden.golden_cases import MODEL_CASES
from tests.gpu_util import need_gpu

pytestmark = pytest.mark.gpu
DECODE = 6


def _run(cfg, w, dtype, prompts, share):
    """Admit prompt 0 first (prefill + publish), then the others in one step;
    decode DECODE steps.  Returns per-request logits of every step, tokens,
    cached token counts and the page stats."""
    eng = E.Engine(cfg, pool_blocks=256, max_seqs=8, max_tokens_per_step=1024, max_blocks_per_seq=32, dtype=dtype)
    eng.load_weights(w)
    pages = E.Pages(256, 16, max_chunks=64 if share else 0)
    ids = list(range(1, len(prompts) + 1))
    logits = {i: [] for i in ids}
    toks = {i: [] for i in ids}
    cached = {}
    owned = {}

    def admit(sid, prompt):
        blocks, c = pages.admit(sid, prompt)
        owned[sid] = blocks
        cached[sid] = c
        eng.admit(sid, prompt, blocks, num_cached=c)

    def grow(active):
        for sid in active:
            need = (eng.cached_tokens(sid) + 1 + 15) // 16
            while len(owned[sid]) < need:
                b = pages.allocate_block(sid)
                owned[sid].append(b)
                eng.append_block(sid, b)

    admit(1, prompts[0])
    out, _ = eng.step([1])
    logits[1].append(eng.logits(1)[0])
    toks[1].append(int(out[0]))
    pages.publish(1, prompts[0])
    for sid, p in zip(ids[1:], prompts[1:]):
        admit(sid, p)
    # request 1 decodes while the others prefill in the same ragged step
    grow([1])
    out, _ = eng.step(ids, flags=E.MS_STEP_TOKENS_FROM_DEVICE)
    lg = eng.logits(len(ids))
    for k, sid in enumerate(ids):
        logits[sid].append(lg[k])
        toks[sid].append(int(out[k]))
    for _ in range(DECODE):
        grow(ids)
        out, _ = eng.step(ids, flags=E.MS_STEP_TOKENS_FROM_DEVICE)
        lg = eng.logits(len(ids))
        for k, sid in enumerate(ids):
            logits[sid].append(lg[k])
            toks[sid].append(int(out[k]))
    st = pages.stats()
    eng.close()
    return logits, toks, cached, st


@pytest.mark.parametrize("dtype,tol", [(E.MS_DTYPE_F32, 1e-4), (E.MS_DTYPE_BF16, 0.25)], ids=["f32", "bf16"])
def test_shared_prefix_pages_match_full_prefill(dtype, tol):
    need_gpu()
    case = MODEL_CASES[1]
    cfg = case["cfg"]
    w = random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
    rng = np.random.default_rng(8)
    base = rng.integers(0, cfg.vocab_size, 77).tolist()
    prompts = [base,                                                   # owner: 4 full chunks + 13
               base[:64] + rng.integers(0, cfg.vocab_size, 21).tolist(),  # shares 4 chunks
               base[:40] + rng.integers(0, cfg.vocab_size, 9).tolist(),   # shares 2 chunks
               base[:64],                                              # exact 4 chunks: shares 3
               rng.integers(0, cfg.vocab_size, 30).tolist()]          # no hit
    lg_s, tk_s, cached, st = _run(cfg, w, dtype, prompts, share=True)
    lg_f, tk_f, cached_f, _ = _run(cfg, w, dtype, prompts, share=False)
    assert cached == {1: 0, 2: 64, 3: 32, 4: 48, 5: 0}, cached
    assert set(cached_f.values()) == {0}
    assert st["hits"] == 3 and st["tokens_saved"] == 144, st
    worst = 0.0
    for sid in lg_s:
        for a, b in zip(lg_s[sid], lg_f[sid]):
            worst = max(worst, float(np.abs(a - b).max()))
        if dtype == E.MS_DTYPE_F32:
            assert tk_s[sid] == tk_f[sid], (sid, tk_s[sid], tk_f[sid])
    assert worst <= tol, worst
