"""Chunked prefill inside the ragged step (ms_step_desc.token_budget).

With a per-step token budget, prompts are prefilled in pieces across steps
(decode rows first, never deferred), flagged MS_FLAG_NO_TOKEN until their
last piece runs.  Each request's tokens must equal those of whole-prompt
prefill (f32 mode: same greedy tokens), whether
its pages were allocated up front or appended piece by piece, and the
logits behind each of those tokens must agree within 1e-4.
"""
import numpy as np
import pytest

from mini_serve_rs_b200 import engine as E
from oracle.qwen_ref import random_weights
from tests.golden.golden_cases import MODEL_CASES
from tests.gpu_util import need_gpu

pytestmark = pytest.mark.gpu
NEW_TOKENS = 8


def _run(cfg, w, prompts, budget, lazy_blocks):
    eng = E.Engine(cfg, pool_blocks=256, max_seqs=8, max_tokens_per_step=1024, max_blocks_per_seq=32,
                   dtype=E.MS_DTYPE_F32)
    eng.load_weights(w)
    ids = list(range(1, len(prompts) + 1))
    nxt = 0
    owned = {}
    for sid, p in zip(ids, prompts):
        # early requests keep decoding while later prompts are still chunked
        n = 1 if lazy_blocks else (len(p) + 200) // 16 + 1
        owned[sid] = list(range(nxt, nxt + n))
        nxt += n
        eng.admit(sid, p, owned[sid])
    gen = {sid: [] for sid in ids}
    lgs = {sid: [] for sid in ids}
    steps = no_token = 0
    while min(len(g) for g in gen.values()) < NEW_TOKENS:
        # the packed rows of this step: decodes, then prompts while budget lasts
        left = budget - sum(1 for s in ids if gen[s]) if budget else None
        packed = []
        for sid, p in zip(ids, prompts):
            if gen[sid]:
                packed.append(sid)
                continue
            rem = len(p) - eng.cached_tokens(sid)
            take = rem if left is None else max(0, min(rem, left))
            if left is not None:
                left -= take
            if take:
                packed.append(sid)
        if lazy_blocks:  # cover what this step can schedule: up to the budget past what is cached
            for sid, p in zip(ids, prompts):
                c = eng.cached_tokens(sid)
                reach = c + 1 if len(gen[sid]) else min(len(p), c + (budget or len(p)))
                while len(owned[sid]) * 16 < reach:
                    owned[sid].append(nxt)
                    eng.append_block(sid, nxt)
                    nxt += 1
        toks, flags = eng.step(ids, flags=E.MS_STEP_TOKENS_FROM_DEVICE, token_budget=budget)
        lg = eng.logits(len(packed))
        steps += 1
        for k, sid in enumerate(ids):
            if flags[k] & E.MS_FLAG_NO_TOKEN:
                no_token += 1
                assert toks[k] == 0
            else:
                gen[sid].append(int(toks[k]))
                lgs[sid].append(lg[packed.index(sid)])
        assert steps < 200
    eng.close()
    return ({s: g[:NEW_TOKENS] for s, g in gen.items()}, {s: np.stack(v[:NEW_TOKENS]) for s, v in lgs.items()},
            steps, no_token)


@pytest.mark.parametrize("budget,lazy", [(32, False), (24, True), (7, False)], ids=["b32", "b24-lazy", "b7"])
def test_chunked_prefill_matches_whole_prompt_prefill(budget, lazy):
    need_gpu()
    case = MODEL_CASES[1]
    cfg = case["cfg"]
    w = random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (70, 45, 100, 3)]
    ref, ref_lg, ref_steps, ref_none = _run(cfg, w, prompts, 0, False)
    got, lg, steps, none = _run(cfg, w, prompts, budget, lazy)
    assert ref_none == 0 and none > 0 and steps > ref_steps
    assert got == ref, (got, ref)
    worst = max(float(np.abs(lg[s] - ref_lg[s]).max()) for s in ref_lg)
    assert worst <= 1e-4, worst
