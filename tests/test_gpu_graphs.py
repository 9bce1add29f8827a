"""CUDA-graph replay of decode steps gives the eager steps' results bit for bit.

Two engines with the same weights and pages run the same request mix: one
with graphs (the default), one with ms_engine_set_graphs(0).  Decode steps
are device-fed (MS_STEP_TOKENS_FROM_DEVICE), blocks are appended lazily when a
sequence crosses a page boundary (block-table deltas inside replayed steps),
contexts outgrow the first graph's capacity (a second capture), and a
sequence leaves half-way (a new batch size, eager warm-up, then capture).
Greedy tokens and f32 logits must be identical at every step.
"""
import numpy as np
import pytest

from mini_serve_rs_b200 import engine as E
from oracle.qwen_ref import random_weights
from tests.golden.golden_cases import MODEL_CASES
from tests.gpu_util import need_gpu

pytestmark = pytest.mark.gpu


def _run(cfg, weights, dtype, graphs, prompts, steps, leave_at):
    eng = E.Engine(cfg, pool_blocks=512, max_seqs=16, max_tokens_per_step=1024, max_blocks_per_seq=64,
                   dtype=dtype)
    eng.load_weights(weights)
    eng.set_graphs(graphs)
    ids = list(range(1, len(prompts) + 1))
    nxt = 0
    owned = {}
    for sid, p in zip(ids, prompts):
        n = (len(p) + 15) // 16
        owned[sid] = list(range(nxt, nxt + n))
        nxt += n
        eng.admit(sid, p, owned[sid])
    ctx = {sid: len(p) for sid, p in zip(ids, prompts)}
    toks_log, logit_log = [], []
    toks, _ = eng.step(ids)
    toks_log.append(toks.copy())
    logit_log.append(eng.logits(len(ids)))
    for s in range(steps):
        if s == leave_at:
            eng.release(ids[0])
            ids = ids[1:]
        for sid in ids:  # the decode token goes to position ctx[sid]
            if ctx[sid] >= 16 * len(owned[sid]):
                owned[sid].append(nxt)
                eng.append_block(sid, nxt)
                nxt += 1
        toks, _ = eng.step(ids, flags=E.MS_STEP_TOKENS_FROM_DEVICE)
        for sid in ids:
            ctx[sid] += 1
        toks_log.append(toks.copy())
        logit_log.append(eng.logits(len(ids)))
    stats = eng.graph_stats()
    eng.close()
    return toks_log, logit_log, stats


@pytest.mark.parametrize("dtype", [E.MS_DTYPE_BF16, E.MS_DTYPE_F32], ids=["bf16", "f32"])
def test_graph_replay_matches_eager_bit_for_bit(dtype):
    need_gpu()
    case = MODEL_CASES[1]  # Qwen3 miniature: QK-norm, tied embeddings
    cfg = case["cfg"]
    w = random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
    rng = np.random.default_rng(7)
    prompts = [list(rng.integers(0, cfg.vocab_size, n)) for n in (5, 17, 30, 33, 64, 100)]
    steps, leave_at = 200, 170
    t_g, l_g, st_g = _run(cfg, w, dtype, True, prompts, steps, leave_at)
    t_e, l_e, st_e = _run(cfg, w, dtype, False, prompts, steps, leave_at)
    assert st_e == (0, 0, 0)
    captures, replays, cached = st_g
    # (6 seqs) warm-up, capture, capacity outgrown -> capture again; (5 seqs) warm-up, capture
    assert captures >= 3, st_g
    assert replays >= steps - 2 * captures - 4, st_g
    assert cached >= 2, st_g
    for k, (a, b) in enumerate(zip(t_g, t_e)):
        assert np.array_equal(a, b), (k, a, b)
    for k, (a, b) in enumerate(zip(l_g, l_e)):
        assert np.array_equal(a, b), (k, float(np.abs(a - b).max()))


def test_graphs_off_by_setting_drops_cache():
    need_gpu()
    case = MODEL_CASES[1]
    cfg = case["cfg"]
    w = random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
    eng = E.Engine(cfg, pool_blocks=64, max_seqs=4, max_tokens_per_step=256, max_blocks_per_seq=16,
                   dtype=E.MS_DTYPE_BF16)
    eng.load_weights(w)
    eng.admit(1, [3, 4, 5], [0, 1, 2])
    eng.step([1])
    for _ in range(5):
        eng.step([1], flags=E.MS_STEP_TOKENS_FROM_DEVICE)
    c, r, n = eng.graph_stats()
    assert c == 1 and r == 3 and n == 1, (c, r, n)
    eng.set_graphs(False)
    assert eng.graph_stats()[2] == 0
    eng.step([1], flags=E.MS_STEP_TOKENS_FROM_DEVICE)
    assert eng.graph_stats()[:2] == (1, 3)
    eng.close()
