"""Tensor parallelism (KV-head sharding; the all-reduce after o_proj and
down_proj either fused with the residual add + RMSNorm over NVLink peer
memory -- the default -- or through NCCL) on two GPUs.

Each of two spawned processes drives one engine (tp_size 2) on its own GPU;
both must reproduce the transformers goldens of the single-GPU tests (logits
within the f32 tolerance, identical greedy tokens) for the Qwen3 miniature
(G = 2 -> one KV head per rank) and the Qwen2.5 miniature (q/k/v bias,
G = 7).  Skipped when fewer than two GPUs are visible.
"""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rank_main(rank, world, uid, case_idx, q, fused=True):
    try:
        os.environ.setdefault("MS_STEP_TIMEOUT_S", "60")
        os.environ["MS_TP_FUSED"] = "1" if fused else "0"
        torch.cuda.set_device(rank)
        from mini_serve_rs_b200 import engine as E
        from oracle.qwen_ref import random_weights
        from tests.golden.golden_cases import MODEL_CASES
        from tests.golden.load import golden
        case = MODEL_CASES[case_idx]
        cfg = case["cfg"]
        comm = E.nccl_comm_init(world, uid, rank, rank)
        eng = E.Engine(cfg, device=rank, pool_blocks=256, max_seqs=8, max_tokens_per_step=512,
                       max_blocks_per_seq=64, dtype=E.MS_DTYPE_F32, tp_rank=rank, tp_size=world, nccl_comm=comm)
        eng.load_weights(random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0)))
        if eng.tp_fused() != fused:
            raise RuntimeError(f"tp_fused() = {eng.tp_fused()}, wanted {fused}")
        g = golden()
        prompts = case["prompts"]
        ids = list(range(1, len(prompts) + 1))
        nb = 0
        for sid, p in zip(ids, prompts):
            need = (len(p) + case["decode_steps"] + 16) // 16 + 1
            eng.admit(sid, p, list(range(nb, nb + need)))
            nb += need
        worst, bad = 0.0, []
        toks, _ = eng.step(ids, flags=E.MS_STEP_KEEP_LOGITS)
        for s in range(case["decode_steps"] + 1):
            lg = eng.logits(len(ids))
            for i in range(len(ids)):
                want = g[f"{case['name']}/p{i}/logits"][s]
                worst = max(worst, float(np.abs(lg[i] - want).max()))
                if int(toks[i]) != int(g[f"{case['name']}/p{i}/tokens"][s]):
                    bad.append((i, s))
            if s == case["decode_steps"]:
                break
            inputs = [int(g[f"{case['name']}/p{i}/tokens"][s]) for i in range(len(ids))]
            pos = [len(p) + s for p in prompts]
            toks, _ = eng.step(ids, inputs, pos, flags=E.MS_STEP_KEEP_LOGITS)
        eng.close()
        E.nccl_comm_destroy(comm)
        q.put((rank, worst, bad, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("case_idx,fused", [(1, True), (2, True), (1, False)],
                         ids=["qwen3_small-fused", "qwen2_small-fused", "qwen3_small-nccl"])
def test_tp2_matches_transformers_goldens(case_idx, fused):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from mini_serve_rs_b200 import engine as E
    uid = E.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, uid, case_idx, q, fused)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, worst, bad, err in results:
        assert err is None, (rank, err)
        assert worst <= 2e-4, (rank, worst)
        assert not bad, (rank, bad)
