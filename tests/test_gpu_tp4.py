"""Tensor parallelism over four GPUs (one KV head per rank, as Qwen2.5-7B
shards at TP=4), with the fused peer-memory all-reduce and with NCCL.

A Qwen2.5-architecture miniature with 4 KV heads (GQA 7, q/k/v bias,
untied lm_head) runs three prompts prefilled in one packed step and four
teacher-forced decode steps on each of four spawned ranks; every rank's f32
logits must match the CPU oracle (oracle.qwen_ref) within 2e-4 and give its
greedy tokens.  Skipped when fewer than four GPUs are visible.
"""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
DECODE = 4


def _cfg():
    from oracle.qwen_ref import Config
    return Config(vocab_size=512, hidden_size=896, intermediate_size=1024, num_hidden_layers=2,
                  num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=4096, head_dim=128,
                  rope_theta=1e6, rms_norm_eps=1e-6, qk_norm=False, attention_bias=True, tie_word_embeddings=False)


def _prompts(cfg):
    rng = np.random.default_rng(44)
    return [rng.integers(0, cfg.vocab_size, n).tolist() for n in (20, 37, 50)]


def _reference(cfg, w, prompts):
    from oracle.qwen_ref import QwenRef, SeqState
    model = QwenRef(cfg, w)
    logits, toks = [], []
    for p in prompts:
        st = SeqState(cfg, len(p) + DECODE + 1)
        lg = [model.forward(p, st, 0).numpy()]
        for s in range(DECODE):
            lg.append(model.forward([int(np.argmax(lg[-1]))], st, len(p) + s).numpy())
        logits.append(np.stack(lg))
        toks.append([int(np.argmax(x)) for x in lg])
    return np.stack(logits, 1), np.array(toks).T  # [step, prompt, vocab], [step, prompt]


def _rank_main(rank, world, uid, fused, ref_logits, ref_toks, q):
    try:
        os.environ.setdefault("MS_STEP_TIMEOUT_S", "60")
        os.environ["MS_TP_FUSED"] = "1" if fused else "0"
        torch.cuda.set_device(rank)
        from mini_serve_rs_b200 import engine as E
        from oracle.qwen_ref import random_weights
        cfg = _cfg()
        prompts = _prompts(cfg)
        comm = E.nccl_comm_init(world, uid, rank, rank)
        eng = E.Engine(cfg, device=rank, pool_blocks=128, max_seqs=4, max_tokens_per_step=256,
                       max_blocks_per_seq=16, dtype=E.MS_DTYPE_F32, tp_rank=rank, tp_size=world, nccl_comm=comm)
        eng.load_weights(random_weights(cfg, 77))
        if eng.tp_fused() != fused:
            raise RuntimeError(f"tp_fused() = {eng.tp_fused()}, wanted {fused}")
        ids = [1, 2, 3]
        for k, (sid, p) in enumerate(zip(ids, prompts)):
            eng.admit(sid, p, list(range(8 * k, 8 * k + 8)))
        worst, bad = 0.0, []
        toks, _ = eng.step(ids)
        for s in range(DECODE + 1):
            lg = eng.logits(len(ids))
            worst = max(worst, float(np.abs(lg - ref_logits[s]).max()))
            bad += [(s, i) for i in range(len(ids)) if int(toks[i]) != int(ref_toks[s][i])]
            if s == DECODE:
                break
            toks, _ = eng.step(ids, [int(t) for t in ref_toks[s]], [len(p) + s for p in prompts])
        eng.close()
        E.nccl_comm_destroy(comm)
        q.put((rank, worst, bad, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "nccl"])
def test_tp4_matches_oracle(fused):
    if torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    from mini_serve_rs_b200 import engine as E
    from oracle.qwen_ref import random_weights
    cfg = _cfg()
    ref_logits, ref_toks = _reference(cfg, random_weights(cfg, 77), _prompts(cfg))
    uid = E.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 4, uid, fused, ref_logits, ref_toks, q)) for r in range(4)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, worst, bad, err in results:
        assert err is None, (rank, err)
        assert worst <= 2e-4, (rank, worst)
        assert not bad, (rank, bad)
