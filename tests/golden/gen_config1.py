"""Generate tests/golden/config1.json: BASELINE config 1 run through the CPU
oracle (the restated Candle f32 path with the reference's scheduling).

Qwen3-0.6B architecture, random init N(0, 0.02) from seed 20261201 (norm
weights 1), four requests with prompt lengths {17, 64, 128, 300} and token ids
uniform in [0, 151936) (seed 7), greedy decode of 32 tokens each under the
restated continuous-batching scheduler with 16-token KV blocks.  Stores per
request the prompt, the 32 greedy tokens, the top-2 logit margin of every
step, and the block table each step used.

Usage: python tests/golden/gen_config1.py   (about a minute on 8 cores)
"""
from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle.kv_cache_ref import KVCacheRef  # noqa: E402
from oracle.qwen_ref import QwenRef, RefBackend, qwen3_0_6b, random_weights  # noqa: E402
from oracle.scheduler_ref import Request, SchedulerRef  # noqa: E402

SEED_WEIGHTS = 20261201
SEED_PROMPTS = 7
PROMPT_LENS = (17, 64, 128, 300)
MAX_TOKENS = 32
POOL_BLOCKS = 1024  # main.rs:26 default


def prompts():
    rng = np.random.Generator(np.random.PCG64(SEED_PROMPTS))
    return [[int(t) for t in rng.integers(0, 151936, n)] for n in PROMPT_LENS]


def main():
    torch.set_num_threads(max(1, torch.get_num_threads()))
    cfg = qwen3_0_6b()
    t0 = time.time()
    model = QwenRef(cfg, random_weights(cfg, SEED_WEIGHTS))
    backend = RefBackend(model)
    margins = {}
    orig_step = backend.step_batch

    def step(seqs):
        toks = orig_step(seqs)
        for s in seqs:
            lg = backend.last_logits[s.request_id]
            top = torch.topk(lg, 2).values
            margins.setdefault(s.request_id, []).append(float(top[0] - top[1]))
        return toks

    sched = SchedulerRef(KVCacheRef(POOL_BLOCKS, 16), step, backend.cancel_sequence, max_batch_size=8)
    ps = prompts()
    for i, p in enumerate(ps):
        sched.submit(Request(f"req-{i}", p, MAX_TOKENS))
    out = sched.run()
    steps = [{"request_ids": r.request_ids, "prefill": r.prefill, "kv_blocks": r.kv_blocks,
              "prompt_lens": r.prompt_lens, "num_outputs": r.num_outputs, "tokens": r.tokens}
             for r in sched.records]
    res = {"config": "BASELINE config 1 (Qwen3-0.6B arch, f32, random init)", "seed_weights": SEED_WEIGHTS,
           "seed_prompts": SEED_PROMPTS, "prompt_lens": PROMPT_LENS, "max_tokens": MAX_TOKENS,
           "pool_blocks": POOL_BLOCKS, "prompts": ps,
           "tokens": {k: v for k, v in out.items()}, "margins": margins, "steps": steps,
           "seconds": round(time.time() - t0, 1), "torch": torch.__version__}
    (HERE / "config1.json").write_text(json.dumps(res) + "\n")
    print("done in", res["seconds"], "s; min margin", min(min(v) for v in margins.values()))


if __name__ == "__main__":
    main()
