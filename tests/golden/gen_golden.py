"""Generate the golden vectors under tests/golden/ (run in a container that has
the reference tree; the outputs are committed, the GPU box only reads them).

Two independent sources pin the oracle:

1. Hugging Face ``transformers`` Qwen2/Qwen3 on CPU f32 with eager attention
   -- the library the reference itself uses as its independent golden
   generator (tests/fixtures/generation/generate_reference.py).  Weights are
   either the deterministic sin construction of
   tests/test_pretrained_numerics.rs:88-100 or seeded N(0, 0.02) draws from
   ``oracle.qwen_ref.random_weights`` (regenerable anywhere from the seed).
2. The torch reference functions of scripts/validate_cuda_kernels.py:21-46
   (``reference_rmsnorm``, ``reference_paged_gqa``) imported from the
   reference tree, on the cases that script runs (:132-251).

Usage: python tests/golden/gen_golden.py [--ref /path/to/mini-serve-rs] [--cases NAME ...]

The reference tree is taken from --ref, else $MS_REFERENCE_ROOT, else the
"reference_path" of BASELINE.json at the repository root.  With --cases only
the named model cases are (re)computed and merged into the existing
golden.npz; every other stored array is kept as it is.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle.qwen_ref import Config, random_weights, sin_fixture_weights  # noqa: E402
from tests.golden.golden_cases import (ATTN_FRAGMENTED_TABLE, ATTN_RAGGED_LENS,  # noqa: E402
                                       ATTN_RAGGED_TABLES, ATTN_SEQ_LENS, MODEL_CASES,
                                       RMSNORM_CASES, attn_inputs, rmsnorm_inputs)


def hf_model(cfg: Config, weights):
    from transformers import Qwen2Config, Qwen2ForCausalLM, Qwen3Config, Qwen3ForCausalLM
    common = dict(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                  intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                  num_attention_heads=cfg.num_attention_heads,
                  num_key_value_heads=cfg.num_key_value_heads,
                  max_position_embeddings=cfg.max_position_embeddings, rope_theta=cfg.rope_theta,
                  rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=cfg.tie_word_embeddings)
    if cfg.qk_norm:
        hc = Qwen3Config(head_dim=cfg.hd(), attention_bias=cfg.attention_bias, **common)
        model = Qwen3ForCausalLM(hc)
    else:
        # Qwen2 always carries q/k/v biases; a bias-free reference config gets zeros.
        assert cfg.hd() == cfg.hidden_size // cfg.num_attention_heads
        hc = Qwen2Config(**common)
        model = Qwen2ForCausalLM(hc)
    hc._attn_implementation = "eager"
    model.config._attn_implementation = "eager"
    sd = model.state_dict()
    with torch.no_grad():
        for name, t in sd.items():
            if name in weights:
                t.copy_(weights[name])
            elif name == "lm_head.weight" and cfg.tie_word_embeddings:
                t.copy_(weights["model.embed_tokens.weight"])
            elif name.endswith(".bias"):
                t.zero_()
            else:
                raise KeyError(name)
    return model.eval().to(torch.float32)


def logits_all(model, ids):
    with torch.no_grad():
        return model(torch.tensor([ids], dtype=torch.long)).logits[0].to(torch.float32)


def gen_model_cases(out, only=None):
    meta = {}
    for case in MODEL_CASES:
        if only and case["name"] not in only:
            continue
        cfg = case["cfg"]
        w = sin_fixture_weights(cfg) if case["weights"] == "sin" else random_weights(
            cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
        model = hf_model(cfg, w)
        for pi, prompt in enumerate(case["prompts"]):
            # prefill logits + greedy continuation, recomputed from scratch each
            # step (no HF cache) so every step is an independent full forward
            seq = list(prompt)
            steps = []
            for s in range(case["decode_steps"] + 1):
                lg = logits_all(model, seq)[-1]
                steps.append(lg.numpy())
                seq.append(int(torch.argmax(lg)))
            key = f"{case['name']}/p{pi}"
            out[key + "/prompt"] = np.asarray(prompt, np.int32)
            out[key + "/logits"] = np.stack(steps).astype(np.float32)
            out[key + "/tokens"] = np.asarray(seq[len(prompt):], np.int32)
            srt = np.sort(np.stack(steps), axis=-1)
            meta[key] = {"min_top2_margin": float((srt[:, -1] - srt[:, -2]).min())}
    return meta


def load_reference_validator(ref_root: Path):
    path = ref_root / "scripts" / "validate_cuda_kernels.py"
    spec = importlib.util.spec_from_file_location("ref_validate_cuda_kernels", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def gen_kernel_cases(out, ref_root: Path):
    ref = load_reference_validator(ref_root)
    eps = 1e-6
    for dt_name, dt in (("f32", torch.float32), ("f16", torch.float16)):
        for rows, dim in RMSNORM_CASES:
            x, w = rmsnorm_inputs(rows, dim)
            y = ref.reference_rmsnorm(torch, torch.from_numpy(x).to(dt), torch.from_numpy(w).to(dt), eps)
            out[f"rmsnorm/{dt_name}/{rows}x{dim}"] = y.to(torch.float32).numpy()
        scale = 1.0 / math.sqrt(128)
        q1, kp, vp, qr = attn_inputs()
        kp_t, vp_t = torch.from_numpy(kp).to(dt), torch.from_numpy(vp).to(dt)
        table = torch.tensor([ATTN_FRAGMENTED_TABLE], dtype=torch.int32)
        for li, L in enumerate(ATTN_SEQ_LENS):
            q = torch.from_numpy(q1[li:li + 1]).to(dt)
            y = ref.reference_paged_gqa(torch, q, kp_t, vp_t, table, [L], scale)
            out[f"paged_gqa/{dt_name}/len{L}"] = y.to(torch.float32).numpy()
        tables = torch.tensor(ATTN_RAGGED_TABLES, dtype=torch.int32)
        y = ref.reference_paged_gqa(torch, torch.from_numpy(qr).to(dt), kp_t, vp_t, tables,
                                    list(ATTN_RAGGED_LENS), scale)
        out[f"paged_gqa/{dt_name}/ragged"] = y.to(torch.float32).numpy()


def reference_root(arg):
    if arg is not None:
        return arg
    if os.environ.get("MS_REFERENCE_ROOT"):
        return Path(os.environ["MS_REFERENCE_ROOT"])
    baseline = ROOT / "BASELINE.json"
    if baseline.exists():
        p = json.loads(baseline.read_text()).get("reference_path")
        if p:
            return Path(p)
    raise SystemExit("reference tree unknown: pass --ref or set MS_REFERENCE_ROOT")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", type=Path, default=None)
    ap.add_argument("--cases", nargs="*", default=None,
                    help="recompute only these model cases and merge them into the existing golden.npz")
    args = ap.parse_args()
    torch.manual_seed(0)
    import transformers
    if args.cases:
        with np.load(HERE / "golden.npz") as z:
            out = {k: z[k] for k in z.files}
        meta_all = json.loads((HERE / "golden_meta.json").read_text())
        meta_all["model_cases"].update(gen_model_cases(out, set(args.cases)))
    else:
        out = {}
        meta = gen_model_cases(out)
        gen_kernel_cases(out, reference_root(args.ref))
        meta_all = {"transformers": transformers.__version__, "torch": torch.__version__,
                    "numpy": np.__version__, "model_cases": meta,
                    "sources": {"model": "transformers Qwen2/Qwen3ForCausalLM, CPU f32, eager",
                                "kernels": "scripts/validate_cuda_kernels.py:21-46 (reference tree)"}}
    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "golden_meta.json").write_text(json.dumps(meta_all, indent=2, sort_keys=True) + "\n")
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
