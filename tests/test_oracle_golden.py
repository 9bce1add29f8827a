"""Pin the CPU oracle against the golden vectors (no GPU needed).

The goldens come from Hugging Face transformers (the reference's own
independent golden generator) and from the reference's kernel validator's
torch functions; see tests/golden/gen_golden.py.
"""
import math

import numpy as np
import pytest
import torch

from oracle import kernels_ref
from oracle.qwen_ref import QwenRef, SeqState, argmax_first, random_weights, sin_fixture_weights
from tests.golden.golden_cases import (ATTN_FRAGMENTED_TABLE, ATTN_RAGGED_LENS,
                                       ATTN_RAGGED_TABLES, ATTN_SEQ_LENS, MODEL_CASES,
                                       RMSNORM_CASES, attn_inputs, rmsnorm_inputs)
from tests.golden.load import golden


def compare(a, b, max_abs, rms):
    """Max-abs and RMS bounds plus an unchanged greedy decision, as
    tests/test_pretrained_numerics.rs:6-41 does."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    assert np.all(np.isfinite(a)) and np.all(np.isfinite(b))
    err = np.abs(a - b)
    assert err.max() <= max_abs, f"max_abs {err.max()}"
    assert math.sqrt((err ** 2).mean()) <= rms, f"rms {math.sqrt((err ** 2).mean())}"


def _weights(case):
    if case["weights"] == "sin":
        return sin_fixture_weights(case["cfg"])
    return random_weights(case["cfg"], case["seed"], norm_std=case.get("norm_std", 0.0))


@pytest.mark.parametrize("case", MODEL_CASES, ids=[c["name"] for c in MODEL_CASES])
def test_oracle_prefill_and_decode_match_transformers(case):
    g = golden()
    cfg = case["cfg"]
    model = QwenRef(cfg, _weights(case))
    for pi, prompt in enumerate(case["prompts"]):
        key = f"{case['name']}/p{pi}"
        want_logits = g[key + "/logits"]
        want_tokens = g[key + "/tokens"]
        st = SeqState(cfg, len(prompt) + case["decode_steps"] + 2)
        lg = model.forward(prompt, st, 0)
        compare(lg.numpy(), want_logits[0], 1e-4, 1e-5)
        assert argmax_first(lg) == want_tokens[0]
        pos = len(prompt)
        for s in range(case["decode_steps"]):
            lg = model.forward([int(want_tokens[s])], st, pos)
            compare(lg.numpy(), want_logits[s + 1], 1e-4, 1e-5)
            assert argmax_first(lg) == want_tokens[s + 1]
            pos += 1


def test_oracle_batched_decode_matches_single_execution():
    """tests/test_pretrained_numerics.rs:174-261 on the sin fixture: batched
    decode equals single execution for 3 teacher-forced steps."""
    case = MODEL_CASES[0]
    cfg = case["cfg"]
    model = QwenRef(cfg, _weights(case))
    singles, batch, inputs, positions = [], [], [], []
    for prompt in case["prompts"]:
        a, b = SeqState(cfg, 128), SeqState(cfg, 128)
        lg = model.forward(prompt, a, 0)
        model.forward(prompt, b, 0)
        singles.append(a)
        batch.append(b)
        inputs.append(argmax_first(lg))
        positions.append(len(prompt))
    for _ in range(3):
        bl = model.step_decode_batch(batch, inputs, positions)
        for i in range(len(singles)):
            sl = model.forward([inputs[i]], singles[i], positions[i])
            compare(bl[i].numpy(), sl.numpy(), 1e-4, 1e-5)
            inputs[i] = argmax_first(sl)
            positions[i] += 1


def test_oracle_prefix_restore_matches_full_prefill():
    """Prefill of a 16-token prefix then the suffix at offset 16 equals the
    full prefill (tests/test_pretrained_numerics.rs:204-222)."""
    case = MODEL_CASES[0]
    cfg = case["cfg"]
    model = QwenRef(cfg, _weights(case))
    ids = case["prompts"][2]
    full = model.forward(ids, SeqState(cfg, 128), 0)
    st = SeqState(cfg, 128)
    model.forward(ids[:16], st, 0)
    resumed = model.forward(ids[16:], st, 16)
    compare(resumed.numpy(), full.numpy(), 1e-4, 1e-5)


@pytest.mark.parametrize("dt_name,dt,atol", [("f32", torch.float32, 1e-5), ("f16", torch.float16, 5e-3)])
def test_oracle_rmsnorm_matches_reference_validator(dt_name, dt, atol):
    g = golden()
    for rows, dim in RMSNORM_CASES:
        x, w = rmsnorm_inputs(rows, dim)
        _, y = kernels_ref.add_rmsnorm(torch.from_numpy(x).to(dt), None, torch.from_numpy(w).to(dt), 1e-6)
        want = g[f"rmsnorm/{dt_name}/{rows}x{dim}"]
        np.testing.assert_allclose(y.to(torch.float32).numpy(), want, atol=atol, rtol=1e-4)


@pytest.mark.parametrize("dt_name,dt,atol", [("f32", torch.float32, 1e-5), ("f16", torch.float16, 5e-3)])
def test_oracle_paged_attention_matches_reference_validator(dt_name, dt, atol):
    g = golden()
    q1, kp, vp, qr = attn_inputs()
    kp_t, vp_t = torch.from_numpy(kp).to(dt), torch.from_numpy(vp).to(dt)
    table = torch.tensor([ATTN_FRAGMENTED_TABLE], dtype=torch.int32)
    scale = 1.0 / math.sqrt(128)
    for li, L in enumerate(ATTN_SEQ_LENS):
        y = kernels_ref.paged_gqa_attention(torch.from_numpy(q1[li:li + 1]).to(dt), kp_t, vp_t,
                                            table, [L], scale)
        np.testing.assert_allclose(y.numpy(), g[f"paged_gqa/{dt_name}/len{L}"], atol=atol, rtol=1e-4)
    y = kernels_ref.paged_gqa_attention(torch.from_numpy(qr).to(dt), kp_t, vp_t,
                                        torch.tensor(ATTN_RAGGED_TABLES, dtype=torch.int32),
                                        ATTN_RAGGED_LENS, scale)
    np.testing.assert_allclose(y.numpy(), g[f"paged_gqa/{dt_name}/ragged"], atol=atol, rtol=1e-4)
