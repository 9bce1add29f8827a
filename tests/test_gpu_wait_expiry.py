"""A bounded wait that runs out inside the decode-attention kernel is reported,
not hung on and not silently ignored.

The kernels poll each K/V page's barrier a bounded number of times.  The test
hook ms_test_set_attention_wait_limit(0) makes those page-loop waits give up
at once, before the page's copy has landed; every copy the kernel started
still lands, because the drain after a failed wait keeps the normal limit, so
no access leaves its buffers and the context stays usable.

* standalone launcher: the status bit shows up in ms_kernel_status, which
  clears it; with the default limit the same launch is correct again;
* engine: the step fails with MS_E_DEVICE (BackendError), the engine is
  quarantined (later steps get NoHealthyWorkers), and a new engine on the same
  device serves the same request correctly.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from mini_serve_rs_b200 import engine as E
from tests.golden.golden_cases import MODEL_CASES

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
WAIT_TIMEOUT_BIT = 1


@pytest.fixture(autouse=True)
def _restore_limit():
    yield
    E.lib().ms_test_set_attention_wait_limit(-1)


def _attention_case(seed=21, batch=64, mb=64, pool=4096):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    rng = np.random.Generator(np.random.PCG64(seed))
    ctx = rng.integers(mb * 8, mb * 16 + 1, batch).astype(np.int32)
    tables = ((np.arange(batch)[:, None] * 97 + np.arange(mb)[None, :] * 13) % pool).astype(np.int32)
    kp = torch.randn(pool, 8, 16, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
    vp = torch.randn(pool, 8, 16, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
    q = torch.randn(batch, 16, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
    return q, kp, vp, torch.from_numpy(tables).to(DEV), torch.from_numpy(ctx).to(DEV)


def _launch(q, kp, vp, tables, ctx):
    out = torch.zeros_like(q)
    p = lambda t: C.c_void_p(t.data_ptr())
    rc = E.lib().launch_paged_gqa_decode_tiled_bf16(p(q), p(kp), p(vp), p(tables), p(ctx), p(out), q.shape[0], 16,
                                                    8, tables.shape[1], 1.0 / math.sqrt(128))
    torch.cuda.synchronize()
    assert rc == 0  # the launch itself succeeds: the failure is inside the kernel
    return out


def test_standalone_launcher_reports_a_wait_that_ran_out():
    lib = E.lib()
    d = _attention_case()
    E.kernel_status(0)
    good = _launch(*d)
    assert E.kernel_status(0) == 0
    assert lib.ms_test_set_attention_wait_limit(0) == 0
    _launch(*d)
    st = E.kernel_status(0)
    assert st & WAIT_TIMEOUT_BIT, st
    assert E.kernel_status(0) == 0  # read and cleared
    assert lib.ms_test_set_attention_wait_limit(-1) == 0
    again = _launch(*d)
    assert E.kernel_status(0) == 0
    assert torch.equal(again, good)


def _engine():
    case = MODEL_CASES[1]  # Qwen3 miniature (head_dim 128, GQA 2)
    from oracle.qwen_ref import random_weights
    eng = E.Engine(case["cfg"], pool_blocks=512, max_seqs=8, max_tokens_per_step=1024, max_blocks_per_seq=64,
                   dtype=E.MS_DTYPE_BF16)
    eng.load_weights(random_weights(case["cfg"], case["seed"], norm_std=case.get("norm_std", 0.0)))
    return case, eng


def _admit_and_prefill(eng, case):
    ids = [1, 2, 3]
    for k, (sid, p) in enumerate(zip(ids, case["prompts"])):
        eng.admit(sid, p, list(range(16 * k, 16 * k + 12)))
    toks, _ = eng.step(ids)  # prefill (tensor-core prefill kernel, not affected by the hook)
    return ids, [int(t) for t in toks], [len(p) for p in case["prompts"]]


def test_engine_step_fails_and_quarantines_when_a_wait_runs_out():
    lib = E.lib()
    case, eng = _engine()  # the healthy result first
    ids, toks, pos = _admit_and_prefill(eng, case)
    want, _ = eng.step(ids, toks, pos)
    eng.close()

    case, eng = _engine()
    ids, toks, pos = _admit_and_prefill(eng, case)
    assert lib.ms_test_set_attention_wait_limit(0) == 0
    with pytest.raises(E.BackendError) as ei:
        eng.step(ids, toks, pos)  # decode rows: the split-K kernel
    assert ei.value.code == E.MS_E_DEVICE
    assert not eng.is_healthy()
    with pytest.raises(E.NoHealthyWorkers):
        eng.step(ids, toks, pos)
    eng.close()
    assert lib.ms_test_set_attention_wait_limit(-1) == 0

    # the context is still usable: a new engine computes the healthy result
    case, eng = _engine()
    ids, toks2, pos = _admit_and_prefill(eng, case)
    assert toks2 == toks
    got, _ = eng.step(ids, toks, pos)
    assert np.array_equal(got, want)
    eng.close()
