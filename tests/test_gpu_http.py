"""The HTTP/SSE driver in front of the real engine: a trace of concurrent
streamed /v1/completions requests (greedy, f32 parity mode, a shared prefix
served from cached pages, chunked prefill) must stream the CPU oracle's
greedy tokens (oracle.qwen_ref, restating qwen2.rs) for every request (one
request may differ: batch shapes change the f32 GEMM rounding, as in the
serving-loop test), every request ends with usage and [DONE], and every page
returns to the pool."""
import numpy as np
import pytest

from mini_serve_rs_b200 import engine as E
from mini_serve_rs_b200.http_driver import (BackgroundHttp, HttpFrontendProcess, ServingServer, StreamResult,
                                            run_trace, summarize_http)
from mini_serve_rs_b200.serving import Request
from oracle.qwen_ref import QwenRef, SeqState, random_weights
from tests.golden.golden_cases import MODEL_CASES
from tests.gpu_util import need_gpu

pytestmark = pytest.mark.gpu


def _oracle_greedy(cfg, w, prompt, n):
    model = QwenRef(cfg, w)
    st = SeqState(cfg, len(prompt) + n + 1)
    toks = [int(np.argmax(model.forward(prompt, st, 0).numpy()))]
    for s in range(n - 1):
        toks.append(int(np.argmax(model.forward([toks[-1]], st, len(prompt) + s).numpy())))
    return toks


@pytest.mark.parametrize("frontend", [BackgroundHttp, HttpFrontendProcess], ids=["thread", "process"])
def test_http_trace_streams_the_oracle_greedy_tokens(frontend):
    need_gpu()
    pytest.importorskip("aiohttp")
    case = MODEL_CASES[1]  # Qwen3 miniature: QK-norm, tied embeddings
    cfg = case["cfg"]
    w = random_weights(cfg, case["seed"], norm_std=case.get("norm_std", 0.0))
    rng = np.random.default_rng(5)
    shared = rng.integers(0, cfg.vocab_size, 40).tolist()
    reqs = []
    for i in range(10):
        own = rng.integers(0, cfg.vocab_size, int(rng.integers(3, 60))).tolist()
        reqs.append(Request(i, (shared + own) if i % 3 == 0 else own, int(rng.integers(4, 12)),
                            arrival=0.004 * i, temperature=0.0))
    eng = E.Engine(cfg, pool_blocks=160, max_seqs=8, max_tokens_per_step=512, max_blocks_per_seq=16,
                   dtype=E.MS_DTYPE_F32)
    eng.load_weights(w)
    pages = E.Pages(160, 16, max_chunks=32)
    srv = ServingServer(eng, pages, model="qwen3-mini", max_active=6, token_budget=40).start()
    http = frontend(srv).start()
    try:
        results, elapsed = run_trace(http.url, "qwen3-mini", reqs, timeout_s=300.0)
    finally:
        http.stop()
        srv.stop()
    st = pages.stats()
    eng.close()
    assert all(isinstance(r, StreamResult) for r in results), results
    bad = []
    for q, r in zip(reqs, results):
        got = [int(x) for x in r.text.split()]
        assert r.tokens == q.max_tokens == len(got) and r.authoritative_usage
        if got != _oracle_greedy(cfg, w, q.prompt, q.max_tokens):
            bad.append(q.rid)
    assert len(bad) <= 1, bad
    s = summarize_http(results, elapsed)
    assert s["failed"] == 0 and s["ttft_ms_p50"] > 0
    assert st["hits"] >= 2, st
    assert st["free_blocks"] + st["cache_only_blocks"] == st["total_blocks"], st
