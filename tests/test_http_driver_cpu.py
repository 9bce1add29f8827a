"""The HTTP/SSE driver on CPU: the real page manager (ms_pages_*) and serving
loop behind a fake engine with the engine's step contract (chunked prefill
under a token budget, one token per sequence per step, MS_FLAG_NO_TOKEN /
MS_FLAG_PREFILLED).  Checks the reference's /v1/completions behaviour
(src/api/routes.rs:144-262): SSE framing, one chunk per token, the final
chunk's finish_reason and usage, [DONE], the non-streamed response, error
payloads and status codes (src/core/errors.rs:52-95), and the trace client's
metrics (examples/bench.rs:61-110)."""
import asyncio
import json
import time

import numpy as np
import pytest

aiohttp = pytest.importorskip("aiohttp")

from mini_serve_rs_b200 import engine as E  # noqa: E402
from mini_serve_rs_b200.http_driver import (BackgroundHttp, HttpFrontendProcess, ServingServer,  # noqa: E402
                                            StreamResult, run_trace, stream_completion, summarize_http)
from mini_serve_rs_b200.serving import Request  # noqa: E402

VOCAB = 1000


def expected_token(prompt, t):
    return (sum(prompt) + 7 * t + 3) % VOCAB


class FakeEngine:
    """Engine stand-in: prompts are consumed under the step's token budget,
    the step that completes one returns its first token (MS_FLAG_PREFILLED),
    later steps one token each; token t of a request is expected_token()."""

    class cfg:
        vocab_size = VOCAB

    def __init__(self, max_blocks_per_seq=64):
        self.max_blocks_per_seq = max_blocks_per_seq
        self.seqs = {}
        self.steps = 0
        self.max_batch = 0

    def admit(self, rid, prompt, blocks, num_cached=0):
        assert rid not in self.seqs
        self.seqs[rid] = {"prompt": list(prompt), "cached": num_cached, "blocks": list(blocks), "out": 0}

    def release(self, rid):
        self.seqs.pop(rid, None)

    def cached_tokens(self, rid):
        return self.seqs[rid]["cached"]

    def append_block(self, rid, b):
        self.seqs[rid]["blocks"].append(b)

    def step(self, ids, flags=0, token_budget=0, temperature=None, top_p=None, seeds=None):
        time.sleep(0.001)  # a step takes device time, so arrivals overlap
        self.steps += 1
        self.max_batch = max(self.max_batch, len(ids))
        budget = token_budget or (1 << 30)
        toks, fl = [], []
        for rid in ids:
            s = self.seqs[rid]
            n = len(s["prompt"])
            if s["cached"] < n:
                take = min(n - s["cached"], budget)
                budget -= take
                s["cached"] += take
                if s["cached"] < n:
                    toks.append(0)
                    fl.append(E.MS_FLAG_NO_TOKEN)
                    continue
                f = E.MS_FLAG_PREFILLED
            else:
                s["cached"] += 1
                f = 0
            assert len(s["blocks"]) * 16 >= s["cached"], "the loop grew the pages before the step"
            toks.append(expected_token(s["prompt"], s["out"]))
            s["out"] += 1
            fl.append(f)
        return np.array(toks, np.int32), np.array(fl, np.int32)


@pytest.fixture(params=["thread", "process"])
def served(request):
    """The server with its HTTP front-end on a thread of this process, or in a
    process of its own (HttpFrontendProcess) talking to the engine over a pipe."""
    eng = FakeEngine()
    pages = E.Pages(512, 16, max_chunks=128)
    srv = ServingServer(eng, pages, model="fake", max_active=8, token_budget=64).start()
    http = (BackgroundHttp if request.param == "thread" else HttpFrontendProcess)(srv).start()
    yield http.url, srv, eng, pages
    http.stop()
    srv.stop()


async def _post(url, body):
    async with aiohttp.ClientSession() as s:
        async with s.post(f"{url}/v1/completions", json=body) as r:
            return r.status, dict(r.headers), await r.read()


async def _get(url, path):
    async with aiohttp.ClientSession() as s:
        async with s.get(f"{url}{path}") as r:
            return r.status, await r.json()


def test_streamed_completion_framing_tokens_and_usage(served):
    url, *_ = served
    prompt = list(range(1, 41))
    status, headers, raw = asyncio.run(_post(url, {"model": "fake", "prompt": prompt, "max_tokens": 5,
                                                   "temperature": 0, "stream": True}))
    assert status == 200 and headers["Content-Type"].startswith("text/event-stream")
    events = [e for e in raw.decode().split("\n\n") if e]
    assert events[-1] == "data: [DONE]"
    chunks = [json.loads(e[len("data: "):]) for e in events[:-1]]
    assert len(chunks) == 6
    for c in chunks:
        assert c["object"] == "text_completion.chunk" and c["model"] == "fake" and c["id"].startswith("cmpl-")
        assert len(c["choices"]) == 1 and c["choices"][0]["index"] == 0
    toks = [int(c["choices"][0]["text"]) for c in chunks[:-1]]
    assert toks == [expected_token(prompt, t) for t in range(5)]
    assert all(c["choices"][0]["finish_reason"] is None and "usage" not in c for c in chunks[:-1])
    last = chunks[-1]
    assert last["choices"][0] == {"text": "", "index": 0, "finish_reason": "length"}
    assert last["usage"] == {"prompt_tokens": 40, "completion_tokens": 5, "total_tokens": 45}


def test_non_streamed_completion_and_string_prompt(served):
    url, *_ = served
    status, _, raw = asyncio.run(_post(url, {"prompt": "5 6 7", "max_tokens": 3, "temperature": 0}))
    body = json.loads(raw)
    assert status == 200 and body["object"] == "text_completion"
    assert body["choices"][0]["text"] == "".join(f" {expected_token([5, 6, 7], t)}" for t in range(3))
    assert body["choices"][0]["finish_reason"] == "length" and body["choices"][0]["logprobs"] is None
    assert body["usage"] == {"prompt_tokens": 3, "completion_tokens": 3, "total_tokens": 6}


@pytest.mark.parametrize("body,status,etype,msg", [
    ({"prompt": "", "max_tokens": 4}, 400, "invalid_request_error", "Invalid request: Prompt cannot be empty"),
    ({"prompt": [], "max_tokens": 4}, 400, "invalid_request_error", "Invalid request: Prompt cannot be empty"),
    ({"prompt": [1, VOCAB], "max_tokens": 4}, 400, "invalid_request_error", "Invalid request: token id"),
    ({"prompt": "hello world", "max_tokens": 4}, 400, "invalid_request_error", "Invalid request: prompt must"),
    ({"prompt": [1, 2], "max_tokens": 64 * 16}, 400, "invalid_request_error", "Token limit exceeded:"),
])
def test_errors_use_the_reference_payload(served, body, status, etype, msg):
    url, *_ = served
    st, _, raw = asyncio.run(_post(url, body))
    err = json.loads(raw)["error"]
    assert st == status and err["type"] == etype and err["code"] == status and err["param"] is None
    assert err["message"].startswith(msg), err["message"]


def test_models_health_ready(served):
    url, *_ = served
    st, models = asyncio.run(_get(url, "/v1/models"))
    assert st == 200 and models["object"] == "list" and models["data"][0]["id"] == "fake"
    st, health = asyncio.run(_get(url, "/health"))
    assert st == 200 and health["status"] == "ok" and health["workers"] == 1
    st, ready = asyncio.run(_get(url, "/ready"))
    assert st == 200 and ready == {"ready": True}


def test_trace_is_batched_and_measured_like_the_reference_bench(served):
    url, srv, eng, pages = served
    rng = np.random.default_rng(0)
    shared = rng.integers(0, VOCAB, 48).tolist()
    reqs = []
    for i in range(24):
        p = (shared if i % 3 == 0 else []) + rng.integers(0, VOCAB, int(rng.integers(5, 150))).tolist()
        reqs.append(Request(i, p, int(rng.integers(2, 12)), arrival=0.002 * i, temperature=0.0))
    results, elapsed = run_trace(url, "fake", reqs)
    assert all(isinstance(r, StreamResult) for r in results), results
    for q, r in zip(reqs, results):
        assert r.tokens == q.max_tokens and r.authoritative_usage
        assert [int(x) for x in r.text.split()] == [expected_token(q.prompt, t) for t in range(q.max_tokens)]
        assert 0 < r.ttft_ms <= r.latency_ms
    s = summarize_http(results, elapsed)
    assert s["failed"] == 0 and s["tokens"] == sum(q.max_tokens for q in reqs)
    assert eng.max_batch > 1, "requests share steps (continuous batching)"
    assert pages.stats()["hits"] > 0, "the shared prefix was served from cached pages"
    assert not eng.seqs and pages.stats()["free_blocks"] + pages.stats()["cache_only_blocks"] == 512


def test_quarantined_engine_fails_requests_and_reports_not_ready(served):
    url, srv, eng, pages = served

    def broken(*a, **k):
        raise E.EngineError("device fault (injected on the host)")
    eng.step = broken
    st, _, raw = asyncio.run(_post(url, {"prompt": [1, 2, 3], "max_tokens": 4, "stream": True}))
    events = [e for e in raw.decode().split("\n\n") if e]
    assert st == 200 and "error" in json.loads(events[-1][len("data: "):])
    st, ready = asyncio.run(_get(url, "/ready"))
    assert st == 503 and ready == {"ready": False}
    st, _, raw = asyncio.run(_post(url, {"prompt": [1, 2, 3], "max_tokens": 4}))
    assert st == 503 and json.loads(raw)["error"]["type"] == "service_unavailable"
    assert pages.stats()["free_blocks"] + pages.stats()["cache_only_blocks"] == 512


def test_trace_client_in_its_own_process(served):
    from mini_serve_rs_b200.http_driver import run_trace_process
    url, srv, eng, pages = served
    reqs = [Request(i, [i + 1, i + 2, i + 3], 4, arrival=0.001 * i, temperature=0.0) for i in range(6)]
    results, elapsed = run_trace_process(url, "fake", reqs, timeout_s=120.0)
    assert all(isinstance(r, StreamResult) for r in results), results
    for q, r in zip(reqs, results):
        assert [int(x) for x in r.text.split()] == [expected_token(q.prompt, t) for t in range(4)]
    assert summarize_http(results, elapsed)["failed"] == 0


def test_client_disconnect_cancels_the_request(served):
    """A client that drops its stream mid-way releases the request's sequence
    and pages (the reference's RequestCancelled path) instead of generating
    to max_tokens."""
    url, srv, eng, pages = served

    async def go():
        async with aiohttp.ClientSession() as s:
            resp = await s.post(f"{url}/v1/completions", json={"prompt": list(range(1, 30)), "max_tokens": 900,
                                                               "temperature": 0, "stream": True})
            assert resp.status == 200
            got = 0
            async for _ in resp.content.iter_any():
                got += 1
                if got >= 3:
                    break
            resp.close()  # drop the connection mid-stream

    asyncio.run(go())
    deadline = time.time() + 10
    while time.time() < deadline and (eng.seqs or srv.cancelled == 0):
        time.sleep(0.01)
    assert srv.cancelled == 1 and not eng.seqs
    st = pages.stats()
    assert st["free_blocks"] + st["cache_only_blocks"] == 512, st
    assert eng.steps < 600  # stopped long before 900 tokens


def test_host_failure_in_the_loop_fails_requests_instead_of_hanging(served):
    url, srv, eng, pages = served

    def boom(*a, **k):
        raise RuntimeError("host-side bug")
    eng.step = boom
    st, _, raw = asyncio.run(_post(url, {"prompt": [4, 5], "max_tokens": 3}))
    assert st == 500 and "serving loop failed" in json.loads(raw)["error"]["message"]
    st, ready = asyncio.run(_get(url, "/ready"))
    assert st == 503


def test_frontend_process_that_cannot_bind_reports_it():
    """A front-end process that dies before serving (here: its port is taken) is a
    clear start-up error, not a hang or a bare EOFError."""
    import socket
    eng = FakeEngine()
    pages = E.Pages(64, 16, max_chunks=16)
    srv = ServingServer(eng, pages, model="fake", max_active=2, token_budget=64).start()
    busy = socket.socket()
    busy.bind(("127.0.0.1", 0))
    busy.listen(1)
    try:
        with pytest.raises(RuntimeError, match="did not start"):
            HttpFrontendProcess(srv, port=busy.getsockname()[1]).start(timeout=60)
    finally:
        busy.close()
        srv.stop()
