"""The trace client's SSE parser (http_driver.CompletionStream) against the
rules of the reference's parser, src/sse.rs, and its tests (:119-173):
arbitrary byte boundaries keep UTF-8 text, token events and usage; truncated
or invalid streams never succeed; the finish chunk is not a token event and
usage is authoritative."""
import json

import pytest

from mini_serve_rs_b200.http_driver import MAX_EVENT_BYTES, CompletionStream, SseError


def fixture() -> bytes:
    s = ": keepalive\r\n\r\n"
    for text in ["café", "", " 終"]:
        s += "data: " + json.dumps({"choices": [{"text": text, "finish_reason": None}]}, ensure_ascii=False) + "\r\n\r\n"
    s += 'data: {"choices":[{"text":"","finish_reason":"length"}],\n'
    s += 'data: "usage":{"completion_tokens":3}}\n\ndata: [DONE]\n\n'
    return s.encode()


def check(parts):
    p = CompletionStream()
    for part in parts:
        p.push(part)
    assert p.finish() == 3
    assert p.token_events == 3
    assert p.text == "café 終"


def test_arbitrary_byte_boundaries_preserve_utf8_events_usage_and_finish():
    s = fixture()
    for split in range(len(s) + 1):
        check([s[:split], s[split:]])
    check([s[i:i + 1] for i in range(len(s))])


def test_errors_and_truncated_streams_never_succeed():
    full = fixture()
    for cut in range(len(full)):
        p = CompletionStream()
        try:
            p.push(full[:cut])
        except SseError:
            continue
        with pytest.raises(SseError):
            p.finish()
    for invalid in [b"data: [DONE]\n\n", b'data: {"error":{"message":"oops"}}\n\n', b"data: invalid\n\n",
                    b'data: {"choices":[]}\n\n']:
        p = CompletionStream()
        with pytest.raises(SseError):
            p.push(invalid)
        with pytest.raises(SseError):
            p.finish()
    p = CompletionStream()
    p.push(full)
    with pytest.raises(SseError):
        p.push(b"data: [DONE]\n\n")
    p = CompletionStream()
    with pytest.raises(SseError):
        p.push(b"x" * (MAX_EVENT_BYTES + 1))


def test_terminal_chunk_is_not_a_token_and_usage_is_authoritative():
    p = CompletionStream()
    p.push(b'data: {"choices":[{"text":"ok","finish_reason":null}]}\n\n'
           b'data: {"choices":[{"text":"","finish_reason":"stop"}],"usage":{"completion_tokens":2}}\n\n'
           b"data: [DONE]\n\n")
    assert p.token_events == 1
    assert p.finish() == 2
