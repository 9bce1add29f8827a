"""The trace client's completion-stream checker (http_driver.CompletionStream)
against the acceptance rules listed in http_driver.py, which are the rules the
reference's client parser enforces, on the vectors of its tests
(src/sse.rs:119-173): arbitrary byte boundaries keep UTF-8 text, token events
and usage; truncated or invalid streams never succeed; the finish chunk is
not a token event and usage is authoritative."""
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


def test_each_rule_is_enforced():
    def stream(*events):
        return b"".join(b"data: " + e + b"\n\n" for e in events)

    tok = b'{"choices":[{"text":"a","finish_reason":null}]}'
    fin = b'{"choices":[{"text":"","finish_reason":"length"}]}'
    usage_only = b'{"choices":[],"usage":{"completion_tokens":1}}'
    ok = CompletionStream()
    ok.push(stream(tok, fin, usage_only, b"[DONE]"))
    assert ok.finish() == 1 and ok.finish_reason == "length"
    bad = {
        "payloads": [stream(b'{"error":null}'), stream(b"[1, 2]")],
        "tokens": [stream(b'{"choices":[{"text":"a"},{"text":"b"}]}'), stream(b'{"choices":[{"text":5}]}')],
        "finish": [stream(tok, fin, tok), stream(tok, b'{"choices":[{"text":"","finish_reason":""}]}'),
                   stream(tok, fin, b'{"choices":[]}')],
        "usage": [stream(b'{"choices":[{"text":"a"}],"usage":{"completion_tokens":-1}}'),
                  stream(b'{"choices":[{"text":"a"}],"usage":{"completion_tokens":true}}'),
                  stream(b'{"choices":[{"text":"a"}],"usage":{"completion_tokens":1}}',
                         b'{"choices":[{"text":"b"}],"usage":{"completion_tokens":2}}')],
        "close": [stream(tok, b"[DONE]"), stream(tok, fin, b"[DONE]", tok)],
        "framing": [b"data: \xff\n\n"],
    }
    for rule, cases in bad.items():
        for data in cases:
            p = CompletionStream()
            with pytest.raises(SseError) as e:
                p.push(data)
            assert e.value.rule == rule, (rule, data, e.value)
            with pytest.raises(SseError):
                p.push(b"")  # a failed stream stays failed
    p = CompletionStream()
    p.push(stream(b'{"choices":[{"text":"a"}],"usage":{"completion_tokens":0}}', fin, b"[DONE]"))
    with pytest.raises(SseError) as e:
        p.finish()  # usage below the token events
    assert e.value.rule == "usage"
