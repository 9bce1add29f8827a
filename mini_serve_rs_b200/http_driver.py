"""HTTP/SSE driver over the serving loop: the reference's completion API in
front of the B200 engine, and a trace client that measures it the way the
reference's benchmark does.

Server (mirrors src/api/routes.rs):
* POST /v1/completions (:144-262): body {model, prompt, max_tokens = 128,
  temperature = 1.0, top_p = 1.0, stream = false, stop = []}
  (src/core/types.rs:84-97, defaults :35-43).  An empty prompt is
  "Invalid request: Prompt cannot be empty" (HTTP 400).  Streaming sends one
  text_completion.chunk per generated token, a final chunk with the
  finish_reason and usage, then "[DONE]"; otherwise one text_completion.
  Errors use the reference's payload and status mapping
  (src/core/errors.rs:52-95).
* GET /v1/models, /health, /ready (:96-139).
The model has random-init weights and no tokenizer, so a prompt is a list of
token ids (a JSON array, or a string of whitespace-separated ids) and each
generated token streams as the text " <id>".  Stop strings are accepted and
ignored; finish_reason is "length".  Streamed chunks carry the request's
start second in "created" (the reference stamps each chunk).

One engine thread owns the ServingLoop (continuous batching: admission,
growth, one ragged ms_step per iteration) and posts each new token to the
waiting handler's asyncio queue.  The aiohttp front-end runs either on a
thread of the engine's process (BackgroundHttp) or in a process of its own
(HttpFrontendProcess), which keeps the per-token SSE work out of the engine
process's interpreter: one pipe message per engine step carries every new
token, and the reference's single tokio process has no such contention.

Client: CompletionStream checks a streamed completion against the rules the
reference's client parser enforces (listed below, src/sse.rs); stream_completion
measures one request as
examples/bench.rs:61-110 does (TTFT = first token event, decode rate over
the events after it), and run_trace replays a trace with real arrival times.
"""
from __future__ import annotations

import asyncio
import json
import queue
import threading
import time
import uuid
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

from . import engine as E
from .serving import Request, ServingLoop

MAX_EVENT_BYTES = 1024 * 1024


# ---------------------------------------------------------------------------------------
# client-side parsing of a streamed completion
#
# What the trace client accepts, as rules (the reference's client, src/sse.rs,
# enforces the same ones):
#   framing   - text/event-stream: lines end in LF or CR LF; the values of the
#               "data" fields of an event (one leading space dropped) are joined
#               by LF; a blank line ends the event; comments and other fields
#               are ignored; a line is decoded as UTF-8 once it is complete;
#               an event may hold at most 1 MiB of line bytes;
#   payloads  - every event but the closing "[DONE]" is a JSON object; one
#               with an "error" member fails the stream;
#   tokens    - a chunk has exactly one choice with a string "text"; without a
#               finish_reason it is one generated-token event;
#   finish    - a non-empty string finish_reason ends the generation: after it
#               only a usage-only chunk (empty choices) or "[DONE]" may come;
#   usage     - usage.completion_tokens, when present, is a non-negative
#               integer that never changes and is the authoritative count;
#               it may not be smaller than the token events seen;
#   close     - "[DONE]" needs a finish_reason before it and ends the stream:
#               nothing may follow, and a stream that never got it, or ends
#               inside an event, is incomplete.
MAX_EVENT_BYTES = 1024 * 1024


class SseError(ValueError):
    """The stream breaks one of the rules above (`rule` names it)."""

    def __init__(self, rule: str, detail: str):
        super().__init__(f"{rule}: {detail}")
        self.rule = rule


class EventFramer:
    """Bytes in, complete event payloads out (the framing rule)."""

    def __init__(self, limit: int = MAX_EVENT_BYTES):
        self.limit = limit
        self.partial = bytearray()   # the current line, not yet terminated
        self.fields: List[str] = []  # data values of the event being built
        self.size = 0                # line bytes of the event being built

    def idle(self) -> bool:
        """No line or event is half received."""
        return not self.partial and not self.fields

    def feed(self, chunk: bytes) -> List[str]:
        events: List[str] = []
        *complete, tail = bytes(chunk).split(b"\n")
        for seg in complete:
            self._grow(len(seg))
            self.partial += seg
            line, self.partial = bytes(self.partial), bytearray()
            if line.endswith(b"\r"):
                line = line[:-1]
            try:
                text = line.decode("utf-8")
            except UnicodeDecodeError:
                raise SseError("framing", "a line is not valid UTF-8") from None
            if text == "":
                if self.fields:  # trailing empty data lines add nothing
                    events.append("\n".join(self.fields).rstrip("\n"))
                self.fields, self.size = [], 0
                continue
            name, _, value = text.partition(":")
            if name == "data" and ":" in text:
                self.fields.append(value[1:] if value.startswith(" ") else value)
        self._grow(len(tail))
        self.partial += tail
        return events

    def _grow(self, n: int):
        self.size += n
        if self.size > self.limit:
            raise SseError("framing", f"an event is longer than {self.limit} bytes")


class CompletionStream:
    """A streamed /v1/completions response, checked against the rules above
    while it arrives.  push() takes bytes as they come (any split); finish()
    returns the completion-token count of a complete stream.  After any broken
    rule the stream stays failed."""

    GENERATING, FINISHED, CLOSED, BROKEN = "generating", "finished", "closed", "broken"

    def __init__(self):
        self.framer = EventFramer()
        self.phase = self.GENERATING
        self.text = ""
        self.token_events = 0
        self.completion_tokens: Optional[int] = None
        self.finish_reason: Optional[str] = None

    def push(self, data: bytes):
        if self.phase == self.BROKEN:
            raise SseError("state", "the stream already failed")
        try:
            for payload in self.framer.feed(data):
                self._take(payload)
        except SseError:
            self.phase = self.BROKEN
            raise

    def finish(self) -> int:
        if self.phase != self.CLOSED or not self.framer.idle():
            raise SseError("close", f"the stream is incomplete (phase {self.phase})")
        if self.completion_tokens is None:
            return self.token_events
        if self.completion_tokens < self.token_events:
            raise SseError("usage", "usage counts fewer tokens than the stream carried")
        return self.completion_tokens

    # -- one event payload
    def _take(self, payload: str):
        if self.phase == self.CLOSED:
            raise SseError("close", "an event arrived after [DONE]")
        if payload == "[DONE]":
            if self.phase != self.FINISHED:
                raise SseError("close", "[DONE] before any finish_reason")
            self.phase = self.CLOSED
            return
        try:
            chunk = json.loads(payload)
        except json.JSONDecodeError as e:
            raise SseError("payloads", f"not JSON ({e})") from None
        if not isinstance(chunk, dict):
            raise SseError("payloads", "not a JSON object")
        if "error" in chunk:
            raise SseError("payloads", "the server sent an error")
        self._usage(chunk.get("usage"))
        choices = chunk.get("choices")
        if not isinstance(choices, list):
            raise SseError("tokens", "no choices list")
        if self.phase == self.FINISHED:
            # after the finish only a usage-only chunk is allowed
            if choices or self.completion_tokens is None:
                raise SseError("finish", "a chunk with choices after the finish_reason")
            return
        if len(choices) != 1 or not isinstance(choices[0], dict):
            raise SseError("tokens", f"{len(choices)} choices in one chunk")
        text = choices[0].get("text")
        if not isinstance(text, str):
            raise SseError("tokens", "a choice without text")
        reason = choices[0].get("finish_reason")
        if isinstance(reason, str):
            if reason == "":
                raise SseError("finish", "an empty finish_reason")
            self.finish_reason = reason
            self.phase = self.FINISHED
        else:
            self.token_events += 1
        self.text += text

    def _usage(self, usage):
        if usage is None:
            return
        n = usage.get("completion_tokens") if isinstance(usage, dict) else None
        if isinstance(n, bool) or not isinstance(n, int) or n < 0:
            raise SseError("usage", "completion_tokens is not a non-negative integer")
        if self.completion_tokens is not None and n != self.completion_tokens:
            raise SseError("usage", "completion_tokens changed within the stream")
        self.completion_tokens = n


# ---------------------------------------------------------------------------------------
# server
class ApiError(Exception):
    """An EngineError variant with its HTTP mapping (src/core/errors.rs:52-95)."""
    KINDS = {
        "AdmissionError": (429, "rate_limit_exceeded", "1", "Queue saturated"),
        "CachePressure": (429, "rate_limit_exceeded", "1", "KV cache capacity exceeded"),
        "NoHealthyWorkers": (503, "service_unavailable", "2", "No healthy workers available"),
        "RequestCancelled": (400, "client_closed_request", None, "Request cancelled"),
        "TokenLimitExceeded": (400, "invalid_request_error", None, "Token limit exceeded"),
        "InvalidRequest": (400, "invalid_request_error", None, "Invalid request"),
        "BackendError": (500, "internal_server_error", None, "Backend error"),
    }

    def __init__(self, kind: str, msg: str):
        super().__init__(f"{self.KINDS[kind][3]}: {msg}")
        self.kind = kind

    def response(self):
        from aiohttp import web
        status, etype, retry, _ = self.KINDS[self.kind]
        payload = {"error": {"message": str(self), "type": etype, "param": None, "code": status}}
        headers = {"Retry-After": retry} if retry else None
        return web.json_response(payload, status=status, headers=headers)


def parse_prompt(prompt, vocab_size: int) -> List[int]:
    """Token ids from a JSON array or a string of whitespace-separated ids."""
    if isinstance(prompt, str):
        parts = prompt.split()
        try:
            ids = [int(p) for p in parts]
        except ValueError:
            raise ApiError("InvalidRequest", "prompt must be token ids (this model has no tokenizer)") from None
    elif isinstance(prompt, list) and all(isinstance(t, int) and not isinstance(t, bool) for t in prompt):
        ids = list(prompt)
    else:
        raise ApiError("InvalidRequest", "prompt must be a string or an array of token ids")
    if not ids:
        raise ApiError("InvalidRequest", "Prompt cannot be empty")
    if any(t < 0 or t >= vocab_size for t in ids):
        raise ApiError("InvalidRequest", f"token id outside [0, {vocab_size})")
    return ids


def _admission_check(healthy: bool, max_context: int, prompt: List[int], max_tokens: int):
    """The checks a submission passes before it reaches the engine."""
    if not healthy:
        raise ApiError("NoHealthyWorkers", "the engine is quarantined")
    if max_tokens < 1:
        raise ApiError("InvalidRequest", "max_tokens must be at least 1")
    if len(prompt) + max_tokens > max_context:
        raise ApiError("TokenLimitExceeded", f"prompt ({len(prompt)}) + max_tokens ({max_tokens}) > {max_context}")


def _deliver(evs):
    for q, ev in evs:
        q.put_nowait(ev)


@dataclass
class _Sub:
    aloop: asyncio.AbstractEventLoop
    q: asyncio.Queue
    req: Request
    sent: int = 0


class ServingServer:
    """The engine thread: owns the ServingLoop and serves submissions from
    any thread; token, done and error events go to each request's asyncio
    queue on its event loop."""

    def __init__(self, eng, pages, *, model: str = "qwen3-0.6b-arch", max_active: int = 256,
                 token_budget: int = 2048, max_context: Optional[int] = None, vocab_size: Optional[int] = None,
                 idle_wait_s: float = 0.002):
        self.model = model
        self.sl = ServingLoop(eng, pages, max_active=max_active, token_budget=token_budget)
        self.vocab_size = vocab_size if vocab_size is not None else eng.cfg.vocab_size
        self.max_context = max_context if max_context is not None else eng.max_blocks_per_seq * 16
        self._inbox: "queue.Queue[_Sub]" = queue.Queue()
        self._subs: Dict[int, _Sub] = {}
        self._rid = 0
        self._rid_lock = threading.Lock()
        self._stop = threading.Event()
        self._idle = idle_wait_s
        self.healthy = True
        self.steps = 0
        self.cancelled = 0
        self._pending: Dict[Optional[asyncio.AbstractEventLoop], List] = {}
        self._thread = threading.Thread(target=self._run, name="ms-engine", daemon=True)
        # a front-end in another process (HttpFrontendProcess): its requests' events go
        # out as one pipe message per flush, under a lock shared with stop messages
        self._remote = None
        self._remote_lock = threading.Lock()
        self._remote_healthy = True

    # -- any thread
    def start(self):
        self.sl._t0 = time.perf_counter()
        self._thread.start()
        return self

    def stop(self, timeout: float = 30.0):
        self._stop.set()
        self._thread.join(timeout)

    def submit(self, prompt: List[int], max_tokens: int, temperature: float, top_p: float,
               aloop: asyncio.AbstractEventLoop, q: asyncio.Queue) -> int:
        _admission_check(self.healthy, self.max_context, prompt, max_tokens)
        with self._rid_lock:
            self._rid += 1
            rid = self._rid
        r = Request(rid, list(prompt), int(max_tokens), temperature=float(temperature), top_p=float(top_p),
                    seed=rid)
        self._inbox.put(_Sub(aloop, q, r))
        return rid

    def cancel(self, rid: int):
        """The client went away: drop the request, or release its sequence and pages."""
        self._inbox.put(rid)

    # -- engine thread
    def _post(self, sub: _Sub, ev: Tuple):
        """Queue an event; _flush hands each event loop its events in one wake-up."""
        self._pending.setdefault(sub.aloop, []).append((sub.q, ev))

    def _flush(self):
        remote = self._pending.pop(None, [])
        for aloop, evs in self._pending.items():
            aloop.call_soon_threadsafe(_deliver, evs)
        self._pending = {}
        if self._remote is not None and (remote or self.healthy != self._remote_healthy):
            self._remote_healthy = self.healthy
            self._remote_send(("ev", self.healthy, remote))

    # -- a front-end process (HttpFrontendProcess)
    def attach_remote(self, conn):
        """Serve the front-end at the other end of `conn` (a duplex multiprocessing
        pipe): it sends ("submit", rid, prompt, max_tokens, temperature, top_p) and
        ("cancel", rid); it receives ("ev", healthy, [(rid, event), ...]) per flush."""
        self._remote = conn
        threading.Thread(target=self._remote_reader, args=(conn,), name="ms-frontend-rx", daemon=True).start()

    def _remote_send(self, msg) -> bool:
        with self._remote_lock:
            conn = self._remote
            if conn is None:
                return False
            try:
                conn.send(msg)
                return True
            except (OSError, EOFError, ValueError):  # the front-end is gone
                self._remote = None
                return False

    def _remote_reader(self, conn):
        while True:
            try:
                msg = conn.recv()
            except (OSError, EOFError):
                return
            if msg[0] == "submit":
                _, rid, prompt, max_tokens, temperature, top_p = msg
                r = Request(rid, list(prompt), int(max_tokens), temperature=float(temperature), top_p=float(top_p),
                            seed=rid)
                self._inbox.put(_Sub(None, rid, r))
            elif msg[0] == "cancel":
                self._inbox.put(msg[1])

    def _drain_inbox(self, block: bool):
        try:
            sub = self._inbox.get(timeout=self._idle) if block else self._inbox.get_nowait()
        except queue.Empty:
            return
        while True:
            if isinstance(sub, _Sub):
                sub.req.arrival = self.sl.clock()
                self.sl.submit(sub.req)
                self._subs[sub.req.rid] = sub
            else:
                self._cancel(sub)
            try:
                sub = self._inbox.get_nowait()
            except queue.Empty:
                return

    def _cancel(self, rid: int):
        sl = self.sl
        sub = self._subs.pop(rid, None)
        if sub is None:  # already finished
            return
        r = sub.req
        if r in sl.queue:
            sl.queue.remove(r)
            sl.pages.release(rid)  # a queued request may already hold its reservation
        elif r in sl.active:
            sl.active.remove(r)
            sl.eng.release(rid)
            sl.pages.release(rid)
        r.error = "Request cancelled: client disconnected"
        r.done_at = sl.clock()
        self.cancelled += 1

    def _publish(self):
        for rid in list(self._subs):
            sub = self._subs[rid]
            r = sub.req
            while sub.sent < len(r.out):
                self._post(sub, ("token", r.out[sub.sent]))
                sub.sent += 1
            if r.done_at is not None or r.error is not None:
                if r.error is None:
                    usage = {"prompt_tokens": len(r.prompt), "completion_tokens": len(r.out),
                             "total_tokens": len(r.prompt) + len(r.out)}
                    self._post(sub, ("done", "length", usage))
                else:
                    self._post(sub, ("error", r.error))
                del self._subs[rid]
        self._flush()

    def _fail_all(self, msg: str):
        """Fail every admitted and queued request; admitted ones give their pages back
        (a quarantined engine has already dropped its own sequence state)."""
        sl = self.sl
        for r in list(sl.active):
            for release in (sl.eng.release, sl.pages.release):
                try:
                    release(r.rid)
                except Exception:  # the engine may be quarantined; pages must still be returned
                    pass
        for r in list(sl.queue):
            sl.pages.release(r.rid)  # reservations of queued requests
        for r in list(sl.active) + list(sl.queue):
            r.error = msg
            r.done_at = sl.clock()
        sl.active.clear()
        sl.queue.clear()
        self._publish()

    def _run(self):
        sl = self.sl
        while not self._stop.is_set():
            self._drain_inbox(block=not (sl.queue or sl.active))
            if not (sl.queue or sl.active):
                continue
            try:
                ran = sl.step(sl.clock())
            except E.EngineError as e:  # quarantined engine: every request fails (candle.rs:689-696)
                self.healthy = False
                self._fail_all(str(e))
                continue
            except Exception as e:  # a host-side failure must not leave handlers waiting for ever
                self.healthy = False
                self._fail_all(f"serving loop failed: {e!r}")
                continue
            if ran:
                self.steps += 1
            self._publish()
            if not ran:
                time.sleep(self._idle)
        self._fail_all("server shutting down")


def make_app(server: ServingServer):
    from aiohttp import web

    async def completions(request: "web.Request"):
        try:
            try:
                body = await request.json()
            except (json.JSONDecodeError, UnicodeDecodeError):
                raise ApiError("InvalidRequest", "body is not JSON") from None
            if not isinstance(body, dict):
                raise ApiError("InvalidRequest", "body is not a JSON object")
            prompt = parse_prompt(body.get("prompt", ""), server.vocab_size)
            max_tokens = int(body.get("max_tokens", 128))
            temperature = float(body.get("temperature", 1.0))
            top_p = float(body.get("top_p", 1.0))
            stream = bool(body.get("stream", False))
            model = str(body.get("model", server.model))
            q: asyncio.Queue = asyncio.Queue()
            rid = server.submit(prompt, max_tokens, temperature, top_p, asyncio.get_running_loop(), q)
        except ApiError as e:
            return e.response()
        except (TypeError, ValueError) as e:
            return ApiError("InvalidRequest", str(e)).response()
        cid = f"cmpl-{uuid.uuid4()}"

        def chunk(text: str, finish: Optional[str], usage: Optional[dict]):
            c = {"id": cid, "object": "text_completion.chunk", "created": int(time.time()), "model": model,
                 "choices": [{"text": text, "index": 0, "finish_reason": finish}]}
            if usage is not None:
                c["usage"] = usage
            return c

        if stream:
            resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
            await resp.prepare(request)
            # a token chunk is this prefix + the token id + this suffix (the same JSON as chunk())
            head = json.dumps(chunk("\x00", None, None))
            pre, post = head.split("\\u0000")
            pre = "data: " + pre + " "
            post = post + "\n\n"
            finished = False
            try:
                while True:
                    ev = await q.get()
                    if ev[0] == "token":
                        await resp.write(f"{pre}{ev[1]}{post}".encode())
                    elif ev[0] == "done":
                        finished = True
                        await resp.write(f"data: {json.dumps(chunk('', ev[1], ev[2]))}\n\ndata: [DONE]\n\n".encode())
                        break
                    else:
                        finished = True
                        err = {"error": {"message": ev[1], "type": "server_error", "code": 500}}
                        await resp.write(f"data: {json.dumps(err)}\n\n".encode())
                        break
                await resp.write_eof()
            except (ConnectionError, asyncio.CancelledError):
                if not finished:  # the client went away mid-stream
                    server.cancel(rid)
                raise
            return resp
        text = []
        while True:
            try:
                ev = await q.get()
            except asyncio.CancelledError:  # the client went away
                server.cancel(rid)
                raise
            if ev[0] == "token":
                text.append(f" {ev[1]}")
            elif ev[0] == "done":
                return web.json_response({
                    "id": cid, "object": "text_completion", "created": int(time.time()), "model": model,
                    "choices": [{"text": "".join(text), "index": 0, "logprobs": None, "finish_reason": ev[1]}],
                    "usage": ev[2]})
            else:
                return ApiError("BackendError", ev[1]).response()

    async def models(_request):
        now = int(time.time())
        return web.json_response({"object": "list", "data": [
            {"id": server.model, "object": "model", "created": now, "owned_by": "rlse"}]})

    async def health(_request):
        return web.json_response({"status": "ok", "model": server.model, "models": [server.model],
                                  "device": "cuda", "workers": 1})

    async def ready(_request):
        return web.json_response({"ready": server.healthy}, status=200 if server.healthy else 503)

    app = web.Application(client_max_size=64 * 1024 * 1024)
    app.router.add_post("/v1/completions", completions)
    app.router.add_get("/v1/models", models)
    app.router.add_get("/health", health)
    app.router.add_get("/ready", ready)
    return app


class BackgroundHttp:
    """The aiohttp app on its own event loop thread (127.0.0.1, port 0 = any free port)."""

    def __init__(self, server: ServingServer, host: str = "127.0.0.1", port: int = 0):
        self.server, self.host, self.port = server, host, port
        self._loop = asyncio.new_event_loop()
        self._ready = threading.Event()
        self._thread = threading.Thread(target=self._main, name="ms-http", daemon=True)
        self._runner = None
        self.url = ""

    def _main(self):
        from aiohttp import web
        asyncio.set_event_loop(self._loop)

        async def up():
            self._runner = web.AppRunner(make_app(self.server), access_log=None)
            await self._runner.setup()
            site = web.TCPSite(self._runner, self.host, self.port)
            await site.start()
            sock = site._server.sockets[0]
            self.url = f"http://{self.host}:{sock.getsockname()[1]}"
            self._ready.set()

        self._loop.run_until_complete(up())
        self._loop.run_forever()

    def start(self, timeout: float = 30.0):
        self._thread.start()
        if not self._ready.wait(timeout):
            raise RuntimeError("HTTP server did not start")
        return self

    def stop(self):
        async def down():
            await self._runner.cleanup()
        asyncio.run_coroutine_threadsafe(down(), self._loop).result(30)
        self._loop.call_soon_threadsafe(self._loop.stop)
        self._thread.join(30)


class _RemoteEngine:
    """The front-end process's view of the ServingServer in the engine process:
    the attributes and calls make_app uses, over a duplex pipe.  Submissions are
    checked here (the same checks and messages as ServingServer.submit); one
    reader thread hands each flush's events to the event loop in one wake-up."""

    def __init__(self, conn, model: str, vocab_size: int, max_context: int):
        self.conn, self.model, self.vocab_size, self.max_context = conn, model, vocab_size, max_context
        self.healthy = True
        self._rid = 1 << 32  # apart from the ids of in-process submissions
        self._subs: Dict[int, asyncio.Queue] = {}
        self._loop: Optional[asyncio.AbstractEventLoop] = None
        self.stopped: Optional[asyncio.Event] = None

    def start(self, loop: asyncio.AbstractEventLoop):
        self._loop = loop
        self.stopped = asyncio.Event()
        threading.Thread(target=self._reader, name="ms-frontend-rx", daemon=True).start()

    def submit(self, prompt: List[int], max_tokens: int, temperature: float, top_p: float,
               aloop: asyncio.AbstractEventLoop, q: asyncio.Queue) -> int:
        _admission_check(self.healthy, self.max_context, prompt, max_tokens)
        self._rid += 1
        rid = self._rid
        self._subs[rid] = q
        try:
            self.conn.send(("submit", rid, list(prompt), int(max_tokens), float(temperature), float(top_p)))
        except (OSError, ValueError):
            self._subs.pop(rid, None)
            raise ApiError("NoHealthyWorkers", "the engine process is gone") from None
        return rid

    def cancel(self, rid: int):
        if self._subs.pop(rid, None) is not None:
            try:
                self.conn.send(("cancel", rid))
            except (OSError, ValueError):
                pass

    def _reader(self):
        while True:
            try:
                msg = self.conn.recv()
            except (OSError, EOFError):
                msg = ("stop",)
            self._loop.call_soon_threadsafe(self._on_message, msg)
            if msg[0] == "stop":
                return

    def _on_message(self, msg):
        if msg[0] == "stop":
            self.healthy = False
            for q in self._subs.values():
                q.put_nowait(("error", "server shutting down"))
            self._subs.clear()
            self.stopped.set()
            return
        _, self.healthy, evs = msg
        for rid, ev in evs:
            q = self._subs.get(rid)
            if q is not None:
                q.put_nowait(ev)
                if ev[0] != "token":
                    del self._subs[rid]


def _frontend_main(conn, model: str, vocab_size: int, max_context: int, host: str, port: int):
    """Entry point of the front-end process: serve make_app over the pipe until
    the engine side sends ("stop",) or closes it."""
    from aiohttp import web

    async def serve():
        eng = _RemoteEngine(conn, model, vocab_size, max_context)
        eng.start(asyncio.get_running_loop())
        runner = web.AppRunner(make_app(eng), access_log=None)
        await runner.setup()
        site = web.TCPSite(runner, host, port)
        await site.start()
        sock = site._server.sockets[0]
        conn.send(("ready", f"http://{host}:{sock.getsockname()[1]}"))
        await eng.stopped.wait()
        await runner.cleanup()

    asyncio.run(serve())
    conn.close()


class HttpFrontendProcess:
    """The aiohttp app in a separate (spawned) process, talking to `server` over
    a pipe.  The engine process then runs no HTTP or SSE code: its interpreter
    is left to the engine thread, which sends one message per step with every
    new token, and per request only a submit or cancel crosses the pipe."""

    def __init__(self, server: ServingServer, host: str = "127.0.0.1", port: int = 0):
        self.server, self.host, self.port = server, host, port
        self._proc = None
        self.url = ""

    def start(self, timeout: float = 120.0):
        import multiprocessing as mp
        ctx = mp.get_context("spawn")
        mine, theirs = ctx.Pipe(duplex=True)
        s = self.server
        self._proc = ctx.Process(target=_frontend_main, name="ms-http-frontend", daemon=True,
                                 args=(theirs, s.model, s.vocab_size, s.max_context, self.host, self.port))
        self._proc.start()
        theirs.close()
        try:
            if not mine.poll(timeout):
                raise EOFError
            kind, self.url = mine.recv()
        except EOFError:  # no answer, or the process died first (e.g. the port is taken; see its stderr)
            self._proc.kill()
            self._proc.join(5)
            raise RuntimeError(f"HTTP front-end process did not start on {self.host}:{self.port}") from None
        assert kind == "ready"
        s.attach_remote(mine)
        return self

    def stop(self, timeout: float = 30.0):
        s = self.server
        s._remote_send(("stop",))
        with s._remote_lock:
            s._remote = None
        self._proc.join(timeout)
        if self._proc.is_alive():
            self._proc.kill()
            self._proc.join(5)


# ---------------------------------------------------------------------------------------
# client
@dataclass
class StreamResult:
    tokens: int
    ttft_ms: float
    latency_ms: float
    end_to_end_tokens_per_sec: float
    observed_decode_tokens_per_sec: Optional[float]
    authoritative_usage: bool
    text: str


async def stream_completion(session, url: str, model: str, prompt, max_tokens: int,
                            temperature: float = 0.0, top_p: float = 1.0) -> StreamResult:
    """One streamed completion, measured as examples/bench.rs:61-110 does."""
    started = time.perf_counter()
    async with session.post(f"{url}/v1/completions", json={
            "model": model, "prompt": prompt, "max_tokens": max_tokens, "temperature": temperature,
            "top_p": top_p, "stream": True}) as resp:
        if resp.status >= 400:
            raise SseError("http", f"HTTP {resp.status}: {await resp.text()}")
        if not resp.headers.get("Content-Type", "").startswith("text/event-stream"):
            raise SseError("http", "the response is not text/event-stream")
        parser = CompletionStream()
        first = last = None
        async for data in resp.content.iter_any():
            before = parser.token_events
            parser.push(data)
            if parser.token_events > before:
                now = time.perf_counter() - started
                if first is None:
                    first = now
                last = now
    tokens = parser.finish()
    elapsed = time.perf_counter() - started
    if first is None:
        raise SseError("tokens", "the completed stream carried no generated token")
    decode = last - first
    return StreamResult(tokens, first * 1000.0, elapsed * 1000.0, tokens / elapsed,
                        (tokens - 1) / decode if tokens > 1 and decode > 0 else None,
                        parser.completion_tokens is not None, parser.text)


async def _run_trace(url: str, model: str, reqs: Sequence[Request], timeout_s: float):
    import aiohttp
    t0 = time.perf_counter()
    timeout = aiohttp.ClientTimeout(total=timeout_s)
    conn = aiohttp.TCPConnector(limit=0)
    async with aiohttp.ClientSession(timeout=timeout, connector=conn) as session:
        async def one(r: Request):
            delay = r.arrival - (time.perf_counter() - t0)
            if delay > 0:
                await asyncio.sleep(delay)
            try:
                return await stream_completion(session, url, model, r.prompt, r.max_tokens, r.temperature,
                                               r.top_p)
            except Exception as e:  # a failed request is counted, not fatal to the trace
                return e
        results = await asyncio.gather(*(one(r) for r in reqs))
    return list(results), time.perf_counter() - t0


def run_trace(url: str, model: str, reqs: Sequence[Request], timeout_s: float = 900.0):
    """Replay `reqs` (arrival offsets in seconds) against the server; returns
    (per-request StreamResult or exception, elapsed seconds)."""
    return asyncio.run(_run_trace(url, model, reqs, timeout_s))


def _trace_child(url: str, model: str, items, timeout_s: float, conn):
    reqs = [Request(i, p, m, arrival=a, temperature=t, top_p=tp) for i, (p, m, a, t, tp) in enumerate(items)]
    results, elapsed = run_trace(url, model, reqs, timeout_s)
    conn.send(([r if isinstance(r, StreamResult) else repr(r) for r in results], elapsed))
    conn.close()


def run_trace_process(url: str, model: str, reqs: Sequence[Request], timeout_s: float = 900.0):
    """run_trace in a separate (spawned) client process, as the reference's
    benchmark is a separate program: the client's SSE parsing does not share
    the server's interpreter.  Failed requests come back as strings."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe(duplex=False)
    items = [(list(r.prompt), int(r.max_tokens), float(r.arrival), float(r.temperature), float(r.top_p))
             for r in reqs]
    proc = ctx.Process(target=_trace_child, args=(url, model, items, timeout_s, child), daemon=True)
    proc.start()
    child.close()
    try:
        if not parent.poll(timeout_s + 120.0):
            raise TimeoutError("trace client did not finish")
        results, elapsed = parent.recv()
    finally:
        proc.join(30)
        if proc.is_alive():
            proc.kill()
    return results, elapsed


def summarize_http(results, elapsed: float) -> Dict[str, float]:
    """Aggregate tokens/s (bench.rs:189) and TTFT / decode-rate percentiles."""
    ok = [r for r in results if isinstance(r, StreamResult)]
    tokens = sum(r.tokens for r in ok)
    ttft = sorted(r.ttft_ms for r in ok)
    dec = sorted(r.observed_decode_tokens_per_sec for r in ok if r.observed_decode_tokens_per_sec)

    def pct(v, q):
        return v[min(len(v) - 1, int(q * len(v)))] if v else float("nan")

    return {"requests": len(results), "failed": len(results) - len(ok), "tokens": tokens, "elapsed_s": elapsed,
            "aggregate_tokens_per_s": tokens / elapsed if elapsed > 0 else 0.0,
            "ttft_ms_p50": pct(ttft, 0.5), "ttft_ms_p90": pct(ttft, 0.9), "ttft_ms_p99": pct(ttft, 0.99),
            "ttft_ms_all": ttft,
            "per_request_decode_tokens_per_s_median": pct(dec, 0.5)}
