"""OpenAI-compatible HTTP server (chat completions, JSON or server-sent events) on top of
the speculative decoder: the reference's ``openai_server.py`` interface (the same response
builders, ``messages_to_prompt``, runners, handler factory and command line), with one
B200 addition: ``BatchingRunner`` gathers the requests that arrive together and decodes
them as one batched session (``dflash_generate_batch_stream``), so concurrent clients share
every weight read instead of queueing behind each other.

    python -m dflash_b200.openai_server --target-model <dir> --draft-model <dir> [--max-batch 16]

Endpoints (reference openai_server.py:274-433): ``GET /health``, ``GET /v1/models``,
``POST /v1/chat/completions`` (``messages``, ``model``, ``max_tokens``, ``temperature``,
``stream``). Streaming answers are ``data: <json>\\n\\n`` events: a role chunk, one chunk
per text delta, a final chunk with ``finish_reason`` and ``usage``, then ``data: [DONE]``.
"""
from __future__ import annotations

import argparse
import json
import queue
import sys
import threading
import time
import uuid
from collections.abc import Iterator
from dataclasses import dataclass, field
from http import HTTPStatus
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any

OWNED_BY = "dflash-mlx"  # the reference's value: clients that list models see the same record


# ---------------------------------------------------------------------------
# response bodies (openai_server.py:15-89)
# ---------------------------------------------------------------------------
def build_health_response() -> dict[str, str]:
    return {"status": "ok"}


def build_models_response(model_id: str) -> dict[str, Any]:
    return {"object": "list", "data": [{"id": model_id, "object": "model", "owned_by": OWNED_BY}]}


def _usage(prompt_tokens: int, completion_tokens: int) -> dict[str, int]:
    return {"prompt_tokens": prompt_tokens, "completion_tokens": completion_tokens,
            "total_tokens": prompt_tokens + completion_tokens}


def build_chat_response(*, model: str, content: str, prompt_tokens: int, completion_tokens: int,
                        finish_reason: str = "stop") -> dict[str, Any]:
    return {
        "id": f"chatcmpl-{uuid.uuid4().hex}", "object": "chat.completion", "created": int(time.time()),
        "model": model,
        "choices": [{"index": 0, "message": {"role": "assistant", "content": content},
                     "finish_reason": finish_reason}],
        "usage": _usage(prompt_tokens, completion_tokens),
    }


def build_chat_stream_chunk(*, chunk_id: str, created: int, model: str, delta: dict[str, str],
                            finish_reason: str | None = None, usage: dict[str, int] | None = None) -> dict[str, Any]:
    out: dict[str, Any] = {"id": chunk_id, "object": "chat.completion.chunk", "created": created, "model": model,
                           "choices": [{"index": 0, "delta": delta, "finish_reason": finish_reason}]}
    if usage is not None:
        out["usage"] = usage
    return out


def _text_of(content: Any) -> str:
    """A message's text: a string, or text parts joined by newlines (text-only server)."""
    if isinstance(content, str):
        return content
    if not isinstance(content, list):
        raise ValueError("Unsupported message content format for text-only server.")
    texts = []
    for part in content:
        if not isinstance(part, dict):
            raise ValueError("Unsupported message content format for text-only server.")
        if part.get("type", "text") != "text":
            raise ValueError("This DFlash OpenAI-compatible server is text-only.")
        if not isinstance(part.get("text"), str):
            raise ValueError("Text content parts must include a string 'text' field.")
        texts.append(part["text"])
    return "\n".join(t for t in texts if t)


_ROLE_LABEL = {"system": "System", "user": "User", "assistant": "Assistant"}


def messages_to_prompt(messages: list[dict[str, Any]]) -> str:
    """``Role: content`` lines and a trailing ``Assistant:`` (openai_server.py:108-130)."""
    if not messages:
        raise ValueError("messages must not be empty")
    lines = []
    for msg in messages:
        if not isinstance(msg, dict):
            raise ValueError("Each message must be an object.")
        role = msg.get("role")
        if not isinstance(role, str) or not role:
            raise ValueError("Each message must include a string role.")
        lines.append(f"{_ROLE_LABEL.get(role, role.capitalize())}: {_text_of(msg.get('content', ''))}")
    lines.append("Assistant:")
    return "\n".join(lines)


# ---------------------------------------------------------------------------
# runners
# ---------------------------------------------------------------------------
@dataclass
class GenerationResult:
    text: str
    prompt_tokens: int
    completion_tokens: int
    finish_reason: str = "stop"


@dataclass
class GenerationChunk:
    delta: str
    text: str
    completion_tokens: int
    prompt_tokens: int = 0
    finish_reason: str | None = None
    finished: bool = False


def _openai_finish(reason: str | None) -> str:
    return "length" if reason == "max_tokens" else (reason or "stop")


class RunnerProtocol:
    def generate(self, *, prompt: str, max_new_tokens: int, temperature: float) -> GenerationResult:
        raise NotImplementedError

    def stream(self, *, prompt: str, max_new_tokens: int, temperature: float) -> Iterator[GenerationChunk]:
        raise NotImplementedError


def collect(chunks: Iterator[GenerationChunk]) -> GenerationResult:
    """The non-streaming result of a chunk stream."""
    last = None
    for c in chunks:
        last = c
    if last is None or not last.finished:
        raise RuntimeError("generation ended without a final chunk")
    return GenerationResult(text=last.text, prompt_tokens=last.prompt_tokens,
                            completion_tokens=last.completion_tokens, finish_reason=last.finish_reason or "stop")


class DFlashRunner(RunnerProtocol):
    """One request at a time through ``DFlashGenerator`` (openai_server.py:170-265)."""

    def __init__(self, *, target_model: str = "", draft_model: str = "", speculative_tokens: int | None = None,
                 verify_mode: str = "parallel-replay", verify_chunk_size: int = 4, seed: int = 0, generator=None):
        if generator is None:
            from .api import DFlashGenerator
            generator = DFlashGenerator(target_model=target_model, draft_model=draft_model, seed=seed)
        self.generator = generator
        self.speculative_tokens = speculative_tokens
        self.verify_mode = verify_mode
        self.verify_chunk_size = verify_chunk_size
        self._lock = threading.Lock()  # one device session at a time

    def _kw(self):
        return dict(speculative_tokens=self.speculative_tokens, verify_mode=self.verify_mode,
                    verify_chunk_size=self.verify_chunk_size, skip_special_tokens=True)

    def generate(self, *, prompt: str, max_new_tokens: int, temperature: float) -> GenerationResult:
        return collect(self.stream(prompt=prompt, max_new_tokens=max_new_tokens, temperature=temperature))

    def stream(self, *, prompt: str, max_new_tokens: int, temperature: float) -> Iterator[GenerationChunk]:
        with self._lock:
            for ev in self.generator.stream(prompt, max_new_tokens=max_new_tokens, temperature=temperature,
                                            **self._kw()):
                n = len(ev.generated_tokens)
                if not ev.finished:
                    yield GenerationChunk(delta=ev.delta, text=ev.text, completion_tokens=n)
                    continue
                if ev.delta:
                    yield GenerationChunk(delta=ev.delta, text=ev.text, completion_tokens=n)
                m = ev.metrics or {}
                yield GenerationChunk(delta="", text=ev.text, completion_tokens=n,
                                      prompt_tokens=int(m.get("num_input_tokens", 0)),
                                      finish_reason=_openai_finish(m.get("finish_reason")), finished=True)


@dataclass
class _Request:
    prompt_ids: list[int]
    max_new_tokens: int
    temperature: float
    out: "queue.Queue" = field(default_factory=queue.Queue)


class BatchingRunner(RunnerProtocol):
    """Requests arriving within ``window_s`` of each other (up to ``max_batch``, same
    temperature) are decoded together as one batched session on a single scheduler thread;
    each request's chunks flow back through its own queue. Greedy results equal the
    single-request decode of the same prompt for batches below four sequences (the same
    kernel forms); from four sequences on the batched GEMM and attention forms apply."""

    def __init__(self, generator, *, max_batch: int = 16, window_s: float = 0.005,
                 speculative_tokens: int | None = None, decode_fn=None):
        self.generator = generator
        self.max_batch = max(1, int(max_batch))
        self.window_s = float(window_s)
        self.speculative_tokens = speculative_tokens
        if decode_fn is None:
            from .runtime import dflash_generate_batch_stream

            def decode_fn(prompts, max_new, temperature):
                g = self.generator
                return dflash_generate_batch_stream(g.target.model, g.draft, prompts, max_new, temperature,
                                                    g.target.stop_token_ids(), self.speculative_tokens,
                                                    seed=getattr(g, "seed", 0))
        self._decode = decode_fn
        self._queue: queue.Queue = queue.Queue()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, name="dflash-batcher", daemon=True)
        self._thread.start()
        self.batches: list[int] = []  # sizes of the batches run (for tests and logs)

    def close(self) -> None:
        self._stop.set()
        self._queue.put(None)
        self._thread.join(timeout=10)

    # request side ----------------------------------------------------------
    def stream(self, *, prompt: str, max_new_tokens: int, temperature: float) -> Iterator[GenerationChunk]:
        req = _Request(list(self.generator.encode_prompt(prompt)), int(max_new_tokens), float(temperature))
        self._queue.put(req)
        while True:
            item = req.out.get()
            if isinstance(item, BaseException):
                raise item
            yield item
            if item.finished:
                return

    def generate(self, *, prompt: str, max_new_tokens: int, temperature: float) -> GenerationResult:
        return collect(self.stream(prompt=prompt, max_new_tokens=max_new_tokens, temperature=temperature))

    # scheduler side --------------------------------------------------------
    def _gather(self, first: _Request) -> list[_Request]:
        batch = [first]
        deadline = time.monotonic() + self.window_s
        while len(batch) < self.max_batch:
            left = deadline - time.monotonic()
            try:
                nxt = self._queue.get(timeout=max(left, 0.0)) if left > 0 else self._queue.get_nowait()
            except queue.Empty:
                break
            if nxt is None:
                self._queue.put(None)
                break
            batch.append(nxt)
        return batch

    def _loop(self) -> None:
        while not self._stop.is_set():
            first = self._queue.get()
            if first is None:
                continue
            batch = self._gather(first)
            groups: dict[float, list[_Request]] = {}
            for r in batch:  # one temperature per session (the sampling path is chosen per session)
                groups.setdefault(r.temperature, []).append(r)
            for temp, reqs in groups.items():
                self._run(reqs, temp)

    def _run(self, reqs: list[_Request], temperature: float) -> None:
        self.batches.append(len(reqs))
        tok = self.generator.target.tokenizer
        ids: list[list[int]] = [[] for _ in reqs]
        texts = [""] * len(reqs)
        try:
            for events in self._decode([r.prompt_ids for r in reqs], [r.max_new_tokens for r in reqs], temperature):
                for ev in events:
                    r = reqs[ev.index]
                    if ev.token_ids:
                        ids[ev.index].extend(ev.token_ids)
                        text = tok.decode(ids[ev.index], skip_special_tokens=True)
                        prev = texts[ev.index]
                        delta = text[len(prev):] if text.startswith(prev) else text
                        texts[ev.index] = text
                        if delta:
                            r.out.put(GenerationChunk(delta=delta, text=text, completion_tokens=len(ids[ev.index])))
                    if ev.finished:
                        r.out.put(GenerationChunk(delta="", text=texts[ev.index],
                                                  completion_tokens=len(ids[ev.index]),
                                                  prompt_tokens=len(r.prompt_ids),
                                                  finish_reason=_openai_finish(ev.finish_reason), finished=True))
        except BaseException as exc:  # noqa: BLE001 - handed to every waiting request
            for r in reqs:
                r.out.put(exc)


# ---------------------------------------------------------------------------
# HTTP
# ---------------------------------------------------------------------------
@dataclass
class ServerConfig:
    host: str
    port: int
    model_id: str
    runner: RunnerProtocol


def _error(kind: str, message: str) -> dict[str, Any]:
    return {"error": {"message": message, "type": kind}}


def make_handler(config: ServerConfig):
    """The request handler class bound to ``config`` (openai_server.py:274-433)."""

    class Handler(BaseHTTPRequestHandler):
        server_version = "dflash-b200-openai/0.1"
        protocol_version = "HTTP/1.1"

        def _json(self, status: int, body: dict[str, Any]) -> None:
            data = json.dumps(body).encode()
            self.send_response(status)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def _event(self, body: dict[str, Any] | str) -> None:
            data = body if isinstance(body, str) else json.dumps(body)
            self.wfile.write(f"data: {data}\n\n".encode())
            self.wfile.flush()

        def _body(self) -> dict[str, Any]:
            raw = self.rfile.read(int(self.headers.get("Content-Length") or 0))
            if not raw:
                raise ValueError("Request body is required.")
            try:
                body = json.loads(raw)
            except json.JSONDecodeError as exc:
                raise ValueError(f"Invalid JSON: {exc.msg}") from exc
            if not isinstance(body, dict):
                raise ValueError("JSON body must be an object.")
            return body

        def do_GET(self) -> None:  # noqa: N802 - http.server naming
            if self.path == "/health":
                self._json(HTTPStatus.OK, build_health_response())
            elif self.path == "/v1/models":
                self._json(HTTPStatus.OK, build_models_response(config.model_id))
            else:
                self._json(HTTPStatus.NOT_FOUND, _error("not_found_error", "Not found"))

        def _stream(self, prompt: str, model: str, max_new_tokens: int, temperature: float) -> None:
            cid, created = f"chatcmpl-{uuid.uuid4().hex}", int(time.time())
            self.send_response(HTTPStatus.OK)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.send_header("Connection", "close")
            self.end_headers()
            self.close_connection = True
            chunk = lambda delta, **kw: build_chat_stream_chunk(  # noqa: E731
                chunk_id=cid, created=created, model=model, delta=delta, **kw)
            self._event(chunk({"role": "assistant"}))
            try:
                final = None
                for c in config.runner.stream(prompt=prompt, max_new_tokens=max_new_tokens, temperature=temperature):
                    if c.finished:
                        final = c
                    elif c.delta:
                        self._event(chunk({"content": c.delta}))
                if final is None:
                    raise RuntimeError("Streaming generation did not produce a final chunk.")
                self._event(chunk({}, finish_reason=final.finish_reason or "stop",
                                  usage=_usage(final.prompt_tokens, final.completion_tokens)))
            except Exception as exc:  # noqa: BLE001 - the status line is already sent
                self._event(_error("server_error", str(exc)))
            finally:
                self._event("[DONE]")

        def do_POST(self) -> None:  # noqa: N802 - http.server naming
            if self.path != "/v1/chat/completions":
                self._json(HTTPStatus.NOT_FOUND, _error("not_found_error", "Not found"))
                return
            try:
                body = self._body()
                messages = body.get("messages")
                if not isinstance(messages, list):
                    raise ValueError("'messages' must be a list.")
                prompt = messages_to_prompt(messages)
                model = str(body.get("model") or config.model_id)
                max_new_tokens = int(body.get("max_tokens", 256))
                temperature = float(body.get("temperature", 0.0))
                if max_new_tokens < 0:
                    raise ValueError("'max_tokens' must be non-negative.")
                if body.get("stream"):
                    self._stream(prompt, model, max_new_tokens, temperature)
                    return
                res = config.runner.generate(prompt=prompt, max_new_tokens=max_new_tokens, temperature=temperature)
                self._json(HTTPStatus.OK, build_chat_response(
                    model=model, content=res.text, prompt_tokens=res.prompt_tokens,
                    completion_tokens=res.completion_tokens, finish_reason=res.finish_reason))
            except ValueError as exc:
                self._json(HTTPStatus.BAD_REQUEST, _error("invalid_request_error", str(exc)))
            except Exception as exc:  # noqa: BLE001 - reported to the client
                self._json(HTTPStatus.INTERNAL_SERVER_ERROR, _error("server_error", str(exc)))

        def log_message(self, fmt: str, *args: Any) -> None:
            sys.stderr.write("[dflash-openai] " + fmt % args + "\n")

    return Handler


def make_server(config: ServerConfig) -> ThreadingHTTPServer:
    server = ThreadingHTTPServer((config.host, config.port), make_handler(config))
    server.daemon_threads = True
    return server


def parse_args(argv: list[str] | None = None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(description="OpenAI-compatible HTTP server for dflash-b200.")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8098)
    ap.add_argument("--model-id", default="dflash-mlx")
    ap.add_argument("--target-model", required=True)
    ap.add_argument("--draft-model", required=True)
    ap.add_argument("--max-speculative-tokens", type=int, default=None)
    ap.add_argument("--verify-mode", default="parallel-replay",
                    choices=["stream", "chunked", "parallel-replay", "parallel-lazy-logits", "parallel-greedy-argmax"])
    ap.add_argument("--verify-chunk-size", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--max-batch", type=int, default=16,
                    help="requests decoded together (1 = one request at a time, as the reference)")
    ap.add_argument("--batch-window-ms", type=float, default=5.0,
                    help="how long the scheduler waits for more requests before starting a batch")
    return ap.parse_args(argv)


def main(argv: list[str] | None = None) -> None:
    args = parse_args(argv)
    if args.max_batch > 1:
        from .api import DFlashGenerator
        gen = DFlashGenerator(target_model=args.target_model, draft_model=args.draft_model, seed=args.seed)
        runner: RunnerProtocol = BatchingRunner(gen, max_batch=args.max_batch, window_s=args.batch_window_ms / 1e3,
                                                speculative_tokens=args.max_speculative_tokens)
    else:
        runner = DFlashRunner(target_model=args.target_model, draft_model=args.draft_model,
                              speculative_tokens=args.max_speculative_tokens, verify_mode=args.verify_mode,
                              verify_chunk_size=args.verify_chunk_size, seed=args.seed)
    config = ServerConfig(host=args.host, port=args.port, model_id=args.model_id, runner=runner)
    server = make_server(config)
    print(f"Serving DFlash OpenAI-compatible API on http://{config.host}:{config.port}")
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        server.server_close()


if __name__ == "__main__":
    main()
