"""OpenAI-compatible server (no GPU): the reference's own expectations for the message
and response shapes (reference tests/test_openai_server.py), the HTTP wire format over a
live 127.0.0.1 socket with a stub runner, and the batching scheduler with a fake decoder."""
import http.client
import json
import threading
import time

import pytest

from dflash_b200 import openai_server as S


# --- the reference's expectations -------------------------------------------------------
def test_server_module_has_main():
    assert callable(S.main)


def test_messages_join_text_parts():
    p = S.messages_to_prompt([{"role": "system", "content": "You are helpful."},
                              {"role": "user", "content": [{"type": "text", "text": "Summarize this."},
                                                           {"type": "text", "text": "Keep it short."}]}])
    assert p == "System: You are helpful.\nUser: Summarize this.\nKeep it short.\nAssistant:"


def test_messages_reject_non_text_parts():
    with pytest.raises(ValueError, match="text-only"):
        S.messages_to_prompt([{"role": "user", "content": [{"type": "image_url", "image_url": {"url": "x"}}]}])
    with pytest.raises(ValueError):
        S.messages_to_prompt([])
    with pytest.raises(ValueError):
        S.messages_to_prompt([{"content": "no role"}])


def test_chat_response_shape():
    d = S.build_chat_response(model="m", content="Hello.", prompt_tokens=12, completion_tokens=4)
    assert d["object"] == "chat.completion" and d["model"] == "m"
    assert d["choices"][0]["message"] == {"role": "assistant", "content": "Hello."}
    assert d["choices"][0]["finish_reason"] == "stop"
    assert d["usage"] == {"prompt_tokens": 12, "completion_tokens": 4, "total_tokens": 16}


def test_stream_chunk_models_health_shapes():
    assert S.build_chat_stream_chunk(chunk_id="c", created=1, model="m", delta={"content": "Hel"}) == {
        "id": "c", "object": "chat.completion.chunk", "created": 1, "model": "m",
        "choices": [{"index": 0, "delta": {"content": "Hel"}, "finish_reason": None}]}
    assert S.build_models_response("m") == {"object": "list",
                                             "data": [{"id": "m", "object": "model", "owned_by": "dflash-mlx"}]}
    assert S.build_health_response() == {"status": "ok"}


# --- HTTP over a live socket ----------------------------------------------------------------
class StubRunner(S.RunnerProtocol):
    def stream(self, *, prompt, max_new_tokens, temperature):
        words = ["Hel", "lo", " world"][:max_new_tokens]
        text = ""
        for w in words:
            text += w
            yield S.GenerationChunk(delta=w, text=text, completion_tokens=len(text))
        yield S.GenerationChunk(delta="", text=text, completion_tokens=len(words), prompt_tokens=len(prompt.split()),
                                finish_reason="length" if max_new_tokens < 3 else "stop", finished=True)

    def generate(self, *, prompt, max_new_tokens, temperature):
        return S.collect(self.stream(prompt=prompt, max_new_tokens=max_new_tokens, temperature=temperature))


@pytest.fixture()
def server():
    srv = S.make_server(S.ServerConfig(host="127.0.0.1", port=0, model_id="local/dflash", runner=StubRunner()))
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    yield srv.server_address[1]
    srv.shutdown()
    srv.server_close()


def _req(port, method, path, body=None):
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=10)
    c.request(method, path, body=json.dumps(body) if isinstance(body, dict) else body,
              headers={"Content-Type": "application/json"})
    r = c.getresponse()
    data = r.read().decode()
    c.close()
    return r.status, r.getheader("Content-Type"), data


def test_http_get_endpoints(server):
    assert _req(server, "GET", "/health")[2] == '{"status": "ok"}'
    st, _, d = _req(server, "GET", "/v1/models")
    assert st == 200 and json.loads(d)["data"][0]["id"] == "local/dflash"
    assert _req(server, "GET", "/nope")[0] == 404


def test_http_chat_json(server):
    st, ct, d = _req(server, "POST", "/v1/chat/completions",
                     {"messages": [{"role": "user", "content": "hi there"}], "max_tokens": 2})
    assert st == 200 and ct == "application/json"
    d = json.loads(d)
    assert d["model"] == "local/dflash"
    assert d["choices"][0]["message"]["content"] == "Hello"
    assert d["choices"][0]["finish_reason"] == "length"
    assert d["usage"]["completion_tokens"] == 2


def test_http_chat_sse(server):
    st, ct, d = _req(server, "POST", "/v1/chat/completions",
                     {"messages": [{"role": "user", "content": "hi"}], "stream": True, "model": "x"})
    assert st == 200 and ct == "text/event-stream"
    events = [e[len("data: "):] for e in d.split("\n\n") if e]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant"}
    assert "".join(c["choices"][0]["delta"].get("content", "") for c in chunks) == "Hello world"
    assert chunks[-1]["choices"][0]["finish_reason"] == "stop" and "usage" in chunks[-1]
    assert all(c["model"] == "x" and c["id"] == chunks[0]["id"] for c in chunks)


def test_http_errors(server):
    assert _req(server, "POST", "/v1/chat/completions", "not json")[0] == 400
    assert _req(server, "POST", "/v1/chat/completions", {"messages": "x"})[0] == 400
    assert _req(server, "POST", "/v1/other", {"messages": []})[0] == 404
    st, _, d = _req(server, "POST", "/v1/chat/completions", {"messages": []})
    assert st == 400 and json.loads(d)["error"]["type"] == "invalid_request_error"


# --- batching scheduler ----------------------------------------------------------------------
class _Tok:
    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(ord("a") + i % 26) for i in ids)


class _Gen:
    seed = 0

    class target:  # noqa: N801 - mirrors LoadedTargetModel's attribute
        tokenizer = _Tok()

    def encode_prompt(self, text):
        return [len(w) for w in text.split()]


def _fake_decode(calls):
    """Every sequence emits its prompt length, then one token per step until max_new;
    a prompt starting with 7 stops early (stop token) after two tokens."""
    from dflash_b200.runtime import BatchStreamEvent

    def decode(prompts, max_new, temperature):
        calls.append((len(prompts), temperature))
        time.sleep(0.05)
        emitted = [0] * len(prompts)
        for step in range(max(max_new) + 1):
            evs = []
            for b, p in enumerate(prompts):
                limit = min(max_new[b], 2) if p and p[0] == 7 else max_new[b]
                if emitted[b] < limit:
                    evs.append(BatchStreamEvent(b, [p[0] + step if p else step]))
                    emitted[b] += 1
                    if emitted[b] == limit:
                        evs.append(BatchStreamEvent(b, [], True, "stop" if limit < max_new[b] else "max_tokens"))
            if evs:
                yield evs
    return decode


def test_batching_runner_groups_concurrent_requests():
    calls = []
    runner = S.BatchingRunner(_Gen(), max_batch=8, window_s=0.2, decode_fn=_fake_decode(calls))
    results = {}

    def client(i, prompt, n, temp):
        results[i] = runner.generate(prompt=prompt, max_new_tokens=n, temperature=temp)

    threads = [threading.Thread(target=client, args=(0, "ab cd", 4, 0.0)),
               threading.Thread(target=client, args=(1, "abcdefg x", 5, 0.0)),
               threading.Thread(target=client, args=(2, "abc", 3, 0.0)),
               threading.Thread(target=client, args=(3, "abc", 2, 0.7))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=20)
    runner.close()
    assert sorted(calls) == [(1, 0.7), (3, 0.0)]  # one session per temperature
    # prompt "ab cd" -> ids [2, 2]: tokens 2, 3, 4, 5 -> "cdef"
    assert results[0].text == "cdef" and results[0].finish_reason == "length"
    assert results[0].prompt_tokens == 2 and results[0].completion_tokens == 4
    # the prompt starting with 7 stops after two tokens
    assert results[1].text == "hi" and results[1].finish_reason == "stop"
    assert results[2].text == "def"
    assert results[3].text == "de"


def test_batching_runner_streams_deltas_and_reports_errors():
    calls = []
    runner = S.BatchingRunner(_Gen(), max_batch=4, window_s=0.0, decode_fn=_fake_decode(calls))
    chunks = list(runner.stream(prompt="abc", max_new_tokens=3, temperature=0.0))
    assert [c.delta for c in chunks if not c.finished] == ["d", "e", "f"]
    assert chunks[-1].finished and chunks[-1].text == "def"

    def boom(prompts, max_new, temperature):
        raise RuntimeError("device lost")
        yield  # pragma: no cover

    runner._decode = boom
    with pytest.raises(RuntimeError, match="device lost"):
        runner.generate(prompt="abc", max_new_tokens=2, temperature=0.0)
    runner.close()


def test_dflash_runner_maps_finish_reasons_with_a_fake_generator():
    """DFlashRunner turns generator events into chunks: deltas, then a final chunk whose
    finish_reason maps max_tokens -> length (openai_server.py:205-262)."""
    from types import SimpleNamespace as NS

    class FakeGen:
        def __init__(self, reason):
            self.reason = reason
            self.kw = None

        def stream(self, prompt, **kw):
            self.kw = kw
            yield NS(delta="ab", text="ab", generated_tokens=[1, 2], finished=False, metrics=None)
            yield NS(delta="c", text="abc", generated_tokens=[1, 2, 3], finished=True,
                     metrics={"num_input_tokens": 7, "finish_reason": self.reason})

    g = FakeGen("max_tokens")
    r = S.DFlashRunner(generator=g, speculative_tokens=8, verify_mode="stream")
    res = r.generate(prompt="x", max_new_tokens=3, temperature=0.0)
    assert (res.text, res.prompt_tokens, res.completion_tokens, res.finish_reason) == ("abc", 7, 3, "length")
    assert g.kw["speculative_tokens"] == 8 and g.kw["verify_mode"] == "stream" and g.kw["skip_special_tokens"]
    chunks = list(S.DFlashRunner(generator=FakeGen("stop")).stream(prompt="x", max_new_tokens=3, temperature=0.0))
    assert [c.delta for c in chunks] == ["ab", "c", ""] and chunks[-1].finish_reason == "stop"


def test_batching_runner_respects_max_batch():
    calls = []
    runner = S.BatchingRunner(_Gen(), max_batch=2, window_s=0.3, decode_fn=_fake_decode(calls))
    out = {}
    threads = [threading.Thread(target=lambda i=i: out.__setitem__(i, runner.generate(
        prompt="abc", max_new_tokens=2, temperature=0.0))) for i in range(5)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=20)
    runner.close()
    assert sum(n for n, _ in calls) == 5 and max(n for n, _ in calls) <= 2
    assert all(out[i].text == "de" for i in range(5))
