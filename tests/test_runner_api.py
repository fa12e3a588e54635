"""Runner + OpenAI API over the mock engine (CPU).

Covers the intent of the reference's runner unit tests
(crates/cascadia-runner/src/lib.rs:1284-2292: failing / stalling / multi-task
engines, cancel semantics) and API tests (crates/cascadia-api/src/lib.rs:2619+).
"""
import json
import threading
import time

import pytest
from fastapi.testclient import TestClient

from cascadia_b200.api.server import ApiConfig, make_app
from cascadia_b200.api.toolcalls import parse_tool_calls
from cascadia_b200.engine import base as eb
from cascadia_b200.engine.mock import MockBuilder, MockEngine
from cascadia_b200.runtime.runner import RelayExit, Runner
from cascadia_b200.types import (Chunk, FinishReason, GenerationTask, PeerLayout, ShardPlan,
                                 ShardSpec)


def _runner():
    r = Runner(MockBuilder(), model_id="mock", device="cpu")
    r.start(PeerLayout(), ShardSpec("mock", 0, 1, 1))
    return r


def test_shard_plan_uniform_remainder_to_last():
    p = ShardPlan.uniform("m", 16, 2048, 32, 128256, 3)
    assert [(s.layer_start, s.layer_end) for s in p.stages] == [(0, 5), (5, 10), (10, 16)]
    assert p.stages[0].is_first_stage and p.stages[-1].is_last_stage
    with pytest.raises(ValueError):
        ShardPlan.uniform("m", 2, 1, 1, 1, 3)


def test_connection_fatal_classification():
    assert eb.Backend("Connection reset by peer").is_connection_fatal()
    assert eb.Backend("socket closed").is_connection_fatal()
    assert not eb.Backend("shape mismatch").is_connection_fatal()
    assert not eb.BatchAborted("connection reset").is_connection_fatal()
    assert eb.NotConnected().is_connection_fatal()
    assert eb.IoError("timeout").is_connection_fatal()
    assert eb.TaskError("t", eb.Backend("broken pipe")).is_connection_fatal()
    assert not eb.QueueFull(1, 1).is_connection_fatal()
    assert eb.classify_exception(ConnectionResetError(104, "x")).is_connection_fatal()


def test_chunk_token_count_and_json():
    assert Chunk.token("t", 1, "a").token_count() == 1
    assert Chunk.final_marker("t").token_count() == 0
    assert Chunk.token("t", 1, "ab").with_n_tokens(3).token_count() == 3
    d = Chunk.final_marker("t").with_finish_reason(FinishReason.LENGTH).to_dict()
    assert d["finish_reason"] == "length" and "n_tokens" not in d


def test_mock_engine_echo_and_finish_reasons():
    e = MockEngine()
    e.submit(GenerationTask("a", "one two three", max_tokens=2))
    out = []
    while True:
        (tid, c), = e.step()
        out.append(c)
        if c.is_final:
            break
    assert "".join(c.text for c in out) == "one two "
    assert out[-1].finish_reason is FinishReason.LENGTH
    e.submit(GenerationTask("b", "x", max_tokens=5))
    e.step()
    (_, c), = e.step()
    assert c.finish_reason is FinishReason.STOP


def test_runner_generate_concurrent_streams():
    r = _runner()
    streams = [r.generate(GenerationTask(f"t{i}", " ".join(f"w{i}_{j}" for j in range(5))))
               for i in range(8)]
    texts = [s.collect() for s in streams]
    for i, t in enumerate(texts):
        assert t.split() == [f"w{i}_{j}" for j in range(5)]
    r.close()


def test_runner_cancel_and_tombstone():
    r = _runner()
    s = r.generate(GenerationTask("c1", " ".join(["w"] * 1000), max_tokens=1000))
    it = iter(s)
    next(it)
    r.cancel("c1")
    rest = list(it)
    assert rest[-1].is_final and rest[-1].finish_reason is FinishReason.CANCELLED
    # A late submit of a cancelled id is dropped immediately.
    s2 = r.generate(GenerationTask("c1", "again"))
    last = list(s2)[-1]
    assert last.finish_reason is FinishReason.CANCELLED
    r.close()


def test_runner_engine_error_fails_streams_then_recovers():
    r = _runner()
    r.engine.fail_next_step("boom")
    s = r.generate(GenerationTask("e1", "a b c"))
    chunks = list(s)
    assert chunks[-1].error is not None and "boom" in chunks[-1].error
    s2 = r.generate(GenerationTask("e2", "a b"))
    assert s2.collect().split() == ["a", "b"]
    r.close()


def test_runner_error_sentinel():
    r = _runner()
    chunks = list(r.generate(GenerationTask("e3", "__engine_error__")))
    assert chunks[-1].error == "mock injected engine failure"
    r.close()


class _Fatal(eb.Engine):
    def __init__(self, fatal_after=2):
        self.n, self.fatal_after = 0, fatal_after

    def submit(self, task):
        pass

    def step(self):
        self.n += 1
        if self.n >= self.fatal_after:
            raise ConnectionResetError(104, "Connection reset by peer")
        raise eb.Backend("transient")


def test_relay_loop_exits_on_connection_fatal():
    r = Runner(MockBuilder())
    r.start_with_engine(_Fatal(2), drive=False)
    t0 = time.time()
    assert r.run_relay_loop() is RelayExit.CONNECTION_FATAL
    assert time.time() - t0 >= 0.19  # one non-fatal backoff


def test_relay_loop_slot_empty_on_close():
    r = Runner(MockBuilder())
    r.start_with_engine(MockEngine(), drive=False)
    threading.Timer(0.1, r.close).start()
    assert r.run_relay_loop() is RelayExit.SLOT_EMPTY


# ------------------------------------------------------------------- API

@pytest.fixture
def client():
    r = _runner()
    app = make_app(r, ApiConfig(model_name="mock"))
    with TestClient(app) as c:
        yield c
    r.close()


def test_health_models_metrics(client):
    assert client.get("/health").json() == {"status": "ok"}
    assert client.get("/v1/models").json()["data"][0]["id"] == "mock"
    assert b"cascadia_http_requests_total" in client.get("/metrics").content


def test_chat_nonstream(client):
    r = client.post("/v1/chat/completions", json={
        "model": "mock", "messages": [{"role": "user", "content": "hello world"}],
        "max_tokens": 50})
    assert r.status_code == 200
    j = r.json()
    assert j["object"] == "chat.completion"
    assert "hello" in j["choices"][0]["message"]["content"]
    assert j["choices"][0]["finish_reason"] == "stop"
    assert j["usage"]["completion_tokens"] > 0


def test_chat_length_finish(client):
    r = client.post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "a b c d e f g"}], "max_tokens": 2})
    assert r.json()["choices"][0]["finish_reason"] == "length"


def test_chat_stream_sse(client):
    with client.stream("POST", "/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "x y"}], "stream": True,
            "stream_options": {"include_usage": True}}) as r:
        body = b"".join(r.iter_bytes()).decode()
    frames = [f for f in body.split("\n\n") if f]
    assert frames[-1] == "data: [DONE]"
    objs = [json.loads(f[6:]) for f in frames[:-1]]
    assert objs[0]["choices"][0]["delta"]["role"] == "assistant"
    assert objs[-1]["usage"]["completion_tokens"] > 0
    assert any(o["choices"] and o["choices"][0]["finish_reason"] == "stop" for o in objs)


def test_stop_sequence_trimmed(client):
    r = client.post("/v1/completions", json={"prompt": "alpha beta STOP gamma", "stop": "STOP",
                                             "max_tokens": 20})
    j = r.json()
    assert j["choices"][0]["text"] == "alpha beta "
    assert j["choices"][0]["finish_reason"] == "stop"


def test_stop_sequence_stream(client):
    with client.stream("POST", "/v1/completions", json={
            "prompt": "alpha beta STOP gamma", "stop": ["STOP"], "stream": True}) as r:
        body = b"".join(r.iter_bytes()).decode()
    objs = [json.loads(f[6:]) for f in body.split("\n\n") if f and f != "data: [DONE]"]
    text = "".join(o["choices"][0]["text"] for o in objs if o["choices"])
    assert text == "alpha beta " and "gamma" not in body


def test_rejections(client):
    assert client.post("/v1/chat/completions", json={"messages": []}).status_code == 400
    big = "a " * 20000
    assert client.post("/v1/completions", json={"prompt": big}).status_code == 413
    assert client.post("/v1/completions", json={"prompt": ["a", "b"]}).status_code == 400
    huge = "x" * (70 * 1024)
    assert client.post("/v1/completions", json={"prompt": huge}).status_code == 413


def test_engine_error_latches_health(client):
    r = client.post("/v1/completions", json={"prompt": "__engine_error__"})
    assert r.status_code == 500
    assert client.get("/health").status_code == 503
    assert client.post("/v1/completions", json={"prompt": "ok"}).status_code == 200
    assert client.get("/health").status_code == 200


def test_cancel_route(client):
    assert client.post("/v1/cancel/abc").json() == {"cancelled": "abc"}


def test_tool_call_dialects():
    c = parse_tool_calls('<tool_call>{"name": "f", "arguments": {"x": "</tool_call>"}}</tool_call>')
    assert c[0].name == "f" and json.loads(c[0].arguments) == {"x": "</tool_call>"}
    c = parse_tool_calls("<tool_call><function=get><parameter=city>Paris</parameter></function>"
                         "</tool_call>")
    assert c[0].name == "get" and json.loads(c[0].arguments) == {"city": "Paris"}
    c = parse_tool_calls("<tool_call>lookup<arg_key>q</arg_key><arg_value>7</arg_value>"
                         "</tool_call>")
    assert c[0].name == "lookup" and json.loads(c[0].arguments) == {"q": 7}
    assert parse_tool_calls('{"name": "Alice", "age": 30}') is None
    c = parse_tool_calls('<|python_tag|>{"name": "f", "parameters": {}}')
    assert c[0].name == "f"
