"""OpenAI API behaviour beyond the basic routes (CPU, mock and tiny engines).

Covers the intent of the reference's API suite
(crates/cascadia-api/src/lib.rs:2619-5133: chat-template precedence and
fallback, tool-call dialects in replies and streams, usage frames, limits)
and of its runner regression tests (crates/cascadia-runner/tests/
token_wait_bound.rs: a stage whose downstream stops answering gives up on
its own deadline, fails only that request and keeps serving), plus a
solo == batched exact-match check of greedy outputs through the live API.
"""
import json
import socket
import threading
import time

import pytest
from fastapi.testclient import TestClient

from cascadia_b200.api.server import ApiConfig, make_app
from cascadia_b200.engine import base as eb
from cascadia_b200.engine.mock import MockBuilder, MockEngine
from cascadia_b200.runtime.runner import Runner
from cascadia_b200.types import Chunk, FinishReason, PeerLayout, ShardSpec

TEMPLATE = ("{% for m in messages %}[{{ m.role }}] {{ m.content }} {% endfor %}"
            "{% if tools %}TOOLS={{ tools | length }} {% endif %}"
            "{% if enable_thinking %}THINK{% else %}NOTHINK{% endif %}")


def _mock_runner(engine=None):
    r = Runner(MockBuilder(), model_id="mock", device="cpu")
    if engine is None:
        r.start(PeerLayout(), ShardSpec("mock", 0, 1, 1))
    else:
        r.start_with_engine(engine)
    return r


@pytest.fixture
def tclient():
    r = _mock_runner()
    with TestClient(make_app(r, ApiConfig(model_name="mock", chat_template=TEMPLATE))) as c:
        yield c
    r.close()


def _chat(c, **kw):
    body = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 64}
    body.update(kw)
    return c.post("/v1/chat/completions", json=body)


def _sse(c, path, body):
    with c.stream("POST", path, json=body) as r:
        text = b"".join(r.iter_bytes()).decode()
    frames = [f for f in text.split("\n\n") if f]
    assert frames[-1] == "data: [DONE]"
    return [json.loads(f[6:]) for f in frames[:-1]]


# ---------------------------------------------------------- chat templates

def test_template_renders_messages_and_thinking_default(tclient):
    # The mock engine echoes the rendered prompt word by word.
    out = _chat(tclient).json()["choices"][0]["message"]["content"]
    assert out.split() == ["[user]", "hi", "THINK"]


def test_thinking_precedence(tclient):
    def rendered(**kw):
        return _chat(tclient, **kw).json()["choices"][0]["message"]["content"].split()[-1]

    assert rendered(enable_thinking=False) == "NOTHINK"
    assert rendered(reasoning_effort="none") == "NOTHINK"
    # chat_template_kwargs wins over the top-level flag and reasoning_effort.
    assert rendered(enable_thinking=False,
                    chat_template_kwargs={"enable_thinking": True}) == "THINK"
    assert rendered(reasoning_effort="none",
                    chat_template_kwargs={"enable_thinking": True}) == "THINK"
    assert rendered(enable_thinking=True,
                    chat_template_kwargs={"enable_thinking": False}) == "NOTHINK"


def test_template_sees_tools_and_content_parts(tclient):
    tools = [{"type": "function", "function": {"name": "f", "parameters": {}}}]
    j = _chat(tclient, tools=tools, tool_choice="none",
              messages=[{"role": "system", "content": "sys"},
                        {"role": "user", "content": [{"type": "text", "text": "part"}]}]).json()
    words = j["choices"][0]["message"]["content"].split()
    assert words[:2] == ["[system]", "sys"] and "TOOLS=1" in words


def test_broken_template_falls_back_to_transcript():
    r = _mock_runner()
    with TestClient(make_app(r, ApiConfig(chat_template="{% for %}"))) as c:
        out = _chat(c).json()["choices"][0]["message"]["content"]
    r.close()
    assert out.split() == ["user:", "hi", "assistant:"]


def test_no_template_uses_transcript():
    r = _mock_runner()
    with TestClient(make_app(r, ApiConfig())) as c:
        out = _chat(c, messages=[{"role": "system", "content": "be brief"},
                                 {"role": "user", "content": "q"}]).json()
    r.close()
    assert out["choices"][0]["message"]["content"].split() == [
        "system:", "be", "brief", "user:", "q", "assistant:"]


# -------------------------------------------------------------- tool calls

CALL = '<tool_call>{"name": "get_weather", "arguments": {"city": "Paris"}}</tool_call>'
TOOLS = [{"type": "function", "function": {"name": "get_weather", "parameters": {}}}]


@pytest.fixture
def plain():
    r = _mock_runner()
    with TestClient(make_app(r, ApiConfig(model_name="mock"))) as c:
        yield c
    r.close()


def test_tool_call_reply(plain):
    # The transcript fallback puts the user text in the prompt; the mock echoes it.
    j = _chat(plain, tools=TOOLS, messages=[{"role": "user", "content": CALL}]).json()
    ch = j["choices"][0]
    assert ch["finish_reason"] == "tool_calls"
    assert ch["message"]["content"] is None
    call = ch["message"]["tool_calls"][0]
    assert call["type"] == "function" and call["function"]["name"] == "get_weather"
    assert json.loads(call["function"]["arguments"]) == {"city": "Paris"}


def test_tool_choice_none_keeps_text(plain):
    j = _chat(plain, tools=TOOLS, tool_choice="none",
              messages=[{"role": "user", "content": CALL}]).json()
    ch = j["choices"][0]
    assert "tool_calls" not in ch["message"] and "get_weather" in ch["message"]["content"]


def test_tool_call_inside_reasoning_is_ignored(plain):
    text = "<think> " + CALL + " </think> plain answer"
    j = _chat(plain, tools=TOOLS, messages=[{"role": "user", "content": text}]).json()
    assert j["choices"][0]["finish_reason"] != "tool_calls"
    # With thinking off the same text is a call.
    j = _chat(plain, tools=TOOLS, enable_thinking=False,
              messages=[{"role": "user", "content": text}]).json()
    assert j["choices"][0]["finish_reason"] == "tool_calls"


def test_tool_call_stream(plain):
    objs = _sse(plain, "/v1/chat/completions", {
        "messages": [{"role": "user", "content": CALL}], "tools": TOOLS, "stream": True})
    calls = [o for o in objs if o["choices"] and o["choices"][0]["delta"].get("tool_calls")]
    assert len(calls) == 1
    tc = calls[0]["choices"][0]["delta"]["tool_calls"][0]
    assert tc["index"] == 0 and tc["function"]["name"] == "get_weather"
    assert objs[-1]["choices"][0]["finish_reason"] == "tool_calls"
    # No call text leaks as content.
    assert not any(o["choices"] and o["choices"][0]["delta"].get("content") for o in objs)


# ------------------------------------------------------------------ usage

def test_usage_nonstream_counts(plain):
    j = plain.post("/v1/completions", json={"prompt": "a b c d", "max_tokens": 3}).json()
    u = j["usage"]
    assert u["completion_tokens"] == 3 and u["total_tokens"] == u["prompt_tokens"] + 3


def test_usage_frame_only_when_asked(plain):
    objs = _sse(plain, "/v1/completions", {"prompt": "a b", "stream": True})
    assert all("usage" not in o for o in objs)
    objs = _sse(plain, "/v1/completions", {"prompt": "a b", "stream": True,
                                           "stream_options": {"include_usage": True}})
    last = objs[-1]
    assert last["choices"] == [] and last["usage"]["completion_tokens"] == 2
    # The usage frame comes after the finishing frame.
    assert objs[-2]["choices"][0]["finish_reason"] == "stop"


def test_chat_stream_first_delta_has_role_once(plain):
    objs = _sse(plain, "/v1/chat/completions", {
        "messages": [{"role": "user", "content": "one two three"}], "stream": True})
    roles = [o for o in objs if o["choices"] and "role" in o["choices"][0]["delta"]]
    assert len(roles) == 1 and roles[0] is objs[0]
    text = "".join(o["choices"][0]["delta"].get("content", "") for o in objs if o["choices"])
    assert text.split() == ["user:", "one", "two", "three", "assistant:"]


def test_invalid_json_and_bad_body(plain):
    r = plain.post("/v1/chat/completions", content=b"{nope", headers={
        "content-type": "application/json"})
    assert r.status_code == 400
    assert plain.post("/v1/completions", json={"prompt": 5}).status_code == 400
    assert plain.post("/v1/completions", json={"prompt": "   "}).status_code == 400


# ------------------------------------------------ concurrency and cancels

class SlowMock(MockEngine):
    def __init__(self, delay=0.02):
        super().__init__()
        self.delay = delay

    def step(self):
        time.sleep(self.delay)
        return super().step()


def test_capacity_limit_rejects_then_recovers():
    eng = SlowMock(0.02)
    r = _mock_runner(eng)
    app = make_app(r, ApiConfig(max_concurrent_requests=2))
    long = " ".join(f"w{i}" for i in range(60))
    with TestClient(app) as c:
        codes = []

        def go():
            codes.append(c.post("/v1/completions", json={"prompt": long,
                                                         "max_tokens": 60}).status_code)

        ts = [threading.Thread(target=go) for _ in range(2)]
        for t in ts:
            t.start()
        deadline = time.time() + 5
        while len(eng.pending) < 2 and time.time() < deadline:
            time.sleep(0.01)
        busy = c.post("/v1/completions", json={"prompt": "x"})
        for t in ts:
            t.join(30)
        assert busy.status_code == 503
        assert codes == [200, 200]
        assert c.post("/v1/completions", json={"prompt": "y z"}).status_code == 200
    r.close()


class LiveServer:
    """The app under uvicorn on a loopback port (the test client buffers a
    whole streamed body, so streaming and disconnects need a real server)."""

    def __init__(self, app):
        import uvicorn

        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        self.port = s.getsockname()[1]
        s.close()
        self.server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=self.port,
                                                    log_level="warning", lifespan="off"))
        self.thread = threading.Thread(target=self.server.run, daemon=True)
        self.thread.start()
        deadline = time.time() + 20
        while not self.server.started and time.time() < deadline:
            time.sleep(0.02)
        assert self.server.started
        self.url = f"http://127.0.0.1:{self.port}"

    def close(self):
        self.server.should_exit = True
        self.thread.join(10)


def test_cancel_route_ends_stream_and_engine_work():
    import httpx

    eng = SlowMock(0.01)
    r = _mock_runner(eng)
    srv = LiveServer(make_app(r, ApiConfig()))
    long = " ".join(f"w{i}" for i in range(400))
    try:
        with httpx.Client(base_url=srv.url, timeout=30) as c:
            frames = []
            with c.stream("POST", "/v1/completions", json={
                    "prompt": long, "max_tokens": 400, "stream": True}) as resp:
                for line in resp.iter_lines():
                    if not line.startswith("data: {"):
                        continue
                    o = json.loads(line[6:])
                    frames.append(o)
                    if len(frames) == 3:
                        assert c.post(f"/v1/cancel/{o['id']}").status_code == 200
            n_text = sum(1 for o in frames if o["choices"] and o["choices"][0]["text"])
            assert n_text < 100
            assert frames[-1]["choices"][0]["finish_reason"] in ("cancelled", "stop")
            time.sleep(0.1)
            assert not eng.pending  # the engine dropped the task
            j = c.post("/v1/completions", json={"prompt": "after cancel"}).json()
            assert j["choices"][0]["text"].split() == ["after", "cancel"]
    finally:
        srv.close()
        r.close()


def test_client_disconnect_cancels_generation():
    import httpx

    eng = SlowMock(0.01)
    r = _mock_runner(eng)
    srv = LiveServer(make_app(r, ApiConfig()))
    long = " ".join(f"w{i}" for i in range(2000))
    try:
        t0 = time.time()
        with httpx.Client(base_url=srv.url, timeout=30) as c:
            with c.stream("POST", "/v1/completions", json={
                    "prompt": long, "max_tokens": 2000, "stream": True}) as resp:
                for line in resp.iter_lines():
                    if line.startswith("data: {"):
                        break  # leave after the first frame
        deadline = time.time() + 10
        while eng.pending and time.time() < deadline:
            time.sleep(0.02)
        assert not eng.pending, "generation kept running after the client left"
        assert time.time() - t0 < 10  # far less than the 20 s the whole stream takes
        with httpx.Client(base_url=srv.url, timeout=30) as c:
            assert c.post("/v1/completions", json={"prompt": "still serving"}).status_code == 200
    finally:
        srv.close()
        r.close()


# ------------------------------------------- bounded wait on a silent peer

class SilentDownstream(eb.Engine):
    """A pipeline head whose step waits for its downstream's reply with a
    bounded first-byte deadline; the downstream accepts the connection and
    never answers until ``answer`` is set, then the engine echoes."""

    def __init__(self, deadline_s=0.3):
        from cascadia_b200.transport.tcp import TensorLink

        self.srv = TensorLink.listen("127.0.0.1", 0)
        box = {}
        th = threading.Thread(
            target=lambda: box.setdefault("peer", TensorLink.accept(self.srv, 10)))
        th.start()
        self.link = TensorLink.connect("127.0.0.1", self.srv.port, 10)
        th.join(10)
        self.peer = box["peer"]
        self.deadline_s = deadline_s
        self.answer = False
        self.tasks = []

    def submit(self, task):
        self.tasks.append(task)

    def cancel(self, task_id):
        self.tasks = [t for t in self.tasks if t.task_id != task_id]

    def has_work(self):
        return bool(self.tasks)

    def step(self):
        if not self.tasks:
            return []
        task = self.tasks.pop(0)
        if not self.answer:
            self.link.recv(first_byte_s=self.deadline_s)  # raises FrameStartTimeout
        return [(task.task_id, Chunk.token(task.task_id, 0, "ok ")),
                (task.task_id, Chunk.final_marker(task.task_id).with_finish_reason(
                    FinishReason.STOP))]


def test_silent_downstream_fails_request_on_deadline_and_keeps_serving():
    from cascadia_b200.transport.tcp import FrameStartTimeout

    assert not FrameStartTimeout("x").is_connection_fatal()
    eng = SilentDownstream(0.3)
    r = _mock_runner(eng)
    with TestClient(make_app(r, ApiConfig())) as c:
        t0 = time.time()
        first = c.post("/v1/completions", json={"prompt": "a"})
        waited = time.time() - t0
        assert first.status_code == 500 and waited < 5.0
        assert eng.link.is_open  # the link is not dropped as connection-fatal
        eng.answer = True
        second = c.post("/v1/completions", json={"prompt": "b"})
        assert second.status_code == 200 and second.json()["choices"][0]["text"] == "ok "
    r.close()
    eng.link.close()
    eng.peer.close()
    eng.srv.close()


# ------------------------------------------- solo == batched (real engine)

def test_solo_equals_batched_greedy_through_api():
    """Greedy token ids of requests served one at a time equal those of the
    same requests served concurrently (continuous batching), on the tiny
    CPU model."""
    import torch

    from cascadia_b200.engine.llm import LLMBuilder

    b = LLMBuilder("tiny-llama", device="cpu", kv_blocks=256, max_model_len=512)
    r = Runner(b, model_id="tiny", device="cpu")
    r.start(PeerLayout(), ShardSpec("tiny", 0, 2, 2))
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(3, 400, (n,), generator=g).tolist() for n in (5, 17, 9, 30)]

    def ask(c, ids):
        j = c.post("/v1/completions", json={"prompt": "x", "prompt_token_ids": ids,
                                            "max_tokens": 8, "logprobs": 1}).json()
        return [e["token_id"] for e in j["choices"][0]["logprobs"]["content"]]

    with TestClient(make_app(r, ApiConfig(model_name="tiny"))) as c:
        solo = [ask(c, p) for p in prompts]
        batched = [None] * len(prompts)

        def go(i):
            batched[i] = ask(c, prompts[i])

        ts = [threading.Thread(target=go, args=(i,)) for i in range(len(prompts))]
        for t in ts:
            t.start()
        for t in ts:
            t.join(120)
    r.close()
    assert all(len(s) == 8 for s in solo)
    assert batched == solo
