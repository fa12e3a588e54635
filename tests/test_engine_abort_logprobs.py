"""Engine behaviour that needs no GPU fault to test:

* a non-zero device status word (what a kernel's bounded wait writes when a
  peer or a copy never arrives) fails the batch that just ran with one error
  chunk per sequence, frees its KV, and the engine then serves the next
  request normally (the reference's BatchAborted semantics);
* per-token logprobs / top_logprobs through the engine and the OpenAI API;
* the engine-step and speculative-decoding metrics are updated.

The status word is written from the host, so no kernel is made to time out.
"""
import math

import torch
from fastapi.testclient import TestClient

from cascadia_b200 import metrics, ops
from cascadia_b200.api.server import ApiConfig, make_app
from cascadia_b200.engine.llm import LLMBuilder, LLMEngine
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.runtime.runner import Runner
from cascadia_b200.types import FinishReason, GenerationTask, PeerLayout, ShardSpec


def _engine(**kw):
    cfg = get_config("tiny-llama")
    m = LlamaModel(cfg, "cpu").init_random(seed=21, gen_device="cpu")
    m.allocate_kv(256)
    return LLMEngine(m, max_model_len=512, **kw)


def _drain(e, ids, max_steps=200):
    out = {t: [] for t in ids}
    for _ in range(max_steps):
        for tid, c in e.step():
            out.setdefault(tid, []).append(c)
        if all(out[t] and out[t][-1].is_final for t in ids):
            break
    return out


def test_device_status_aborts_batch_then_engine_serves_next():
    e = _engine()
    status = ops.status_buffer(torch.device("cpu"))
    status.zero_()
    for i in range(2):
        e.submit(GenerationTask(f"a{i}", "", max_tokens=20, prompt_ids=list(range(5, 20 + i))))
    first = e.step()  # prefill: one token per sequence
    assert {tid for tid, _ in first} == {"a0", "a1"}
    status.fill_(301)  # as a peer-signal timeout inside the next forward would
    out = e.step()
    errs = [c for _, c in out if c.error is not None]
    assert sorted(c.task_id for c in errs) == ["a0", "a1"]
    assert all(c.is_final and "batch aborted" in c.error and "301" in c.error for c in errs)
    assert not [c for _, c in out if c.error is None]  # no token from the failed forward
    assert int(status.item()) == 0                     # cleared by the read
    assert e.aborted_batches == 1
    assert e.model.kv.allocator.num_free == e.model.kv.num_blocks
    assert not e.has_work()
    # The next request runs to completion, with the tokens of a fresh engine.
    res = _drain(e, ["b"]) if e.submit(GenerationTask("b", "", max_tokens=4,
                                                      prompt_ids=[7, 8, 9])) is None else None
    fresh = _engine()
    fresh.submit(GenerationTask("b", "", max_tokens=4, prompt_ids=[7, 8, 9]))
    ref = _drain(fresh, ["b"])
    assert res["b"][-1].finish_reason in (FinishReason.LENGTH, FinishReason.STOP)
    assert [c.token_id for c in res["b"] if not c.is_final] == \
        [c.token_id for c in ref["b"] if not c.is_final]


def test_abort_in_prefill_fails_only_that_batch():
    e = _engine()
    status = ops.status_buffer(torch.device("cpu"))
    status.fill_(104)
    e.submit(GenerationTask("p", "", max_tokens=3, prompt_ids=[3, 4, 5, 6]))
    out = e.step()
    assert len(out) == 1 and out[0][1].error is not None and "104" in out[0][1].error
    status.zero_()
    e.submit(GenerationTask("q", "", max_tokens=3, prompt_ids=[3, 4, 5, 6]))
    res = _drain(e, ["q"])
    assert res["q"][-1].error is None and res["q"][-1].is_final


def test_engine_logprobs_match_log_softmax_of_greedy_path():
    e = _engine()
    e.submit(GenerationTask("l", "", max_tokens=5, logprobs=3, prompt_ids=[9, 10, 11, 12]))
    res = _drain(e, ["l"])
    toks = [c for c in res["l"] if not c.is_final or c.token_id]
    lps = [c.logprobs for c in res["l"] if c.logprobs is not None]
    assert len(lps) == 5
    for lp in lps:
        assert len(lp.top_logprobs) == 3
        vals = [t.logprob for t in lp.top_logprobs]
        assert vals == sorted(vals, reverse=True) and all(v <= 0 for v in vals)
        # Greedy: the chosen token is the most likely one.
        assert lp.token_id == lp.top_logprobs[0].token_id
        assert math.isclose(lp.logprob, vals[0], rel_tol=1e-6, abs_tol=1e-6)
        assert sum(math.exp(v) for v in vals) <= 1.0 + 1e-5
    assert toks


def test_api_logprobs_chat_and_completions():
    b = LLMBuilder("tiny-llama", device="cpu", kv_blocks=256, max_model_len=512)
    r = Runner(b, model_id="tiny", device="cpu")
    r.start(PeerLayout(), ShardSpec("tiny", 0, 2, 2))
    with TestClient(make_app(r, ApiConfig(model_name="tiny"))) as c:
        j = c.post("/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hello"}], "max_tokens": 4,
            "logprobs": True, "top_logprobs": 2}).json()
        content = j["choices"][0]["logprobs"]["content"]
        assert len(content) == j["usage"]["completion_tokens"]
        assert all(len(x["top_logprobs"]) == 2 and x["logprob"] <= 0 for x in content)
        # logprobs without top_logprobs: one alternative (the reference's default).
        j = c.post("/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hello"}], "max_tokens": 3,
            "logprobs": True}).json()
        assert all(len(x["top_logprobs"]) == 1 for x in j["choices"][0]["logprobs"]["content"])
        # Not requested: no logprobs object on chat choices.
        j = c.post("/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hello"}], "max_tokens": 3}).json()
        assert "logprobs" not in j["choices"][0]
        # Legacy completions: `logprobs` is the count.
        j = c.post("/v1/completions", json={"prompt": "hi there", "max_tokens": 3,
                                            "logprobs": 4}).json()
        content = j["choices"][0]["logprobs"]["content"]
        assert len(content) == 3 and all(len(x["top_logprobs"]) == 4 for x in content)
        # Streaming: every frame with text carries the logprobs of its tokens.
        with c.stream("POST", "/v1/chat/completions", json={
                "messages": [{"role": "user", "content": "hello"}], "max_tokens": 3,
                "stream": True, "logprobs": True}) as resp:
            body = b"".join(resp.iter_bytes()).decode()
        import json as _json
        frames = [_json.loads(l[6:]) for l in body.splitlines()
                  if l.startswith("data: {")]
        n = sum(len(f["choices"][0].get("logprobs", {}).get("content", []))
                for f in frames if f.get("choices"))
        assert n >= 1
    r.close()


def test_step_metrics_recorded():
    def count(phase):
        for m in metrics.STEP_SECONDS.collect():
            for s in m.samples:
                if s.name.endswith("_count") and s.labels.get("phase") == phase \
                        and s.labels.get("model") == "mtest":
                    return s.value
        return 0.0

    e = _engine(model_id="mtest")
    before = count("decode"), count("prefill")
    e.submit(GenerationTask("m", "", max_tokens=3, prompt_ids=[3, 4, 5]))
    _drain(e, ["m"])
    assert count("prefill") > before[1] and count("decode") > before[0]
