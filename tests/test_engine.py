"""Continuous-batching LLM engine: CPU oracle path (and the same on GPU)."""
import pytest
import torch
from fastapi.testclient import TestClient

from cascadia_b200.api.server import ApiConfig, make_app
from cascadia_b200.engine.llm import LLMBuilder, LLMEngine
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.runtime.generator import BatchGenerator
from cascadia_b200.runtime.runner import Runner
from cascadia_b200.types import (FinishReason, GenerationTask, PeerLayout, SamplingParams,
                                 ShardSpec)


def _engine(device="cpu", **kw):
    cfg = get_config("tiny-llama")
    m = LlamaModel(cfg, device).init_random(seed=21, gen_device="cpu")
    m.allocate_kv(kw.pop("blocks", 256))
    return LLMEngine(m, max_model_len=512, **kw)


def _run(engine, tasks, max_steps=400):
    for t in tasks:
        engine.submit(t)
    out = {t.task_id: [] for t in tasks}
    for _ in range(max_steps):
        for tid, c in engine.step():
            out[tid].append(c)
        if all(out[t.task_id] and out[t.task_id][-1].is_final for t in tasks):
            break
    return out


def _ids(chunks):
    return [c.token_id for c in chunks if not c.is_final]


@pytest.mark.parametrize("device", ["cpu", pytest.param("cuda", marks=pytest.mark.gpu)])
def test_engine_matches_batch_generator(device):
    e = _engine(device)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(3, 500, (n,), generator=g).tolist() for n in (5, 40, 17)]
    tasks = [GenerationTask(f"t{i}", "", max_tokens=6, prompt_ids=p) for i, p in enumerate(prompts)]
    out = _run(e, tasks)
    for t in tasks:
        assert out[t.task_id][-1].finish_reason in (FinishReason.LENGTH, FinishReason.STOP)
        assert out[t.task_id][-1].prompt_tokens == len(t.prompt_ids)
    # Solo runs through the same engine give identical greedy tokens.
    for i, t in enumerate(tasks):
        solo = _run(e, [GenerationTask(f"s{i}", "", max_tokens=6, prompt_ids=t.prompt_ids)])
        assert _ids(solo[f"s{i}"]) == _ids(out[t.task_id])
    assert e.model.kv.allocator.num_free == e.model.kv.num_blocks


def test_chunked_prefill_equals_whole_prefill():
    e1 = _engine()
    e2 = _engine()
    e2.sched.max_prefill_tokens = 16  # forces 3 prefill chunks for 40 tokens
    p = list(range(3, 43))
    a = _run(e1, [GenerationTask("a", "", max_tokens=5, prompt_ids=p)])
    b = _run(e2, [GenerationTask("b", "", max_tokens=5, prompt_ids=p)])
    assert _ids(a["a"]) == _ids(b["b"])


def test_prefix_cache_hit_reuses_blocks():
    e = _engine(prefix_cache_blocks=64)
    p = list(range(3, 70))  # 67 tokens -> 4 full blocks cacheable
    a = _run(e, [GenerationTask("a", "", max_tokens=4, prompt_ids=p)])
    s = e.sched
    assert len(s.prefix.map) == 4
    b = _run(e, [GenerationTask("b", "", max_tokens=4, prompt_ids=p)])
    assert _ids(a["a"]) == _ids(b["b"])


def test_cancel_frees_kv():
    e = _engine()
    e.submit(GenerationTask("c", "", max_tokens=100, prompt_ids=list(range(3, 30))))
    e.step()
    e.step()
    assert "c" in e.model.kv.seqs
    e.cancel("c")
    assert e.model.kv.allocator.num_free == e.model.kv.num_blocks
    assert not e.has_work()


def test_sampling_path_and_seed_determinism():
    e = _engine()
    sp = SamplingParams(top_k=20, top_p=0.9, seed=7)
    a = _run(e, [GenerationTask("a", "", max_tokens=6, temperature=0.9, sampling=sp,
                                prompt_ids=[5, 6, 7])])
    b = _run(e, [GenerationTask("b", "", max_tokens=6, temperature=0.9, sampling=sp,
                                prompt_ids=[5, 6, 7])])
    assert _ids(a["a"]) == _ids(b["b"])


def test_api_over_llm_engine():
    b = LLMBuilder("tiny-llama", device="cpu", kv_blocks=256, max_model_len=512)
    r = Runner(b, model_id="tiny", device="cpu")
    r.start(PeerLayout(), ShardSpec("tiny", 0, 2, 2))
    with TestClient(make_app(r, ApiConfig(model_name="tiny"))) as c:
        j = c.post("/v1/completions", json={"prompt": "hi there", "max_tokens": 5}).json()
        assert j["usage"]["completion_tokens"] == 5
        assert j["choices"][0]["finish_reason"] in ("length", "stop")
        with c.stream("POST", "/v1/chat/completions", json={
                "messages": [{"role": "user", "content": "hello"}], "max_tokens": 4,
                "stream": True}) as resp:
            body = b"".join(resp.iter_bytes()).decode()
        assert body.rstrip().endswith("data: [DONE]")
    r.close()


def test_sliding_window_generation_frees_old_blocks():
    """A window model decodes past its window: CPU attention sees only the
    window (+ sinks) and blocks wholly before it return to the pool."""
    import dataclasses

    cfg = dataclasses.replace(get_config("tiny-llama"), sliding_window=32, attention_sinks=4)
    m = LlamaModel(cfg, "cpu").init_random(seed=3, gen_device="cpu")
    m.allocate_kv(64)
    gen = BatchGenerator(m, use_graph=False)
    prompt = list(range(3, 60))
    ids = ["w"]
    gen.prefill(ids, [prompt])
    held = [b for b in m.kv.seqs["w"].blocks if b >= 0]
    assert all(b >= 0 for b in m.kv.seqs["w"].blocks)  # the prompt's queries need them all
    last = [5]
    for _ in range(20):
        last = [int(t) for t in gen.decode(ids, last, 8)]
    s = m.kv.seqs["w"]
    assert s.length == 57 + 20
    # At position 76 the window starts at 45: block 1 (16..31) went back to
    # the pool, the sink block 0 stays.
    assert s.blocks[0] >= 0 and s.blocks[1] < 0
    assert sum(b >= 0 for b in s.blocks) <= 4  # sink block + 3 window blocks
    assert len(held) >= sum(b >= 0 for b in s.blocks)
    m.kv.free_sequence("w")
    assert m.kv.allocator.num_free == m.kv.num_blocks


@pytest.mark.parametrize("preset", ["tiny-glm5", "tiny-gemma4", "tiny-gemma4-moe", "tiny-mla",
                                    "tiny-moe"])
def test_builder_serves_every_model_family(preset):
    """The builder picks the model class from the config and the engine
    serves a request end to end (CPU oracle path)."""
    from cascadia_b200.types import GenerationTask

    b = LLMBuilder(preset, device="cpu", kv_blocks=128, max_model_len=256, max_running=4)
    n = get_config(preset).num_layers
    for _ in b.load(ShardSpec(preset, 0, n, n, device="cpu")):
        pass
    e = b.build()
    out = _run(e, [GenerationTask("t", "", max_tokens=3, prompt_ids=list(range(3, 23)))])
    assert out["t"][-1].is_final and len(_ids(out["t"])) == 3


def test_builder_spec_mtp_equals_plain():
    """``--spec mtp`` through the builder: GLM-5 with its MTP head drafting
    gives the same greedy tokens as plain decoding."""
    from cascadia_b200.types import GenerationTask

    outs = []
    for spec in (None, "mtp"):
        b = LLMBuilder("tiny-glm5", device="cpu", kv_blocks=128, max_model_len=256,
                       max_running=4, spec=spec, spec_k=2)
        n = get_config("tiny-glm5").num_layers
        for _ in b.load(ShardSpec("tiny-glm5", 0, n, n, device="cpu")):
            pass
        e = b.build()
        out = _run(e, [GenerationTask("t", "", max_tokens=6, prompt_ids=list(range(3, 23)))])
        outs.append(_ids(out["t"]))
    assert outs[0] == outs[1] and len(outs[0]) == 6
