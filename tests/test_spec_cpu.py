"""Speculative decoding: n-gram draft, acceptance / reconcile arithmetic, and
spec output == plain greedy output (CPU oracle path)."""
import torch

from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.runtime.generator import BatchGenerator
from cascadia_b200.runtime.spec import (NGramDraft, SpecDecoder, count_accepted,
                                        reconcile_after_round)


def test_ngram_longest_match_and_most_recent():
    d = NGramDraft(k=4)
    d.extend([1, 2, 3, 4, 1, 2, 3, 5])
    # trailing "2 3 5"... history ends in 3,5 -> no continuation yet
    assert d.propose() == []
    d.extend([1, 2, 3])
    # 4-gram (5,1,2,3) unseen; 3-gram (1,2,3) -> most recent follower 5
    assert d.propose(1) == [5]
    assert d.propose(3)[:1] == [5]


def test_ngram_rewind_keeps_table():
    d = NGramDraft()
    d.extend([7, 8, 9, 7, 8])
    assert d.propose(1) == [9]
    d.rewind(2)
    assert d.history == [7, 8, 9]
    assert (7, 8) in d.table


def test_count_accepted_and_reconcile():
    assert count_accepted([1, 2, 3], [1, 2, 4, 9]) == 2
    assert count_accepted([], [5]) == 0
    r = reconcile_after_round(4, 2, False, False)
    assert (r.history_pop, r.kv_rewind, r.new_tokens) == (2, 2, 3)
    r = reconcile_after_round(4, 4, True, True)
    assert r.kv_rewind == 0 and r.new_tokens == 5
    r = reconcile_after_round(4, 1, False, True)
    assert r.kv_rewind == 2


def _model(seed, name="tiny-llama"):
    m = LlamaModel(get_config(name), "cpu").init_random(seed=seed, gen_device="cpu")
    m.allocate_kv(256)
    return m


def _prompts():
    g = torch.Generator().manual_seed(3)
    rep = torch.randint(3, 500, (6,), generator=g).tolist()
    return [rep * 4, torch.randint(3, 500, (11,), generator=g).tolist()]


def test_spec_ngram_equals_greedy():
    target = _model(5)
    prompts = _prompts()
    ref = BatchGenerator(target).generate(prompts, 20)
    sd = SpecDecoder(target, draft=None, ngram_k=4)
    out = sd.generate(prompts, 20)
    assert out == ref
    assert sd.stats.emitted == sum(len(o) - 1 for o in out)


def test_spec_self_draft_accepts_everything():
    target = _model(5)
    draft = _model(5)  # identical weights: every draft token is accepted
    prompts = _prompts()
    ref = BatchGenerator(target).generate(prompts, 17)
    sd = SpecDecoder(target, draft=draft, k=4)
    out = sd.generate(prompts, 17)
    assert out == ref
    assert sd.stats.accept_rate > 0.9


def test_spec_foreign_draft_still_exact():
    target = _model(5)
    draft = _model(99)
    prompts = _prompts()
    ref = BatchGenerator(target).generate(prompts, 13)
    out = SpecDecoder(target, draft=draft, k=3).generate(prompts, 13)
    assert out == ref
    # KV fully returned to the pools
    assert target.kv.allocator.num_free == target.kv.allocator.num_blocks
    assert draft.kv.allocator.num_free == draft.kv.allocator.num_blocks


def _engine_outputs(spec, draft=None, k=4):
    from cascadia_b200.engine.llm import LLMEngine
    from cascadia_b200.types import GenerationTask

    m = _model(5)
    e = LLMEngine(m, max_model_len=256, spec=spec, draft_model=draft, spec_k=k)
    tasks = [GenerationTask(f"t{i}", "", max_tokens=14, prompt_ids=p)
             for i, p in enumerate(_prompts())]
    for t in tasks:
        e.submit(t)
    out = {t.task_id: [] for t in tasks}
    fin = set()
    for _ in range(200):
        for tid, c in e.step():
            if c.is_final:
                fin.add(tid)
            else:
                out[tid].append(c.token_id)
        if len(fin) == len(tasks):
            break
    return [out[t.task_id] for t in tasks], e


def test_engine_spec_modes_equal_plain_greedy():
    plain, _ = _engine_outputs(None)
    ng, e1 = _engine_outputs("ngram")
    dr, e2 = _engine_outputs("draft", draft=_model(5))
    assert ng == plain and dr == plain
    assert e2.spec_stats.accept_rate > 0.9
    assert all(len(o) == 14 for o in plain)
    assert e1.model.kv.allocator.num_free == e1.model.kv.allocator.num_blocks
