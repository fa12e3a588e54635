"""Grammar-constrained decoding: forced runs cost one forward each and give
the same tokens as feeding them one by one; free slots take the best
allowed token."""
import torch

from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel, build_batch
from cascadia_b200.runtime.grammar import TemplateGrammar, generate_constrained, masked_argmax


def _model():
    cfg = get_config("tiny-llama")
    m = LlamaModel(cfg, "cpu").init_random(seed=4, gen_device="cpu")
    m.allocate_kv(128)
    return m


def _one_by_one(m, prompt, grammar, max_tokens):
    """Oracle: every token fed by its own forward."""
    m.kv.add_sequence("ref")
    b = build_batch(m, ["ref"], [len(prompt)], [0], False)
    hid = m.embed_tokens(torch.tensor(prompt, dtype=torch.int32))
    m.forward(b, hid)
    logits = m.head(hid[-1:].contiguous())[0]
    out, pos = [], len(prompt)
    while len(out) < max_tokens and not grammar.can_end(out):
        run = grammar.forced_run(out)
        t = run[0] if run else masked_argmax(logits, grammar.allowed(out, m.cfg.vocab_size))
        out.append(t)
        b = build_batch(m, ["ref"], [1], [pos], True)
        hid = m.embed_tokens(torch.tensor([t], dtype=torch.int32))
        m.forward(b, hid)
        logits = m.head(hid)[0]
        pos += 1
    m.kv.free_sequence("ref")
    return out


def test_forced_runs_are_batched_and_match_one_by_one():
    m = _model()
    prompt = list(range(3, 20))
    template = [100, 101, 102, None, 103, 104, None, None, 105]
    choices = [7, 8, 9, 10, 11]
    g = TemplateGrammar(template, choices)
    res = generate_constrained(m, "s", prompt, g, 20)
    want = _one_by_one(m, prompt, g, 20)
    assert res.tokens == want
    assert len(res.tokens) == len(template)
    for t, slot in zip(res.tokens, template):
        assert t == slot if slot is not None else t in choices
    # prompt + 3 forced runs + free slots fed by their own forward (one of
    # them is folded into the following forced run).
    assert res.forwards < len(res.tokens)
    assert m.kv.allocator.num_free == m.kv.num_blocks


def test_free_grammar_is_plain_greedy():
    from cascadia_b200.runtime.generator import BatchGenerator

    m = _model()
    prompt = list(range(30, 41))
    g = TemplateGrammar([None] * 6)
    res = generate_constrained(m, "s", prompt, g, 6)
    want = BatchGenerator(m, use_graph=False).generate([prompt], 6)[0]
    assert res.tokens == want
