"""Speculative decoding on the GPU kernels: verify forward (ragged prefill
attention + LM head on every row + device verify kernel), paged-KV rewind,
draft model through CUDA-graph decode."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.runtime.generator import BatchGenerator
from cascadia_b200.runtime.spec import SpecDecoder

pytestmark = pytest.mark.gpu


def _model(seed):
    m = LlamaModel(get_config("tiny-llama-128"), "cuda").init_random(seed=seed, gen_device="cpu")
    m.allocate_kv(256)
    return m


def _prompts():
    g = torch.Generator().manual_seed(3)
    rep = torch.randint(3, 1000, (6,), generator=g).tolist()
    return [rep * 4, torch.randint(3, 1000, (11,), generator=g).tolist(),
            torch.randint(3, 1000, (40,), generator=g).tolist()]


def _agree(a, b):
    """Common-prefix length (the verify path and the decode path use
    different attention kernels, so near-tied argmaxes may differ)."""
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


@pytest.mark.parametrize("mode", ["self", "foreign", "ngram"])
def test_spec_matches_greedy(mode):
    target = _model(5)
    ref = BatchGenerator(target).generate(_prompts(), 24)
    draft = {"self": lambda: _model(5), "foreign": lambda: _model(77), "ngram": lambda: None}[mode]()
    sd = SpecDecoder(target, draft=draft, k=4, ngram_k=4)
    out = sd.generate(_prompts(), 24)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    assert [len(o) for o in out] == [24, 24, 24]
    agree = sum(_agree(a, b) for a, b in zip(out, ref))
    assert agree >= 0.8 * 72, (out, ref)
    if mode == "self":
        assert sd.stats.accept_rate > 0.8
    assert target.kv.allocator.num_free == target.kv.allocator.num_blocks


def test_verify_graph_matches_eager_logits():
    """The captured verify step (a decode step over B*T rows) computes the
    same logits as the eager verify forward (ragged prefill attention) for
    every row, and the verify kernel's result agrees with the argmax of
    those logits."""
    from cascadia_b200.models.llama import build_batch
    from cascadia_b200.runtime.spec import VerifyGraph

    target = _model(5)
    prompts = _prompts()
    gen = BatchGenerator(target)
    ids = [f"q{i}" for i in range(len(prompts))]
    first = gen.prefill(ids, prompts).cpu().tolist()
    g = torch.Generator().manual_seed(4)
    T = 5
    rows = [[f] + torch.randint(3, 1000, (T - 1,), generator=g).tolist() for f in first]
    kv_lens = [len(p) for p in prompts]
    batch = build_batch(target, ids, [T] * len(ids), kv_lens, False)
    hid = target.embed_tokens(torch.tensor([t for r in rows for t in r], dtype=torch.int32,
                                           device="cuda"))
    target.forward(batch, hid)
    want = target.head(hid).float()
    vg = VerifyGraph(target, len(ids), T, 64)
    vg.stage(ids, rows, kv_lens)
    res = vg.verify()
    got = vg.logits.float()
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    scale = want.abs().max().item()
    err = (got - want).abs().max().item()
    assert err <= 0.02 * scale, (err, scale)
    picks = got.argmax(-1).view(len(ids), T).cpu().tolist()
    for r, p, out in zip(rows, picks, res):
        acc = 0
        while acc < T - 1 and r[1 + acc] == p[acc]:
            acc += 1
        assert out == r[1:1 + acc] + [p[acc]], (out, r, p)
    for sid in ids:
        target.kv.free_sequence(sid)


def test_early_exit_draft():
    """Self-speculation: the draft is the target's first layer (shared
    weights, own KV)."""
    target = _model(5)
    ref = BatchGenerator(target).generate(_prompts(), 24)
    draft = target.early_exit(1)
    draft.allocate_kv(256)
    sd = SpecDecoder(target, draft=draft, k=3)
    out = sd.generate(_prompts(), 24)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    assert sum(_agree(a, b) for a, b in zip(out, ref)) >= 0.8 * 72
    assert draft.kv.allocator.num_free == draft.kv.allocator.num_blocks
