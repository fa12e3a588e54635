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
