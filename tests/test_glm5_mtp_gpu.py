"""GLM-5 MTP drafting on the GPU kernels: the head's ragged catch-up
forward and chain steps run the MLA / DSA / MoE kernels on its own paged
KV; speculative decoding with it reproduces greedy decoding (up to
near-tied argmaxes between the verify and decode kernels).  The index top-k
covers the whole context here: near-tied indexer scores would otherwise
select different positions in the verify and decode kernels and the two
greedy runs would part for that reason alone."""
import dataclasses

import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.glm5 import GLM5MTP, GLM5Model
from cascadia_b200.runtime.generator import BatchGenerator
from cascadia_b200.runtime.spec import SpecDecoder

pytestmark = pytest.mark.gpu


def _agree(a, b):
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def test_mtp_spec_matches_greedy_on_gpu():
    cfg = dataclasses.replace(get_config("tiny-glm5"), index_topk=2048)
    target = GLM5Model(cfg, "cuda").init_random(4, std=0.05, gen_device="cpu")
    target.allocate_kv(128)
    mtp = GLM5MTP(target).init_random(11, std=0.05, gen_device="cpu")
    mtp.allocate_kv(128)
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(2, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 24, 40)]
    ref = BatchGenerator(target).generate(prompts, 16, prefix="r")
    sd = SpecDecoder(target, k=3, mtp=mtp)
    out = sd.generate(prompts, 16)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    assert [len(o) for o in out] == [16, 16, 16]
    assert sum(_agree(a, b) for a, b in zip(out, ref)) >= 0.8 * 48, (out, ref)
    assert sd.stats.drafted > 0
    assert mtp.kv.allocator.num_free == mtp.kv.allocator.num_blocks
