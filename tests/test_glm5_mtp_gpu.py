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


def _close(a, b, frac=0.08):
    # Absorbed-latent MLA on the GPU vs the expanded fp32 oracle: up to ~7 %
    # of the largest value on this model (as in test_glm5_gpu.py).
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item()
    assert err <= frac * scale + 1e-3, (err, scale)


def _models(device, cfg):
    target = GLM5Model(cfg, device).init_random(4, std=0.05, gen_device="cpu")
    target.allocate_kv(128)
    mtp = GLM5MTP(target).init_random(11, std=0.05, gen_device="cpu")
    mtp.allocate_kv(128)
    return target, mtp


def test_mtp_head_matches_cpu():
    """The head's ragged catch-up forward (MLA / DSA / MoE kernels on its own
    paged KV) and one chain step against the CPU oracle, from the same
    target hidden rows."""
    from cascadia_b200.models.llama import build_batch

    cfg = dataclasses.replace(get_config("tiny-glm5"), index_topk=2048)
    (tc, mc), (tg, mg) = _models("cpu", cfg), _models("cuda", cfg)
    g = torch.Generator().manual_seed(8)
    lens = [9, 24]
    toks = [torch.randint(2, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    hid = torch.randn(sum(lens), cfg.hidden_size, generator=g).to(torch.bfloat16)
    flat = torch.tensor([t for tt in toks for t in tt], dtype=torch.int32)
    outs = []
    drafts = None
    for m, dev in ((mc, "cpu"), (mg, "cuda")):
        for sid in ("a", "b"):
            m.kv.add_sequence(sid)
        b = build_batch(m.block, ["a", "b"], lens, [0, 0], False)
        h, d = m.step(b, flat.to(dev), hid.to(dev), from_target=True)
        last = torch.tensor(b.last_rows, device=dev)
        hl = h.index_select(0, last).contiguous()
        if drafts is None:  # both chain steps take the oracle's drafts
            drafts = d.index_select(0, last).to(torch.int32).cpu()
        b2 = build_batch(m.block, ["a", "b"], [1, 1], lens, True)
        h2, _ = m.step(b2, drafts.to(dev), hl, from_target=False)
        outs.append((h, h2))
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    _close(outs[1][0], outs[0][0])
    _close(outs[1][1], outs[0][1])


def test_mtp_spec_decoding_runs_on_gpu():
    """Speculative decoding with the MTP head on the GPU: every sequence gets
    its tokens, the head's KV is returned, and the output follows greedy
    decoding.  Exact equality is checked on the CPU (the verify forward
    batches several rows, so its MoE and attention kernels differ from the
    single-row decode kernels and near-tied argmaxes may part the two
    runs)."""
    cfg = dataclasses.replace(get_config("tiny-glm5"), index_topk=2048)
    target, mtp = _models("cuda", cfg)
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(2, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 24, 40)]
    ref = BatchGenerator(target).generate(prompts, 16, prefix="r")
    sd = SpecDecoder(target, k=3, mtp=mtp)
    out = sd.generate(prompts, 16)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    assert [len(o) for o in out] == [16, 16, 16]
    assert [o[0] for o in out] == [r[0] for r in ref]   # the prefill's token
    assert sum(_agree(a, b) for a, b in zip(out, ref)) >= 0.5 * 48, (out, ref)
    assert sd.stats.drafted > 0
    assert mtp.kv.allocator.num_free == mtp.kv.allocator.num_blocks
    assert target.kv.allocator.num_free == target.kv.allocator.num_blocks
