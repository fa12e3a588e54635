"""End-to-end model parity: our sm_100a kernel path vs the CPU fp32 oracle."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.runtime.generator import BatchGenerator

pytestmark = pytest.mark.gpu


def _models(name, seed=5):
    cfg = get_config(name)
    cpu = LlamaModel(cfg, "cpu").init_random(seed=seed, gen_device="cpu")
    gpu = LlamaModel(cfg, "cuda").init_random(seed=seed, gen_device="cpu")
    cpu.allocate_kv(128)
    gpu.allocate_kv(128)
    return cfg, cpu, gpu


@pytest.mark.parametrize("name", ["tiny-llama", "tiny-llama-128"])
def test_prefill_logits_match_oracle(name):
    cfg, cpu, gpu = _models(name)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (3, 40, 90)]
    from cascadia_b200.models.llama import build_batch

    for m in (cpu, gpu):
        for i in range(3):
            m.kv.add_sequence(f"p{i}")
    outs = []
    for m in (cpu, gpu):
        b = build_batch(m, ["p0", "p1", "p2"], [len(p) for p in prompts], [0, 0, 0], False)
        ids = torch.tensor([t for p in prompts for t in p], dtype=torch.int32).to(m.device)
        hid = m.embed_tokens(ids)
        m.forward(b, hid)
        last = torch.tensor(b.last_rows, device=m.device)
        outs.append(m.head(hid.index_select(0, last).contiguous()).float().cpu())
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    c, gg = outs
    err = (c - gg).abs().max().item()
    scale = c.abs().max().item()
    assert err <= 0.05 * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("use_graph", [False, True])
def test_greedy_generation_matches_oracle(use_graph):
    cfg, cpu, gpu = _models("tiny-llama-128", seed=7)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (4, 19, 50)]
    out_c = BatchGenerator(cpu).generate(prompts, 12)
    out_g = BatchGenerator(gpu, use_graph=use_graph).generate(prompts, 12)
    assert ops.read_status(torch.device("cuda")) == 0
    same = sum(a == b for oc, og in zip(out_c, out_g) for a, b in zip(oc, og))
    total = sum(len(o) for o in out_c)
    # Both paths round activations to bf16 at the same points; only the
    # accumulation order differs, so greedy paths agree except on near-ties.
    assert [o[0] for o in out_c] == [o[0] for o in out_g]
    assert same >= 0.8 * total, (out_c, out_g)


def test_solo_equals_batched_on_gpu():
    cfg, _, gpu = _models("tiny-llama-128", seed=9)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (7, 33)]
    gen = BatchGenerator(gpu, use_graph=True)
    batched = gen.generate(prompts, 8, prefix="b")
    solo = [gen.generate([p], 8, prefix=f"s{i}")[0] for i, p in enumerate(prompts)]
    assert batched == solo
