"""MLA on the GPU (absorbed latent attention kernel, swizzled latent cache)
against the CPU oracle of the reference's expanded per-head attention."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import build_batch
from cascadia_b200.models.mla import MLAModel

pytestmark = pytest.mark.gpu


def _logits(m, prompts):
    ids = [f"p{i}" for i in range(len(prompts))]
    m.allocate_kv(64)
    for s in ids:
        m.kv.add_sequence(s)
    b = build_batch(m, ids, [len(p) for p in prompts], [0] * len(prompts), False)
    hid = m.embed_tokens(torch.tensor([t for p in prompts for t in p], dtype=torch.int32,
                                      device=m.device))
    m.forward(b, hid)
    rows = torch.tensor(b.last_rows, device=m.device)
    pre = m.head(hid.index_select(0, rows).contiguous()).float().cpu()
    outs = [pre]
    for step in range(2):
        b2 = build_batch(m, ids, [1] * len(prompts), [len(p) + step for p in prompts], True)
        hid2 = m.embed_tokens(torch.tensor([3 + step] * len(prompts), dtype=torch.int32,
                                           device=m.device))
        m.forward(b2, hid2)
        outs.append(m.head(hid2).float().cpu())
    return outs


def test_mla_model_matches_oracle():
    cfg = get_config("tiny-mla")
    g = torch.Generator().manual_seed(2)
    # 40 tokens: several 16-token blocks, a partial last block
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 7)]
    cpu = MLAModel(cfg, "cpu").init_random(seed=5, gen_device="cpu")
    gpu = MLAModel(cfg, "cuda").init_random(seed=5, gen_device="cpu")
    oc, og = _logits(cpu, prompts), _logits(gpu, prompts)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    for c, gg in zip(oc, og):
        scale = c.abs().max().item()
        assert (c - gg).abs().max().item() <= 0.05 * scale + 1e-3


def test_mla_decode_graph_equals_eager():
    from cascadia_b200.runtime.generator import BatchGenerator

    cfg = get_config("tiny-mla")
    outs = []
    for use_graph in (False, True):
        m = MLAModel(cfg, "cuda").init_random(seed=1, gen_device="cpu")
        m.allocate_kv(64)
        outs.append(BatchGenerator(m, use_graph=use_graph).generate([[5, 6, 7], [8] * 20], 6))
    assert ops.read_status(torch.device("cuda")) == 0
    assert outs[0] == outs[1]
