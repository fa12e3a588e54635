"""Gemma-4 on the GPU (sliding-window head_dim-256 attention, head_dim-512
full attention split over two CTAs per head, shared-KV layers, per-layer
inputs) against the CPU oracle path of the same model (itself checked
against HuggingFace in test_gemma4_cpu.py)."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.gemma4 import Gemma4Model
from cascadia_b200.models.llama import build_batch
from cascadia_b200.runtime.generator import BatchGenerator

pytestmark = pytest.mark.gpu


def _pair(seed=3, preset="tiny-gemma4"):
    cfg = get_config(preset)
    cpu = Gemma4Model(cfg, "cpu").init_random(seed=seed, gen_device="cpu")
    gpu = Gemma4Model(cfg, "cuda").init_random(seed=seed, gen_device="cpu")
    for m in (cpu, gpu):
        m.allocate_kv(64)
        g = torch.Generator().manual_seed(seed + 100)
        for lw in m.layers:  # moderate attention sharpness (see test_gemma4_cpu)
            lw.q_norm.fill_(0.2)
            lw.k_norm.fill_(0.2)
            if lw.moe is not None:
                # Router logits of std ~1 (the random init is near uniform,
                # where CPU/GPU rounding would swap near-tied experts).
                r = (torch.randn(lw.moe.router.shape, generator=g) / 16).to(torch.bfloat16)
                lw.moe.router.copy_(r.to(lw.moe.router.device))
    return cfg, cpu, gpu


def _close(a, b, frac=0.05):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item()
    assert err <= frac * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("preset", ["tiny-gemma4", "tiny-gemma4-moe"])
def test_prefill_beyond_window_then_decode_matches_cpu(preset):
    cfg, cpu, gpu = _pair(preset=preset)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (5, 40)]
    ids = ["a", "b"]
    lens = [len(p) for p in prompts]
    outs = []
    for m in (cpu, gpu):
        for s in ids:
            m.kv.add_sequence(s)
        b = build_batch(m, ids, lens, [0, 0], False)
        hid = m.embed_tokens(torch.cat(prompts).to(torch.int32).to(m.device))
        m.forward(b, hid)
        last = torch.tensor(b.last_rows, device=m.device)
        logits = [m.head(hid.index_select(0, last).contiguous())]
        for step in range(2):
            b = build_batch(m, ids, [1, 1], [l + step for l in lens], True)
            hid = m.embed_tokens(torch.tensor([7 + step, 9], dtype=torch.int32, device=m.device))
            m.forward(b, hid)
            logits.append(m.head(hid))
        outs.append(logits)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    for c, gg in zip(*outs):
        _close(gg, c)


@pytest.mark.parametrize("preset", ["tiny-gemma4", "tiny-gemma4-moe"])
def test_graph_generation_matches_eager(preset):
    cfg, _, gpu = _pair(seed=5, preset=preset)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (6, 30)]
    eager = BatchGenerator(gpu, use_graph=False).generate(prompts, 6, prefix="e")
    graph = BatchGenerator(gpu, use_graph=True).generate(prompts, 6, prefix="g")
    assert ops.read_status(torch.device("cuda")) == 0
    assert graph == eager
