"""GLM-5 on the GPU: the DSA indexer kernel, MLA decode restricted to the
selected positions, and the whole model (IndexShare preset) against the CPU
oracle path (itself checked against HuggingFace in test_glm5_cpu.py)."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.glm5 import GLM5Model
from cascadia_b200.models.llama import build_batch

pytestmark = pytest.mark.gpu


def test_dsa_scores_kernel_matches_torch():
    g = torch.Generator().manual_seed(0)
    T, H, L, NB = 5, 16, 2, 12
    lens = [1, 16, 17, 70, 150]
    cache = (torch.randn(L, NB, 16, 128, generator=g) * 0.5).to(torch.bfloat16)
    # Each token gets its own shuffled block list.
    width = 10
    bt = torch.stack([torch.randperm(NB, generator=g)[:width] for _ in range(T)]).to(torch.int32)
    q = (torch.randn(T, H, 128, generator=g) * 0.5).to(torch.bfloat16)
    w = torch.randn(T, H, generator=g)
    out = torch.empty(T, width * 16, device="cuda")
    layer = 1
    ops.ext().dsa_scores(q.cuda(), w.cuda(), cache.cuda(), bt.cuda(),
                         torch.tensor(lens, dtype=torch.int32, device="cuda"), out, layer)
    torch.cuda.synchronize()
    for t in range(T):
        keys = cache[layer, bt[t].long()].reshape(-1, 128)[:lens[t]].float()
        s = torch.relu(q[t].float() @ keys.t())             # [H, len]
        want = (w[t][:, None] * s).sum(0)
        got = out[t].cpu()
        assert torch.allclose(got[:lens[t]], want, rtol=1e-4, atol=1e-4)
        assert torch.isinf(got[lens[t]:]).all() and (got[lens[t]:] < 0).all()


def _pair(seed=3):
    cfg = get_config("tiny-glm5")
    cpu = GLM5Model(cfg, "cpu").init_random(seed=seed, gen_device="cpu")
    gpu = GLM5Model(cfg, "cuda").init_random(seed=seed, gen_device="cpu")
    cpu.allocate_kv(64)
    gpu.allocate_kv(64)
    return cfg, cpu, gpu


def _close(a, b, frac=0.08):
    # Absorbed-latent MLA on the GPU (q and the latent output rounded to
    # bf16 around the 192/256-wide head projections) vs the expanded fp32
    # oracle: up to ~7 % of the largest logit on this 3-layer model.
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item()
    assert err <= frac * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("n", [7, 40])
def test_model_matches_cpu_with_the_same_selection(n):
    """Both paths attend over the CPU indexer's selection (near-tie swaps of
    the indexer are checked separately); the GPU indexer's own scores must
    match the CPU ones closely."""
    cfg, cpu, gpu = _pair()
    ids = torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(n))
    sels = []
    orig_cpu, orig_gpu = cpu._index, gpu._index

    def rec(slot, ind, x, qa, batch):
        r = orig_cpu(slot, ind, x, qa, batch)
        sels.append(r)
        return r

    it = iter(sels)

    def replay(slot, ind, x, qa, batch):
        own = orig_gpu(slot, ind, x, qa, batch)
        sc, thr = next(it)
        ld = own[0].shape[1]
        want = torch.full((sc.shape[0], ld), float("-inf"))
        want[:, :sc.shape[1]] = sc
        valid = torch.isfinite(want)
        # Same inputs up to bf16 rounding upstream: scores close.
        assert torch.allclose(own[0].cpu()[valid], want[valid], rtol=0.1, atol=0.05)
        return want.cuda(), thr.cuda()

    cpu._index, gpu._index = rec, replay
    outs = []
    for m in (cpu, gpu):
        m.kv.add_sequence("s")
        b = build_batch(m, ["s"], [n], [0], False)
        hid = m.embed_tokens(ids.to(torch.int32).to(m.device))
        m.forward(b, hid)
        logits = [m.head(hid)]
        for step in range(2):
            b = build_batch(m, ["s"], [1], [n + step], True)
            hid = m.embed_tokens(torch.tensor([5 + step], dtype=torch.int32, device=m.device))
            m.forward(b, hid)
            logits.append(m.head(hid))
        outs.append(logits)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    for c, gg in zip(*outs):
        _close(gg, c)
