"""Sparse-MoE kernels (router/top-k, permute, grouped INT4 expert GEMM,
combine) and the MoE model vs plain PyTorch fp32 references."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import build_batch
from cascadia_b200.models.moe import MoEModel, ref_topk_gate
from cascadia_b200.ops import reference as ref
from cascadia_b200.quant import Int4Weight

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("scoring,E,k,norm,scale", [(0, 128, 8, True, 1.0), (0, 64, 4, False, 1.0),
                                                   (1, 384, 8, True, 2.827), (1, 16, 2, True, 1.0)])
def test_topk_gate(scoring, E, k, norm, scale):
    g = torch.Generator().manual_seed(E + k)
    T, H = 37, 512
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    wg = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(E, generator=g) * 0.1) if scoring == 1 else None
    ids, w = ops.moe_topk_gate(x.to(DEV), wg.to(DEV), k, scoring, norm, scale,
                               bias.to(DEV) if bias is not None else None)
    rid, rw = ref_topk_gate(x, wg, bias, k, scoring, norm, scale)
    ids, w = ids.cpu(), w.cpu()
    # Same expert set per token (order of near-equal scores may differ).
    agree = sum(set(a.tolist()) == set(b.tolist()) for a, b in zip(ids, rid))
    assert agree >= T - 1
    for t in range(T):
        if set(ids[t].tolist()) != set(rid[t].tolist()):
            continue
        a = dict(zip(ids[t].tolist(), w[t].tolist()))
        b = dict(zip(rid[t].tolist(), rw[t].tolist()))
        for e in a:
            assert abs(a[e] - b[e]) <= 1e-3 * max(1.0, abs(b[e]))


@pytest.mark.parametrize("T,k,E", [(1, 8, 128), (64, 8, 128), (300, 2, 8), (2048, 8, 128)])
def test_permute(T, k, E):
    g = torch.Generator().manual_seed(T)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    x = torch.randn(T, 256, generator=g).to(torch.bfloat16)
    offsets, perm, inv, xp = ops.moe_permute(ids.to(DEV), E, x.to(DEV))
    offsets, perm, inv, xp = offsets.cpu(), perm.cpu(), inv.cpu(), xp.cpu()
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    assert offsets[0] == 0 and torch.equal(offsets[1:].long(), torch.cumsum(counts, 0))
    n = T * k
    assert sorted(perm[:n].tolist()) == list(range(n))
    flat = ids.flatten()
    for e in range(E):
        seg = perm[offsets[e]:offsets[e + 1]].long()
        assert bool((flat[seg] == e).all())
    assert torch.equal(inv[perm[:n].long()], torch.arange(n, dtype=torch.int32))
    assert torch.equal(xp[:n], x[perm[:n].long() // k])


def _grouped_case(G, rows, N, K, gs, epi, seed=0):
    g = torch.Generator().manual_seed(seed)
    ws = [Int4Weight.random(N, K, 0.05, gs, generator=g) for _ in range(G)]
    offs = [0]
    for r in rows:
        offs.append(offs[-1] + r)
    M = offs[-1]
    x = (torch.randn(max(M, 1), K, generator=g) * 0.5).to(torch.bfloat16)
    inter = epi == ops.EPI_SILU
    blob = torch.cat([w.to(DEV).blob(interleave_gate_up=inter) for w in ws])
    out = ops.w4a16_gemm_grouped(x.to(DEV), blob, N, gs, epi,
                                 torch.tensor(offs, dtype=torch.int32, device=DEV), G,
                                 max(rows) if rows else 0)
    torch.cuda.synchronize()
    assert ops.read_status(DEV) == 0
    out = out.float().cpu()
    for e in range(G):
        if rows[e] == 0:
            continue
        xs = x[offs[e]:offs[e + 1]].float()
        y = xs @ ws[e].dequant_bf16().float().t()
        if inter:
            y = ref.silu_mul(y[:, :N // 2], y[:, N // 2:])
        got = out[offs[e]:offs[e + 1]]
        err = (got - y).abs().max().item()
        assert err <= 0.02 * y.abs().max().item() + 1e-2, (e, err)


@pytest.mark.parametrize("gs", [128, 32])
@pytest.mark.parametrize("epi", [ops.EPI_STORE, ops.EPI_SILU])
def test_grouped_gemm_decode_shapes(gs, epi):
    rows = [3, 0, 1, 7, 0, 0, 12, 2]
    _grouped_case(len(rows), rows, 512, 256, gs, epi, seed=gs + epi)


def test_grouped_gemm_large_groups():
    rows = [130, 0, 64, 1, 257]
    _grouped_case(len(rows), rows, 256, 512, 128, ops.EPI_STORE, seed=3)


@pytest.mark.parametrize("dynamic", [False, True])
@pytest.mark.parametrize("rows", [[3, 0, 1, 7, 0, 0, 12, 2], [1, 1, 1, 1], [0, 0, 20, 0]])
@pytest.mark.parametrize("epi", [ops.EPI_STORE, ops.EPI_SILU])
def test_grouped_small_m(rows, epi, dynamic):
    """Grouped small-M kernel on prepared activations (fp16, scaled, with
    offset corrections), including experts with more than 8 rows; static
    and dynamic (atomic counter) unit order.  The dynamic counter is run
    twice to check that it resets itself."""
    g = torch.Generator().manual_seed(sum(rows) + epi)
    G, N, K = len(rows), 512, 768
    ws = [Int4Weight.random(N, K, 0.05, 128, generator=g) for _ in range(G)]
    offs = [0]
    for r in rows:
        offs.append(offs[-1] + r)
    M = offs[-1]
    x = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16)
    x[0, :5] = 3e4  # one huge activation: exercises the per-row fp16 scaling
    inter = epi == ops.EPI_SILU
    blob = torch.cat([w.to(DEV).blob(interleave_gate_up=inter) for w in ws])
    x16, xs = ops.moe_prep_fp16(x.to(DEV), M)
    sched = torch.zeros(2, dtype=torch.int32, device=DEV) if dynamic else None
    for _ in range(2 if dynamic else 1):
        out = ops.w4a16_gemv_grouped(x16, xs, blob, N, epi,
                                     torch.tensor(offs, dtype=torch.int32, device=DEV), G,
                                     sched=sched)
    torch.cuda.synchronize()
    if dynamic:
        assert sched.tolist() == [0, 0]
    assert ops.read_status(DEV) == 0
    out = out.float().cpu()
    for e in range(G):
        if rows[e] == 0:
            continue
        wq = (ws[e].unpack().float() - 8.0) * ws[e].scales.float().repeat_interleave(128, dim=1)
        y = x[offs[e]:offs[e + 1]].float() @ wq.t()
        if inter:
            y = ref.silu_mul(y[:, :N // 2], y[:, N // 2:])
        got = out[offs[e]:offs[e + 1]]
        err = (got - y).abs().max().item()
        assert err <= 0.01 * y.abs().max().item() + 1e-2, (e, err)


@pytest.mark.parametrize("epi", [ops.EPI_STORE, ops.EPI_SILU])
def test_grouped_small_m_many_units(epi):
    """The decode down-projection shape (K 512: four X buffers in flight)
    with many experts of 0 to 3 rows, so every CTA runs through several
    units and the X ring wraps; dynamic unit order."""
    g = torch.Generator().manual_seed(11 + epi)
    G, N, K = 64, 2048, 512
    rows = torch.randint(0, 4, (G,), generator=g).tolist()
    ws = [Int4Weight.random(N, K, 0.05, 128, generator=g) for _ in range(G)]
    offs = [0]
    for r in rows:
        offs.append(offs[-1] + r)
    M = offs[-1]
    x = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16)
    inter = epi == ops.EPI_SILU
    blob = torch.cat([w.to(DEV).blob(interleave_gate_up=inter) for w in ws])
    x16, xs = ops.moe_prep_fp16(x.to(DEV), M)
    sched = torch.zeros(2, dtype=torch.int32, device=DEV)
    out = ops.w4a16_gemv_grouped(x16, xs, blob, N, epi,
                                 torch.tensor(offs, dtype=torch.int32, device=DEV), G,
                                 sched=sched)
    torch.cuda.synchronize()
    assert ops.read_status(DEV) == 0 and sched.tolist() == [0, 0]
    out = out.float().cpu()
    for e in range(G):
        if rows[e] == 0:
            continue
        wq = (ws[e].unpack().float() - 8.0) * ws[e].scales.float().repeat_interleave(128, dim=1)
        y = x[offs[e]:offs[e + 1]].float() @ wq.t()
        if inter:
            y = ref.silu_mul(y[:, :N // 2], y[:, N // 2:])
        err = (out[offs[e]:offs[e + 1]] - y).abs().max().item()
        assert err <= 0.01 * y.abs().max().item() + 1e-2, (e, err)


def test_combine():
    g = torch.Generator().manual_seed(4)
    T, k, H = 33, 4, 384
    y = torch.randn(T * k, H, generator=g).to(torch.bfloat16)
    inv = torch.randperm(T * k, generator=g).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    add = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out = ops.moe_combine(y.to(DEV), inv.to(DEV), w.to(DEV), add=add.to(DEV)).float().cpu()
    refo = (y.float()[inv.long()].view(T, k, H) * w[:, :, None]).sum(1) + add.float()
    assert (out - refo).abs().max().item() <= 0.02 * refo.abs().max().item()


def _kimi_route_cfg():
    cfg = get_config("tiny-moe")
    cfg.router, cfg.routed_scaling_factor, cfg.num_shared_experts = "sigmoid", 2.5, 1
    cfg.first_k_dense_replace, cfg.group_size, cfg.qk_norm = 1, 32, False
    return cfg


@pytest.mark.parametrize("cfg_fn", [lambda: get_config("tiny-moe"), _kimi_route_cfg])
def test_moe_model_matches_oracle(cfg_fn):
    cfg = cfg_fn()
    cpu = MoEModel(cfg, "cpu").init_random(seed=3, gen_device="cpu")
    gpu = MoEModel(cfg, "cuda").init_random(seed=3, gen_device="cpu")
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 23)]
    outs = []
    for m in (cpu, gpu):
        m.allocate_kv(64)
        for i in range(2):
            m.kv.add_sequence(f"p{i}")
        b = build_batch(m, ["p0", "p1"], [len(p) for p in prompts], [0, 0], False)
        ids = torch.tensor([t for p in prompts for t in p], dtype=torch.int32).to(m.device)
        hid = m.embed_tokens(ids)
        m.forward(b, hid)
        last = torch.tensor(b.last_rows, device=m.device)
        pre = m.head(hid.index_select(0, last).contiguous()).float().cpu()
        b2 = build_batch(m, ["p0", "p1"], [1, 1], [len(p) for p in prompts], True)
        hid2 = m.embed_tokens(torch.tensor([3, 4], dtype=torch.int32, device=m.device))
        m.forward(b2, hid2)
        outs.append((pre, m.head(hid2).float().cpu()))
    torch.cuda.synchronize()
    assert ops.read_status(DEV) == 0
    for c, gg in zip(outs[0], outs[1]):
        scale = c.abs().max().item()
        assert (c - gg).abs().max().item() <= 0.05 * scale + 1e-3


def test_moe_engine_generates():
    from cascadia_b200.runtime.generator import BatchGenerator

    cfg = get_config("tiny-moe")
    m = MoEModel(cfg, "cuda").init_random(seed=1, gen_device="cpu")
    m.allocate_kv(64)
    out_e = BatchGenerator(m, use_graph=False).generate([[5, 6, 7], [8] * 20], 8)
    m2 = MoEModel(cfg, "cuda").init_random(seed=1, gen_device="cpu")
    m2.allocate_kv(64)
    out_g = BatchGenerator(m2, use_graph=True).generate([[5, 6, 7], [8] * 20], 8)
    assert ops.read_status(DEV) == 0
    assert out_e == out_g
