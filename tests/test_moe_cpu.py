"""Sparse-MoE model on the CPU oracle path: routing semantics and the
expert-block arithmetic against a dense restatement."""
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import build_batch
from cascadia_b200.models.moe import MoEModel, ref_topk_gate
from cascadia_b200.ops import reference as ref


def test_softmax_topk_renormalises():
    g = torch.Generator().manual_seed(0)
    h = torch.randn(5, 64, generator=g).to(torch.bfloat16)
    wg = torch.randn(16, 64, generator=g).to(torch.bfloat16)
    ids, w = ref_topk_gate(h, wg, None, 4, 0, True, 1.0)
    assert ids.shape == (5, 4) and torch.allclose(w.sum(-1), torch.ones(5))
    p = torch.softmax(h.float() @ wg.float().t(), -1)
    assert torch.equal(ids.long(), torch.topk(p, 4).indices)


def test_sigmoid_bias_only_chooses():
    g = torch.Generator().manual_seed(1)
    h = torch.randn(3, 64, generator=g).to(torch.bfloat16)
    wg = torch.randn(8, 64, generator=g).to(torch.bfloat16)
    bias = torch.zeros(8)
    bias[7] = 100.0  # expert 7 always chosen, but weighted by its sigmoid only
    ids, w = ref_topk_gate(h, wg, bias, 2, 1, False, 2.0)
    s = torch.sigmoid(h.float() @ wg.float().t())
    assert bool((ids == 7).any(-1).all())
    for t in range(3):
        for j in range(2):
            assert abs(w[t, j].item() - 2.0 * s[t, ids[t, j]].item()) < 1e-6


def test_moe_layer_equals_dense_restatement():
    cfg = get_config("tiny-moe")
    cfg.num_layers = 1
    m = MoEModel(cfg, "cpu").init_random(seed=2, gen_device="cpu")
    lw = m.layers[0]
    g = torch.Generator().manual_seed(3)
    h = torch.randn(4, cfg.hidden_size, generator=g).to(torch.bfloat16)
    hidden = torch.randn(4, cfg.hidden_size, generator=g).to(torch.bfloat16)
    expect = hidden.float().clone()
    ids, w = ref_topk_gate(h, lw.router, None, cfg.num_experts_per_tok, 0, True, 1.0)
    bank = lw.experts
    for t in range(4):
        acc = torch.zeros(cfg.hidden_size)
        for j in range(cfg.num_experts_per_tok):
            e = int(ids[t, j])
            gu = h[t].float() @ bank.gu_ref[e].t()
            a = ref.silu_mul(gu[:bank.inter], gu[bank.inter:]).to(torch.bfloat16).float()
            acc += w[t, j] * (a @ bank.dn_ref[e].t()).to(torch.bfloat16).float()
        expect[t] += acc
    m._moe(lw, h, hidden)
    assert torch.allclose(hidden.float(), expect.to(torch.bfloat16).float(), atol=1e-2)


def test_moe_model_prefill_and_decode_consistent():
    """Prefill of n+1 tokens and prefill of n then decode 1 give the same
    last-token logits (KV cache + routing per token)."""
    cfg = get_config("tiny-moe")
    m = MoEModel(cfg, "cpu").init_random(seed=4, gen_device="cpu")
    m.allocate_kv(32)
    toks = [5, 9, 13, 2, 7, 7, 30]
    m.kv.add_sequence("a")
    b = build_batch(m, ["a"], [len(toks)], [0], False)
    hid = m.embed_tokens(torch.tensor(toks, dtype=torch.int32))
    m.forward(b, hid)
    full = m.head(hid[-1:].contiguous()).float()
    m.kv.add_sequence("b")
    b = build_batch(m, ["b"], [len(toks) - 1], [0], False)
    hid = m.embed_tokens(torch.tensor(toks[:-1], dtype=torch.int32))
    m.forward(b, hid)
    b = build_batch(m, ["b"], [1], [len(toks) - 1], True)
    hid = m.embed_tokens(torch.tensor(toks[-1:], dtype=torch.int32))
    m.forward(b, hid)
    step = m.head(hid).float()
    assert (full - step).abs().max().item() <= 0.02 * full.abs().max().item() + 1e-3


def test_moe_builder_rejects_dense():
    import pytest

    from cascadia_b200.engine.base import InvalidConfig
    from cascadia_b200.engine.llm import MoEBuilder

    with pytest.raises(InvalidConfig):
        MoEBuilder("tiny-llama", device="cpu").model_class(get_config("tiny-llama"))
    assert MoEBuilder("tiny-moe", device="cpu").model_class(get_config("tiny-moe")) is MoEModel


def test_moe_engine_cpu_generates():
    from cascadia_b200.engine.llm import MoEBuilder
    from cascadia_b200.runtime.runner import Runner
    from cascadia_b200.types import GenerationTask, PeerLayout, ShardSpec

    b = MoEBuilder("tiny-moe", device="cpu", kv_blocks=64, max_running=4, max_model_len=256)
    r = Runner(b, model_id="tiny-moe", device="cpu")
    r.start(PeerLayout(), ShardSpec("tiny-moe", 0, 2, 2))
    chunks = list(r.generate(GenerationTask("m1", "", max_tokens=6, prompt_ids=[5, 6, 7, 8])))
    r.close()
    assert chunks[-1].is_final
    assert sum(1 for c in chunks if not c.is_final) == 6


def test_expert_load_metric_observed():
    import torch

    from cascadia_b200 import metrics
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.moe import MoEModel

    def count():
        for m in metrics.EXPERT_LOAD.collect():
            for s in m.samples:
                if s.name.endswith("_count") and s.labels.get("model") == "qwen3_moe":
                    return s.value
        return 0.0

    cfg = get_config("tiny-moe")
    m = MoEModel(cfg, "cpu").init_random(seed=3, gen_device="cpu")
    m.allocate_kv(64)
    from cascadia_b200.runtime.generator import BatchGenerator

    before = count()
    BatchGenerator(m, use_graph=False).generate([[3, 4, 5, 6]], max_new_tokens=2)
    # One observation per expert for the sampled layer calls.
    assert count() >= before + cfg.num_experts
