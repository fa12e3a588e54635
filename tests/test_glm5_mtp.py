"""GLM-5 MTP draft head: speculative decoding with the head as drafter
equals plain greedy decoding; the head's paged KV built incrementally over
verify rounds gives the same drafts as building it in one pass; the HF
checkpoint layout (``layers.{num_layers}`` + enorm / hnorm / eh_proj /
shared_head.norm) loads."""
import dataclasses

import pytest
import torch

from cascadia_b200.models.config import get_config
from cascadia_b200.models.glm5 import GLM5MTP, GLM5Model, load_hf_weights, load_mtp_weights
from cascadia_b200.runtime.generator import BatchGenerator
from cascadia_b200.runtime.spec import MTPDrafter, SpecDecoder


def _pair(seed=0, blocks=64):
    cfg = get_config("tiny-glm5")
    target = GLM5Model(cfg, "cpu").init_random(seed, std=0.05)
    target.allocate_kv(blocks)
    mtp = GLM5MTP(target).init_random(seed + 7, std=0.05)
    mtp.allocate_kv(blocks)
    return cfg, target, mtp


def _prompts(cfg, n, lens, seed=3):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(2, cfg.vocab_size, (L,), generator=g).tolist() for L in lens[:n]]


def test_mtp_spec_equals_greedy():
    cfg, target, mtp = _pair()
    prompts = _prompts(cfg, 3, [5, 11, 20])
    ref = BatchGenerator(target, use_graph=False).generate(prompts, 12, prefix="r")
    sd = SpecDecoder(target, k=3, use_graph=False, mtp=mtp)
    out = sd.generate(prompts, 12)
    assert out == ref
    assert sd.stats.drafted > 0 and sd.stats.emitted == sum(len(o) - 1 for o in out)
    assert target.kv.allocator.num_free == target.kv.allocator.num_blocks
    assert mtp.kv.allocator.num_free == mtp.kv.allocator.num_blocks


def test_mtp_incremental_kv_matches_one_pass():
    cfg, target, mtp = _pair(seed=1)
    toks = _prompts(cfg, 1, [30], seed=9)[0]
    gen = BatchGenerator(target, use_graph=False)
    first = int(gen.prefill(["t"], [toks])[0])
    hid = gen.last_hidden
    nxt = toks[1:] + [first]
    N = len(toks)

    one = MTPDrafter(mtp)
    one.observe("a", 0, nxt, hid)
    want = one.propose(["a"], [toks], 3, 4)
    one.release("a")

    inc = MTPDrafter(mtp)
    cut = [0, 9, 10, 22, N]
    for lo, hi in zip(cut[:-1], cut[1:]):
        inc.observe("b", lo, nxt[lo:hi], hid[lo:hi])
        got = inc.propose(["b"], [toks[:hi]], 3, 4)
        inc.accept("b", 0, 3)
        assert mtp.kv.seqs["b"].length == hi   # chain rows rewound
    inc.release("b")
    assert got == want
    target.kv.free_sequence("t")


def _hf_state_dict(cfg, seed=0):
    """A glm_moe_dsa-style state dict with one extra (MTP) layer, from our
    own random model's layer structure: float tensors under HF names."""
    hf = pytest.importorskip("transformers.models.glm_moe_dsa.modeling_glm_moe_dsa")
    hfc = pytest.importorskip("transformers.models.glm_moe_dsa.configuration_glm_moe_dsa")
    L = cfg.num_layers
    hcfg = hfc.GlmMoeDsaConfig(
        vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
        intermediate_size=cfg.intermediate_size, moe_intermediate_size=cfg.moe_intermediate_size,
        num_hidden_layers=L + 1, num_attention_heads=cfg.num_heads,
        num_key_value_heads=cfg.num_heads, n_shared_experts=1, n_routed_experts=cfg.num_experts,
        routed_scaling_factor=cfg.routed_scaling_factor, kv_lora_rank=512,
        q_lora_rank=cfg.q_lora_rank, qk_rope_head_dim=64, v_head_dim=cfg.v_head_dim,
        qk_nope_head_dim=cfg.qk_nope_head_dim, n_group=1, topk_group=1,
        num_experts_per_tok=cfg.num_experts_per_tok, norm_topk_prob=True, rms_norm_eps=cfg.rms_eps,
        index_topk=cfg.index_topk, index_head_dim=128, index_n_heads=cfg.index_n_heads,
        mlp_layer_types=["dense"] * cfg.first_k_dense_replace +
        ["sparse"] * (L + 1 - cfg.first_k_dense_replace),
        rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta},
        tie_word_embeddings=False)
    torch.manual_seed(seed)
    m = hf.GlmMoeDsaForCausalLM(hcfg).eval()
    g = torch.Generator().manual_seed(seed + 1)
    sd = {}
    for k, v in m.state_dict().items():
        v = v.float()
        if v.dim() >= 2:
            v = torch.randn(v.shape, generator=g) * 0.05
        elif "k_norm.bias" in k:
            v = torch.zeros_like(v)
        else:
            v = 1.0 + 0.1 * torch.randn(v.shape, generator=g)
        sd[k] = v
    H = cfg.hidden_size
    p = f"model.layers.{L}."
    for n in ("enorm.weight", "hnorm.weight", "shared_head.norm.weight"):
        sd[p + n] = 1.0 + 0.1 * torch.randn(H, generator=g)
    sd[p + "eh_proj.weight"] = torch.randn(H, 2 * H, generator=g) * 0.05
    return sd


def test_mtp_loads_hf_layout_and_decodes():
    cfg = dataclasses.replace(get_config("tiny-glm5"), indexer_types=None)
    sd = _hf_state_dict(cfg)
    target = load_hf_weights(GLM5Model(cfg, "cpu"), sd)
    target.allocate_kv(64)
    mtp = load_mtp_weights(GLM5MTP(target), sd)
    mtp.allocate_kv(64)
    L = cfg.num_layers
    assert len(target.layers) == L and len(mtp.block.layers) == 1
    blk = mtp.block.layers[0]
    assert torch.equal(blk.router.float(), sd[f"model.layers.{L}.mlp.gate.weight"].bfloat16().float())
    assert blk.qkv.indexer is not None
    assert torch.equal(mtp.eh_proj.w, sd[f"model.layers.{L}.eh_proj.weight"].bfloat16())
    prompts = _prompts(cfg, 2, [7, 13])
    ref = BatchGenerator(target, use_graph=False).generate(prompts, 8, prefix="r")
    assert SpecDecoder(target, k=2, use_graph=False, mtp=mtp).generate(prompts, 8) == ref


def test_config_reads_nextn_layers():
    from cascadia_b200.models.config import ModelConfig

    c = ModelConfig.from_hf({"model_type": "glm_moe_dsa", "vocab_size": 1000, "hidden_size": 64,
                             "num_hidden_layers": 4, "num_attention_heads": 4,
                             "num_key_value_heads": 4, "intermediate_size": 128,
                             "kv_lora_rank": 512, "q_lora_rank": 64, "qk_rope_head_dim": 64,
                             "qk_nope_head_dim": 64, "v_head_dim": 64, "index_topk": 16,
                             "num_nextn_predict_layers": 1, "indexer_types": ["full"] * 4})
    assert c.num_nextn_predict_layers == 1
    assert c.layer_has_indexer(4)     # the MTP layer owns an indexer


def _engine_run(target, spec=None, mtp=None, prompts=()):
    from cascadia_b200.engine.llm import LLMEngine
    from cascadia_b200.types import GenerationTask

    e = LLMEngine(target, max_model_len=128, spec=spec, spec_k=3, mtp_head=mtp)
    tasks = [GenerationTask(f"t{i}", "", max_tokens=10 if i else 1, prompt_ids=p)
             for i, p in enumerate(prompts)]
    for t in tasks:
        e.submit(t)
    out = {t.task_id: [] for t in tasks}
    fin = set()
    for _ in range(100):
        for tid, c in e.step():
            if c.is_final:
                fin.add(tid)
            else:
                out[tid].append(c.token_id)
        if len(fin) == len(tasks):
            break
    return [out[t.task_id] for t in tasks], e


def test_engine_mtp_mode_equals_plain_greedy():
    cfg, target, mtp = _pair(seed=2)
    prompts = _prompts(cfg, 3, [6, 19, 33])
    plain, _ = _engine_run(target, prompts=prompts)
    got, e = _engine_run(target, "mtp", mtp, prompts)
    assert got == plain
    assert e.spec_stats.drafted > 0
    assert not e.drafter.queue and not e.drafter.kv_len
    assert mtp.kv.allocator.num_free == mtp.kv.allocator.num_blocks


def test_engine_mtp_with_a_sampled_request():
    """A sampled request beside greedy ones decodes normally; the head never
    holds rows for it."""
    from cascadia_b200.engine.llm import LLMEngine
    from cascadia_b200.types import GenerationTask

    cfg, target, mtp = _pair(seed=4)
    prompts = _prompts(cfg, 2, [8, 15])
    e = LLMEngine(target, max_model_len=128, spec="mtp", spec_k=2, mtp_head=mtp)
    e.submit(GenerationTask("g", "", max_tokens=6, prompt_ids=prompts[0]))
    e.submit(GenerationTask("s", "", max_tokens=6, prompt_ids=prompts[1], temperature=0.8))
    fin = set()
    for _ in range(60):
        for tid, c in e.step():
            if c.is_final:
                fin.add(tid)
        assert "s" not in e.drafter.queue
        if len(fin) == 2:
            break
    assert fin == {"g", "s"}
    assert not e.drafter.queue and mtp.kv.allocator.num_free == mtp.kv.allocator.num_blocks


def test_engine_mtp_refuses_prefix_cache():
    from cascadia_b200.engine.llm import LLMEngine
    from cascadia_b200.engine.base import InvalidConfig

    cfg, target, mtp = _pair(seed=2)
    with pytest.raises(InvalidConfig):
        LLMEngine(target, spec="mtp", mtp_head=mtp, prefix_cache_blocks=8)
    with pytest.raises(InvalidConfig):
        LLMEngine(target, spec="mtp")
