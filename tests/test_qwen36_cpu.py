"""Qwen3.5/3.6 hybrid (Gated DeltaNet + gated attention + MoE): our CPU
oracle path against the published HuggingFace model definition
(transformers ``qwen3_5_moe``), prefill and decode steps, on a tiny random
model whose projection weights are INT4-representable (so both sides use the
same effective weights)."""
import pytest
import torch

from cascadia_b200.models.config import ModelConfig, get_config
from cascadia_b200.models.llama import build_batch
from cascadia_b200.models.qwen36 import HybridMoEModel, load_hf_weights
from cascadia_b200.quant import Int4Weight

hf = pytest.importorskip("transformers.models.qwen3_5_moe.modeling_qwen3_5_moe")
hfc = pytest.importorskip("transformers.models.qwen3_5_moe.configuration_qwen3_5_moe")


def _hf_model(ours: ModelConfig, seed=0):
    cfg = hfc.Qwen3_5MoeTextConfig(
        vocab_size=ours.vocab_size, hidden_size=ours.hidden_size,
        num_hidden_layers=ours.num_layers, num_attention_heads=ours.num_heads,
        num_key_value_heads=ours.num_kv_heads, head_dim=ours.head_dim, rms_norm_eps=ours.rms_eps,
        linear_num_key_heads=ours.linear_num_key_heads,
        linear_num_value_heads=ours.linear_num_value_heads, linear_key_head_dim=128,
        linear_value_head_dim=128, linear_conv_kernel_dim=4,
        moe_intermediate_size=ours.moe_intermediate_size,
        shared_expert_intermediate_size=ours.shared_expert_intermediate_size,
        num_experts=ours.num_experts, num_experts_per_tok=ours.num_experts_per_tok,
        rope_parameters={"rope_type": "default", "rope_theta": ours.rope_theta,
                         "partial_rotary_factor": ours.partial_rotary_factor,
                         "mrope_section": [11, 11, 10]},
        tie_word_embeddings=False)
    torch.manual_seed(seed)
    m = hf.Qwen3_5MoeForCausalLM(cfg).eval()
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "norm" in name and p.dim() == 1:
                if "linear_attn.norm" in name:
                    p.copy_((1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(torch.bfloat16))
                else:  # zero-centred: make 1 + w exact in bf16
                    one_w = (1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(torch.bfloat16)
                    p.copy_(one_w.float() - 1.0)
            elif name.endswith("dt_bias") or name.endswith("A_log"):
                continue
            elif "conv1d" in name or "embed" in name or "mlp.gate.weight" in name or \
                    "shared_expert_gate" in name:
                if "mlp.gate.weight" in name:
                    p.normal_(0, 0.3, generator=g)
                p.copy_(p.to(torch.bfloat16).float())
            elif p.dim() >= 2:
                if p.dim() == 2 and "lm_head" not in name:
                    p.normal_(0, 0.05, generator=g)
                flat = p.reshape(-1, p.shape[-1])
                q = Int4Weight.quantize(flat.float(), 128).dequant_bf16().float()
                p.copy_(q.view_as(p))
    return m


def _ours(cfg, sd):
    m = HybridMoEModel(cfg, "cpu")
    load_hf_weights(m, sd)
    m.allocate_kv(64, max_seqs=4)
    return m


def _close(a, b, frac=0.05):
    # The HF model itself, run in bf16, differs from its fp32 run by 3-4 % of
    # the largest logit on this model; we round activations to bf16 too.
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item()
    assert err <= frac * scale + 1e-3, (err, scale)


def test_hf_config_maps_to_hybrid_preset():
    cfg = ModelConfig.from_hf({
        "model_type": "qwen3_5_moe_text", "vocab_size": 248320, "hidden_size": 2048,
        "num_hidden_layers": 40, "num_attention_heads": 16, "num_key_value_heads": 2,
        "head_dim": 256, "rms_norm_eps": 1e-6, "num_experts": 256, "num_experts_per_tok": 8,
        "moe_intermediate_size": 512, "shared_expert_intermediate_size": 512,
        "linear_num_key_heads": 16, "linear_num_value_heads": 32,
        "rope_parameters": {"rope_theta": 1e7, "partial_rotary_factor": 0.25},
        "layer_types": ["linear_attention"] * 3 + ["full_attention"]})
    ref = get_config("qwen3.6-35b-a3b")
    for f in ("hidden_size", "num_layers", "num_heads", "num_kv_heads", "head_dim", "num_experts",
              "num_experts_per_tok", "moe_intermediate_size", "full_attention_interval",
              "linear_num_key_heads", "linear_num_value_heads", "rot_dim", "attn_output_gate",
              "shared_expert_gate", "qk_norm"):
        assert getattr(cfg, f) == getattr(ref, f), f
    assert [cfg.is_linear_layer(i) for i in range(8)] == [True] * 3 + [False] + [True] * 3 + [False]


def test_prefill_and_decode_match_hf():
    cfg = get_config("tiny-qwen36")
    hfm = _hf_model(cfg)
    ours = _ours(cfg, hfm.state_dict())
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (11,), generator=g)
    with torch.no_grad():
        out = hfm(ids.view(1, -1), use_cache=True)
    pkv = out.past_key_values
    want = out.logits[0, -1]

    ours.kv.add_sequence("s")
    b = build_batch(ours, ["s"], [len(ids)], [0], False)
    hid = ours.embed_tokens(ids.to(torch.int32))
    ours.forward(b, hid)
    got = ours.head(hid[-1:].contiguous())[0]
    _close(got, want)

    # Three decode steps through both caches (HF: recurrent form).
    pos = len(ids)
    for step in range(3):
        tok = int(torch.argmax(want))
        with torch.no_grad():
            out = hfm(torch.tensor([[tok]]), past_key_values=pkv, use_cache=True)
        pkv = out.past_key_values
        want = out.logits[0, -1]
        b = build_batch(ours, ["s"], [1], [pos], True)
        hid = ours.embed_tokens(torch.tensor([tok], dtype=torch.int32))
        ours.forward(b, hid)
        got = ours.head(hid)[0]
        _close(got, want)
        pos += 1


def test_two_sequences_keep_separate_state():
    cfg = get_config("tiny-qwen36")
    hfm = _hf_model(cfg, seed=4)
    sd = hfm.state_dict()
    g = torch.Generator().manual_seed(5)
    p1 = torch.randint(0, cfg.vocab_size, (7,), generator=g)
    p2 = torch.randint(0, cfg.vocab_size, (4,), generator=g)
    solo = []
    for p in (p1, p2):
        m = _ours(cfg, sd)
        m.kv.add_sequence("x")
        b = build_batch(m, ["x"], [len(p)], [0], False)
        hid = m.embed_tokens(p.to(torch.int32))
        m.forward(b, hid)
        solo.append(m.head(hid[-1:].contiguous())[0])
    m = _ours(cfg, sd)
    for s in ("a", "b"):
        m.kv.add_sequence(s)
    b = build_batch(m, ["a", "b"], [7, 4], [0, 0], False)
    hid = m.embed_tokens(torch.cat([p1, p2]).to(torch.int32))
    m.forward(b, hid)
    both = m.head(hid[[6, 10]].contiguous())
    # Batched CPU matmuls may round differently from solo ones; states must
    # not leak between the sequences (that would be a gross difference).
    _close(both[0], solo[0], 0.01)
    _close(both[1], solo[1], 0.01)
    with pytest.raises(NotImplementedError):
        m.kv.truncate("a", 3)


def _hybrid_engine(device, **kw):
    from cascadia_b200.engine.llm import LLMEngine

    cfg = get_config("tiny-qwen36")
    m = HybridMoEModel(cfg, device).init_random(seed=21, gen_device="cpu")
    m.allocate_kv(128, max_seqs=8)
    return LLMEngine(m, max_model_len=256, max_running=8, **kw)


def _run(engine, tasks, max_steps=400):
    for t in tasks:
        engine.submit(t)
    out = {t.task_id: [] for t in tasks}
    for _ in range(max_steps):
        for tid, c in engine.step():
            out[tid].append(c)
        if all(out[t.task_id] and out[t.task_id][-1].is_final for t in tasks):
            break
    return {k: [c.token_id for c in v if not c.is_final] for k, v in out.items()}


@pytest.mark.parametrize("device", ["cpu", pytest.param("cuda", marks=pytest.mark.gpu)])
def test_hybrid_engine_batched_solo_and_chunked(device):
    from cascadia_b200.types import GenerationTask

    e = _hybrid_engine(device)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(3, 500, (n,), generator=g).tolist() for n in (5, 24, 11)]
    tasks = [GenerationTask(f"t{i}", "", max_tokens=4, prompt_ids=p) for i, p in enumerate(prompts)]
    batched = _run(e, tasks)
    def same(a, b):
        # CPU: bit-identical.  GPU: batch size changes the cuBLAS algorithm
        # of the shared-expert gate and the attention split plan, so a late
        # near-tie may flip; leaked state would change every token.
        if device == "cpu":
            return a == b
        return a[:2] == b[:2]

    for i, t in enumerate(tasks):
        solo = _run(e, [GenerationTask(f"s{i}", "", max_tokens=4, prompt_ids=t.prompt_ids)])
        assert same(solo[f"s{i}"], batched[t.task_id]), (solo, batched)
    # Prefill in chunks carries the conv and recurrent state across chunks.
    e.sched.max_prefill_tokens = 8
    chunked = _run(e, [GenerationTask("c", "", max_tokens=4, prompt_ids=prompts[1])])
    assert same(chunked["c"], batched["t1"]), (chunked, batched)
    assert not e.model.kv.slot_of and len(e.model.kv.free_slots) == 8
