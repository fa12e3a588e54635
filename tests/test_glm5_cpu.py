"""GLM-5 (MLA + DSA indexer + sigmoid-routed MoE): our CPU oracle path
against the published HuggingFace definition (transformers ``glm_moe_dsa``)
on a tiny random model with INT4-representable projections.  The index top-k
is 8, so prompts longer than 8 tokens exercise the sparse selection."""
import dataclasses

import pytest
import torch

from cascadia_b200.models.config import ModelConfig, get_config
from cascadia_b200.models.glm5 import GLM5Model, load_hf_weights
from cascadia_b200.models.llama import build_batch
from cascadia_b200.quant import Int4Weight

hf = pytest.importorskip("transformers.models.glm_moe_dsa.modeling_glm_moe_dsa")
hfc = pytest.importorskip("transformers.models.glm_moe_dsa.configuration_glm_moe_dsa")


def _cfg_all_full():
    # HF's definition gives every layer its own indexer (no IndexShare).
    return dataclasses.replace(get_config("tiny-glm5"), indexer_types=None)


def _hf_model(ours: ModelConfig, seed=0):
    cfg = hfc.GlmMoeDsaConfig(
        vocab_size=ours.vocab_size, hidden_size=ours.hidden_size,
        intermediate_size=ours.intermediate_size, moe_intermediate_size=ours.moe_intermediate_size,
        num_hidden_layers=ours.num_layers, num_attention_heads=ours.num_heads,
        num_key_value_heads=ours.num_heads, n_shared_experts=1,
        n_routed_experts=ours.num_experts, routed_scaling_factor=ours.routed_scaling_factor,
        kv_lora_rank=512, q_lora_rank=ours.q_lora_rank, qk_rope_head_dim=64,
        v_head_dim=ours.v_head_dim, qk_nope_head_dim=ours.qk_nope_head_dim, n_group=1,
        topk_group=1, num_experts_per_tok=ours.num_experts_per_tok, norm_topk_prob=True,
        rms_norm_eps=ours.rms_eps, index_topk=ours.index_topk, index_head_dim=128,
        index_n_heads=ours.index_n_heads,
        mlp_layer_types=["dense"] * ours.first_k_dense_replace +
        ["sparse"] * (ours.num_layers - ours.first_k_dense_replace),
        rope_parameters={"rope_type": "default", "rope_theta": ours.rope_theta},
        tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    m = hf.GlmMoeDsaForCausalLM(cfg).eval()
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if p.dim() == 1:
                if "indexer.k_norm" in name:
                    p.copy_((1.0 if name.endswith("weight") else 0.0) +
                            0.1 * torch.randn(p.shape, generator=g))
                else:  # RMSNorm weights: bf16-exact
                    p.copy_((1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(torch.bfloat16))
            elif "embed" in name or "mlp.gate.weight" in name or "weights_proj" in name:
                p.normal_(0, 0.3 if "gate" in name else 0.05, generator=g)
                p.copy_(p.to(torch.bfloat16).float())
            else:
                if "lm_head" not in name:
                    p.normal_(0, 0.05, generator=g)
                flat = p.reshape(-1, p.shape[-1])
                p.copy_(Int4Weight.quantize(flat.float(), 128).dequant_bf16().float().view_as(p))
        for mod in m.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.copy_(0.1 * torch.randn(
                    mod.e_score_correction_bias.shape, generator=g))
    return m


def _ours(cfg, sd):
    m = GLM5Model(cfg, "cpu")
    load_hf_weights(m, sd)
    m.allocate_kv(64)
    return m


def _close(a, b, frac=0.05):
    # bf16 activations on our side vs HF fp32 (HF's own bf16 run differs by
    # a few percent of the largest logit on these models).
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item()
    assert err <= frac * scale + 1e-3, (err, scale)


def test_hf_config_maps_to_glm5_preset():
    cfg = ModelConfig.from_hf({
        "model_type": "glm_moe_dsa", "vocab_size": 154880, "hidden_size": 6144,
        "num_hidden_layers": 78, "num_attention_heads": 64, "num_key_value_heads": 64,
        "intermediate_size": 12288, "moe_intermediate_size": 2048, "n_routed_experts": 256,
        "n_shared_experts": 1, "num_experts_per_tok": 8, "routed_scaling_factor": 2.5,
        "kv_lora_rank": 512, "q_lora_rank": 2048, "qk_rope_head_dim": 64, "v_head_dim": 256,
        "qk_nope_head_dim": 192, "index_topk": 2048, "index_n_heads": 32, "index_head_dim": 128,
        "rope_parameters": {"rope_theta": 8e6}, "mlp_layer_types": ["dense"] * 3 + ["sparse"] * 75})
    ref = get_config("glm-5")
    for f in ("hidden_size", "num_layers", "num_heads", "q_lora_rank", "kv_lora_rank",
              "qk_nope_head_dim", "v_head_dim", "index_topk", "index_n_heads", "num_experts",
              "first_k_dense_replace", "router", "routed_scaling_factor", "mla_rope_interleaved",
              "rope_theta"):
        assert getattr(cfg, f) == getattr(ref, f), f


def _capture_hf(hfm, ids):
    """HF logits plus, per layer, the indexer's inputs and its top-k output."""
    inputs, sel = {}, {}

    def pre(mod, args, kwargs):
        x = kwargs.get("hidden_states", args[0] if args else None)
        qa = kwargs.get("q_resid", args[1] if len(args) > 1 else None)
        inputs.setdefault(mod.layer_idx, (x[0], qa[0]))

    def post(mod, args, kwargs, out):
        sel.setdefault(mod.layer_idx, out[0])

    hooks = []
    for layer in hfm.model.layers:
        hooks.append(layer.self_attn.indexer.register_forward_pre_hook(pre, with_kwargs=True))
        hooks.append(layer.self_attn.indexer.register_forward_hook(post, with_kwargs=True))
    with torch.no_grad():
        out = hfm(ids.view(1, -1), use_cache=True)
    for h in hooks:
        h.remove()
    return out, inputs, sel


def test_indexer_selection_matches_hf_on_the_same_inputs():
    """Our indexer (CPU path) fed HF's own per-layer inputs picks HF's top-k,
    except where two scores tie within rounding."""
    cfg = _cfg_all_full()
    hfm = _hf_model(cfg)
    ours = _ours(cfg, hfm.state_dict())
    n = 21
    ids = torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(7))
    _, inputs, hf_sel = _capture_hf(hfm, ids)
    ours.kv.add_sequence("s")
    b = build_batch(ours, ["s"], [n], [0], False)
    for layer in range(cfg.num_layers):
        x, qa = inputs[layer]
        ind = ours.layers[layer].qkv.indexer
        sc, thr = ours._index(ours.idx_slot[layer], ind, x.to(torch.bfloat16),
                              qa.to(torch.bfloat16), b)
        for q in range(n):
            mine = set(torch.nonzero(sc[q, :q + 1] >= thr[q]).flatten().tolist())
            theirs = set(int(t) for t in hf_sel[layer][q].tolist() if t <= q)
            if mine != theirs:  # only a near-tie at the boundary may differ
                diff = sorted(mine ^ theirs)
                v = sc[q, diff]
                spread = (sc[q, :q + 1].max() - sc[q, :q + 1].min()).item()
                assert (v.max() - v.min()).item() <= 0.01 * spread, (layer, q, diff, v)


@pytest.mark.parametrize("n", [6, 21])
def test_prefill_and_decode_match_hf_given_hf_selection(n):
    """Attention restricted to HF's own top-k positions (so near-tie swaps in
    the indexer cannot move a row elsewhere): every logit row matches."""
    cfg = _cfg_all_full()
    hfm = _hf_model(cfg)
    ours = _ours(cfg, hfm.state_dict())
    ids = torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(3 + n))
    out, _, hf_sel = _capture_hf(hfm, ids)
    pkv, want = out.past_key_values, out.logits[0]
    forced = {}

    def fixed(slot, ind, x, qa, batch):
        top = forced[slot]                      # [T, k] HF indices
        T = top.shape[0]
        ld = max(batch.ctx_lens)
        sc = torch.zeros(T, ld)
        sc.scatter_(1, top.clamp(max=ld - 1).long(), 1.0)
        return sc, torch.ones(T)

    forced.update(hf_sel)
    ours._index = fixed
    ours.kv.add_sequence("s")
    b = build_batch(ours, ["s"], [n], [0], False)
    hid = ours.embed_tokens(ids.to(torch.int32))
    ours.forward(b, hid)
    _close(ours.head(hid), want)
    pos = n
    for step in range(2):
        tok = int(torch.argmax(want[-1]))
        cap = {}

        def post(mod, args, kwargs, o):
            cap.setdefault(mod.layer_idx, o[0])

        hooks = [layer.self_attn.indexer.register_forward_hook(post, with_kwargs=True)
                 for layer in hfm.model.layers]
        with torch.no_grad():
            out = hfm(torch.tensor([[tok]]), past_key_values=pkv, use_cache=True)
        for h in hooks:
            h.remove()
        pkv, want = out.past_key_values, out.logits[0]
        forced.update(cap)
        b = build_batch(ours, ["s"], [1], [pos], True)
        hid = ours.embed_tokens(torch.tensor([tok], dtype=torch.int32))
        ours.forward(b, hid)
        _close(ours.head(hid), want)
        pos += 1
