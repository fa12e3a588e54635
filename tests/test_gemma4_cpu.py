"""Gemma-4 text model: our CPU oracle path against the published
HuggingFace definition (transformers ``gemma4``) on a tiny random model with
sliding (head_dim 256, window 16) and full (head_dim 512, K = V) layers,
shared-KV layers with double-wide MLPs, per-layer inputs and soft-capped
logits; prefill beyond the window, then decode steps."""
import pytest
import torch

from cascadia_b200.models.config import ModelConfig, get_config
from cascadia_b200.models.gemma4 import Gemma4Model, load_hf_weights
from cascadia_b200.models.llama import build_batch
from cascadia_b200.quant import Int4Weight

hf = pytest.importorskip("transformers.models.gemma4.modeling_gemma4")
hfc = pytest.importorskip("transformers.models.gemma4.configuration_gemma4")


def _hf_model(ours: ModelConfig, seed=0):
    cfg = hfc.Gemma4TextConfig(
        vocab_size=ours.vocab_size, hidden_size=ours.hidden_size,
        intermediate_size=ours.intermediate_size, num_hidden_layers=ours.num_layers,
        num_attention_heads=ours.num_heads, num_key_value_heads=ours.num_kv_heads,
        head_dim=ours.head_dim, global_head_dim=ours.global_head_dim,
        num_global_key_value_heads=ours.num_global_kv_heads,
        attention_k_eq_v=ours.attention_k_eq_v, sliding_window=ours.local_window,
        num_kv_shared_layers=ours.num_kv_shared_layers,
        use_double_wide_mlp=ours.use_double_wide_mlp,
        hidden_size_per_layer_input=ours.hidden_size_per_layer_input,
        vocab_size_per_layer_input=ours.vocab_size_per_layer_input,
        final_logit_softcapping=ours.final_logit_softcapping, rms_norm_eps=ours.rms_eps,
        layer_types=list(ours.layer_types), tie_word_embeddings=True,
        **(dict(enable_moe_block=True, num_experts=ours.num_experts,
                top_k_experts=ours.num_experts_per_tok,
                moe_intermediate_size=ours.moe_intermediate_size) if ours.gemma_moe else {}))
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    m = hf.Gemma4ForCausalLM(cfg).eval()
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "router.scale" in name:
                # Ones (HF's init): the scale * H^-1/2 fold into the router
                # rows is then exact.
                p.fill_(1.0)
            elif "router.proj" in name:
                # A spread-out router: random near-ties between the k-th and
                # (k+1)-th expert would flip with bf16 rounding of the input.
                p.normal_(0, 1.0, generator=g)
                p.copy_(p.to(torch.bfloat16).float())
            elif p.dim() == 1 and ("q_norm" in name or "k_norm" in name):
                # Attention is unscaled (scale 1 on RMS-normalised q and k):
                # small norm weights keep the random model's softmax from
                # being near one-hot, where bf16 rounding alone (HF's own
                # bf16 run included) would pick other keys.
                p.copy_((0.2 + 0.02 * torch.randn(p.shape, generator=g)).to(torch.bfloat16))
            elif p.dim() == 1:
                p.copy_((1.0 + 0.1 * torch.randn(p.shape, generator=g)).to(torch.bfloat16))
            elif "embed_tokens_per_layer" in name:
                p.normal_(0, 0.05, generator=g)
                p.copy_(p.to(torch.bfloat16).float())
            elif "embed" in name:  # also the tied LM head: INT4-representable
                p.normal_(0, 0.05, generator=g)
                p.copy_(Int4Weight.quantize(p.float(), 128).dequant_bf16().float())
            else:  # 3-D expert tensors: groups along the last (input) dim
                p.normal_(0, 0.05, generator=g)
                flat = p.reshape(-1, p.shape[-1]).float()
                p.copy_(Int4Weight.quantize(flat, 128).dequant_bf16().float().view_as(p))
        for name, b in m.named_buffers():
            if name.endswith("layer_scalar"):
                b.copy_(torch.tensor([0.75]))
    return m


def _ours(cfg, sd):
    m = Gemma4Model(cfg, "cpu")
    # Tied head: the HF lm_head is the embedding (its INT4 copy on our side).
    sd = dict(sd)
    bufs = {k: v for k, v in sd.items()}
    load_hf_weights(m, bufs)
    m.allocate_kv(64)
    return m


def _close(a, b, frac=0.05):
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item()
    assert err <= frac * scale + 1e-3, (err, scale)


def test_hf_config_maps_to_gemma4():
    cfg = ModelConfig.from_hf({
        "model_type": "gemma4_text", "vocab_size": 262144, "hidden_size": 2560,
        "num_hidden_layers": 42, "num_attention_heads": 8, "num_key_value_heads": 2,
        "head_dim": 256, "global_head_dim": 512, "num_global_key_value_heads": 1,
        "attention_k_eq_v": True, "sliding_window": 512, "num_kv_shared_layers": 18,
        "hidden_size_per_layer_input": 256, "vocab_size_per_layer_input": 262144,
        "final_logit_softcapping": 30.0, "intermediate_size": 10240,
        "layer_types": (["sliding_attention"] * 5 + ["full_attention"]) * 7,
        "rope_parameters": {"sliding_attention": {"rope_theta": 10000.0},
                            "full_attention": {"rope_theta": 1e6, "partial_rotary_factor": 0.25}}})
    assert cfg.is_gemma4 and cfg.global_head_dim == 512 and cfg.local_window == 512
    assert cfg.global_partial_rotary == 0.25 and cfg.rope_theta == 1e6
    assert cfg.num_kv_shared_layers == 18 and cfg.attention_k_eq_v


@pytest.mark.parametrize("preset", ["tiny-gemma4", "tiny-gemma4-moe"])
def test_prefill_and_decode_match_hf(preset):
    cfg = get_config(preset)
    hfm = _hf_model(cfg)
    ours = _ours(cfg, hfm.state_dict())
    n = 27  # longer than the 16-token window
    ids = torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        out = hfm(ids.view(1, -1), use_cache=True)
    pkv, want = out.past_key_values, out.logits[0]
    ours.kv.add_sequence("s")
    b = build_batch(ours, ["s"], [n], [0], False)
    hid = ours.embed_tokens(ids.to(torch.int32))
    ours.forward(b, hid)
    _close(ours.head(hid), want)
    pos = n
    for step in range(3):
        tok = int(torch.argmax(want[-1]))
        with torch.no_grad():
            out = hfm(torch.tensor([[tok]]), past_key_values=pkv, use_cache=True)
        pkv, want = out.past_key_values, out.logits[0]
        b = build_batch(ours, ["s"], [1], [pos], True)
        hid = ours.embed_tokens(torch.tensor([tok], dtype=torch.int32))
        ours.forward(b, hid)
        _close(ours.head(hid), want)
        pos += 1


def test_hf_config_maps_moe_block():
    cfg = ModelConfig.from_hf({
        "model_type": "gemma4_text", "vocab_size": 262144, "hidden_size": 2816,
        "num_hidden_layers": 30, "num_attention_heads": 16, "num_key_value_heads": 8,
        "head_dim": 256, "global_head_dim": 512, "sliding_window": 1024,
        "intermediate_size": 2112, "enable_moe_block": True, "num_experts": 128,
        "top_k_experts": 8, "moe_intermediate_size": 704,
        "layer_types": (["sliding_attention"] * 5 + ["full_attention"]) * 5})
    assert cfg.gemma_moe and cfg.num_experts == 128 and cfg.num_experts_per_tok == 8
    assert cfg.moe_intermediate_size == 704 and cfg.router == "softmax"
