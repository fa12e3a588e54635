"""Model configurations for the architectures the engine serves.

The field names follow HF ``config.json`` (what the reference reads through
``load_model_config``, crates/cascadia-engine-openvino/src/rotary.rs:186) so a
real config can be loaded with :meth:`ModelConfig.from_hf`.
"""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass, field
from typing import Optional

import torch


@dataclass
class ModelConfig:
    arch: str = "llama"  # llama | qwen3_moe | kimi_k2 (deepseek-v3 style MLA + MoE)
    vocab_size: int = 128256
    hidden_size: int = 4096
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    rope_theta: float = 500000.0
    rope_scaling: Optional[dict] = None
    rms_eps: float = 1e-5
    tie_word_embeddings: bool = False
    partial_rotary_factor: float = 1.0
    max_position: int = 131072
    group_size: int = 128
    # Sliding-window attention (0: full causal): keys within the last
    # `sliding_window` positions plus the first `attention_sinks` ones.
    sliding_window: int = 0
    attention_sinks: int = 0
    eos_token_ids: tuple = (128001, 128009)
    # --- sparse MoE ---
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    num_shared_experts: int = 0
    router: str = "softmax"  # softmax | sigmoid
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 1.0
    first_k_dense_replace: int = 0
    qk_norm: bool = False
    # --- MLA ---
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_rope_head_dim: int = 0
    qk_nope_head_dim: int = 0
    v_head_dim: int = 0
    # --- DSA sparse attention (GLM-5 / DeepSeek-V3.2 lightning indexer) ---
    index_topk: int = 0                # 0: dense attention
    index_n_heads: int = 0
    index_head_dim: int = 128
    indexer_types: Optional[tuple] = None  # per layer "full" | "shared" (None: all full)
    mla_rope_interleaved: bool = True  # False: checkpoint rotates split halves (NeoX)
    num_nextn_predict_layers: int = 0  # MTP draft layers stored after the last layer
    # --- Gemma-4 (per-layer attention types, PLE, shared KV) ---
    layer_types: Optional[tuple] = None   # per layer "sliding_attention" | "full_attention"
    local_window: int = 0                 # window of the sliding layers
    global_head_dim: int = 0
    num_global_kv_heads: int = 0
    attention_k_eq_v: bool = False
    num_kv_shared_layers: int = 0
    use_double_wide_mlp: bool = False
    hidden_size_per_layer_input: int = 0
    vocab_size_per_layer_input: int = 0
    final_logit_softcapping: float = 0.0
    rope_theta_local: float = 10000.0
    global_partial_rotary: float = 1.0
    gemma_moe: bool = False               # MoE block beside every layer's MLP (enable_moe_block)
    # --- hybrid linear attention (Qwen3.5 / Qwen3.6: Gated DeltaNet layers,
    # every full_attention_interval-th layer full attention) ---
    full_attention_interval: int = 0   # 0: no linear-attention layers
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    attn_output_gate: bool = False     # full attention output * sigmoid(gate)
    shared_expert_gate: bool = False   # shared expert output * sigmoid(w . x)
    shared_expert_intermediate_size: int = 0

    @property
    def is_gemma4(self) -> bool:
        return self.arch == "gemma4"

    @property
    def is_dsa(self) -> bool:
        return self.index_topk > 0

    def layer_has_indexer(self, li: int) -> bool:
        """Layer li computes its own DSA top-k (IndexShare: "shared" layers
        reuse the previous indexer layer's selection)."""
        if not self.is_dsa:
            return False
        # The MTP layer (index num_layers) owns its indexer.
        if self.indexer_types is None or li >= len(self.indexer_types):
            return True
        return self.indexer_types[li] == "full"

    @property
    def is_hybrid(self) -> bool:
        return self.full_attention_interval > 0

    def is_linear_layer(self, li: int) -> bool:
        """Layer li is a Gated DeltaNet layer (the rest are full attention)."""
        return self.is_hybrid and (li + 1) % self.full_attention_interval != 0

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @property
    def rot_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def to_json(self) -> str:
        return json.dumps(asdict(self), indent=1)

    @staticmethod
    def from_dict(d: dict) -> "ModelConfig":
        known = {f for f in ModelConfig.__dataclass_fields__}
        kw = {k: v for k, v in d.items() if k in known}
        if "eos_token_ids" in kw and isinstance(kw["eos_token_ids"], list):
            kw["eos_token_ids"] = tuple(kw["eos_token_ids"])
        return ModelConfig(**kw)

    @staticmethod
    def from_hf(d: dict) -> "ModelConfig":
        """Map a HuggingFace config.json dict (Llama/Qwen3-MoE/DeepSeek-V3)."""
        d = d.get("text_config", d)
        heads = d["num_attention_heads"]
        hidden = d["hidden_size"]
        c = ModelConfig(
            vocab_size=d["vocab_size"],
            hidden_size=hidden,
            num_layers=d["num_hidden_layers"],
            num_heads=heads,
            num_kv_heads=d.get("num_key_value_heads", heads),
            head_dim=d.get("head_dim") or hidden // heads,
            intermediate_size=d.get("intermediate_size", 0),
            rope_theta=float(d.get("rope_theta", 10000.0)),
            rope_scaling=d.get("rope_scaling"),
            rms_eps=float(d.get("rms_norm_eps", 1e-5)),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            partial_rotary_factor=float(d.get("partial_rotary_factor", 1.0)),
            max_position=int(d.get("max_position_embeddings", 131072)),
        )
        if d.get("sliding_window") and d.get("use_sliding_window", True) and \
                d.get("model_type", "") in ("mistral", "mixtral", "qwen2", "starcoder2"):
            c.sliding_window = int(d["sliding_window"])
        eos = d.get("eos_token_id")
        if eos is not None:
            c.eos_token_ids = tuple(eos) if isinstance(eos, list) else (eos,)
        mt = d.get("model_type", "")
        if d.get("num_experts") or d.get("n_routed_experts"):
            c.num_experts = d.get("num_experts") or d.get("n_routed_experts")
            c.num_experts_per_tok = d.get("num_experts_per_tok") or d.get("top_k_experts")
            c.moe_intermediate_size = d["moe_intermediate_size"]
            c.num_shared_experts = d.get("n_shared_experts", 0) or 0
            c.norm_topk_prob = bool(d.get("norm_topk_prob", True))
            c.routed_scaling_factor = float(d.get("routed_scaling_factor", 1.0))
            c.first_k_dense_replace = int(d.get("first_k_dense_replace", 0))
            c.router = "sigmoid" if d.get("scoring_func") == "sigmoid" else "softmax"
            c.arch = "kimi_k2" if d.get("kv_lora_rank") else "qwen3_moe"
        if d.get("kv_lora_rank"):
            c.q_lora_rank = d.get("q_lora_rank") or 0
            c.kv_lora_rank = d["kv_lora_rank"]
            c.qk_rope_head_dim = d["qk_rope_head_dim"]
            c.qk_nope_head_dim = d["qk_nope_head_dim"]
            c.v_head_dim = d["v_head_dim"]
        if mt == "glm_moe_dsa" or d.get("index_topk"):
            rp = d.get("rope_parameters") or {}
            c.arch = "glm5"
            c.rope_theta = float(rp.get("rope_theta", d.get("rope_theta", c.rope_theta)))
            c.rope_scaling = None
            c.index_topk = int(d["index_topk"])
            c.index_n_heads = int(d.get("index_n_heads", 32))
            c.index_head_dim = int(d.get("index_head_dim", 128))
            if d.get("indexer_types"):
                c.indexer_types = tuple(d["indexer_types"])
            c.mla_rope_interleaved = False
            c.num_nextn_predict_layers = int(d.get("num_nextn_predict_layers", 0))
            c.router = "sigmoid"
            types = d.get("mlp_layer_types")
            c.first_k_dense_replace = types.index("sparse") if types and "sparse" in types else \
                int(d.get("first_k_dense_replace", 3))
        if mt.startswith("gemma4"):
            rp = d.get("rope_parameters") or {}
            c.arch = "gemma4"
            c.layer_types = tuple(d["layer_types"])
            c.local_window = int(d.get("sliding_window", 512))
            c.global_head_dim = int(d.get("global_head_dim") or c.head_dim)
            c.num_global_kv_heads = int(d.get("num_global_key_value_heads") or c.num_kv_heads)
            c.attention_k_eq_v = bool(d.get("attention_k_eq_v", False))
            c.num_kv_shared_layers = int(d.get("num_kv_shared_layers", 0))
            c.use_double_wide_mlp = bool(d.get("use_double_wide_mlp", False))
            c.hidden_size_per_layer_input = int(d.get("hidden_size_per_layer_input") or 0)
            c.vocab_size_per_layer_input = int(d.get("vocab_size_per_layer_input") or 0)
            c.final_logit_softcapping = float(d.get("final_logit_softcapping") or 0.0)
            c.rope_theta_local = float(rp.get("sliding_attention", {}).get("rope_theta", 10000.0))
            fa = rp.get("full_attention", {})
            c.rope_theta = float(fa.get("rope_theta", 1e6))
            c.global_partial_rotary = float(fa.get("partial_rotary_factor", 1.0))
            c.rope_scaling = None
            c.tie_word_embeddings = bool(d.get("tie_word_embeddings", True))
            if d.get("enable_moe_block"):
                c.gemma_moe = True
                c.num_experts = int(d["num_experts"])
                c.num_experts_per_tok = int(d["top_k_experts"])
                c.moe_intermediate_size = int(d["moe_intermediate_size"])
                c.router = "softmax"
                c.norm_topk_prob = True
        if mt.startswith("qwen3"):
            c.qk_norm = True
        if mt.startswith("qwen3_5") or mt.startswith("qwen3_next"):
            rp = d.get("rope_parameters") or {}
            c.arch = "qwen3_5_moe"
            c.rope_theta = float(rp.get("rope_theta", d.get("rope_theta", 10000000.0)))
            c.partial_rotary_factor = float(rp.get("partial_rotary_factor",
                                                   d.get("partial_rotary_factor", 0.25)))
            c.rope_scaling = None
            types = d.get("layer_types")
            c.full_attention_interval = (types.index("full_attention") + 1) if types else int(
                d.get("full_attention_interval", 4))
            c.linear_num_key_heads = d["linear_num_key_heads"]
            c.linear_num_value_heads = d["linear_num_value_heads"]
            c.linear_key_head_dim = d.get("linear_key_head_dim", 128)
            c.linear_value_head_dim = d.get("linear_value_head_dim", 128)
            c.linear_conv_kernel_dim = d.get("linear_conv_kernel_dim", 4)
            c.attn_output_gate = True
            if d.get("shared_expert_intermediate_size"):
                c.shared_expert_gate = True
                c.shared_expert_intermediate_size = d["shared_expert_intermediate_size"]
                c.num_shared_experts = 1
        return c


LLAMA3_SCALING = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                  "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}

PRESETS = {
    # BASELINE config #2 (north-star).
    "llama-3.1-8b": ModelConfig(rope_scaling=dict(LLAMA3_SCALING)),
    # BASELINE config #1 and the spec-decode draft.
    "llama-3.2-1b": ModelConfig(hidden_size=2048, num_layers=16, num_heads=32, num_kv_heads=8,
                                head_dim=64, intermediate_size=8192,
                                rope_scaling=dict(LLAMA3_SCALING, factor=32.0),
                                tie_word_embeddings=True),
    # BASELINE config #4.
    "qwen3-30b-a3b": ModelConfig(arch="qwen3_moe", vocab_size=151936, hidden_size=2048,
                                 num_layers=48, num_heads=32, num_kv_heads=4, head_dim=128,
                                 intermediate_size=6144, rope_theta=1000000.0, rms_eps=1e-6,
                                 num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768,
                                 router="softmax", norm_topk_prob=True, qk_norm=True,
                                 eos_token_ids=(151645, 151643)),
    # BASELINE config #5 (DeepSeek-V3-style MLA + MoE), INT4 group 32.
    "kimi-k2": ModelConfig(arch="kimi_k2", vocab_size=163840, hidden_size=7168, num_layers=61,
                           num_heads=64, num_kv_heads=64, head_dim=192, intermediate_size=18432,
                           rope_theta=50000.0, rms_eps=1e-6, num_experts=384,
                           num_experts_per_tok=8, moe_intermediate_size=2048,
                           num_shared_experts=1, router="sigmoid", norm_topk_prob=True,
                           routed_scaling_factor=2.827, first_k_dense_replace=1,
                           q_lora_rank=1536, kv_lora_rank=512, qk_rope_head_dim=64,
                           qk_nope_head_dim=128, v_head_dim=128, group_size=32,
                           rope_scaling={"rope_type": "yarn", "factor": 64.0, "beta_fast": 32.0,
                                         "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0,
                                         "original_max_position_embeddings": 4096},
                           eos_token_ids=(163586,)),
    # GLM-5 (HF glm_moe_dsa): MLA + DSA lightning indexer (top-2048), 3 dense
    # + 75 MoE layers (256 experts top-8, sigmoid + bias, 1 shared).
    "glm-5": ModelConfig(arch="glm5", vocab_size=154880, hidden_size=6144, num_layers=78,
                         num_heads=64, num_kv_heads=64, head_dim=256, intermediate_size=12288,
                         rope_theta=8000000.0, rms_eps=1e-5, num_experts=256,
                         num_experts_per_tok=8, moe_intermediate_size=2048, num_shared_experts=1,
                         router="sigmoid", norm_topk_prob=True, routed_scaling_factor=2.5,
                         first_k_dense_replace=3, q_lora_rank=2048, kv_lora_rank=512,
                         qk_rope_head_dim=64, qk_nope_head_dim=192, v_head_dim=256,
                         index_topk=2048, index_n_heads=32, index_head_dim=128,
                         mla_rope_interleaved=False, group_size=32, max_position=202752,
                         num_nextn_predict_layers=1, eos_token_ids=(1,)),
    # Qwen3.6-35B-A3B (HF qwen3_5_moe): 30 Gated DeltaNet + 10 gated
    # full-attention layers (head_dim 256, rotary on 64 dims), 256 experts
    # top-8 + a sigmoid-gated shared expert.
    "qwen3.6-35b-a3b": ModelConfig(arch="qwen3_5_moe", vocab_size=248320, hidden_size=2048,
                                   num_layers=40, num_heads=16, num_kv_heads=2, head_dim=256,
                                   intermediate_size=512, rope_theta=10000000.0,
                                   partial_rotary_factor=0.25, rms_eps=1e-6, num_experts=256,
                                   num_experts_per_tok=8, moe_intermediate_size=512,
                                   num_shared_experts=1, router="softmax", norm_topk_prob=True,
                                   qk_norm=True, full_attention_interval=4,
                                   linear_num_key_heads=16, linear_num_value_heads=32,
                                   attn_output_gate=True, shared_expert_gate=True,
                                   shared_expert_intermediate_size=512,
                                   max_position=262144, eos_token_ids=(248046, 248044)),
    # Small shapes for tests (same code paths).
    "tiny-llama": ModelConfig(vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                              num_kv_heads=2, head_dim=64, intermediate_size=512,
                              rope_scaling=dict(LLAMA3_SCALING), eos_token_ids=(1,)),
    "tiny-llama-128": ModelConfig(vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8,
                                  num_kv_heads=2, head_dim=128, intermediate_size=1024,
                                  eos_token_ids=(1,)),
    # Eight KV heads: splits over up to 8 tensor-parallel ranks.
    "tiny-llama-kv8": ModelConfig(vocab_size=1024, hidden_size=1024, num_layers=2, num_heads=8,
                                  num_kv_heads=8, head_dim=128, intermediate_size=1024,
                                  eos_token_ids=(1,)),
    "tiny-moe": ModelConfig(arch="qwen3_moe", vocab_size=512, hidden_size=256, num_layers=2,
                            num_heads=4, num_kv_heads=2, head_dim=64, intermediate_size=512,
                            num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
                            router="softmax", qk_norm=True, eos_token_ids=(1,)),
    # Kimi-K2 layer structure at small width; the MLA latent (512) and rope
    # (64) widths are the real ones (the decode kernel is built for them).
    "tiny-mla": ModelConfig(arch="kimi_k2", vocab_size=512, hidden_size=256, num_layers=3,
                            num_heads=20, num_kv_heads=20, head_dim=192, intermediate_size=512,
                            num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
                            num_shared_experts=1, router="sigmoid", routed_scaling_factor=2.5,
                            first_k_dense_replace=1, q_lora_rank=128, kv_lora_rank=512,
                            qk_rope_head_dim=64, qk_nope_head_dim=128, v_head_dim=128,
                            group_size=32, rope_theta=50000.0,
                            rope_scaling={"rope_type": "yarn", "factor": 64.0, "beta_fast": 32.0,
                                          "beta_slow": 1.0, "mscale": 1.0,
                                          "mscale_all_dim": 1.0,
                                          "original_max_position_embeddings": 4096},
                            eos_token_ids=(1,)),
    # Gemma-4 layer structure at small width: sliding (head_dim 256, window
    # 16) and full (head_dim 512, K = V, one KV head) layers, 2 shared-KV
    # layers with double-wide MLPs, per-layer inputs, soft-capped logits.
    "tiny-gemma4": ModelConfig(arch="gemma4", vocab_size=512, hidden_size=256, num_layers=6,
                               num_heads=4, num_kv_heads=2, head_dim=256, intermediate_size=512,
                               rms_eps=1e-6, tie_word_embeddings=True,
                               layer_types=("sliding_attention", "sliding_attention",
                                            "full_attention", "sliding_attention",
                                            "sliding_attention", "full_attention"),
                               local_window=16, global_head_dim=512, num_global_kv_heads=1,
                               attention_k_eq_v=True, num_kv_shared_layers=2,
                               use_double_wide_mlp=True, hidden_size_per_layer_input=128,
                               vocab_size_per_layer_input=512, final_logit_softcapping=30.0,
                               rope_theta=1000000.0, rope_theta_local=10000.0,
                               global_partial_rotary=0.25, eos_token_ids=(1,)),
    # The MoE-block variant (dense MLP + routed experts in every layer).
    "tiny-gemma4-moe": ModelConfig(arch="gemma4", vocab_size=512, hidden_size=256, num_layers=4,
                                   num_heads=4, num_kv_heads=2, head_dim=256,
                                   intermediate_size=256, rms_eps=1e-6, tie_word_embeddings=True,
                                   layer_types=("sliding_attention", "sliding_attention",
                                                "sliding_attention", "full_attention"),
                                   local_window=16, global_head_dim=512, num_global_kv_heads=1,
                                   attention_k_eq_v=True, final_logit_softcapping=30.0,
                                   rope_theta=1000000.0, rope_theta_local=10000.0,
                                   global_partial_rotary=0.25, gemma_moe=True, num_experts=8,
                                   num_experts_per_tok=2, moe_intermediate_size=128,
                                   router="softmax", norm_topk_prob=True, eos_token_ids=(1,)),
    # GLM-5 layer structure at small width: MLA (latent 512, rope 64; nope
    # 192 / v 256 as in GLM-5), DSA indexer with top-8 (so selection matters
    # at test lengths), IndexShare on layer 2, 1 dense + 2 MoE layers.
    "tiny-glm5": ModelConfig(arch="glm5", vocab_size=512, hidden_size=256, num_layers=3,
                             num_heads=8, num_kv_heads=8, head_dim=256, intermediate_size=512,
                             rope_theta=8000000.0, rms_eps=1e-5, num_experts=8,
                             num_experts_per_tok=2, moe_intermediate_size=128,
                             num_shared_experts=1, router="sigmoid", norm_topk_prob=True,
                             routed_scaling_factor=2.5, first_k_dense_replace=1, q_lora_rank=256,
                             kv_lora_rank=512, qk_rope_head_dim=64, qk_nope_head_dim=192,
                             v_head_dim=256, index_topk=8, index_n_heads=16, index_head_dim=128,
                             indexer_types=("full", "full", "shared"), mla_rope_interleaved=False,
                             num_nextn_predict_layers=1, eos_token_ids=(1,)),
    # Qwen3.6 layer structure at small width (linear head dims are the real
    # 128; full attention head_dim 256 as in the real model).
    "tiny-qwen36": ModelConfig(arch="qwen3_5_moe", vocab_size=512, hidden_size=256, num_layers=4,
                               num_heads=4, num_kv_heads=2, head_dim=256, intermediate_size=128,
                               rope_theta=10000000.0, partial_rotary_factor=0.25, rms_eps=1e-6,
                               num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
                               num_shared_experts=1, router="softmax", norm_topk_prob=True,
                               qk_norm=True, full_attention_interval=4, linear_num_key_heads=2,
                               linear_num_value_heads=4, attn_output_gate=True,
                               shared_expert_gate=True, shared_expert_intermediate_size=128,
                               eos_token_ids=(1,)),
}


def get_config(name: str) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    from copy import deepcopy

    return deepcopy(PRESETS[name])


def rope_inv_freq(cfg: ModelConfig, rot: Optional[int] = None) -> torch.Tensor:
    rot = rot or cfg.rot_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
    sc = cfg.rope_scaling
    if sc and sc.get("rope_type", sc.get("type")) == "llama3":
        # crates/cascadia-engine-openvino/src/rotary.rs:111-140
        factor = sc["factor"]
        low, high = sc["low_freq_factor"], sc["high_freq_factor"]
        old = float(sc["original_max_position_embeddings"])
        low_wl, high_wl = old / low, old / high
        wl = 2 * math.pi / inv
        smooth = (old / wl - low) / (high - low)
        mid = (1 - smooth) * inv / factor + smooth * inv
        inv = torch.where(wl < high_wl, inv, torch.where(wl > low_wl, inv / factor, mid))
    elif sc and sc.get("rope_type", sc.get("type")) == "yarn":
        # YaRN blend of extrapolated and interpolated frequencies
        # (crates/cascadia-int4-gemm/src/shell.rs:395-429, the published
        # YaRN correction-dimension ramp).
        factor = float(sc["factor"])
        base = cfg.rope_theta
        old = float(sc.get("original_max_position_embeddings", 4096))
        beta_fast = float(sc.get("beta_fast", 32.0))
        beta_slow = float(sc.get("beta_slow", 1.0))

        def corr_dim(n_rot):
            return (rot * math.log(old / (n_rot * 2 * math.pi))) / (2 * math.log(base))
        low = max(math.floor(corr_dim(beta_fast)), 0.0)
        high = min(math.ceil(corr_dim(beta_slow)), rot - 1.0)
        denom = high - low if abs(high - low) > 1e-6 else 0.001
        i = torch.arange(rot // 2, dtype=torch.float64)
        ramp = ((i - low) / denom).clamp(0.0, 1.0)
        inv_mask = 1.0 - ramp
        inv = (inv / factor) * (1.0 - inv_mask) + inv * inv_mask
    return inv.float()


def rope_mscale(cfg: ModelConfig) -> float:
    """Attention scale factor folded into cos / sin (YaRN mscale ratio)."""
    sc = cfg.rope_scaling
    if not (sc and sc.get("rope_type", sc.get("type")) == "yarn"):
        return 1.0

    def get(scale, m):
        return 1.0 if scale <= 1.0 else 0.1 * m * math.log(scale) + 1.0
    f = float(sc["factor"])
    return get(f, float(sc.get("mscale", 1.0))) / get(f, float(sc.get("mscale_all_dim", 1.0)))


def rope_table(cfg: ModelConfig, max_pos: int, rot: Optional[int] = None,
               device="cpu") -> torch.Tensor:
    """[max_pos, rot] fp32: cos in the first rot/2 columns, sin in the rest."""
    inv = rope_inv_freq(cfg, rot)
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv)
    ms = rope_mscale(cfg)
    return (torch.cat([ang.cos(), ang.sin()], dim=1) * ms).to(device)
