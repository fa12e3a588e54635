"""The `shard` checkpoint layout: per-stage INT4 weights plus stage manifests.

Directory layout and manifest keys follow the reference's exporter
(tools/export_shards.py:1562-1593 stage meta, :2197-2212 pipeline meta;
docs/SHARDING.md:27-39):

    <out>/pipeline_config.json
    <out>/tokenizer/                 (copied when a tokenizer exists)
    <out>/stage_<i>/stage_config.json
    <out>/stage_<i>/model.safetensors

Instead of OpenVINO IR, each stage holds safetensors of the canonical INT4
form (``<layer>.<proj>.packed`` int32 [N, K/8] + ``.scales`` fp16 [N, K/G],
symmetric group-128 — the NNCF INT4_SYM g128 the reference exports), the
layer norms, and the embedding (first stage) / final norm + LM head (last
stage).  ``stage_config.json`` additionally carries ``format`` and the full
``model_config`` so a stage loads without the original HF config.
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Optional

import torch
from safetensors.torch import load_file, save_file

from ..models.config import ModelConfig
from ..quant import Int4Weight
from ..types import ShardPlan, ShardSpec

EXPORT_VERSION = "b200_v1_int4"
PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def stage_plan(num_layers: int, num_stages: int, layer_split: Optional[List[int]] = None):
    """[(start, end)] per stage; explicit split (--layer-split) or uniform with
    the remainder on the last stage (tools/export_shards.py:517-566)."""
    if layer_split:
        if sum(layer_split) != num_layers or len(layer_split) != num_stages:
            raise ValueError(f"layer split {layer_split} does not cover {num_layers} layers "
                             f"in {num_stages} stages")
        out, c = [], 0
        for n in layer_split:
            out.append((c, c + n))
            c += n
        return out
    plan = ShardPlan.uniform("m", num_layers, 1, 1, 1, num_stages)
    return [(s.layer_start, s.layer_end) for s in plan.stages]


def _layer_tensors(cfg: ModelConfig, li: int, seed: int, std: float, device) -> Dict[str, torch.Tensor]:
    from ..models.llama import _layer_generator, random_int4

    g = _layer_generator(seed, li, device)
    h, d, gs = cfg.hidden_size, cfg.head_dim, cfg.group_size
    shapes = {"q_proj": (cfg.num_heads * d, h), "k_proj": (cfg.num_kv_heads * d, h),
              "v_proj": (cfg.num_kv_heads * d, h), "o_proj": (h, cfg.num_heads * d),
              "gate_proj": (cfg.intermediate_size, h), "up_proj": (cfg.intermediate_size, h),
              "down_proj": (h, cfg.intermediate_size)}
    t = {}
    for name in PROJ:
        w = random_int4(*shapes[name], g, device, std, gs)
        t[f"{name}.packed"] = w.packed.cpu()
        t[f"{name}.scales"] = w.scales.cpu()
    t["input_layernorm"] = torch.ones(h, dtype=torch.bfloat16)
    t["post_attention_layernorm"] = torch.ones(h, dtype=torch.bfloat16)
    return t


def write_random_shards(cfg: ModelConfig, out_dir: str, num_stages: int, model_id: str,
                        seed: int = 0, std: float = 0.02, layer_split=None,
                        device: str = "cpu", tokenizer_dir: Optional[str] = None) -> dict:
    """Random-init N(0, std) -> INT4 sym g128 shard tree (the BASELINE
    random-weights mode).  Uses the same per-layer seeds as
    ``LlamaModel.init_random`` so a shard loads into the same model."""
    from ..models.llama import _layer_generator

    os.makedirs(out_dir, exist_ok=True)
    plan = stage_plan(cfg.num_layers, num_stages, layer_split)
    quant = f"int4_sym_g{cfg.group_size}"
    for si, (ls, le) in enumerate(plan):
        sdir = os.path.join(out_dir, f"stage_{si}")
        os.makedirs(sdir, exist_ok=True)
        tensors: Dict[str, torch.Tensor] = {}
        has_embed, has_head = si == 0, si == len(plan) - 1
        embed = None
        if has_embed or (has_head and cfg.tie_word_embeddings):
            g = _layer_generator(seed, 100000, device)
            embed = (torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g, device=device)
                     * std).to(torch.bfloat16)
            if has_embed:
                tensors["embed_tokens"] = embed.cpu()
        for li in range(ls, le):
            for k, v in _layer_tensors(cfg, li, seed, std, device).items():
                tensors[f"layers.{li}.{k}"] = v
        if has_head:
            tensors["norm"] = torch.ones(cfg.hidden_size, dtype=torch.bfloat16)
            if cfg.tie_word_embeddings:
                head = Int4Weight.quantize(embed.float(), cfg.group_size)
            else:
                from ..models.llama import random_int4

                g = _layer_generator(seed, 100001, device)
                head = random_int4(cfg.vocab_size, cfg.hidden_size, g, device, std,
                                   cfg.group_size)
            tensors["lm_head.packed"] = head.packed.cpu()
            tensors["lm_head.scales"] = head.scales.cpu()
        save_file({k: v.contiguous() for k, v in tensors.items()},
                  os.path.join(sdir, "model.safetensors"))
        meta = {
            "stage": si, "layer_start": ls, "layer_end": le, "has_embed": has_embed,
            "has_head": has_head, "quantization": quant, "hidden_size": cfg.hidden_size,
            "vocab_size": cfg.vocab_size, "num_layers_total": cfg.num_layers,
            "num_kv_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "stateful": True,
            "rope_theta": cfg.rope_theta, "partial_rotary_factor": cfg.partial_rotary_factor,
            "arch_tag": cfg.arch, "target": "cuda", "static_seq": None, "static_context": None,
            "static_prefill_seq": None, "static_prefill_context": None,
            "inputs": "input_ids/hidden_states, positions, paged KV (block 16)",
            "cache_reorder": False, "export_version": EXPORT_VERSION,
            "format": quant, "model_config": json.loads(cfg.to_json()),
        }
        with open(os.path.join(sdir, "stage_config.json"), "w") as f:
            json.dump(meta, f, indent=2)
    pipeline = {
        "model_id": model_id, "num_stages": len(plan), "num_layers": cfg.num_layers,
        "hidden_size": cfg.hidden_size, "num_attention_heads": cfg.num_heads,
        "num_key_value_heads": cfg.num_kv_heads, "vocab_size": cfg.vocab_size,
        "rope_theta": cfg.rope_theta, "partial_rotary_factor": cfg.partial_rotary_factor,
        "arch_tag": cfg.arch, "quantization": quant, "export_version": EXPORT_VERSION,
        "model_config": json.loads(cfg.to_json()),
    }
    with open(os.path.join(out_dir, "pipeline_config.json"), "w") as f:
        json.dump(pipeline, f, indent=2)
    if tokenizer_dir and os.path.isdir(tokenizer_dir):
        import shutil

        shutil.copytree(tokenizer_dir, os.path.join(out_dir, "tokenizer"), dirs_exist_ok=True)
    return pipeline


def read_pipeline(dir_: str) -> dict:
    with open(os.path.join(dir_, "pipeline_config.json")) as f:
        return json.load(f)


def read_stage(dir_: str, stage: int) -> dict:
    with open(os.path.join(dir_, f"stage_{stage}", "stage_config.json")) as f:
        return json.load(f)


def stage_for_layers(dir_: str, shard: ShardSpec) -> int:
    p = read_pipeline(dir_)
    for i in range(p["num_stages"]):
        m = read_stage(dir_, i)
        if m["layer_start"] == shard.layer_start and m["layer_end"] == shard.layer_end:
            return i
    raise ValueError(f"no stage covers layers [{shard.layer_start}, {shard.layer_end})")


def load_stage_model(dir_: str, shard: ShardSpec, device, tp=None, stage: Optional[int] = None):
    """Build a LlamaModel for one stage of a shard tree (TP-sliced on load)."""
    from ..models.llama import LlamaModel, QLinear

    if os.path.exists(os.path.join(dir_, "stage_config.json")):
        sdir = dir_
    else:
        if stage is None:
            stage = stage_for_layers(dir_, shard)
        sdir = os.path.join(dir_, f"stage_{stage}")
    with open(os.path.join(sdir, "stage_config.json")) as f:
        meta = json.load(f)
    cfg = ModelConfig.from_dict(meta["model_config"])
    gs = int(meta["format"].rsplit("g", 1)[1]) if "format" in meta else cfg.group_size
    t = load_file(os.path.join(sdir, "model.safetensors"))
    m = LlamaModel(cfg, device, tp=tp, layer_start=meta["layer_start"],
                   layer_end=meta["layer_end"], has_embed=meta["has_embed"],
                   has_head=meta["has_head"])
    from ..models.config import rope_table

    m.cos_sin = rope_table(cfg, min(cfg.max_position, 1 << 16), device=m.device)
    if meta["has_embed"]:
        m.embed = t["embed_tokens"].to(m.device)
    for li in range(meta["layer_start"], meta["layer_end"]):
        pre = f"layers.{li}."
        m.load_layer(li, {k[len(pre):]: v for k, v in t.items() if k.startswith(pre)}, gs)
    if meta["has_head"]:
        m.final_norm = t["norm"].to(torch.bfloat16).to(m.device)
        head = Int4Weight(t["lm_head.packed"], t["lm_head.scales"], gs)
        m.lm_head = QLinear(m._vocab_shard(head), m.device)
    return m
