"""`shard` layout: writer/reader round trip and stage planning (CPU)."""
import json
import os

import torch

from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.runtime.generator import BatchGenerator
from cascadia_b200.shard.format import (load_stage_model, read_pipeline, read_stage, stage_plan,
                                        write_random_shards)
from cascadia_b200.types import ShardSpec

STAGE_KEYS = {"stage", "layer_start", "layer_end", "has_embed", "has_head", "quantization",
              "hidden_size", "vocab_size", "num_layers_total", "num_kv_heads", "head_dim",
              "stateful", "rope_theta", "partial_rotary_factor", "arch_tag", "target",
              "inputs", "cache_reorder", "export_version", "format"}
PIPE_KEYS = {"model_id", "num_stages", "num_layers", "hidden_size", "num_attention_heads",
             "num_key_value_heads", "vocab_size", "rope_theta", "partial_rotary_factor",
             "arch_tag", "quantization", "export_version"}


def test_stage_plan():
    assert stage_plan(16, 2) == [(0, 8), (8, 16)]
    assert stage_plan(32, 3) == [(0, 10), (10, 20), (20, 32)]
    assert stage_plan(10, 2, [3, 7]) == [(0, 3), (3, 10)]


def test_write_and_load_roundtrip(tmp_path):
    cfg = get_config("tiny-llama")
    d = str(tmp_path / "shards")
    write_random_shards(cfg, d, 2, "tiny", seed=5)
    p = read_pipeline(d)
    assert PIPE_KEYS <= set(p) and p["num_stages"] == 2
    s0, s1 = read_stage(d, 0), read_stage(d, 1)
    assert STAGE_KEYS <= set(s0) and s0["has_embed"] and not s0["has_head"]
    assert s1["has_head"] and s1["format"] == "int4_sym_g128"
    # Stage models chained == one random-init model with the same seed.
    full = LlamaModel(cfg, "cpu").init_random(seed=5, gen_device="cpu")
    m0 = load_stage_model(d, ShardSpec("tiny", 0, 1, 2, "cpu", True, False), "cpu")
    m1 = load_stage_model(d, ShardSpec("tiny", 1, 2, 2, "cpu", False, True), "cpu")
    for m in (full, m0, m1):
        m.allocate_kv(16)
        m.kv.add_sequence("x")
    from cascadia_b200.models.llama import build_batch

    ids = torch.tensor([5, 9, 33, 2], dtype=torch.int32)
    bf = build_batch(full, ["x"], [4], [0], False)
    h = full.embed_tokens(ids)
    full.forward(bf, h)
    ref = full.head(h[-1:])
    b0 = build_batch(m0, ["x"], [4], [0], False)
    h0 = m0.embed_tokens(ids)
    m0.forward(b0, h0)
    b1 = build_batch(m1, ["x"], [4], [0], False)
    m1.forward(b1, h0)
    out = m1.head(h0[-1:])
    assert torch.equal(out, ref)
