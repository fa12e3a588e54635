"""Sparse-MoE model directory: manifest + F1 expert bins round trip."""
import json
import os

import torch

from cascadia_b200.models import llama
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import build_batch
from cascadia_b200.quant import Int4Weight
from cascadia_b200.shard.moe_format import load_moe_model, read_expert_bin, write_expert_bin, write_moe_model


def test_f1_expert_bin_layout(tmp_path):
    g = torch.Generator().manual_seed(0)
    gate, up = (Int4Weight.random(64, 128, 0.05, 32, generator=g) for _ in range(2))
    down = Int4Weight.random(128, 64, 0.05, 32, generator=g)
    p = os.path.join(tmp_path, "e.bin")
    write_expert_bin(p, gate, up, down)
    raw = open(p, "rb").read()
    assert len(raw) == 3 * (64 * 128 // 2 + 64 * 128 // 32 * 2)
    # even column in the low nibble of byte 0
    q = gate.unpack()
    assert raw[0] & 0x0F == int(q[0, 0]) and raw[0] >> 4 == int(q[0, 1])
    g2, u2, d2 = read_expert_bin(p, 128, 64)
    for a, b in ((gate, g2), (up, u2), (down, d2)):
        assert torch.equal(a.packed, b.packed)
        assert torch.equal(a.scales.to(torch.bfloat16), b.scales)


def _logits(m):
    m.allocate_kv(16)
    m.kv.add_sequence("s")
    b = build_batch(m, ["s"], [5], [0], False)
    hid = m.embed_tokens(torch.tensor([3, 1, 4, 1, 5], dtype=torch.int32))
    m.forward(b, hid)
    return m.head(hid[-1:].contiguous()).float()


def test_moe_model_dir_round_trip(tmp_path):
    from cascadia_b200.models.mla import MLAModel

    cfg = get_config("tiny-mla")
    llama.KEEP_INT4 = True
    try:
        m = MLAModel(cfg, "cpu").init_random(seed=4, gen_device="cpu")
    finally:
        llama.KEEP_INT4 = False
    write_moe_model(m, str(tmp_path))
    man = json.load(open(os.path.join(tmp_path, "manifest.json")))
    assert man["experts_format"] == "int4_bin" and man["num_experts"] == cfg.num_experts
    assert os.path.exists(os.path.join(tmp_path, "experts", "layer_01", "expert_007.bin"))
    m2 = load_moe_model(str(tmp_path), "cpu")
    assert torch.allclose(_logits(m), _logits(m2))
