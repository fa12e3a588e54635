"""Sparse-MoE model directory (the reference's layout,
crates/cascadia-engine-sparse-moe/src/lib.rs:10-19 and manifest.rs:21-70):

    manifest.json                     arch, counts, dims, experts_format = "int4_bin"
    embed.safetensors / head.safetensors
    shells/layer_NN.safetensors       attention, norms, router (+bias), shared expert
    dense/layer_NN.bin                dense FFN of the first layers (F1)
    experts/layer_NN/expert_XXX.bin   one routed expert (F1)

F1 expert file: gate_packed, gate_scale, up_packed, up_scale, down_packed,
down_scale back to back, no header; packed = int32 [out, in/8] little endian
with column 8i+j in bits 4j (even column in the low nibble of each byte),
scale = bf16 [out, in/32]; value = (nibble - 8) * scale
(crates/cascadia-int4-gemm/src/kernel.rs:31-71, format.rs:1-17).
Other INT4 tensors (attention, shared expert, head) are stored in the shell
files as `<name>.packed` (int32) + `<name>.scales`.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Tuple

import numpy as np
import torch
from safetensors.torch import load_file, save_file

from ..models.config import ModelConfig
from ..quant import Int4Weight

F1_GROUP = 32


def _f1_bytes(w: Int4Weight) -> bytes:
    assert w.group_size == F1_GROUP, "F1 expert files are group 32"
    return (w.packed.cpu().contiguous().numpy().astype("<i4").tobytes() +
            w.scales.cpu().to(torch.bfloat16).contiguous().view(torch.int16).numpy()
            .astype("<i2").tobytes())


def _f1_read(buf: memoryview, off: int, n: int, k: int) -> Tuple[Int4Weight, int]:
    pk = n * k // 2
    sc = n * (k // F1_GROUP) * 2
    packed = torch.from_numpy(np.frombuffer(buf, dtype="<i4", count=pk // 4, offset=off)
                              .copy()).view(n, k // 8)
    scales = torch.from_numpy(np.frombuffer(buf, dtype="<i2", count=sc // 2, offset=off + pk)
                              .copy()).view(torch.bfloat16).view(n, k // F1_GROUP)
    return Int4Weight(packed, scales, F1_GROUP), off + pk + sc


def write_expert_bin(path: str, gate: Int4Weight, up: Int4Weight, down: Int4Weight):
    with open(path, "wb") as f:
        for w in (gate, up, down):
            f.write(_f1_bytes(w))


def read_expert_bin(path: str, hidden: int, inter: int):
    buf = memoryview(open(path, "rb").read())
    gate, off = _f1_read(buf, 0, inter, hidden)
    up, off = _f1_read(buf, off, inter, hidden)
    down, off = _f1_read(buf, off, hidden, inter)
    assert off == len(buf), f"{path}: {len(buf)} bytes, expected {off}"
    return gate, up, down


def manifest_for(cfg: ModelConfig, arch: str) -> dict:
    return {
        "arch": arch, "num_layers": cfg.num_layers,
        "dense_layers": list(range(cfg.first_k_dense_replace)),
        "num_experts": cfg.num_experts, "top_k": cfg.num_experts_per_tok,
        "hidden_size": cfg.hidden_size, "num_kv_heads": cfg.num_kv_heads,
        "qk_head_dim": (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim) if cfg.is_mla
        else cfg.head_dim,
        "v_head_dim": cfg.v_head_dim if cfg.is_mla else cfg.head_dim,
        "vocab_size": cfg.vocab_size, "eos_token_ids": list(cfg.eos_token_ids),
        "experts_format": "int4_bin", "shell_backend": "cascadia_b200",
        "exported_layers": [], "expert_intermediate": cfg.moe_intermediate_size,
        # Our additions: the full config, so the directory is self-describing.
        "config": json.loads(cfg.to_json()),
    }


def _split_gu(w: Int4Weight) -> Tuple[Int4Weight, Int4Weight]:
    i = w.n // 2
    return w.rows(0, i), w.rows(i, w.n)


def _put(t: Dict[str, torch.Tensor], name: str, w: Int4Weight):
    t[name + ".packed"] = w.packed.cpu().contiguous()
    t[name + ".scales"] = w.scales.cpu().contiguous()


def _get(t: Dict[str, torch.Tensor], name: str, gs: int) -> Int4Weight:
    return Int4Weight(t[name + ".packed"], t[name + ".scales"], gs)


def write_moe_model(model, out_dir: str):
    """Write a MoE / MLA model built with ``models.llama.KEEP_INT4 = True``."""
    cfg = model.cfg
    os.makedirs(os.path.join(out_dir, "shells"), exist_ok=True)
    os.makedirs(os.path.join(out_dir, "dense"), exist_ok=True)
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest_for(cfg, cfg.arch), f, indent=1)
    save_file({"embed": model.embed.cpu().contiguous()}, os.path.join(out_dir, "embed.safetensors"))
    head = {"final_norm": model.final_norm.cpu()}
    _put(head, "lm_head", model.lm_head.int4)
    save_file(head, os.path.join(out_dir, "head.safetensors"))
    for li, lw in enumerate(model.layers):
        t = {"in_norm": lw.in_norm.cpu(), "post_norm": lw.post_norm.cpu()}
        if cfg.is_mla:
            a = lw.qkv
            if a.q_a is not None:
                _put(t, "q_a", a.q_a.int4)
                t["q_a_norm"] = a.q_a_norm.cpu()
            _put(t, "q_b", a.q_b.int4)
            _put(t, "kv_a", a.kv_a.int4)
            t["kv_a_norm"] = a.kv_a_norm.cpu()
            t["w_uk"] = a.w_uk.to(torch.bfloat16).cpu().contiguous()
            t["w_uv"] = a.w_uv.to(torch.bfloat16).cpu().contiguous()
            _put(t, "o", a.o.int4)
        else:
            t["qkv"] = lw.qkv.w.cpu().contiguous()
            t["o"] = lw.o.w.cpu().contiguous()
            if lw.q_norm is not None:
                t["q_norm"], t["k_norm"] = lw.q_norm.cpu(), lw.k_norm.cpu()
        if lw.router is not None:
            t["router"] = lw.router.cpu()
            if lw.router_bias is not None:
                t["router_bias"] = lw.router_bias.cpu()
        if lw.shared is not None:
            _put(t, "shared_gate_up", lw.shared[0].int4)
            _put(t, "shared_down", lw.shared[1].int4)
        save_file(t, os.path.join(out_dir, "shells", f"layer_{li:02d}.safetensors"))
        if lw.dense is not None:
            g, u = _split_gu(lw.dense[0].int4)
            write_expert_bin(os.path.join(out_dir, "dense", f"layer_{li:02d}.bin"), g, u,
                             lw.dense[1].int4)
        if lw.experts is not None:
            d = os.path.join(out_dir, "experts", f"layer_{li:02d}")
            os.makedirs(d, exist_ok=True)
            gus, dns = lw.experts.int4
            for e, (gu, dn) in enumerate(zip(gus, dns)):
                g, u = _split_gu(gu)
                write_expert_bin(os.path.join(d, f"expert_{e:03d}.bin"), g, u, dn)


def load_moe_model(model_dir: str, device, ep=None):
    """Build a MoE / MLA model (this rank's experts when ``ep`` is given)
    from a directory written by :func:`write_moe_model`."""
    from ..models.llama import QLinear
    from ..models.mla import MLAAttention, MLAModel
    from ..models.moe import BF16Linear, ExpertBank, MoELayer, MoEModel
    from ..models.config import rope_table

    man = json.load(open(os.path.join(model_dir, "manifest.json")))
    cfg = ModelConfig.from_dict(man["config"])
    cls = MLAModel if cfg.is_mla else MoEModel
    m = cls(cfg, device, ep=ep) if cls is MoEModel else cls(cfg, device, ep=ep)
    dev = torch.device(device)
    gs = cfg.group_size
    m.cos_sin = rope_table(cfg, min(cfg.max_position, 1 << 16),
                           rot=cfg.qk_rope_head_dim if cfg.is_mla else None, device=dev)
    m.embed = load_file(os.path.join(model_dir, "embed.safetensors"))["embed"].to(dev)
    head = load_file(os.path.join(model_dir, "head.safetensors"))
    m.final_norm = head["final_norm"].to(dev)
    m.lm_head = QLinear(_get(head, "lm_head", gs), dev)
    lo, hi = (ep.lo, ep.hi) if ep is not None else (0, cfg.num_experts)
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    for li in range(cfg.num_layers):
        t = load_file(os.path.join(model_dir, "shells", f"layer_{li:02d}.safetensors"))
        if cfg.is_mla:
            cpu = dev.type != "cuda"
            w_uk = t["w_uk"].float() if cpu else t["w_uk"].to(dev)
            w_uv = t["w_uv"].float() if cpu else t["w_uv"].to(dev)
            o = QLinear(_get(t, "o", gs), dev)
            qkv = MLAAttention(
                q_a=QLinear(_get(t, "q_a", gs), dev) if "q_a.packed" in t else None,
                q_a_norm=t["q_a_norm"].to(dev) if "q_a_norm" in t else None,
                q_b=QLinear(_get(t, "q_b", gs), dev), kv_a=QLinear(_get(t, "kv_a", gs), dev),
                kv_a_norm=t["kv_a_norm"].to(dev), w_uk=w_uk, w_uv=w_uv, o=o)
        else:
            qkv, o = BF16Linear(t["qkv"], dev), BF16Linear(t["o"], dev)
        dense = bank = shared = None
        if li in man["dense_layers"]:
            g, u, d = read_expert_bin(os.path.join(model_dir, "dense", f"layer_{li:02d}.bin"),
                                      H, cfg.intermediate_size)
            dense = (QLinear(Int4Weight.cat_rows([g, u]), dev, interleave_gate_up=True),
                     QLinear(d, dev))
        else:
            gus, dns = [], []
            for e in range(lo, hi):
                g, u, d = read_expert_bin(os.path.join(model_dir, "experts", f"layer_{li:02d}",
                                                       f"expert_{e:03d}.bin"), H, I)
                gus.append(Int4Weight.cat_rows([g, u]))
                dns.append(d)
            bank = ExpertBank(gus, dns, dev)
        if "shared_gate_up.packed" in t:
            shared = (QLinear(_get(t, "shared_gate_up", gs), dev, interleave_gate_up=True),
                      QLinear(_get(t, "shared_down", gs), dev))
        m.layers.append(MoELayer(
            in_norm=t["in_norm"].to(dev), post_norm=t["post_norm"].to(dev), qkv=qkv, o=o,
            q_norm=t["q_norm"].to(dev) if "q_norm" in t else None,
            k_norm=t["k_norm"].to(dev) if "k_norm" in t else None, dense=dense,
            router=t["router"].to(dev) if "router" in t else None,
            router_bias=t["router_bias"].to(dev) if "router_bias" in t else None,
            experts=bank, shared=shared))
    return m
