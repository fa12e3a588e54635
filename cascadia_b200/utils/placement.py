"""Parallelism placement for one 8-GPU box (`cascadia_b200 place`).

The reference solves an exact branch-and-bound ILP assigning pipeline stages
to heterogeneous devices under memory caps (crates/cascadia-cli/src/placement.rs:134-377).
On one B200 box the devices are identical and uniformly connected, so the
decision is the factorisation PP x TP x EP of the GPU count.  We enumerate
every factorisation, reject those that do not fit in memory (weights + KV +
activations), and rank the rest by a decode cost model:

  t_step = weight_bytes / (tp * ep_fraction * HBM) / pp-pipelining
         + kv_bytes / (tp * HBM)
         + collectives (2 per layer for TP, 2 all-to-all per MoE layer for EP)
           at measured NVLink latency / bandwidth
         + pipeline bubble (pp - 1) micro-batch stage times

with the HBM / NVLink figures measured on this pool.  Exhaustive search over a
handful of factorisations is exact, like the reference's ILP, for this size.
"""
from __future__ import annotations

from typing import Dict, List

HBM_GBS = 6500.0
NVLINK_GBS = 770.0
COLL_LAT_US = 8.0


def _model_bytes(cfg) -> Dict[str, float]:
    h, L = cfg.hidden_size, cfg.num_layers
    d = cfg.head_dim
    attn = (cfg.num_heads * d * h * 2 + cfg.num_kv_heads * d * h * 2) * 0.5  # int4
    if cfg.is_moe:
        expert = 3 * h * cfg.moe_intermediate_size * 0.5
        ffn_total = cfg.num_experts * expert + cfg.num_shared_experts * expert
        ffn_active = (cfg.num_experts_per_tok + cfg.num_shared_experts) * expert
    else:
        ffn_total = ffn_active = 3 * h * cfg.intermediate_size * 0.5
    head = cfg.vocab_size * h * 0.5 + cfg.vocab_size * h * 2
    return {"total": L * (attn + ffn_total) + head, "active": L * (attn + ffn_active) + head,
            "kv_per_token": 2 * L * cfg.num_kv_heads * d * 2}


def factorizations(n: int) -> List[tuple]:
    out = []
    for pp in range(1, n + 1):
        if n % pp:
            continue
        for tp in range(1, n // pp + 1):
            if (n // pp) % tp:
                continue
            out.append((pp, tp, n // (pp * tp)))
    return out


def choose_parallelism(model: str, gpus: int, batch: int, context: int,
                       gpu_mem_gb: float = 180.0) -> dict:
    from ..models.config import get_config

    cfg = get_config(model)
    mb = _model_bytes(cfg)
    cands = []
    for pp, tp, ep in factorizations(gpus):
        if cfg.num_heads % tp or cfg.num_kv_heads % tp and cfg.num_kv_heads >= tp:
            continue
        if ep > 1 and not cfg.is_moe:
            continue
        if cfg.is_moe and cfg.num_experts % ep:
            continue
        per_gpu_w = mb["total"] / (pp * tp * ep)
        kv = batch * context * mb["kv_per_token"] / (pp * tp)
        mem = (per_gpu_w + kv) / 2**30 + 4.0
        if mem > gpu_mem_gb:
            continue
        stage_t = (mb["active"] / (pp * tp * max(1, ep if cfg.is_moe else 1)) + kv) / (HBM_GBS * 1e3)
        coll = 0.0
        layers_per_stage = cfg.num_layers / pp
        if tp > 1:
            coll += layers_per_stage * 2 * (COLL_LAT_US + batch * cfg.hidden_size * 2 / NVLINK_GBS / 1e3)
        if ep > 1:
            coll += layers_per_stage * 2 * (COLL_LAT_US + batch * cfg.num_experts_per_tok
                                            * cfg.hidden_size * 2 / NVLINK_GBS / 1e3)
        step_us = stage_t + coll
        # pp stages overlap micro-batches; the bubble adds (pp-1) stage times / micro-batches.
        mbs = max(1, min(pp, batch))
        total_us = step_us * (pp + (pp - 1) / mbs) / pp * pp if pp > 1 else step_us
        cands.append({"pp": pp, "tp": tp, "ep": ep, "mem_gb_per_gpu": round(mem, 1),
                      "decode_step_us": round(total_us, 1),
                      "tokens_per_s": round(batch / (total_us / 1e6), 1)})
    cands.sort(key=lambda c: c["decode_step_us"])
    return {"model": model, "gpus": gpus, "batch": batch, "context": context,
            "best": cands[0] if cands else None, "candidates": cands}
