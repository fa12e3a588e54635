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

Inputs are measured where a measurement exists: the HBM copy bandwidth
from the box's peak file (``MEASURED_PEAKS.json`` beside the repository, or
``--peaks``), and, with ``--calibrate``, the per-layer decode time of the
model on this GPU (a short timed run of two of its layers at the requested
batch and context), which replaces the bytes / bandwidth estimate of a
stage.  Exhaustive search over the handful of factorisations is exact, like
the reference's ILP, for this size.

``--launch`` runs the chosen split under a small supervisor: it starts
``python -m torch.distributed.run ... -m cascadia_b200 run --tp T --pp P``
(one rank per GPU) and restarts it after a crash, up to a restart budget
(the reference's placement runner keeps its stage processes up the same
way, crates/cascadia-cli/src/placement.rs).
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import time
from typing import Callable, Dict, List, Optional

HBM_GBS = 6432.0      # default: measured B200 copy bandwidth on this pool
NVLINK_GBS = 770.0    # measured peer copy, per direction
COLL_LAT_US = 25.0    # measured per fused all-reduce at TP=8, batch 64 (sync-bound)


def measured_hbm_gbs(path: Optional[str] = None) -> float:
    """HBM bandwidth from a peaks file (``hbm_gbs``), else the default."""
    cands = [path] if path else [os.path.join(os.path.dirname(os.path.dirname(
        os.path.dirname(os.path.abspath(__file__)))), "MEASURED_PEAKS.json")]
    for c in cands:
        try:
            with open(c) as f:
                v = float(json.load(f)["hbm_gbs"])
            if v > 0:
                return v
        except (OSError, KeyError, ValueError, TypeError):
            continue
    return HBM_GBS


def calibrate_layer_us(model: str, batch: int, context: int, layers: int = 2,
                       steps: int = 5) -> float:
    """Measured decode time per layer (us) of `model` at `batch` sequences
    of `context` tokens on the local GPU: `layers` layers, CUDA-graph decode
    steps timed with CUDA events, minus nothing (embedding and head are
    included once and amortised by the caller's layer count)."""
    import dataclasses

    import torch

    from ..models.config import get_config
    from ..models.llama import LlamaModel
    from ..runtime.generator import BatchGenerator
    from ..runtime.kv_cache import BLOCK_SIZE

    cfg = dataclasses.replace(get_config(model), num_layers=layers)
    dev = torch.device("cuda")
    m = LlamaModel(cfg, dev).init_random(seed=1)
    width = -(-(context + steps + 4) // BLOCK_SIZE)
    m.allocate_kv(batch * width + 8)
    gen = BatchGenerator(m)
    ids = [f"c{i}" for i in range(batch)]
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (batch, context), generator=g).tolist()
    last = []
    chunk = max(1, 8192 // context)
    for i in range(0, batch, chunk):
        last.extend(gen.prefill(ids[i:i + chunk], prompt[i:i + chunk]).tolist())
    for _ in range(2):
        last = gen.decode(ids, last, width).tolist()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        last = gen.decode(ids, last, width).tolist()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000.0 / steps / layers


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
                       gpu_mem_gb: float = 180.0, hbm_gbs: Optional[float] = None,
                       layer_us: Optional[float] = None) -> dict:
    """Rank every PP x TP x EP split.  `hbm_gbs`: measured bandwidth;
    `layer_us`: measured single-GPU decode time of one layer at this batch
    and context (replaces the bandwidth estimate of the layer work)."""
    from ..models.config import get_config

    cfg = get_config(model)
    mb = _model_bytes(cfg)
    hbm = hbm_gbs or HBM_GBS
    cands = []
    for pp, tp, ep in factorizations(gpus):
        if cfg.num_heads % tp or cfg.num_kv_heads % tp and cfg.num_kv_heads >= tp:
            continue
        if ep > 1 and not cfg.is_moe:
            continue
        if cfg.is_moe and tp > 1:
            # The MoE engines shard experts (EP, data-parallel attention)
            # and layers (PP); their attention is not tensor-parallel.
            continue
        if cfg.is_moe and cfg.num_experts % ep:
            continue
        per_gpu_w = mb["total"] / (pp * tp * ep)
        kv = batch * context * mb["kv_per_token"] / (pp * tp)
        mem = (per_gpu_w + kv) / 2**30 + 4.0
        if mem > gpu_mem_gb:
            continue
        if layer_us is not None:
            # Measured per-layer time split over the TP ranks (weights and KV
            # both shard), the stage's share of the layers.
            stage_t = layer_us * cfg.num_layers / pp / (tp * max(1, ep if cfg.is_moe else 1))
        else:
            stage_t = (mb["active"] / (pp * tp * max(1, ep if cfg.is_moe else 1)) + kv) / (
                hbm * 1e3)
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
            "inputs": {"hbm_gbs": hbm, "layer_us": layer_us, "nvlink_gbs": NVLINK_GBS,
                       "collective_latency_us": COLL_LAT_US},
            "best": cands[0] if cands else None, "candidates": cands}


def launch_command(model: str, choice: dict, api: str = "0.0.0.0:8000",
                   port: int = 29500, extra: Optional[List[str]] = None) -> List[str]:
    """torchrun command line that serves `choice` (one rank per GPU)."""
    n = choice["pp"] * choice["tp"] * choice["ep"]
    if choice["ep"] > 1:
        raise ValueError("expert-parallel serving is launched by bench.py, not `run`")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           "-m", "cascadia_b200", "run", "--model", model, "--api", api,
           "--tp", str(choice["tp"]), "--pp", str(choice["pp"])]
    return cmd + list(extra or [])


def supervise(cmd: List[str], max_restarts: int = 3, backoff_s: float = 2.0,
              popen: Callable = subprocess.Popen, sleep: Callable = time.sleep) -> int:
    """Run `cmd`; restart it after a non-zero exit, up to `max_restarts`
    times with a growing back-off.  Returns the last exit code (0 = the
    command ended cleanly)."""
    restarts = 0
    while True:
        proc = popen(cmd)
        try:
            code = proc.wait()
        except KeyboardInterrupt:
            proc.terminate()
            proc.wait()
            return 130
        if code == 0 or restarts >= max_restarts:
            return code
        restarts += 1
        sleep(backoff_s * restarts)
