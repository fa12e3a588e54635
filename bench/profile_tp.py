"""Per-op device times of one tensor-parallel decode step (every rank).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        bench/profile_tp.py --batch 64 [--layers 2] [--tp-comm fused|nccl]

ncu cannot wrap a multi-rank command, so this times the ops of an eager
decode step with CUDA events on the launching stream: each of our kernel
wrappers (GEMMs, attention, norms, RoPE/KV write, the fused all-reduce, the
argmax merge, NCCL collectives) is wrapped while the step runs.  Two warm-up
steps first; then K steps are timed and the per-op sums averaged.  Rank 0
prints one JSON line per op category with the time per step (max over ranks)
and the share of the step.  The events serialise nothing the stream does not
already serialise, but an eager step is slower than a graph replay: compare
shares, not the total, with bench.py.
"""
from __future__ import annotations

import argparse
import collections
import datetime
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


class OpTimer:
    def __init__(self):
        self.active = False
        self.events = []  # (name, start, end)

    def wrap(self, name, fn):
        def timed(*a, **k):
            if not self.active:
                return fn(*a, **k)
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            r = fn(*a, **k)
            e.record()
            self.events.append((name, s, e))
            return r
        return timed

    def totals(self):
        torch.cuda.synchronize()
        t = collections.defaultdict(float)
        n = collections.Counter()
        for name, s, e in self.events:
            t[name] += s.elapsed_time(e)
            n[name] += 1
        self.events.clear()
        return t, n


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--prompt-len", type=int, default=1024)
    p.add_argument("--layers", type=int, default=0)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--model", default="llama-3.1-8b")
    p.add_argument("--tp-comm", default="fused", choices=["fused", "push", "multimem", "nccl"])
    a = p.parse_args()

    from cascadia_b200 import ops
    from cascadia_b200.models import llama as llama_mod
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel, TPGroup
    from cascadia_b200.runtime.generator import BatchGenerator
    from cascadia_b200.runtime.kv_cache import BLOCK_SIZE

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD
    cfg = get_config(a.model)
    if a.layers:
        cfg.num_layers = a.layers
    tp = TPGroup(rank, world, group)
    if world > 1 and a.tp_comm in ("fused", "push", "multimem"):
        from cascadia_b200.parallel.tp import FusedTP

        tp.fused = FusedTP(group, rank, world, dev, cfg.hidden_size, max(64, a.batch),
                           push=a.tp_comm == "push", multimem=a.tp_comm == "multimem")
    model = LlamaModel(cfg, dev, tp=tp).init_random(seed=1234)
    width = -(-(a.prompt_len + a.steps + 8) // BLOCK_SIZE)
    model.allocate_kv(a.batch * width + 16)
    gen = BatchGenerator(model, use_graph=False)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab_size, (a.batch, a.prompt_len), generator=g).tolist()
    ids = [f"b{i}" for i in range(a.batch)]
    last = []
    chunk = max(1, 16384 // a.prompt_len)
    for i in range(0, a.batch, chunk):
        last.extend(gen.prefill(ids[i:i + chunk], prompts[i:i + chunk]).tolist())

    timer = OpTimer()
    # Wrap the op entry points the model calls through the module attribute.
    for name in ("w4a16_gemm", "attn_decode", "rmsnorm", "rope_kv_write", "embedding",
                 "argmax"):
        setattr(ops, name, timer.wrap(name, getattr(ops, name)))
    if tp.fused is not None:
        tp.fused.allreduce = timer.wrap("fused_allreduce_rmsnorm", tp.fused.allreduce)
    TPGroup.all_reduce = timer.wrap("nccl_all_reduce", TPGroup.all_reduce)
    TPGroup.all_gather_rows = timer.wrap("nccl_all_gather", TPGroup.all_gather_rows)

    for _ in range(2):
        last = gen.decode(ids, last, width).tolist()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    timer.active = True
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.steps):
        last = gen.decode(ids, last, width).tolist()
    e.record()
    torch.cuda.synchronize()
    timer.active = False
    step_ms = s.elapsed_time(e) / a.steps
    tot, cnt = timer.totals()
    names = sorted(tot)
    if world > 1:
        # Same op set on every rank (same code path); max over ranks.
        allnames = [None] * world
        dist.all_gather_object(allnames, names)
        names = sorted(set().union(*allnames))
        v = torch.tensor([tot.get(n, 0.0) for n in names] + [step_ms], dtype=torch.float64,
                         device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        vals = v.tolist()
        step_ms = vals[-1]
        tot = dict(zip(names, vals[:-1]))
    if rank == 0:
        ops_ms = sum(tot.values()) / a.steps
        print(json.dumps({"what": "tp decode step per-op device time (eager, CUDA events)",
                          "model": a.model + (f"-L{a.layers}" if a.layers else ""),
                          "tp": world, "batch": a.batch, "tp_comm": a.tp_comm if world > 1
                          else None, "step_ms": round(step_ms, 4),
                          "ops_ms": round(ops_ms, 4)}))
        for n in sorted(tot, key=lambda k: -tot[k]):
            ms = tot[n] / a.steps
            print(json.dumps({"op": n, "ms_per_step": round(ms, 4),
                              "launches_per_step": cnt[n] // a.steps,
                              "share_of_step": round(ms / step_ms, 3)}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
