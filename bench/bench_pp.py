"""Pipeline-parallel decode benchmark: Llama-3.1-8B-shaped INT4 split into
N stages (one GPU each), global batch split into M micro-batches, NCCL p2p
between stages with micro-batch overlap (parallel.pp_decode).

    torchrun --nproc-per-node N bench/bench_pp.py [--micro M] [--batch 64] [--steps 20]

Each stage's micro-batch step is a CUDA graph replay; hidden rows and the
returning tokens travel by NCCL send/recv on NCCL's streams.  Timed on the
device (CUDA events, barrier + synchronize on both sides), max over ranks.
"""
import argparse
import datetime
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cascadia_b200 import ops  # noqa: E402
from cascadia_b200.models.config import get_config  # noqa: E402
from cascadia_b200.models.llama import LlamaModel  # noqa: E402
from cascadia_b200.parallel.pp_decode import PipelinedDecoder, pp_prefill  # noqa: E402
from cascadia_b200.runtime.kv_cache import BLOCK_SIZE  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama-3.1-8b")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--micro", type=int, default=2)
    p.add_argument("--prompt-len", type=int, default=1024)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    a = p.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    ops.ext()
    cfg = get_config(a.model)
    per = cfg.num_layers // world
    lo = rank * per
    hi = cfg.num_layers if rank == world - 1 else lo + per
    m = LlamaModel(cfg, dev, layer_start=lo, layer_end=hi, has_embed=rank == 0,
                   has_head=rank == world - 1).init_random(seed=1234)
    B, M, P = a.batch, a.micro, a.prompt_len
    assert B % M == 0
    width = -(-(P + a.warmup + a.steps + 8) // BLOCK_SIZE)
    m.allocate_kv(B * width + 16)
    g = torch.Generator().manual_seed(42)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=g).tolist()
    mbs = [[f"s{i}" for i in range(k * B // M, (k + 1) * B // M)] for k in range(M)]
    firsts = []
    for k, ids in enumerate(mbs):
        sub = prompts[k * B // M:(k + 1) * B // M]
        tok = []
        for c in range(0, len(ids), 16):  # prefill in chunks of 16 sequences
            tok.extend(pp_prefill(m, rank, world, ids[c:c + 16], sub[c:c + 16]))
        firsts.append(tok)
    dec = PipelinedDecoder(m, rank, world, mbs, width)
    if rank == 0:
        for k in range(M):
            dec.set_tokens(k, firsts[k])
    for i in range(a.warmup):
        dec.step(capture_now=True)
    dec.finish()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        dec.step()
    dec.finish()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms)
    st = ops.read_status(dev)
    if rank == 0:
        print(json.dumps({
            "metric": "pipeline-parallel decode tok/s (max over ranks)", "model": a.model,
            "stages": world, "micro_batches": M, "global_batch": B, "prompt_len": P,
            "steps": a.steps, "warmup": a.warmup, "tok_s": round(B * a.steps / (ms / 1000), 1),
            "ms_per_step": round(ms / a.steps, 3), "device_status": st,
            "transport": "NCCL p2p send/recv (NVLink), async, overlapped per micro-batch",
            "data": "synthetic: random-init N(0,0.02) INT4 weights, seeded uniform prompt ids"}))
    del dec
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
