"""Decode-step profiling driver (for ncu launch lists and kernel captures).

Builds the Llama-3.1-8B-shaped INT4 model (or a MoE preset) on cuda:0, prefills
`--batch` prompts of `--prompt-len` tokens, then runs `--steps` decode steps
eagerly (no CUDA graph) inside cudaProfilerStart/Stop so that

    ncu --profile-from-start off --metrics gpu__time_duration.sum \
        --clock-control none --csv python bench/profile_decode.py

lists exactly the kernels of the decode steps.  `--layers` shrinks the model
for small `--set full` captures of one kernel.
"""
import argparse
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from cascadia_b200 import ops  # noqa: E402
from cascadia_b200.models.config import get_config  # noqa: E402
from cascadia_b200.models.llama import LlamaModel  # noqa: E402
from cascadia_b200.runtime.generator import BatchGenerator  # noqa: E402
from cascadia_b200.runtime.kv_cache import BLOCK_SIZE  # noqa: E402


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama-3.1-8b")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--prompt-len", type=int, default=1024)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--layers", type=int, default=0)
    p.add_argument("--prefill", action="store_true", help="profile one prefill instead")
    a = p.parse_args()
    cfg = get_config(a.model)
    if a.layers:
        cfg.num_layers = a.layers
    dev = torch.device("cuda", 0)
    t0 = time.time()
    if cfg.is_moe or cfg.is_gemma4:
        from cascadia_b200.engine.llm import LLMBuilder

        m = LLMBuilder.model_class(None, cfg)(cfg, dev).init_random(seed=1)
    else:
        m = LlamaModel(cfg, dev).init_random(seed=1)
    width = -(-(a.prompt_len + a.steps + 8) // BLOCK_SIZE)
    if cfg.is_hybrid:
        m.allocate_kv(a.batch * width + 8, max_seqs=a.batch)
    else:
        m.allocate_kv(a.batch * width + 8)
    gen = BatchGenerator(m, use_graph=False)
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, cfg.vocab_size, (a.batch, a.prompt_len), generator=g).tolist()
    ids = [f"s{i}" for i in range(a.batch)]
    if a.prefill:
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        first = gen.prefill(ids, prompts)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        print("prefill done", time.time() - t0)
        return
    chunk = max(1, (4096 if cfg.is_moe else 16384) // a.prompt_len)
    last = []
    for i in range(0, a.batch, chunk):
        last.extend(gen.prefill(ids[i:i + chunk], prompts[i:i + chunk]).tolist())
    last = gen.decode(ids, last, width).tolist()  # warm-up (plans, workspaces)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    for _ in range(a.steps):
        last = gen.decode(ids, last, width).tolist()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print("decode done", time.time() - t0, "status", ops.read_status(dev))


if __name__ == "__main__":
    main()
