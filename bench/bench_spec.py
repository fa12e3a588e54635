"""Speculative-decoding benchmark (the distributed spec-decode config's shapes,
on one GPU).

    python bench/bench_spec.py [--batch 1] [--k 4] [--gen 256] [--prompt-len 512]
                               [--draft llama-3.2-1b | ngram]

Target: Llama-3.1-8B-shaped INT4; draft: Llama-3.2-1B-shaped INT4 on the same
GPU, sharing the target's embedding and LM head (their first 2048 columns:
the draft's hidden size).  Times the whole generation after prefill (draft
rounds, verify forwards, host bookkeeping) with CUDA events, and the same
generation without speculation.  Prints one JSON line.  Random weights: the
acceptance rate is whatever the two random models give and is reported next
to the throughput; `common_prefix` compares the speculative output with plain
greedy decoding token by token (the verify forward and the decode step run
different attention kernels, so near-tied argmaxes can differ).
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from cascadia_b200 import ops  # noqa: E402
from cascadia_b200.models.config import get_config  # noqa: E402
from cascadia_b200.models.llama import (LlamaModel, QLinear, _layer_generator,  # noqa: E402
                                        random_int4)
from cascadia_b200.runtime.generator import BatchGenerator  # noqa: E402
from cascadia_b200.runtime.kv_cache import BLOCK_SIZE  # noqa: E402
from cascadia_b200.runtime.spec import SpecDecoder  # noqa: E402


def share_embedding_and_head(draft, target, seed: int):
    """Give the draft the target's embedding and LM head, restricted to the
    draft's hidden width."""
    hd = draft.cfg.hidden_size
    draft.embed = target.embed[:, :hd].contiguous()
    tc = target.cfg
    g = _layer_generator(seed, 100001, target.device)
    head = random_int4(tc.vocab_size, tc.hidden_size, g, target.device, 0.02, tc.group_size)
    draft.lm_head = QLinear(head.cols(0, hd), draft.device)
    del head


def timed(fn):
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    out = fn()
    b.record()
    torch.cuda.synchronize()
    return out, a.elapsed_time(b)


def common_prefix(a, b):
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--k", type=int, default=4)
    p.add_argument("--gen", type=int, default=256)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--target", default="llama-3.1-8b")
    p.add_argument("--draft", default="llama-3.2-1b", help="draft preset or 'ngram'")
    p.add_argument("--reps", type=int, default=2)
    args = p.parse_args()
    dev = torch.device("cuda")
    ops.ext()
    seed = 1234
    target = LlamaModel(get_config(args.target), dev).init_random(seed=seed)
    B, P, N = args.batch, args.prompt_len, args.gen
    width = -(-(P + N + args.k + 8) // BLOCK_SIZE)
    target.allocate_kv(B * width * 2 + 64)
    draft = None
    if args.draft != "ngram":
        draft = LlamaModel(get_config(args.draft), dev).init_random(seed=seed + 1)
        share_embedding_and_head(draft, target, seed)
        draft.allocate_kv(B * width * 2 + 64)
    g = torch.Generator().manual_seed(42)
    prompts = torch.randint(0, target.cfg.vocab_size, (B, P), generator=g).tolist()

    plain = BatchGenerator(target)
    plain.generate(prompts, 8, prefix="w")  # warm-up + graph capture
    ref, _ = timed(lambda: plain.generate(prompts, N, prefix="p"))
    _, t_pre = timed(lambda: plain.prefill(["x0"], prompts[:1]))
    target.kv.free_sequence("x0")
    t_plain = min(timed(lambda: plain.generate(prompts, N, prefix="p"))[1]
                  for _ in range(args.reps))

    sd = SpecDecoder(target, draft=draft, k=args.k, ngram_k=args.k)
    sd.generate(prompts, 8, prefix="ws")
    best, out = None, None
    for _ in range(args.reps):
        sd.stats = type(sd.stats)()
        out, t = timed(lambda: sd.generate(prompts, N))
        best = t if best is None else min(best, t)
    stats = sd.stats
    pre_b = t_pre * B  # batch-1 prefill x B (upper bound of the batched prefill)
    dec_tokens = B * (N - 1)
    res = {
        "metric": "speculative decode tok/s (after prefill), greedy, one GPU",
        "target": args.target, "draft": args.draft, "k": args.k, "batch": B,
        "prompt_len": P, "gen": N,
        "spec_tok_s": round(dec_tokens / ((best - pre_b) / 1000), 2),
        "plain_tok_s": round(dec_tokens / ((t_plain - pre_b) / 1000), 2),
        "spec_total_ms": round(best, 2), "plain_total_ms": round(t_plain, 2),
        "prefill_ms_b1": round(t_pre, 2),
        "accept_rate": round(stats.accept_rate, 4),
        "tokens_per_round": round(stats.emitted / max(1, stats.rounds) / B, 3),
        "rounds": stats.rounds,
        "common_prefix_mean": round(sum(common_prefix(a, b) for a, b in zip(out, ref)) / B, 1),
        "device_status": ops.read_status(dev),
        "data": "synthetic: random-init N(0,0.02) INT4 weights, seeded uniform prompt ids",
    }
    print(json.dumps(res))


if __name__ == "__main__":
    main()
