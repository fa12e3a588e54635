"""Speculative-decoding benchmark (the distributed spec-decode config's shapes).

    python bench/bench_spec.py [--batch 1] [--k 4] [--gen 256] [--prompt-len 512]
                               [--draft llama-3.2-1b | ngram | self:L]
                               [--emulate-accept 0.62]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        bench/bench_spec.py ...          # target at TP=N, the draft on rank 0

Target: Llama-3.1-8B-shaped INT4 (tensor-parallel over the ranks when run
under torchrun); draft: Llama-3.2-1B-shaped INT4 on rank 0's GPU, sharing the
target's embedding and LM head (their first 2048 columns: the draft's hidden
size), or the target's first L layers (``self:L``, early-exit drafting), or
n-gram prompt lookup.  Times the generation after prefill (draft rounds,
draft broadcast, verify forwards, host bookkeeping) with CUDA events on every
rank (max over ranks), and the same generation without speculation.

Random weights make two different models disagree on every argmax, so the
measured acceptance of a random draft is ~0.  ``--emulate-accept A`` keeps
the draft's work (the draft model still runs every step) but replaces its
proposals: position j of a round carries the target's own next token with
probability q (else a wrong token), q chosen so that the expected accepted /
drafted ratio is A.  The target's own tokens come from a first speculative
pass whose drafts are all wrong (its corrections are exactly the tokens the
verify path produces).  This gives the throughput the engine reaches at a
stated acceptance (the reference's published k=4 acceptance is 0.62 / 0.50).
Prints one JSON line per mode.
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
from cascadia_b200.models.llama import (LlamaModel, QLinear, TPGroup,  # noqa: E402
                                        _layer_generator, random_int4)
from cascadia_b200.runtime.generator import BatchGenerator  # noqa: E402
from cascadia_b200.runtime.kv_cache import BLOCK_SIZE  # noqa: E402
from cascadia_b200.runtime.spec import SpecDecoder  # noqa: E402


def share_embedding_and_head(draft, target_cfg, target_embed, seed: int, dev):
    """Give the draft the target's embedding and LM head, restricted to the
    draft's hidden width."""
    hd = draft.cfg.hidden_size
    draft.embed = target_embed[:, :hd].contiguous()
    g = _layer_generator(seed, 100001, dev)
    head = random_int4(target_cfg.vocab_size, target_cfg.hidden_size, g, dev, 0.02,
                       target_cfg.group_size)
    draft.lm_head = QLinear(head.cols(0, hd), draft.device)
    del head


def accept_prob(rate: float, k: int) -> float:
    """Per-position match probability q with (q + q^2 + .. + q^k) / k = rate
    (accepted / drafted when each position matches independently)."""
    lo, hi = 0.0, 1.0
    for _ in range(60):
        q = (lo + hi) / 2
        if sum(q ** i for i in range(1, k + 1)) / k < rate:
            lo = q
        else:
            hi = q
    return (lo + hi) / 2


class EmulatedDrafter:
    """Runs the real drafter (its cost stays in the timing), then proposes
    the target's own continuation per position with probability q."""

    def __init__(self, inner, oracle, prompt_lens, q, vocab, seed=7):
        self.inner, self.oracle, self.plen = inner, oracle, prompt_lens
        self.q, self.vocab = q, vocab
        self.g = torch.Generator().manual_seed(seed)
        self.idx = {}

    def propose(self, seq_ids, histories, k, width):
        real = self.inner.propose(seq_ids, histories, k, width) if self.inner else None
        out = []
        for i, (sid, h) in enumerate(zip(seq_ids, histories)):
            b = int(sid.split("_")[-1])
            gen = len(h) - self.plen[b]          # tokens generated so far
            want = self.oracle[b][gen:gen + k]
            r = torch.rand(len(want), generator=self.g).tolist()
            d = [t if x < self.q else (t + 1) % self.vocab for t, x in zip(want, r)]
            if real is not None:
                d = d[:len(real[i])] if len(real[i]) < len(d) else d
            out.append(d)
        return out

    def accept(self, sid, accepted, k):
        if self.inner:
            self.inner.accept(sid, accepted, k)

    def release(self, sid):
        if self.inner:
            self.inner.release(sid)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--k", type=int, default=4)
    p.add_argument("--gen", type=int, default=256)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--target", default="llama-3.1-8b")
    p.add_argument("--draft", default="llama-3.2-1b",
                   help="draft preset, 'ngram', or 'self:L' (the target's first L layers)")
    p.add_argument("--emulate-accept", type=float, nargs="*", default=[],
                   help="also time with emulated acceptance rates (accepted / drafted)")
    p.add_argument("--reps", type=int, default=2)
    args = p.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD
    ops.ext()
    seed = 1234
    tcfg = get_config(args.target)
    tp = TPGroup(rank, world, group)
    if world > 1:
        from cascadia_b200.parallel.tp import FusedTP

        tp.fused = FusedTP(group, rank, world, dev, tcfg.hidden_size, 64)
    target = LlamaModel(tcfg, dev, tp=tp).init_random(seed=seed)
    B, P, N = args.batch, args.prompt_len, args.gen
    width = -(-(P + N + args.k + 8) // BLOCK_SIZE)
    target.allocate_kv(B * width * 2 + 64)
    draft = None
    if rank == 0 and args.draft.startswith("self:"):
        assert world == 1, "early-exit drafting shares the whole target: one GPU"
        draft = target.early_exit(int(args.draft.split(":")[1]))
        draft.allocate_kv(B * width * 2 + 64)
    elif rank == 0 and args.draft != "ngram":
        dcfg = get_config(args.draft)
        draft = LlamaModel(dcfg, dev).init_random(seed=seed + 1)
        share_embedding_and_head(draft, tcfg, target.embed, seed, dev)
        draft.allocate_kv(B * width * 2 + 64)
    remote = world > 1 and args.draft != "ngram" and rank != 0
    g = torch.Generator().manual_seed(42)
    prompts = torch.randint(0, tcfg.vocab_size, (B, P), generator=g).tolist()

    def timed(fn):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out = fn()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return out, float(ms)

    plain = BatchGenerator(target)
    plain.generate(prompts, 8, prefix="w")  # warm-up + graph capture
    _, t_pre = timed(lambda: plain.prefill(["x0"], prompts[:1]))
    target.kv.free_sequence("x0")
    t_plain = min(timed(lambda: plain.generate(prompts, N, prefix="p"))[1]
                  for _ in range(args.reps))
    pre_b = t_pre * B  # batch-1 prefill x B (upper bound of the batched prefill)
    dec_tokens = B * (N - 1)
    plain_tok_s = dec_tokens / ((t_plain - pre_b) / 1000)

    def run(sd, tag):
        sd.generate(prompts, 8, prefix=f"w{tag}_")  # warm-up; graphs are keyed by 64-block width buckets
        best, out = None, None
        for i in range(args.reps):
            sd.stats = type(sd.stats)()
            out, t = timed(lambda: sd.generate(prompts, N, prefix=f"{tag}{i}_"))
            best = t if best is None else min(best, t)
        return out, best, sd.stats

    def report(mode, best, stats, extra):
        if rank != 0:
            return
        res = {
            "metric": "speculative decode tok/s (after prefill), greedy",
            "mode": mode, "target": args.target, "tp": world,
            "draft": args.draft + (" (rank 0)" if world > 1 else ""),
            "k": args.k, "batch": B, "prompt_len": P, "gen": N,
            "spec_tok_s": round(dec_tokens / ((best - pre_b) / 1000), 2),
            "plain_tok_s": round(plain_tok_s, 2),
            "spec_total_ms": round(best, 2), "plain_total_ms": round(t_plain, 2),
            "prefill_ms_b1": round(t_pre, 2),
            "accept_rate": round(stats.accept_rate, 4),
            "tokens_per_round": round(stats.emitted / max(1, stats.rounds) / B, 3),
            "rounds": stats.rounds,
            "ms_per_round_draft": round(1000 * stats.draft_s / max(1, stats.rounds), 3),
            "ms_per_round_verify": round(1000 * stats.verify_s / max(1, stats.rounds), 3),
            "device_status": ops.read_status(dev),
            "data": "synthetic: random-init N(0,0.02) INT4 weights, seeded uniform prompt ids",
        }
        res.update(extra)
        print(json.dumps(res), flush=True)

    sd = SpecDecoder(target, draft=draft, k=args.k, ngram_k=args.k, remote_draft=remote)
    _, best, stats = run(sd, "s")
    report("measured", best, stats, {})

    if args.emulate_accept:
        # Oracle: a speculative pass whose every draft is wrong emits exactly
        # the verify path's own tokens.
        assert world == 1 or args.draft != "ngram", "emulation at TP>1 needs a draft model"
        plens = [len(x) for x in prompts]
        real = sd.drafter
        if rank == 0:
            sd.drafter = EmulatedDrafter(real, [[-1] * (N + args.k)] * B, plens, 0.0,
                                         tcfg.vocab_size)
        oracle = sd.generate(prompts, N, prefix="o_")
        for rate in args.emulate_accept:
            q = accept_prob(rate, args.k)
            if rank == 0:
                sd.drafter = EmulatedDrafter(real, [o + [0] * (args.k + 1) for o in oracle],
                                             plens, q, tcfg.vocab_size)
            out, best, stats = run(sd, f"e{int(rate * 100)}")
            same = sum(a == b for a, b in zip(out, oracle))
            report("emulated", best, stats, {"emulated_accept": rate, "q_per_position": round(q, 4),
                                             "outputs_equal_oracle": f"{same}/{B}"})
    if world > 1:
        # CUDA graphs that captured NCCL calls keep the communicator busy:
        # release every graph before tearing the process group down.
        import gc

        plain.graphs.clear()
        sd.vgraphs.clear()
        for d in (sd.drafter, getattr(sd.drafter, "inner", None)):
            if d is not None and hasattr(d, "gen"):
                d.gen.graphs.clear()
        del plain, sd
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
