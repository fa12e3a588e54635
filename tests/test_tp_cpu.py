"""Tensor-parallel sharding on CPU ranks (gloo): TP=2 == TP=1 (greedy)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prefill_logits(m, prompts):
    from cascadia_b200.models.llama import build_batch

    ids = [f"p{i}" for i in range(len(prompts))]
    for s in ids:
        m.kv.add_sequence(s)
    b = build_batch(m, ids, [len(p) for p in prompts], [0] * len(prompts), False)
    hid = m.embed_tokens(torch.tensor([t for p in prompts for t in p], dtype=torch.int32))
    m.forward(b, hid)
    last = hid[torch.tensor(b.last_rows)]
    return m.full_logits(m.head(last)).float()


def _worker(rank, world, port, prompts, steps, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cascadia_b200.models.config import get_config
        from cascadia_b200.models.llama import LlamaModel, TPGroup
        from cascadia_b200.runtime.generator import BatchGenerator

        cfg = get_config("tiny-llama")
        m = LlamaModel(cfg, "cpu", tp=TPGroup(rank, world, dist.group.WORLD))
        m.init_random(seed=11, gen_device="cpu")
        m.allocate_kv(64)
        logits = _prefill_logits(m, prompts)
        if rank == 0:
            q.put(logits)
    finally:
        dist.destroy_process_group()


def test_tp2_matches_tp1():
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel

    cfg = get_config("tiny-llama")
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (6, 21)]
    m = LlamaModel(cfg, "cpu").init_random(seed=11, gen_device="cpu")
    m.allocate_kv(64)
    ref = _prefill_logits(m, prompts)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompts, 0, q)) for r in range(2)]
    for p in procs:
        p.start()
    import queue as _queue
    out = None
    for _ in range(240):
        try:
            out = q.get(timeout=1)
            break
        except _queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        if out is None:
            p.kill()
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out is not None
    assert out.shape == ref.shape
    # Sharded partial sums are rounded to bf16 before the all-reduce, so
    # compare with a tolerance relative to the logit scale.
    err = (out - ref).abs().max().item()
    assert err <= 0.03 * ref.abs().max().item() + 1e-4, err
