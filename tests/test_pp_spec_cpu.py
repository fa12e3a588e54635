"""Distributed speculative decoding across two pipeline stages (gloo ranks
on CPU): the tokens must equal plain greedy decoding of the full target,
with a draft model on rank 0 (here the target itself, so every draft is
accepted) and with n-gram drafts."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, prompts, n_new, mode, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from cascadia_b200.models.config import get_config
        from cascadia_b200.models.llama import LlamaModel
        from cascadia_b200.parallel.pp_spec import PipelinedSpecDecoder

        cfg = get_config("tiny-llama")
        per = cfg.num_layers // world
        m = LlamaModel(cfg, "cpu", layer_start=rank * per, layer_end=(rank + 1) * per,
                       has_embed=rank == 0, has_head=rank == world - 1).init_random(
                           seed=13, gen_device="cpu")
        m.allocate_kv(256)
        draft = None
        if mode == "draft" and rank == 0:
            draft = LlamaModel(cfg, "cpu").init_random(seed=13, gen_device="cpu")
            draft.allocate_kv(256)
        dec = PipelinedSpecDecoder(m, rank, world, k=3, draft=draft, use_graph=False)
        out = dec.generate(prompts, n_new)
        q.put((rank, out, dec.stats.accepted, dec.stats.drafted))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["draft", "ngram"])
def test_distributed_spec_equals_greedy(mode):
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel
    from cascadia_b200.runtime.generator import BatchGenerator

    cfg = get_config("tiny-llama")
    g = torch.Generator().manual_seed(8)
    base = torch.randint(3, 500, (6,), generator=g).tolist()
    prompts = [base * 3, torch.randint(3, 500, (9,), generator=g).tolist()]
    n_new = 10
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, prompts, n_new, mode, q))
          for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = LlamaModel(cfg, "cpu").init_random(seed=13, gen_device="cpu")
    ref.allocate_kv(256)
    want = BatchGenerator(ref, use_graph=False).generate(prompts, n_new)
    for rank, out, acc, drafted in res:
        assert out == want, (rank, out, want)
        if mode == "draft":
            assert drafted > 0 and acc == drafted  # identical draft: all accepted


def _tp_worker(rank, world, port, prompts, n_new, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from cascadia_b200.models.config import get_config
        from cascadia_b200.models.llama import LlamaModel, TPGroup
        from cascadia_b200.runtime.spec import SpecDecoder

        cfg = get_config("tiny-llama")
        m = LlamaModel(cfg, "cpu", tp=TPGroup(rank, world, dist.group.WORLD)).init_random(
            seed=13, gen_device="cpu")
        m.allocate_kv(256)
        draft = None
        if rank == 0:
            # The whole target as the draft: every draft must be accepted.
            draft = LlamaModel(cfg, "cpu").init_random(seed=13, gen_device="cpu")
            draft.allocate_kv(256)
        dec = SpecDecoder(m, draft=draft, k=3, use_graph=False, remote_draft=rank != 0)
        out = dec.generate(prompts, n_new)
        q.put((rank, out, dec.stats.accepted, dec.stats.drafted))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tp_target_draft_on_rank0_equals_greedy():
    """Target at TP=2, draft model on rank 0 only; the drafts reach rank 1 by
    a broadcast each round.  Both ranks emit plain greedy tokens of the
    full target."""
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel
    from cascadia_b200.runtime.generator import BatchGenerator

    cfg = get_config("tiny-llama")
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(3, 500, (n,), generator=g).tolist() for n in (7, 12)]
    n_new = 9
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_tp_worker, args=(r, 2, port, prompts, n_new, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = LlamaModel(cfg, "cpu").init_random(seed=13, gen_device="cpu")
    ref.allocate_kv(256)
    want = BatchGenerator(ref, use_graph=False).generate(prompts, n_new)
    for rank, out, acc, drafted in res:
        assert out == want, (rank, out, want)
        assert drafted > 0 and acc == drafted
