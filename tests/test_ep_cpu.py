"""Expert parallelism on CPU ranks (gloo): each rank holds half the experts
and its own sequences; logits must match the single-process MoE model."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run_model(m, prompts, tag):
    from cascadia_b200.models.llama import build_batch

    ids = [f"{tag}{i}" for i in range(len(prompts))]
    m.allocate_kv(64)
    for s in ids:
        m.kv.add_sequence(s)
    b = build_batch(m, ids, [len(p) for p in prompts], [0] * len(prompts), False)
    hid = m.embed_tokens(torch.tensor([t for p in prompts for t in p], dtype=torch.int32))
    m.forward(b, hid)
    pre = m.head(hid.index_select(0, torch.tensor(b.last_rows)).contiguous()).float()
    b2 = build_batch(m, ids, [1] * len(prompts), [len(p) for p in prompts], True)
    hid2 = m.embed_tokens(torch.tensor([5 + i for i in range(len(prompts))], dtype=torch.int32))
    m.forward(b2, hid2)
    return pre, m.head(hid2).float()


def _worker(rank, world, port, cfg_name, prompts_per_rank, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cascadia_b200.models.config import get_config
        from cascadia_b200.models.moe import MoEModel
        from cascadia_b200.parallel.ep import ExpertParallel

        cfg = get_config(cfg_name)
        ep = ExpertParallel(dist.group.WORLD, rank, world, "cpu", cfg.num_experts,
                            cfg.hidden_size, cfg.num_experts_per_tok, max_tokens=64)
        m = MoEModel(cfg, "cpu", ep=ep).init_random(seed=11, gen_device="cpu")
        assert m.layers[-1].experts.E == cfg.num_experts // world
        q.put((rank, _run_model(m, prompts_per_rank[rank], f"r{rank}_")))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ep2_matches_single_process():
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.moe import MoEModel

    cfg = get_config("tiny-moe")
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (6, 11, 3)]
    per_rank = [prompts[:2], prompts[2:]]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, "tiny-moe", per_rank, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        ref = MoEModel(cfg, "cpu").init_random(seed=11, gen_device="cpu")
        pre_ref, dec_ref = _run_model(ref, per_rank[r], "s")
        pre, dec = got[r]
        for a, b in ((pre, pre_ref), (dec, dec_ref)):
            assert (a - b).abs().max().item() <= 0.02 * b.abs().max().item() + 1e-3
