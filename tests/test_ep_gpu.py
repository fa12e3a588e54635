"""Expert parallelism on 2+ GPUs: the fused peer-memory path (dispatch,
expert GEMMs with peer-store epilogue, combine) and the NCCL all-to-all
baseline against the single-GPU MoE model.  Child processes, one per GPU."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0


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
    hid = m.embed_tokens(torch.tensor([t for p in prompts for t in p], dtype=torch.int32,
                                      device=m.device))
    m.forward(b, hid)
    rows = torch.tensor(b.last_rows, device=m.device)
    pre = m.head(hid.index_select(0, rows).contiguous()).float().cpu()
    b2 = build_batch(m, ids, [1] * len(prompts), [len(p) for p in prompts], True)
    hid2 = m.embed_tokens(torch.tensor([5 + i for i in range(len(prompts))], dtype=torch.int32,
                                       device=m.device))
    m.forward(b2, hid2)
    return pre, m.head(hid2).float().cpu()


def _worker(rank, world, port, prompts_per_rank, fused, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from cascadia_b200 import ops
        from cascadia_b200.models.config import get_config
        from cascadia_b200.models.moe import MoEModel
        from cascadia_b200.parallel.ep import ExpertParallel

        cfg = get_config("tiny-moe")
        ep = ExpertParallel(dist.group.WORLD, rank, world, dev, cfg.num_experts,
                            cfg.hidden_size, cfg.num_experts_per_tok, max_tokens=64, fused=fused)
        m = MoEModel(cfg, dev, ep=ep).init_random(seed=11, gen_device="cpu")
        out = _run_model(m, prompts_per_rank[rank], f"r{rank}_")
        torch.cuda.synchronize()
        q.put((rank, out, ops.read_status(dev)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(world, fused, per_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, per_rank, fused, q))
          for r in range(world)]
    for p in ps:
        p.start()
    got = {}
    for _ in range(world):
        r, out, st = q.get(timeout=300)
        got[r] = (out, st)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


@pytest.mark.skipif(WORLD < 2, reason="needs >= 2 GPUs")
@pytest.mark.parametrize("fused", [True, False])
def test_ep_matches_single_gpu(fused):
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.moe import MoEModel

    cfg = get_config("tiny-moe")
    world = 2
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (6, 11, 3)]
    per_rank = [prompts[:2], prompts[2:]]
    got = _run(world, fused, per_rank)
    for r in range(world):
        (pre, dec), st = got[r]
        assert st == 0
        ref = MoEModel(cfg, "cuda:0").init_random(seed=11, gen_device="cpu")
        pre_ref, dec_ref = _run_model(ref, per_rank[r], "s")
        for a, b in ((pre, pre_ref), (dec, dec_ref)):
            assert (a - b).abs().max().item() <= 0.03 * b.abs().max().item() + 1e-3
