"""Pipelined decode on 2 GPUs (NCCL p2p, CUDA-graph micro-batch steps):
tokens equal single-GPU greedy generation (same kernels, bf16 hand-off)."""
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


def _worker(rank, world, port, prompts, steps, q):
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
        from cascadia_b200.models.llama import LlamaModel
        from cascadia_b200.parallel.pp_decode import PipelinedDecoder, pp_prefill

        cfg = get_config("tiny-llama-128")
        per = cfg.num_layers // world
        m = LlamaModel(cfg, dev, layer_start=rank * per, layer_end=(rank + 1) * per,
                       has_embed=rank == 0, has_head=rank == world - 1).init_random(
                           seed=13, gen_device="cpu")
        m.allocate_kv(128)
        mbs = [["a0", "a1"], ["b0", "b1"]]
        firsts = [pp_prefill(m, rank, world, ids, prompts[2 * i:2 * i + 2])
                  for i, ids in enumerate(mbs)]
        dec = PipelinedDecoder(m, rank, world, mbs, 8)
        out = [[f] for f in firsts]
        if rank == 0:
            for i in range(2):
                dec.set_tokens(i, firsts[i])
        for _ in range(steps):
            dec.step(capture_now=True)
            dec.finish()
            if rank == 0:
                for i in range(2):
                    out[i].append(dec.tokens(i))
        torch.cuda.synchronize()
        if rank == 0:
            q.put((out, ops.read_status(dev)))
        del dec
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(WORLD < 2, reason="needs >= 2 GPUs")
def test_pipelined_decode_two_gpus():
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel
    from cascadia_b200.runtime.generator import BatchGenerator

    cfg = get_config("tiny-llama-128")
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(3, 1000, (n,), generator=g).tolist() for n in (5, 40, 3, 17)]
    steps = 6
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, prompts, steps, q)) for r in range(2)]
    for p in ps:
        p.start()
    out, st = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert st == 0
    ref = LlamaModel(cfg, "cuda:0").init_random(seed=13, gen_device="cpu")
    ref.allocate_kv(128)
    want = BatchGenerator(ref).generate(prompts, steps + 1)
    got = [[out[i][0][j]] + [out[i][s][j] for s in range(1, steps + 1)]
           for i in range(2) for j in range(2)]
    assert got == want
