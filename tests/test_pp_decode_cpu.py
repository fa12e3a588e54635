"""Pipelined decode with micro-batch overlap (gloo ranks on CPU): tokens must
equal single-process greedy generation."""
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


def _worker(rank, world, port, prompts, steps, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cascadia_b200.models.config import get_config
        from cascadia_b200.models.llama import LlamaModel
        from cascadia_b200.parallel.pp_decode import PipelinedDecoder, pp_prefill

        cfg = get_config("tiny-llama")
        per = cfg.num_layers // world
        m = LlamaModel(cfg, "cpu", layer_start=rank * per, layer_end=(rank + 1) * per,
                       has_embed=rank == 0, has_head=rank == world - 1).init_random(
                           seed=13, gen_device="cpu")
        m.allocate_kv(128)
        mbs = [["a0", "a1"], ["b0", "b1"]]
        width = 8
        firsts = [pp_prefill(m, rank, world, ids, prompts[2 * i:2 * i + 2])
                  for i, ids in enumerate(mbs)]
        dec = PipelinedDecoder(m, rank, world, mbs, width, use_graph=False)
        out = [[f] for f in firsts] if rank == 0 else None
        if rank == 0:
            for i in range(2):
                dec.set_tokens(i, firsts[i])
        for _ in range(steps):
            dec.step()
            dec.finish()
            if rank == 0:
                for i in range(2):
                    out[i].append(dec.tokens(i))
        if rank == 0:
            q.put(out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_pipelined_decode_matches_single_stage():
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel
    from cascadia_b200.runtime.generator import BatchGenerator

    cfg = get_config("tiny-llama")
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(3, 500, (n,), generator=g).tolist() for n in (5, 12, 3, 9)]
    steps = 6
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, prompts, steps, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = q.get(timeout=300)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = LlamaModel(cfg, "cpu").init_random(seed=13, gen_device="cpu")
    ref.allocate_kv(128)
    want = BatchGenerator(ref).generate(prompts, steps + 1)
    got = []
    for i in range(2):
        for j in range(2):
            got.append([out[i][0][j]] + [out[i][s][j] for s in range(1, steps + 1)])
    assert got == want
