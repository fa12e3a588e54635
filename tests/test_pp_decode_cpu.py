"""Pipelined decode with micro-batch overlap (gloo ranks on CPU): tokens must
equal single-process greedy generation.  One code path for every family:
dense Llama, the hybrid Gated DeltaNet MoE (recurrent state per stage) and
GLM-5 (MLA + DSA indexer + MoE)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _build(preset, device, **kw):
    from cascadia_b200.engine.llm import LLMBuilder
    from cascadia_b200.models.config import get_config

    cfg = get_config(preset)
    cls = LLMBuilder.model_class(None, cfg)
    m = cls(cfg, device, **kw).init_random(seed=13, gen_device="cpu")
    if cfg.is_hybrid:
        m.allocate_kv(128, max_seqs=8)
    else:
        m.allocate_kv(128)
    return cfg, m


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, prompts, steps, q, preset="tiny-llama"):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cascadia_b200.models.config import get_config
        from cascadia_b200.parallel.pp_decode import PipelinedDecoder, pp_prefill

        L = get_config(preset).num_layers
        per = L // world
        end = L if rank == world - 1 else (rank + 1) * per
        cfg, m = _build(preset, "cpu", layer_start=rank * per, layer_end=end,
                        has_embed=rank == 0, has_head=rank == world - 1)
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


@pytest.mark.parametrize("preset", ["tiny-llama", "tiny-qwen36", "tiny-glm5", "tiny-gemma4"])
def test_pipelined_decode_matches_single_stage(preset):
    from cascadia_b200.runtime.generator import BatchGenerator

    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(3, 500, (n,), generator=g).tolist() for n in (5, 12, 3, 9)]
    steps = 6
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, prompts, steps, q, preset))
          for r in range(2)]
    for p in ps:
        p.start()
    out = q.get(timeout=300)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    _, ref = _build(preset, "cpu")
    want = BatchGenerator(ref).generate(prompts, steps + 1)
    got = []
    for i in range(2):
        for j in range(2):
            got.append([out[i][0][j]] + [out[i][s][j] for s in range(1, steps + 1)])
    assert got == want
