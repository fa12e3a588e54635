"""Tensor parallelism on 2+ GPUs: peer-memory fused all-reduce, the GEMM
that pushes its partial into every rank's slots, NCCL, and TP=1.

Runs as child processes (one per GPU, NCCL).  Skipped when fewer than two
GPUs are visible.
"""
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


def _logits(m, prompts, decode_tokens):
    from cascadia_b200.models.llama import build_batch

    ids = [f"p{i}" for i in range(len(prompts))]
    for s in ids:
        m.kv.add_sequence(s)
    b = build_batch(m, ids, [len(p) for p in prompts], [0] * len(prompts), False)
    flat = torch.tensor([t for p in prompts for t in p], dtype=torch.int32, device=m.device)
    hid = m.embed_tokens(flat)
    m.forward(b, hid)
    rows = torch.tensor(b.last_rows, device=m.device)
    pre = m.full_logits(m.head(hid.index_select(0, rows).contiguous())).float().cpu()
    # One decode step (exercises the decode-attention path and the fused AR).
    starts = [len(p) for p in prompts]
    b2 = build_batch(m, ids, [1] * len(prompts), starts, True)
    hid2 = m.embed_tokens(torch.tensor(decode_tokens, dtype=torch.int32, device=m.device))
    m.forward(b2, hid2)
    dec = m.full_logits(m.head(hid2)).float().cpu()
    return pre, dec


def _worker(rank, world, port, prompts, decode_tokens, mode, q, cfg_name="tiny-llama-128"):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from cascadia_b200 import ops
        from cascadia_b200.models.config import get_config
        from cascadia_b200.models.llama import LlamaModel, TPGroup
        from cascadia_b200.parallel.tp import FusedTP

        cfg = get_config(cfg_name)
        tp = TPGroup(rank, world, dist.group.WORLD)
        if mode in ("fused", "push", "multimem"):
            tp.fused = FusedTP(dist.group.WORLD, rank, world, dev, cfg.hidden_size, 64,
                               push=mode == "push", multimem=mode == "multimem")
        m = LlamaModel(cfg, dev, tp=tp).init_random(seed=17, gen_device="cpu")
        m.allocate_kv(64)
        out = _logits(m, prompts, decode_tokens)
        torch.cuda.synchronize()
        st = ops.read_status(dev)
        if rank == 0:
            q.put((out, st))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(world, mode, prompts, decode_tokens, cfg_name="tiny-llama-128"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, prompts, decode_tokens, mode, q,
                                            cfg_name))
          for r in range(world)]
    for p in ps:
        p.start()
    out = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


@pytest.mark.skipif(WORLD < 2, reason="needs >= 2 GPUs")
def test_fused_tp_matches_nccl_and_tp1():
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel

    cfg = get_config("tiny-llama-128")
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 33)]
    decode_tokens = [7, 11]
    m = LlamaModel(cfg, torch.device("cuda", 0)).init_random(seed=17, gen_device="cpu")
    m.allocate_kv(64)
    ref_pre, ref_dec = _logits(m, prompts, decode_tokens)
    world = 2 if WORLD < 4 else min(WORLD, 4)
    (f_pre, f_dec), st = _run(world, "fused", prompts, decode_tokens)
    assert st == 0
    (p_pre, p_dec), st = _run(world, "push", prompts, decode_tokens)
    assert st == 0
    (n_pre, n_dec), _ = _run(world, "nccl", prompts, decode_tokens)
    (m_pre, m_dec), st = _run(world, "multimem", prompts, decode_tokens)
    assert st == 0
    scale = ref_pre.abs().max().item()
    for a, b in ((f_pre, ref_pre), (f_dec, ref_dec), (n_pre, ref_pre), (n_dec, ref_dec),
                 (p_pre, ref_pre), (p_dec, ref_dec), (m_pre, ref_pre), (m_dec, ref_dec)):
        assert (a - b).abs().max().item() <= 0.03 * scale + 1e-3
    # Prefill rows run the same GEMM kernel and sum the same bf16 partials
    # in rank order either way: pushing changes nothing in the result.
    assert torch.equal(p_pre, f_pre)


@pytest.mark.skipif(WORLD < 8, reason="needs 8 GPUs")
def test_push_tp8_matches_tp1():
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel

    cfg = get_config("tiny-llama-kv8")
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist() for n in (17, 40)]
    decode_tokens = [5, 9]
    m = LlamaModel(cfg, torch.device("cuda", 0)).init_random(seed=17, gen_device="cpu")
    m.allocate_kv(64)
    ref_pre, ref_dec = _logits(m, prompts, decode_tokens)
    (p_pre, p_dec), st = _run(8, "push", prompts, decode_tokens, "tiny-llama-kv8")
    assert st == 0
    scale = ref_pre.abs().max().item()
    for a, b in ((p_pre, ref_pre), (p_dec, ref_dec)):
        assert (a - b).abs().max().item() <= 0.03 * scale + 1e-3
