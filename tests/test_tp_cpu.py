"""Tensor-parallel sharding on CPU ranks (gloo): TP=2 and TP=4 equal TP=1.

TP=4 runs a vocabulary (1000) that does not divide by 4 x 128, so the LM
head's per-rank shard is padded to the GEMM's 128-row tile; the padded rows
must stay out of full_logits and the greedy merge.  The 8B-shape test builds
the kernel blobs of every sharded projection at TP 2/4/8 (the check that the
GEMM accepts each shard's rows and columns)."""
import dataclasses
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


def _config(name):
    from cascadia_b200.models.config import get_config

    if name == "tiny-llama-tp4":
        # 8 heads / 4 KV heads split 4 ways; vocab 1000 -> 256-row shards,
        # the last rank holding 232 real rows.
        return dataclasses.replace(get_config("tiny-llama"), vocab_size=1000, num_heads=8,
                                   num_kv_heads=4)
    return get_config(name)


def _prefill(m, prompts):
    from cascadia_b200.models.llama import build_batch

    ids = [f"p{i}" for i in range(len(prompts))]
    for s in ids:
        m.kv.add_sequence(s)
    b = build_batch(m, ids, [len(p) for p in prompts], [0] * len(prompts), False)
    hid = m.embed_tokens(torch.tensor([t for p in prompts for t in p], dtype=torch.int32))
    m.forward(b, hid)
    last = hid[torch.tensor(b.last_rows)]
    logits = m.head(last)
    return m.full_logits(logits).float(), m.greedy(logits)


def _worker(rank, world, port, cfg_name, prompts, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cascadia_b200.models.llama import LlamaModel, TPGroup

        m = LlamaModel(_config(cfg_name), "cpu", tp=TPGroup(rank, world, dist.group.WORLD))
        m.init_random(seed=11, gen_device="cpu")
        m.allocate_kv(64)
        logits, toks = _prefill(m, prompts)
        if rank == 0:
            q.put((logits, toks))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cfg_name", [(2, "tiny-llama"), (4, "tiny-llama-tp4")])
def test_tp_matches_tp1(world, cfg_name):
    from cascadia_b200.models.llama import LlamaModel

    cfg = _config(cfg_name)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (6, 21)]
    m = LlamaModel(cfg, "cpu").init_random(seed=11, gen_device="cpu")
    m.allocate_kv(64)
    ref, ref_toks = _prefill(m, prompts)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg_name, prompts, q))
             for r in range(world)]
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
    logits, toks = out
    assert logits.shape == ref.shape == (len(prompts), cfg.vocab_size)
    # Sharded partial sums are rounded to bf16 before the all-reduce, so
    # compare with a tolerance relative to the logit scale.
    err = (logits - ref).abs().max().item()
    assert err <= 0.03 * ref.abs().max().item() + 1e-4, err
    # The merged greedy pick is the argmax of the gathered logits (never a
    # padded row) and agrees with TP=1 wherever the top-2 margin exceeds the
    # rounding tolerance.
    assert torch.equal(toks.long(), logits.argmax(-1))
    assert int(toks.max()) < cfg.vocab_size
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2 * err
    assert torch.equal(toks.long()[clear], ref_toks.long()[clear])


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_llama8b_shards_pack_at_tp(tp):
    """Every sharded projection of Llama-3.1-8B packs into kernel blobs at
    TP=tp on every rank (K reduced to 128 where it is not the sharded axis,
    which leaves the row-tile check the same), and the padded vocab shards
    cover the vocabulary exactly once."""
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel, TPGroup
    from cascadia_b200.quant import Int4Weight, pack_blob

    cfg = get_config("llama-3.1-8b")
    h, d = cfg.hidden_size, cfg.head_dim

    def w(n, k):
        return Int4Weight(torch.full((n, k // 8), -2004318072, dtype=torch.int32),
                          torch.ones(n, k // cfg.group_size, dtype=torch.float16),
                          cfg.group_size)

    covered = 0
    for r in range(tp):
        m = LlamaModel(cfg, "meta", tp=TPGroup(r, tp))
        # Column-parallel outputs with a short K; row-parallel inputs full.
        q, k, v = w(cfg.num_heads * d, 128), w(cfg.num_kv_heads * d, 128), w(cfg.num_kv_heads * d, 128)
        gate, up = w(cfg.intermediate_size, 128), w(cfg.intermediate_size, 128)
        o, down = w(128, cfg.num_heads * d), w(128, cfg.intermediate_size)
        hq, hkv, it = m.hq, m.hkv, m.inter
        qkv = Int4Weight.cat_rows([q.rows(r * hq * d, (r + 1) * hq * d),
                                   k.rows(r * hkv * d, (r + 1) * hkv * d),
                                   v.rows(r * hkv * d, (r + 1) * hkv * d)])
        gu = Int4Weight.cat_rows([gate.rows(r * it, (r + 1) * it), up.rows(r * it, (r + 1) * it)])
        shards = [(qkv, False), (gu, True), (o.cols(r * hq * d, (r + 1) * hq * d), False),
                  (down.cols(r * it, (r + 1) * it), False)]
        head = m._vocab_shard(w(cfg.vocab_size, 128))
        shards.append((head, False))
        assert head.n == m.vocab_shard and m.vocab_shard % 128 == 0
        for s, inter in shards:
            blob = pack_blob(s.unpack(), s.scales, s.group_size, inter)
            assert blob.numel() > 0
        covered += m.vocab_valid
        # Padded rows dequantise to exactly zero.
        if m.vocab_valid < m.vocab_shard:
            assert head.dequant_bf16()[m.vocab_valid:].abs().max().item() == 0.0
    assert covered == cfg.vocab_size
