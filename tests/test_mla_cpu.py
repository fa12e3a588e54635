"""MLA model (Kimi-K2 layer structure, small width) on the CPU oracle path."""
import math

import torch

from cascadia_b200.models.config import get_config, rope_inv_freq, rope_table
from cascadia_b200.models.llama import build_batch
from cascadia_b200.models.mla import MLAModel, rope_pairs


def _run(m, toks, sid, start=0):
    b = build_batch(m, [sid], [len(toks)], [start], start > 0 and len(toks) == 1)
    hid = m.embed_tokens(torch.tensor(toks, dtype=torch.int32))
    m.forward(b, hid)
    return m.head(hid[-1:].contiguous()).float()


def test_mla_prefill_equals_incremental_decode():
    cfg = get_config("tiny-mla")
    m = MLAModel(cfg, "cpu").init_random(seed=3, gen_device="cpu")
    m.allocate_kv(32)
    toks = [5, 9, 13, 2, 7, 30, 11]
    m.kv.add_sequence("a")
    full = _run(m, toks, "a")
    m.kv.add_sequence("b")
    _run(m, toks[:-1], "b")
    step = _run(m, toks[-1:], "b", start=len(toks) - 1)
    assert (full - step).abs().max().item() <= 0.02 * full.abs().max().item() + 1e-3


def test_yarn_table_and_pair_rotation():
    cfg = get_config("kimi-k2")
    inv = rope_inv_freq(cfg, 64)
    # High-frequency pairs keep the base frequency, low-frequency ones are
    # divided by the YaRN factor.
    assert math.isclose(float(inv[0]), 1.0, rel_tol=1e-6)
    base = 1.0 / (cfg.rope_theta ** (62 / 64))
    assert math.isclose(float(inv[-1]), base / 64.0, rel_tol=1e-5)
    cs = rope_table(cfg, 8, rot=64)
    x = torch.randn(3, 2, 64)
    y = rope_pairs(x, torch.tensor([0, 1, 7]), cs)
    assert torch.allclose(y[0], x[0])            # position 0: identity
    # rotation preserves each pair's norm
    n0 = x[..., 0::2] ** 2 + x[..., 1::2] ** 2
    n1 = y[..., 0::2] ** 2 + y[..., 1::2] ** 2
    assert torch.allclose(n0, n1, atol=1e-5)
