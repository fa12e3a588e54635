"""The q/k/v GEMM with RoPE and the paged-KV write in its epilogue against
the separate GEMM + rope_kv kernels: same logits, same K/V cache contents,
for prefill rows and for a decode batch above the small-M threshold."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel, build_batch

pytestmark = pytest.mark.gpu


def _run(fuse: bool):
    ops.FUSE_ROPE = fuse
    try:
        cfg = get_config("tiny-llama-128")
        m = LlamaModel(cfg, "cuda").init_random(seed=9, gen_device="cpu")
        m.allocate_kv(128)
        g = torch.Generator().manual_seed(2)
        prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist()
                   for n in (5, 19, 33, 7, 12, 9, 40, 3, 21, 16, 11, 2)]
        ids = [f"s{i}" for i in range(len(prompts))]
        for s in ids:
            m.kv.add_sequence(s)
        b = build_batch(m, ids, [len(p) for p in prompts], [0] * len(prompts), False)
        hid = m.embed_tokens(torch.tensor([t for p in prompts for t in p], dtype=torch.int32,
                                          device="cuda"))
        m.forward(b, hid)
        pre = m.head(hid).float()
        toks = torch.randint(3, cfg.vocab_size, (len(prompts),), generator=g)
        b2 = build_batch(m, ids, [1] * len(prompts), [len(p) for p in prompts], True)
        h2 = m.embed_tokens(toks.to(torch.int32).cuda())
        m.forward(b2, h2)
        dec = m.head(h2).float()
        torch.cuda.synchronize()
        assert ops.read_status(torch.device("cuda")) == 0
        return pre.cpu(), dec.cpu(), m.kv.k.float().cpu(), m.kv.v.float().cpu()
    finally:
        ops.FUSE_ROPE = True


def test_fused_rope_kv_matches_separate_kernels():
    assert ops.rope_fusable(12, 128, 128, 128)
    a = _run(True)
    b = _run(False)
    for x, y in zip(a, b):
        scale = y.abs().max().item() + 1e-6
        assert (x - y).abs().max().item() <= 1e-2 * scale
    # The caches hold the same rotated keys and values.
    assert (a[2] - b[2]).abs().max().item() <= 1e-2 * b[2].abs().max().item()
