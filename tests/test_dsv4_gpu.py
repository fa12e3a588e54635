"""DeepSeek-V4 on the GPU: the Hyper-Connections pre-mix kernel against the
fp32 PyTorch path, and the tiny exported model's greedy tokens on CUDA."""
import json
import os

import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models import dsv4
from cascadia_b200.models.dsv4 import DSV4Model

pytestmark = pytest.mark.gpu
FIX = os.path.join(os.path.dirname(__file__), "fixtures", "dsv4_tiny")


@pytest.mark.parametrize("T,hc,dim", [(1, 4, 64), (7, 4, 256), (33, 4, 4096), (3, 2, 96)])
def test_hc_pre_kernel(T, hc, dim):
    g = torch.Generator().manual_seed(T + dim)
    copies = dsv4.bf16r(torch.randn(T, hc, dim, generator=g))
    nm = (2 + hc) * hc
    fn = torch.randn(nm, hc * dim, generator=g) * 0.02
    base = torch.randn(nm, generator=g) * 0.1
    scale = torch.tensor([1.0, 0.7, 1.3])
    flat = copies.reshape(T, -1)
    r = 1.0 / torch.sqrt((flat * flat).mean(-1, keepdim=True) + 1e-6)
    pre, post, comb = dsv4.hc_coeffs((flat @ fn.t()) * r, scale, base, hc, 20, 1e-6)
    y = dsv4.bf16r((pre[:, :, None] * copies).sum(1))
    gy, gpost, gcomb, gpre = ops.hc_pre(copies.cuda(), fn.cuda(), base.cuda(), scale.cuda(), 20,
                                        1e-6, 1e-6)
    torch.cuda.synchronize()
    assert torch.allclose(gpre.cpu(), pre, atol=1e-5)
    assert torch.allclose(gpost.cpu(), post, atol=1e-5)
    assert torch.allclose(gcomb.cpu(), comb, atol=1e-4)
    # y is bf16-rounded: allow one bf16 step.
    assert ((gy.cpu() - y).abs() <= 1e-2 * y.abs().clamp_min(1e-2)).all()


def test_tiny_model_greedy_on_cuda():
    with open(os.path.join(FIX, "reference.json")) as f:
        ref = json.load(f)
    m = DSV4Model(FIX, "cuda", max_seq=64)
    out = m.generate(ref["prompt_ids"], len(ref["generated"]))
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0
    assert out == ref["generated"]
    lg = m.prefill(ref["prompt_ids"]).cpu()
    want = torch.tensor(ref["prefill_logits"])
    assert (lg - want).abs().max() <= 0.1 * want.abs().max()
