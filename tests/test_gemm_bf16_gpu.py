"""tcgen05 bf16 GEMM against an fp32 PyTorch reference: token tiles 32..256,
ragged M / N / K (TMA zero fill at the edges), split-K (forced and chosen),
residual epilogue, strided input and output, and the split-K counters
returning to zero."""
import pytest
import torch

from cascadia_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ref(x, w, r=None):
    y = x.float() @ w.float().t()
    if r is not None:
        y = y + r.float()
    return y


def _check(y, want):
    err = (y.float() - want).abs().max().item()
    scale = want.abs().max().item() + 1e-3
    assert err <= 1.5e-2 * scale, (err, scale)


@pytest.mark.parametrize("m,n,k", [(1, 128, 64), (5, 200, 136), (32, 5120, 2048),
                                   (64, 2048, 4096), (100, 384, 1024), (300, 640, 512),
                                   (1024, 1024, 2048)])
@pytest.mark.parametrize("resid", [False, True])
def test_bf16_gemm(m, n, k, resid):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    r = torch.randn(m, n, generator=g, device=DEV).to(torch.bfloat16) if resid else None
    y = ops.bf16_gemm(x, w, r)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device(DEV)) == 0
    _check(y, _ref(x, w, r))


@pytest.mark.parametrize("splits", [1, 2, 3, 8])
def test_bf16_gemm_splits_deterministic(splits):
    g = torch.Generator(device=DEV).manual_seed(splits)
    x = torch.randn(48, 2048, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(1024, 2048, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    ws = ops.default_workspace(torch.device(DEV))
    a = ops.bf16_gemm(x, w, splits=splits)
    b = ops.bf16_gemm(x, w, splits=splits)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device(DEV)) == 0
    assert torch.equal(a, b)
    _check(a, _ref(x, w))
    assert int(ws.counters.abs().sum()) == 0


def test_bf16_gemm_strided_out_and_input():
    g = torch.Generator(device=DEV).manual_seed(3)
    big = torch.randn(16, 3 * 512, generator=g, device=DEV).to(torch.bfloat16)
    x = big[:, 512:1024]          # row stride 1536 elements
    w = (torch.randn(256, 512, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    out = torch.zeros(16, 2 * 256, dtype=torch.bfloat16, device=DEV)
    ops.bf16_gemm(x, w, out=out[:, 256:])
    torch.cuda.synchronize()
    _check(out[:, 256:], _ref(x, w))
    assert int(out[:, :256].abs().sum()) == 0
