"""The persistent stream-K W4A16 GEMM (decode batches up to 64 rows) against
the fp32 reference: every epilogue, both group sizes, shapes that take each
work decomposition (row-tile pairs or single tiles, two- or one-k-block
steps, pairs split between CTAs), repeated launches (the arrival counters
must return to zero) and bitwise run-to-run determinism."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.ops import reference as ref
from cascadia_b200.quant import Int4Weight

pytestmark = pytest.mark.gpu
DEV = "cuda"
STREAM = -1  # forced kernel choice: the persistent stream kernel


def _expect(x, qw, epi, r):
    full = x.float() @ qw.dequant_bf16().float().t()
    if epi == ops.EPI_SILU:
        i = full.shape[1] // 2
        return ref.silu_mul(full[:, :i], full[:, i:])
    if epi == ops.EPI_RESID:
        return full + r.float()
    return full


def _check(m, n, k, gs, epi, seed):
    g = torch.Generator().manual_seed(seed)
    qw = Int4Weight.random(n, k, group_size=gs, generator=g, std=0.05)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16)
    r = torch.randn(m, n, generator=g).to(torch.bfloat16)
    blob = qw.blob(interleave_gate_up=(epi == ops.EPI_SILU)).to(DEV)
    plan = ops.w4a16_plan(m, n, k, STREAM)
    assert plan[0] == 1, plan  # the stream kernel takes this shape
    outs = []
    for _ in range(3):  # repeated: counters back to zero, results identical
        rd = r.to(DEV) if epi == ops.EPI_RESID else None
        outs.append(ops.w4a16_gemm(x.to(DEV), blob, n, gs, epi, rd, splits=STREAM))
    torch.cuda.synchronize()
    assert ops.read_status(torch.device(DEV)) == 0
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    expect = _expect(x, qw, epi, r)
    err = (outs[0].float().cpu() - expect).abs()
    tol = 2e-2 + 1e-2 * expect.abs()
    assert (err > tol).sum().item() == 0, f"max err {err.max().item():.4g} plan {plan}"
    return plan


@pytest.mark.parametrize("m", [1, 7, 16, 17, 33, 64])
@pytest.mark.parametrize("n,k", [
    (384, 1024),     # odd tile count: single tiles, one-k-block steps, 8 contributors a tile
    (1024, 512),     # small GEMM: fine steps
    (256, 384),      # odd k-block count: a last step of one k-block
    (6144, 4096),    # tile pairs, two-k-block steps
    (4096, 14336),   # long K: every pair split between ~10 CTAs
])
def test_stream_store(m, n, k):
    _check(m, n, k, 128, ops.EPI_STORE, m * 31 + n + k)


@pytest.mark.parametrize("m", [3, 32, 64])
@pytest.mark.parametrize("epi", [ops.EPI_SILU, ops.EPI_RESID])
@pytest.mark.parametrize("gs", [128, 32])
def test_stream_epilogues(m, epi, gs):
    _check(m, 2048, 2048, gs, epi, m + epi * 7 + gs)


def test_stream_gate_up_shape_matches_splitk():
    """Llama-3.1-8B gate_up at decode batch 64: stream kernel vs the split-K
    tcgen05 kernel on the same inputs."""
    g = torch.Generator().manual_seed(1)
    n, k, m = 28672, 4096, 64
    qw = Int4Weight.random(n, k, generator=g, std=0.02)
    x = (torch.randn(m, k, generator=g)).to(torch.bfloat16).to(DEV)
    blob = qw.blob(interleave_gate_up=True).to(DEV)
    a = ops.w4a16_gemm(x, blob, n, 128, ops.EPI_SILU, splits=STREAM)
    b = ops.w4a16_gemm(x, blob, n, 128, ops.EPI_SILU, splits=1)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device(DEV)) == 0
    err = (a.float() - b.float()).abs()
    assert (err > 1e-2 + 1e-2 * b.float().abs()).sum().item() == 0, err.max().item()


def test_kernel_choice():
    for m in (1, 8):
        assert ops.w4a16_plan(m, 4096, 4096, 0)[0] == 2      # small-M kernel
    for m in (9, 64, 65):
        assert ops.w4a16_plan(m, 4096, 4096, 0)[0] == 0      # split-K tcgen05 kernel
    assert ops.w4a16_plan(64, 4096, 4096, STREAM)[0] == 1    # stream kernel on request


@pytest.mark.parametrize("m,n,k", [(64, 2048, 4096), (16, 2048, 4096), (64, 4096, 14336)])
def test_stream_residual_in_place(m, n, k):
    """out and residual are the same tensor (the decoder's residual stream):
    every element must be read and written once."""
    g = torch.Generator().manual_seed(m + n + k)
    qw = Int4Weight.random(n, k, generator=g, std=0.02)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16)
    r = torch.randn(m, n, generator=g).to(torch.bfloat16)
    blob = qw.blob().to(DEV)
    h = r.to(DEV)
    ops.w4a16_gemm(x.to(DEV), blob, n, 128, ops.EPI_RESID, residual=h, out=h, splits=STREAM)
    other = ops.w4a16_gemm(x.to(DEV), blob, n, 128, ops.EPI_RESID, residual=r.to(DEV),
                           splits=STREAM)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device(DEV)) == 0
    expect = _expect(x, qw, ops.EPI_RESID, r)
    for got in (other, h):
        err = (got.float().cpu() - expect).abs()
        assert (err > 2e-2 + 1e-2 * expect.abs()).sum().item() == 0, err.max().item()


@pytest.mark.parametrize("m,n,k", [(64, 2048, 4096), (16, 2048, 4096), (64, 384, 1024),
                                   (64, 8192, 2048)])
def test_stream_counters_return_to_zero(m, n, k):
    """After each launch every arrival counter is zero again, and back-to-back
    launches give identical results."""
    g = torch.Generator().manual_seed(n + k)
    qw = Int4Weight.random(n, k, generator=g, std=0.02)
    x = (torch.randn(m, k, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    blob = qw.blob().to(DEV)
    ws = ops.default_workspace(torch.device(DEV))
    outs = []
    for _ in range(3):
        outs.append(ops.w4a16_gemm(x, blob, n, 128, ops.EPI_STORE, splits=STREAM))
        torch.cuda.synchronize()
        nz = torch.nonzero(ws.counters).flatten().tolist()
        assert nz == [], f"counters left non-zero at {nz[:16]} (row tile = index // 4)"
    assert ops.read_status(torch.device(DEV)) == 0
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    expect = x.float().cpu() @ qw.dequant_bf16().float().t()
    err = (outs[0].float().cpu() - expect).abs()
    assert (err > 2e-2 + 1e-2 * expect.abs()).sum().item() == 0, err.max().item()
