"""Activation-sparse SwiGLU FFN (single-token decode option): mask
semantics, CHESS calibration, the CPU path against the dense FFN, and the
GPU kernels against the CPU path."""
import pytest
import torch

from cascadia_b200.ops.ffn_sparse import SparseFFN, build_active_mask, calibrate_tau
from cascadia_b200.quant import Int4Weight

H, I = 512, 1024


def _weights(seed=0, gs=128):
    g = torch.Generator().manual_seed(seed)
    gate = Int4Weight.random(I, H, std=0.05, group_size=gs, generator=g)
    up = Int4Weight.random(I, H, std=0.05, group_size=gs, generator=g)
    down = Int4Weight.random(H, I, std=0.05, group_size=gs, generator=g)
    x = (torch.randn(1, H, generator=g)).to(torch.bfloat16)
    return gate, up, down, x


def _dense(gate, up, down, x):
    xf = x[0].float()
    a = torch.nn.functional.silu(gate.dequant_bf16().float() @ xf) * (up.dequant_bf16().float() @ xf)
    return a @ down.dequant_bf16().float().t()


def test_mask_semantics_and_uniform_per_channel_equals_global():
    g = torch.randn(I, generator=torch.Generator().manual_seed(1))
    s, act = build_active_mask(g, 0.1)
    mx = torch.nn.functional.silu(g).abs().max()
    assert torch.equal(act, torch.nonzero(s.abs() >= 0.1 * mx).flatten())
    _, act2 = build_active_mask(g, torch.full((I,), 0.1))
    assert torch.equal(act, act2)
    _, dense = build_active_mask(g, 0.0)
    assert dense.numel() == I


def test_calibrated_taus_hit_the_active_fraction():
    samples = torch.randn(400, I, generator=torch.Generator().manual_seed(2))
    tau = calibrate_tau(samples, 0.4)
    frac = sum(build_active_mask(samples[i], tau)[1].numel() for i in range(400)) / (400 * I)
    assert abs(frac - 0.4) < 0.03


def test_cpu_sparse_ffn_tau0_equals_dense_and_error_grows_with_tau():
    gate, up, down, x = _weights()
    want = _dense(gate, up, down, x)
    ffn0 = SparseFFN(gate, up, down, "cpu", tau_all=0.0)
    got = ffn0(x)[0].float()
    # tau 0 with the re-quantised transposed down is the dense arithmetic ...
    down_t = ffn0.down_t_w.dequant_bf16().float()
    exact = _dense(gate, up, Int4Weight.quantize(down_t.t().contiguous(), 128), x)
    xf = x[0].float()
    a = torch.nn.functional.silu(gate.dequant_bf16().float() @ xf) * (up.dequant_bf16().float() @ xf)
    assert torch.allclose(got, (a @ down_t).to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)
    # ... and the second rounding of down (INT4 on a new grid) costs up to
    # ~10 % of the largest output on random weights.
    assert (got - want).abs().max() <= 0.15 * want.abs().max()
    del exact
    errs = []
    for tau in (0.02, 0.1, 0.3):
        f = SparseFFN(gate, up, down, "cpu", tau_all=tau)
        errs.append((f(x)[0].float() - want).abs().max().item())
        assert f.active_fraction(x) < 1.0
    assert errs[0] <= errs[-1]


@pytest.mark.gpu
@pytest.mark.parametrize("per_channel", [False, True])
def test_gpu_sparse_ffn_matches_cpu(per_channel):
    gate, up, down, x = _weights(seed=5)
    tau = torch.rand(I, generator=torch.Generator().manual_seed(3)) * 0.2 if per_channel else None
    cpu = SparseFFN(gate, up, down, "cpu", tau_all=0.08, tau=tau)
    gpu = SparseFFN(gate, up, down, "cuda", tau_all=0.08, tau=tau)
    res = torch.randn(1, H, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    want = cpu(x, residual=res)
    for _ in range(2):  # the fp32 accumulator must be left zero for the next call
        got = gpu(x.cuda(), residual=res.cuda())
        torch.cuda.synchronize()
        err = (got.cpu().float() - want.float()).abs().max().item()
        # A lane whose |silu(g)| sits within rounding of the threshold may
        # flip between the CPU and GPU gate sums; its contribution is small.
        assert err <= 0.05 * want.float().abs().max().item() + 1e-2, err


@pytest.mark.gpu
def test_llama_decode_with_sparse_ffn_gpu_matches_cpu():
    from cascadia_b200.models import llama
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel
    from cascadia_b200.runtime.generator import BatchGenerator

    cfg = get_config("tiny-llama-128")
    llama.KEEP_INT4 = True
    try:
        cpu = LlamaModel(cfg, "cpu").init_random(seed=4, gen_device="cpu")
        gpu = LlamaModel(cfg, "cuda").init_random(seed=4, gen_device="cpu")
    finally:
        llama.KEEP_INT4 = False
    for m in (cpu, gpu):
        m.allocate_kv(64)
        m.enable_ffn_sparsity(0.05)
    prompt = [torch.randint(0, cfg.vocab_size, (9,), generator=torch.Generator().manual_seed(6)).tolist()]
    want = BatchGenerator(cpu, use_graph=False).generate(prompt, 8)
    got = BatchGenerator(gpu, use_graph=True).generate(prompt, 8)
    assert got[0][:3] == want[0][:3]
    assert sum(a == b for a, b in zip(got[0], want[0])) >= 6
