"""Programmatic dependent launch: kernels that start before their predecessor
finishes must still read its results.  Chains of dependent kernels are run
with the launch attribute on and off (eagerly and inside CUDA graphs); the
outputs must be bitwise identical, since the same kernels run either way."""
import pytest
import torch

from cascadia_b200 import ops
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.quant import Int4Weight
from cascadia_b200.runtime.generator import BatchGenerator

pytestmark = pytest.mark.gpu


def _chain(x, layers, norm_w):
    """rmsnorm -> GEMM (SiLU) -> GEMM (+residual) per layer, residual stream in h."""
    h = x.clone()
    y = torch.empty_like(h)
    for gu, dn, inter in layers:
        ops.rmsnorm(h, norm_w, y, 1e-5)
        act = ops.w4a16_gemm(y, gu, 2 * inter, 128, ops.EPI_SILU)
        ops.w4a16_gemm(act, dn, h.shape[1], 128, ops.EPI_RESID, residual=h, out=h)
    return h


@pytest.mark.parametrize("m", [1, 8, 64])
def test_pdl_chain_matches_serial(m):
    torch.manual_seed(0)
    H, inter = 2048, 4096
    g = torch.Generator().manual_seed(1)
    layers = []
    for _ in range(4):
        gu = Int4Weight.random(2 * inter, H, generator=g).blob(True).to("cuda")
        dn = Int4Weight.random(H, inter, generator=g).blob().to("cuda")
        layers.append((gu, dn, inter))
    x = (torch.randn(m, H, device="cuda") * 0.5).to(torch.bfloat16)
    nw = (torch.rand(H, device="cuda") + 0.5).to(torch.bfloat16)
    ext = ops.ext()
    was = ext.pdl_enabled()
    try:
        ext.set_pdl(False)
        ref = _chain(x, layers, nw)
        ext.set_pdl(True)
        for _ in range(3):
            assert torch.equal(_chain(x, layers, nw), ref)
        # The same chain captured in a graph and replayed several times.
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            _chain(x, layers, nw)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = _chain(x, layers, nw)
        for _ in range(5):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        del graph
    finally:
        ext.set_pdl(was)
    assert ops.read_status(torch.device("cuda")) == 0


def test_pdl_generation_identical():
    cfg = get_config("tiny-llama-128")
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (4, 19, 50)]
    ext = ops.ext()
    was = ext.pdl_enabled()
    outs = []
    try:
        for on in (False, True):
            ext.set_pdl(on)
            model = LlamaModel(cfg, "cuda").init_random(seed=7, gen_device="cpu")
            model.allocate_kv(128)
            outs.append(BatchGenerator(model, use_graph=True).generate(prompts, 12))
    finally:
        ext.set_pdl(was)
    assert outs[0] == outs[1]
    assert ops.read_status(torch.device("cuda")) == 0
