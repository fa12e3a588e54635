"""DeepSeek-V4 against the reference's exported tiny model (4 layers,
hidden 64, 4 HC copies, ratio 4 / 16 compressed layers with the indexer,
a hash-routed first layer) and its recorded outputs.

The recorded logits come from the bf16 model while the export carries int4
experts, so logits agree to the int4 error (a few percent of their range)
and the greedy tokens agree exactly."""
import json
import os

import pytest
import torch

from cascadia_b200.models import dsv4
from cascadia_b200.models.dsv4 import DSV4Model

FIX = os.path.join(os.path.dirname(__file__), "fixtures", "dsv4_tiny")


def _ref():
    with open(os.path.join(FIX, "reference.json")) as f:
        return json.load(f)


def test_prefill_and_decode_logits_and_greedy_tokens():
    ref = _ref()
    m = DSV4Model(FIX, "cpu", max_seq=64)
    lg = m.prefill(ref["prompt_ids"])
    want = torch.tensor(ref["prefill_logits"])
    assert (lg - want).abs().max() <= 0.1 * want.abs().max()
    assert int(lg.argmax()) == int(want.argmax())
    d0 = m.decode(int(lg.argmax()), len(ref["prompt_ids"]))
    want0 = torch.tensor(ref["decode0_logits"])
    assert (d0 - want0).abs().max() <= 0.12 * want0.abs().max()
    assert m.generate(ref["prompt_ids"], len(ref["generated"])) == ref["generated"]


def test_token_by_token_drive_equals_prefill():
    """Every prompt token through the stateful decode path (ring, compressor
    windows, indexer cache) gives the same greedy continuation as the
    batched prefill, and reset() makes the model reusable."""
    ref = _ref()
    m = DSV4Model(FIX, "cpu", max_seq=64)
    prompt = ref["prompt_ids"]
    for _ in range(2):
        m.reset()
        for p, t in enumerate(prompt):
            lg = m.decode(t, p)
        out = [int(lg.argmax())]
        while len(out) < len(ref["generated"]):
            out.append(int(m.decode(out[-1], len(prompt) + len(out) - 1).argmax()))
        assert out == ref["generated"]


def test_quant_sims_on_their_grids():
    x = torch.tensor([[0.3, -1.7, 5.9, 100.0, 1e-3, -0.0, 2.5, 0.75] * 8])
    y = dsv4.fp8_sim(x, 64)
    s = dsv4.pow2_ceil(x.abs().max().clamp_min(1e-4) / 448.0)
    q = (y / s)
    assert torch.equal(q.to(torch.float8_e4m3fn).float(), q)  # on the e4m3 grid
    z = dsv4.fp4_sim(x, 32)
    grid = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    for g in z.view(-1, 32):
        sc = dsv4.pow2_ceil(g.abs().max() / 6.0 + 1e-30)
        assert torch.isin((g.abs() / sc), grid).all()
    # ties to the even mantissa: 2.5 -> 2, 0.75 -> 1 (grid units)
    assert dsv4._round_e2m1(torch.tensor([2.5, 0.75, -5.0, 1.25])).tolist() == [2.0, 1.0, -4.0,
                                                                               1.0]
    assert dsv4.pow2_ceil(torch.tensor([3.0, 4.0, 0.3])).tolist() == [4.0, 4.0, 0.5]


def test_sinkhorn_is_doubly_stochastic():
    g = torch.Generator().manual_seed(0)
    hc = 4
    mixes = torch.randn(5, (2 + hc) * hc, generator=g)
    pre, post, comb = dsv4.hc_coeffs(mixes, torch.ones(3), torch.zeros((2 + hc) * hc), hc, 20,
                                     1e-6)
    assert torch.allclose(comb.sum(-2), torch.ones(5, hc), atol=1e-4)
    assert torch.allclose(comb.sum(-1), torch.ones(5, hc), atol=1e-3)
    assert (post > 0).all() and (post < 2).all() and (pre > 0).all()


def test_engine_serves_through_api():
    """The V4 engine behind the runner and the OpenAI API: greedy tokens of
    the recorded prompt, and a second request served after the first."""
    from fastapi.testclient import TestClient

    from cascadia_b200.api.server import ApiConfig, make_app
    from cascadia_b200.engine.dsv4 import DSV4Builder
    from cascadia_b200.runtime.runner import Runner
    from cascadia_b200.types import PeerLayout, ShardSpec

    ref = _ref()
    r = Runner(DSV4Builder(FIX, "cpu", max_seq=64), model_id="dsv4-tiny", device="cpu")
    r.start(PeerLayout(), ShardSpec("dsv4-tiny", 0, 4, 4))
    with TestClient(make_app(r, ApiConfig(model_name="dsv4-tiny"))) as c:
        for _ in range(2):
            j = c.post("/v1/completions", json={
                "prompt": "x", "prompt_token_ids": ref["prompt_ids"],
                "max_tokens": len(ref["generated"]), "logprobs": 0}).json()
            assert j["usage"]["completion_tokens"] == len(ref["generated"])
            assert j["usage"]["prompt_tokens"] == len(ref["prompt_ids"])
        too_long = c.post("/v1/completions", json={"prompt": "x",
                                                   "prompt_token_ids": list(range(70))})
        assert too_long.status_code == 500
    r.close()


def test_engine_greedy_tokens():
    from cascadia_b200.engine.dsv4 import DSV4Engine
    from cascadia_b200.types import GenerationTask

    ref = _ref()
    e = DSV4Engine(DSV4Model(FIX, "cpu", max_seq=64))
    e.submit(GenerationTask("a", "x", max_tokens=len(ref["generated"]),
                            prompt_ids=ref["prompt_ids"]))
    e.submit(GenerationTask("b", "x", max_tokens=3, prompt_ids=ref["prompt_ids"]))
    toks = {"a": [], "b": []}
    fins = {}
    for _ in range(50):
        for tid, ch in e.step():
            if ch.is_final:
                fins[tid] = ch.finish_reason
            elif ch.error is None:
                toks[tid].append(ch.token_id)
        if not e.has_work():
            break
    assert toks["a"] == ref["generated"] and toks["b"] == ref["generated"][:3]
    assert fins["b"].name == "LENGTH"
