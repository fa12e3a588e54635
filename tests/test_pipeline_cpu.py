"""Pipeline parallelism over the native TCP transport on CPU (loopback).

Two stages in one process (threads): stage 0 = LLMEngine + PipelineHead,
stage 1 = PipelineWorker driven by Runner.run_relay_loop.  Greedy output must
equal the single-stage engine (both stages hold slices of the same
random-init model).  Also covers the transport framing, the seq-echo guard and
connection-fatal exits.
"""
import threading

import pytest
import torch

from cascadia_b200.engine import base as eb
from cascadia_b200.engine.llm import LLMEngine
from cascadia_b200.models.config import get_config
from cascadia_b200.models.llama import LlamaModel
from cascadia_b200.parallel.pp import PipelineHead, PipelineWorker, TcpChannel
from cascadia_b200.runtime.runner import RelayExit, Runner
from cascadia_b200.transport.tcp import FrameStartTimeout, TensorLink
from cascadia_b200.types import GenerationTask

rt = pytest.importorskip("cascadia_b200._runtime")


def _pair():
    srv = TensorLink.listen("127.0.0.1", 0)
    out = {}
    th = threading.Thread(target=lambda: out.setdefault("a", TensorLink.accept(srv, 10)))
    th.start()
    client = TensorLink.connect("127.0.0.1", srv.port, 10)
    th.join()
    return out["a"], client, srv


def test_tensor_frames_roundtrip():
    a, b, srv = _pair()
    for t in (torch.arange(12, dtype=torch.int32).view(3, 4), torch.randn(2, 3, 5),
              torch.randn(7, 9).to(torch.bfloat16), torch.tensor([1, 2], dtype=torch.int64)):
        b.send(t)
        r = a.recv()
        assert r.dtype == t.dtype and torch.equal(r.reshape(t.shape), t)
    b.send_raw(b"\x01\x02\x03\x04")
    assert a.recv_raw(4) == b"\x01\x02\x03\x04"
    with pytest.raises(FrameStartTimeout) as ei:
        a.recv(first_byte_s=0.2)
    assert not ei.value.is_connection_fatal()
    b.close()
    with pytest.raises(eb.EngineError) as ei2:
        a.recv(first_byte_s=2.0)
    assert ei2.value.is_connection_fatal()
    a.close()
    srv.close()


def _models(cfg, seed=3):
    full = LlamaModel(cfg, "cpu").init_random(seed=seed, gen_device="cpu")
    half = cfg.num_layers // 2
    s0 = LlamaModel(cfg, "cpu", layer_start=0, layer_end=half, has_embed=True,
                    has_head=False).init_random(seed=seed, gen_device="cpu")
    s1 = LlamaModel(cfg, "cpu", layer_start=half, layer_end=cfg.num_layers, has_embed=False,
                    has_head=True).init_random(seed=seed, gen_device="cpu")
    for m in (full, s0, s1):
        m.allocate_kv(128)
    return full, s0, s1


def test_two_stage_pipeline_matches_single_stage():
    cfg = get_config("tiny-llama")
    full, s0, s1 = _models(cfg)
    down, up, srv = _pair()  # stage0.down = client side, stage1.up = accepted side
    head = PipelineHead(s0, TcpChannel(down=up))
    worker = PipelineWorker(s1, TcpChannel(up=down), is_last=True)
    r1 = Runner(None)
    r1.start_with_engine(worker, drive=False)
    exit_code = {}
    th = threading.Thread(target=lambda: exit_code.setdefault("x", r1.run_relay_loop()))
    th.start()
    e0 = LLMEngine(s0, max_model_len=512)
    e0.pipeline = head
    ref = LLMEngine(full, max_model_len=512)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(3, 500, (n,), generator=g).tolist() for n in (7, 30)]

    def run(e):
        tasks = [GenerationTask(f"t{i}", "", max_tokens=6, prompt_ids=p)
                 for i, p in enumerate(prompts)]
        for t in tasks:
            e.submit(t)
        out = {t.task_id: [] for t in tasks}
        for _ in range(50):
            for tid, c in e.step():
                if not c.is_final:
                    out[tid].append(c.token_id)
            if not e.has_work():
                break
        return out

    assert run(e0) == run(ref)
    head.shutdown()
    th.join(timeout=10)
    assert exit_code["x"] is RelayExit.CONNECTION_FATAL or exit_code["x"] is RelayExit.SLOT_EMPTY
    up.close()
    down.close()
    srv.close()


def test_worker_exits_connection_fatal_when_upstream_dies():
    cfg = get_config("tiny-llama")
    _, _, s1 = _models(cfg)
    down, up, srv = _pair()
    worker = PipelineWorker(s1, TcpChannel(up=down), is_last=True)
    r = Runner(None)
    r.start_with_engine(worker, drive=False)
    res = {}
    th = threading.Thread(target=lambda: res.setdefault("x", r.run_relay_loop()))
    th.start()
    up.close()  # upstream stage crashed
    th.join(timeout=10)
    assert res["x"] is RelayExit.CONNECTION_FATAL
    srv.close()
