"""CPU 2-stage loopback pipeline (the reference's CPU pipeline config, our
timed CPU baseline): Llama-3.2-1B-shaped INT4 g128 decoder split in two
stages, two processes connected by the native TCP stage transport (20-byte
frame header) over 127.0.0.1, batch 1, a 128-token seeded prompt, greedy
decode of 64 tokens.  Weights are dequantised once to fp32 on the CPU (the
oracle path), so the arithmetic is exact INT4 dequant + fp32 GEMV.

    python bench/bench_cpu_pipeline.py [--model llama-3.2-1b] [--gen 64] [--prompt-len 128]

Prints one JSON line: decode tok/s (wall clock, after the first token) and
TTFT.
"""
import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def stage1(model_name, port_q, seed):
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel
    from cascadia_b200.parallel.pp import PipelineWorker, TcpChannel
    from cascadia_b200.runtime.runner import Runner
    from cascadia_b200.transport.tcp import TensorLink

    cfg = get_config(model_name)
    half = cfg.num_layers // 2
    m = LlamaModel(cfg, "cpu", layer_start=half, layer_end=cfg.num_layers, has_embed=False,
                   has_head=True).init_random(seed=seed, gen_device="cpu")
    m.allocate_kv(64)
    srv = TensorLink.listen("127.0.0.1", 0)
    port_q.put(srv.port)
    link = TensorLink.accept(srv, 120)
    r = Runner(None)
    r.start_with_engine(PipelineWorker(m, TcpChannel(up=link), is_last=True), drive=False)
    r.run_relay_loop()
    link.close()
    srv.close()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama-3.2-1b")
    p.add_argument("--gen", type=int, default=64)
    p.add_argument("--prompt-len", type=int, default=128)
    p.add_argument("--threads", type=int, default=0)
    a = p.parse_args()
    if a.threads:
        torch.set_num_threads(a.threads)
    from cascadia_b200.engine.llm import LLMEngine
    from cascadia_b200.models.config import get_config
    from cascadia_b200.models.llama import LlamaModel
    from cascadia_b200.parallel.pp import PipelineHead, TcpChannel
    from cascadia_b200.transport.tcp import TensorLink
    from cascadia_b200.types import GenerationTask

    seed = 7
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    proc = ctx.Process(target=stage1, args=(a.model, q, seed))
    proc.start()
    cfg = get_config(a.model)
    half = cfg.num_layers // 2
    t0 = time.time()
    m = LlamaModel(cfg, "cpu", layer_start=0, layer_end=half, has_embed=True,
                   has_head=False).init_random(seed=seed, gen_device="cpu")
    m.allocate_kv(64)
    load_s = time.time() - t0
    link = TensorLink.connect("127.0.0.1", q.get(timeout=600), 600)
    head = PipelineHead(m, TcpChannel(down=link))
    e = LLMEngine(m, max_model_len=a.prompt_len + a.gen + 8)
    e.pipeline = head
    g = torch.Generator().manual_seed(42)
    prompt = torch.randint(3, cfg.vocab_size, (a.prompt_len,), generator=g).tolist()
    e.submit(GenerationTask("b0", "", max_tokens=a.gen, prompt_ids=prompt))
    t_start = time.perf_counter()
    t_first, n = None, 0
    while e.has_work():
        for _, c in e.step():
            if not c.is_final:
                n += 1
                if t_first is None:
                    t_first = time.perf_counter()
    t_end = time.perf_counter()
    head.shutdown()
    proc.join(timeout=60)
    link.close()
    dec = (n - 1) / (t_end - t_first) if n > 1 else 0.0
    print(json.dumps({
        "metric": "CPU 2-stage loopback pipeline: greedy decode tok/s, batch 1",
        "model": a.model, "prompt_len": a.prompt_len, "generated": n,
        "decode_tok_s": round(dec, 2), "ttft_ms": round((t_first - t_start) * 1000, 1),
        "threads": torch.get_num_threads(), "load_s": round(load_s, 1),
        "transport": "native C++ TCP frames over 127.0.0.1",
        "data": "synthetic: random-init N(0,0.02) INT4 g128 weights, seeded prompt ids"}))


if __name__ == "__main__":
    main()
