"""Command line: ``python -m cascadia_b200 <command>``.

Commands and flag names follow the reference CLI where the semantics carry
over (crates/cascadia-cli/src/lib.rs:144-770): ``worker`` (one stage / rank,
``--rank --total --layer-start --layer-end --model --listen --next --api
--engine``), ``run`` (single-process server), ``shard`` (write the per-stage
INT4 layout), ``engines``, ``doctor`` (CUDA / sm_100 / NCCL / NVLink checks)
and ``place`` (choose a PP x TP x EP split for the GPUs of one box).
"""
from __future__ import annotations

import argparse
import json
import logging
import os
import signal
import sys
import threading

ENGINES = {
    "mock": "word-echo engine for tests (no weights)",
    "llama": "dense Llama-family INT4 engine (continuous batching, paged KV, TP, PP)",
    "moe": "sparse-MoE INT4 engine (Qwen3-MoE / Kimi-K2 shapes, expert parallel)",
    "spec": "distributed speculative decoding (draft stage + target stages)",
    "dsv4": "DeepSeek-V4 export directory (--model DIR): hyper-connections, compressed KV",
}


def _init_logging(level: str):
    logging.basicConfig(level=getattr(logging, level.upper(), logging.INFO),
                        format="%(asctime)s %(levelname)s %(name)s: %(message)s")


def _parse_hostport(s: str, default_host="127.0.0.1"):
    if s is None:
        return None
    host, _, port = s.rpartition(":")
    return (host or default_host), int(port)


def _env(name: str, default, cast=str):
    """Flag default from CASCADIA_<NAME> when set (command line > env >
    built-in default)."""
    v = os.environ.get("CASCADIA_" + name)
    if v is None or v == "":
        return default
    try:
        return cast(v)
    except ValueError:
        raise SystemExit(f"CASCADIA_{name}={v!r} is not a valid {cast.__name__}")


def _common(p: argparse.ArgumentParser):
    p.add_argument("--model", required=False, default=_env("MODEL", "tiny-llama"),
                   help="shard directory or model preset (random-init weights); "
                        "env CASCADIA_MODEL")
    p.add_argument("--served-model-name", default=_env("SERVED_MODEL_NAME", None))
    p.add_argument("--engine", default=_env("ENGINE", "llama"), choices=sorted(ENGINES))
    p.add_argument("--device", default=_env("DEVICE", "cuda"))
    p.add_argument("--max-model-len", type=int, default=_env("MAX_MODEL_LEN", 8192, int))
    p.add_argument("--max-running", type=int, default=_env("MAX_RUNNING", 64, int))
    p.add_argument("--kv-blocks", type=int, default=_env("KV_BLOCKS", 0, int))
    p.add_argument("--kv-fraction", type=float, default=_env("KV_FRACTION", 0.5, float))
    p.add_argument("--kv-prefix-cache-size", type=int, default=_env("KV_PREFIX_CACHE_SIZE", 0, int),
                   help="blocks kept for prefix reuse (0 disables)")
    p.add_argument("--no-cuda-graph", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--log-level", default="info")
    p.add_argument("--max-concurrent", type=int, default=16)
    p.add_argument("--spec", default=None, choices=["ngram", "draft", "mtp"],
                   help="speculative decoding of greedy requests")
    p.add_argument("--spec-k", type=int, default=4, help="draft tokens per round")
    p.add_argument("--draft-model", default=None, help="draft model preset (--spec draft)")


def _serve(runner, api: str, model_name: str, max_concurrent: int):
    import uvicorn

    from .api.server import ApiConfig, make_app

    host, port = _parse_hostport(api, "0.0.0.0")
    topo = None
    try:
        from .topology import local_gpu_topology

        topo = local_gpu_topology(api_port=port, engines=[model_name])
    except Exception:  # no GPU / no CUDA: serve an empty topology
        topo = None
    app = make_app(runner, ApiConfig(model_name=model_name,
                                     max_concurrent_requests=max_concurrent), topology=topo)
    uvicorn.run(app, host=host, port=port, log_level="warning")


def _builder(args, tp=None):
    from .engine.llm import LLMBuilder
    from .engine.mock import MockBuilder

    if args.engine == "mock":
        return MockBuilder()
    if args.engine == "dsv4":
        from .engine.dsv4 import DSV4Builder

        return DSV4Builder(args.model, device=args.device, max_seq=args.max_model_len)
    if args.engine == "moe":
        from .engine.llm import MoEBuilder

        return MoEBuilder(args.model, device=args.device, kv_blocks=args.kv_blocks,
                          max_running=args.max_running, max_model_len=args.max_model_len,
                          seed=args.seed)
    return LLMBuilder(args.model, device=args.device, kv_blocks=args.kv_blocks,
                      kv_fraction=args.kv_fraction, max_running=args.max_running,
                      max_model_len=args.max_model_len,
                      prefix_cache_blocks=args.kv_prefix_cache_size,
                      use_graph=not args.no_cuda_graph, seed=args.seed, tp=tp,
                      tokenizer_path=args.tokenizer, spec=args.spec, spec_k=args.spec_k,
                      draft_model=args.draft_model)


def validate_run_flags(args) -> None:
    """Reject flag combinations that cannot run, before any model loads
    (the reference's validate_worker_runtime_flags does the same for its
    worker, crates/cascadia-cli/src/lib.rs:1493-1589)."""
    def bad(msg):
        raise SystemExit(f"invalid flags: {msg}")

    if args.max_model_len <= 0 or args.max_running <= 0:
        bad("--max-model-len and --max-running must be positive")
    if args.kv_blocks < 0 or args.kv_prefix_cache_size < 0:
        bad("--kv-blocks and --kv-prefix-cache-size must be >= 0")
    if not 0.0 < args.kv_fraction <= 1.0:
        bad("--kv-fraction must be in (0, 1]")
    if args.kv_blocks and args.kv_prefix_cache_size >= args.kv_blocks:
        bad("--kv-prefix-cache-size must be smaller than --kv-blocks")
    tp, pp, ep = getattr(args, "tp", 1), getattr(args, "pp", 1), getattr(args, "ep", 1)
    if tp < 1 or pp < 1 or ep < 1:
        bad("--tp, --pp and --ep must be >= 1")
    if ep > 1:
        from .models.config import PRESETS

        cfg = PRESETS.get(args.model)
        if tp > 1 or pp > 1:
            bad("--ep serves the whole model per rank group: no --tp / --pp with it")
        if cfg is None or not cfg.is_moe:
            bad("--ep needs a sparse-MoE model preset")
        elif cfg.num_experts % ep:
            bad(f"--ep {ep} must divide the model's {cfg.num_experts} experts")
    if args.engine in ("mock", "dsv4") and (tp > 1 or pp > 1):
        bad(f"--engine {args.engine} serves on one device (expert parallelism runs through "
            "bench.py)")
    if args.spec is not None and pp > 1:
        bad("--spec runs on a single stage (distributed speculative decoding across stages "
            "is --engine spec)")
    if args.spec == "draft" and not args.draft_model:
        bad("--spec draft needs --draft-model")
    if tp > 1 and not os.path.isdir(str(args.model)):
        from .models.config import PRESETS

        cfg = PRESETS.get(args.model)
        if cfg is not None and (cfg.num_heads % tp or cfg.num_kv_heads % tp):
            bad(f"--tp {tp} must divide the model's {cfg.num_heads} heads and "
                f"{cfg.num_kv_heads} KV heads")
    if getattr(args, "prompt_ids", None) and not getattr(args, "prompt", None):
        bad("--prompt-ids needs --prompt (the one-shot prompt mode)")


def cmd_run(args):
    """Serve the model: one process on one device, or, under
    ``torch.distributed.run``, one rank per GPU with ``--tp`` or ``--pp``."""
    from .runtime.runner import Runner
    from .types import PeerLayout, ShardSpec

    validate_run_flags(args)
    _init_logging(args.log_level)
    if (int(os.environ.get("WORLD_SIZE", "1")) > 1 or args.tp > 1 or args.pp > 1
            or args.ep > 1):
        return _run_distributed(args)
    name = args.served_model_name or os.path.basename(str(args.model).rstrip("/"))
    runner = Runner(_builder(args), model_id=name, device=args.device)
    nl = _num_layers(args.model)
    runner.start(PeerLayout(), ShardSpec(name, 0, nl, nl, args.device, True, True))
    try:
        _serve_or_prompt(runner, args, name)
    finally:
        runner.close()


def _run_distributed(args):
    """Ranks of one box (torch.distributed.run): tensor parallel with a
    replicated scheduler (--tp) or an NCCL pipeline (--pp); rank 0 serves the
    API (or, with --prompt, generates once and prints)."""
    import torch.distributed as dist

    from .parallel.serve import (DistContext, ReplicatedEngine, build_pp_stage, build_tp_engine,
                                 follower_loop)
    from .runtime.runner import RelayExit, Runner

    ctx = DistContext.from_env("cuda" if args.device.startswith("cuda") else "cpu",
                               timeout_s=args.dist_timeout)
    if getattr(args, "ep", 1) > 1:
        from .parallel.serve import build_ep_engine

        if args.ep != ctx.world:
            raise SystemExit(f"--ep {args.ep} must equal the {ctx.world} ranks")
        try:
            engine, name = build_ep_engine(args, ctx)
            if ctx.rank != 0:
                follower_loop(engine, ctx.control)
                return
            eng = ReplicatedEngine(engine, ctx.control)
            runner = Runner(None, model_id=name, device=str(ctx.device))
            runner.start_with_engine(eng)
            try:
                _serve_or_prompt(runner, args, name)
            finally:
                runner.close()
        finally:
            if dist.is_initialized():
                dist.destroy_process_group()
        return
    tp = args.tp if args.tp > 1 else (1 if args.pp > 1 else ctx.world)
    pp = args.pp
    if tp * pp != ctx.world:
        raise SystemExit(f"--tp {tp} x --pp {pp} must equal the {ctx.world} ranks")
    code = 0
    try:
        if tp > 1 and pp > 1:
            from .parallel.serve import build_pp_tp_stage

            engine, worker, name, control0 = build_pp_tp_stage(args, ctx, pp, tp)
            if worker is not None:
                r = Runner(None, model_id=name, device=str(ctx.device))
                r.start_with_engine(worker, drive=False)
                code = 1 if r.run_relay_loop() is RelayExit.CONNECTION_FATAL else 0
                return
            if ctx.rank != 0:
                # A replica of the first stage's scheduler; its pipeline
                # head tells its downstream counterparts to stop afterwards.
                follower_loop(engine, control0)
                engine.pipeline.shutdown()
                return
            eng = ReplicatedEngine(engine, control0)
            runner = Runner(None, model_id=name, device=str(ctx.device))
            runner.start_with_engine(eng)
            try:
                _serve_or_prompt(runner, args, name)
            finally:
                runner.close()
                engine.pipeline.shutdown()
        elif pp == 1:
            engine, name = build_tp_engine(args, ctx)
            if ctx.rank != 0:
                follower_loop(engine, ctx.control)
                return
            eng = ReplicatedEngine(engine, ctx.control)
            eng.warmup()
            runner = Runner(None, model_id=name, device=str(ctx.device))
            runner.start_with_engine(eng)
            try:
                _serve_or_prompt(runner, args, name)
            finally:
                runner.close()
        else:
            engine, worker, name = build_pp_stage(args, ctx)
            if worker is not None:
                r = Runner(None, model_id=name, device=str(ctx.device))
                r.start_with_engine(worker, drive=False)
                code = 1 if r.run_relay_loop() is RelayExit.CONNECTION_FATAL else 0
                return
            runner = Runner(None, model_id=name, device=str(ctx.device))
            runner.start_with_engine(engine)
            try:
                _serve_or_prompt(runner, args, name)
            finally:
                engine.pipeline.shutdown()
                runner.close()
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
        if code:
            sys.exit(code)


def _serve_or_prompt(runner, args, name: str):
    if getattr(args, "prompt", None):
        import uuid

        from .types import GenerationTask

        ids = [int(x) for x in args.prompt_ids.split(",")] if args.prompt_ids else None
        s = runner.generate(GenerationTask("cli-" + uuid.uuid4().hex[:8], args.prompt,
                                           max_tokens=args.max_tokens, prompt_ids=ids))
        chunks = list(s)
        print(json.dumps({"text": "".join(c.text for c in chunks),
                          "token_ids": [c.token_id for c in chunks if not c.is_final],
                          "error": chunks[-1].error if chunks else None}), flush=True)
        return
    _serve(runner, args.api, name, args.max_concurrent)


def _num_layers(model: str) -> int:
    if os.path.isfile(os.path.join(model, "manifest.json")):
        import json

        with open(os.path.join(model, "manifest.json")) as f:
            return int(json.load(f).get("num_layers", 1))  # export directory (V4 / MoE)
    if os.path.isdir(model):
        from .shard.format import read_pipeline

        return read_pipeline(model)["num_layers"]
    from .models.config import PRESETS

    return PRESETS[model].num_layers if model in PRESETS else 1


def cmd_worker(args):
    """One pipeline stage.  Rank 0 serves the API (or a stdin prompt loop);
    other ranks run the relay loop and exit non-zero on a dead link so a
    supervisor (systemd Restart=on-failure) rebuilds the stage."""
    from .engine.llm import LLMBuilder
    from .parallel.pp import PipelineHead, PipelineWorker, TcpChannel
    from .runtime.runner import RelayExit, Runner
    from .transport.tcp import TensorLink
    from .types import PeerLayout, ShardPlan, ShardSpec

    _init_logging(args.log_level)
    if args.rank >= args.total:
        raise SystemExit(f"--rank {args.rank} must be < --total {args.total}")
    name = args.served_model_name or os.path.basename(str(args.model).rstrip("/"))
    nl = _num_layers(args.model)
    if args.layer_start is not None and args.layer_end is not None:
        ls, le = args.layer_start, args.layer_end
    else:
        st = ShardPlan.uniform(name, nl, 1, 1, 1, args.total).stages[args.rank]
        ls, le = st.layer_start, st.layer_end
    first, last = args.rank == 0, args.rank == args.total - 1
    shard = ShardSpec(name, ls, le, nl, args.device, first, last)
    builder = LLMBuilder(args.model, device=args.device, kv_blocks=args.kv_blocks or 2048,
                         max_running=args.max_running, max_model_len=args.max_model_len,
                         use_graph=False, seed=args.seed)
    # Links: listen for upstream first (downstream stages start first), then dial.
    up = down = None
    if not first:
        srv = TensorLink.listen(*_parse_hostport(args.listen, "0.0.0.0"))
        logging.info("rank %d listening on %s", args.rank, args.listen)
        up = TensorLink.accept(srv, timeout_s=args.connect_timeout)
    if not last:
        down = TensorLink.connect(*_parse_hostport(args.next), total_s=args.connect_timeout)
    for p in builder.load(shard):
        logging.info("load: %s", p.message)
    model = builder.model
    if not first:
        worker = PipelineWorker(model, TcpChannel(up=up, down=down), is_last=last)
        r = Runner(None, model_id=name, device=args.device)
        r.start_with_engine(worker, drive=False)
        code = r.run_relay_loop()
        logging.info("relay loop exit: %s", code.value)
        sys.exit(1 if code is RelayExit.CONNECTION_FATAL else 0)
    engine = builder.build()
    if not last:
        engine.pipeline = PipelineHead(model, TcpChannel(down=down))
    runner = Runner(None, model_id=name, device=args.device)
    runner.start_with_engine(engine)
    if args.api:
        try:
            _serve(runner, args.api, name, args.max_concurrent)
        finally:
            if engine.pipeline is not None:
                engine.pipeline.shutdown()
            runner.close()
    else:
        from .types import GenerationTask

        import uuid
        for line in sys.stdin:
            if not line.strip():
                continue
            s = runner.generate(GenerationTask("stdin-" + uuid.uuid4().hex[:8], line.strip(),
                                               max_tokens=args.max_tokens))
            print(s.collect(), flush=True)
        if engine.pipeline is not None:
            engine.pipeline.shutdown()
        runner.close()


def cmd_shard(args):
    from .models.config import get_config
    from .shard.format import write_random_shards

    cfg = get_config(args.model)
    if cfg.is_moe:
        # Sparse-MoE directory (manifest + shells + F1 expert bins).
        from .models import llama
        from .models.mla import MLAModel
        from .models.moe import MoEModel
        from .shard.moe_format import write_moe_model

        llama.KEEP_INT4 = True
        cls = MLAModel if cfg.is_mla else MoEModel
        m = cls(cfg, "cpu").init_random(seed=args.seed, gen_device="cpu")
        write_moe_model(m, args.output_dir)
        print(json.dumps({"output_dir": args.output_dir, "format": "sparse-moe int4_bin"}))
        return
    split = [int(x) for x in args.layer_split.split(",")] if args.layer_split else None
    meta = write_random_shards(cfg, args.output_dir, args.num_stages, args.model,
                               seed=args.seed, layer_split=split, device=args.device,
                               tokenizer_dir=args.tokenizer)
    print(json.dumps(meta, indent=1))


def cmd_engines(args):
    for k, v in ENGINES.items():
        print(f"{k:6s} {v}")


def cmd_doctor(args):
    from .utils.doctor import run_doctor

    report = run_doctor()
    print(json.dumps(report, indent=1))
    sys.exit(0 if report.get("ok") else 1)


def cmd_topology(args):
    """Print this host's GPU topology (with --probe: measured NVLink edges)."""
    from .topology import local_gpu_topology

    print(json.dumps(local_gpu_topology(probe=args.probe, probe_mb=args.probe_mb).to_json(),
                     indent=1))


def cmd_place(args):
    from .utils import placement as pl

    layer_us = None
    if args.calibrate:
        layer_us = pl.calibrate_layer_us(args.model, args.batch, args.context)
    res = pl.choose_parallelism(args.model, args.gpus, args.batch, args.context,
                                gpu_mem_gb=args.gpu_mem_gb,
                                hbm_gbs=pl.measured_hbm_gbs(args.peaks), layer_us=layer_us)
    best = res["best"]
    if best is not None and best["ep"] == 1:
        res["launch"] = " ".join(pl.launch_command(args.model, best, args.api))
    print(json.dumps(res, indent=1), flush=True)
    if args.launch:
        if best is None:
            sys.exit("no split fits in memory")
        sys.exit(pl.supervise(pl.launch_command(args.model, best, args.api),
                              max_restarts=args.max_restarts))


def main(argv=None):
    p = argparse.ArgumentParser(prog="cascadia_b200")
    sub = p.add_subparsers(dest="cmd", required=True)

    r = sub.add_parser("run", help="serve the model (one process, or one rank per GPU "
                                   "under torch.distributed.run with --tp / --pp)")
    _common(r)
    r.add_argument("--api", default="0.0.0.0:8000")
    r.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks (torchrun)")
    r.add_argument("--pp", type=int, default=1, help="pipeline stages over NCCL (torchrun)")
    r.add_argument("--ep", type=int, default=1,
                   help="expert-parallel ranks for sparse-MoE models (torchrun)")
    r.add_argument("--dist-timeout", type=float, default=300.0,
                   help="process-group timeout, seconds")
    r.add_argument("--prompt", default=None,
                   help="generate once for this prompt, print JSON, exit (no API)")
    r.add_argument("--prompt-ids", default=None, help="comma-separated token ids for --prompt")
    r.add_argument("--max-tokens", type=int, default=64)
    r.set_defaults(fn=cmd_run)

    w = sub.add_parser("worker", help="run one pipeline stage")
    _common(w)
    w.add_argument("--rank", type=int, required=True)
    w.add_argument("--total", type=int, required=True)
    w.add_argument("--layer-start", type=int, default=None)
    w.add_argument("--layer-end", type=int, default=None)
    w.add_argument("--listen", default=None, help="host:port for the upstream stage")
    w.add_argument("--next", default=None, help="host:port of the downstream stage")
    w.add_argument("--api", default=None, help="rank 0: serve the OpenAI API here")
    w.add_argument("--connect-timeout", type=float, default=30.0)
    w.add_argument("--max-tokens", type=int, default=256)
    w.set_defaults(fn=cmd_worker)

    s = sub.add_parser("shard", help="write the per-stage INT4 shard layout")
    s.add_argument("--model", required=True, help="model preset (random-init weights)")
    s.add_argument("--output-dir", required=True)
    s.add_argument("--num-stages", type=int, default=1)
    s.add_argument("--layer-split", default=None, help="comma-separated layers per stage")
    s.add_argument("--seed", type=int, default=0)
    s.add_argument("--device", default="cpu")
    s.add_argument("--tokenizer", default=None)
    s.set_defaults(fn=cmd_shard)

    sub.add_parser("engines", help="list engines").set_defaults(fn=cmd_engines)
    sub.add_parser("doctor", help="check CUDA / NCCL / NVLink").set_defaults(fn=cmd_doctor)
    tp_ = sub.add_parser("topology", help="GPU nodes and measured NVLink links (JSON)")
    tp_.add_argument("--probe", action="store_true", help="measure peer bandwidth / latency")
    tp_.add_argument("--probe-mb", type=int, default=256)
    tp_.set_defaults(fn=cmd_topology)

    pl = sub.add_parser("place", help="choose a PP x TP x EP split")
    pl.add_argument("--model", required=True)
    pl.add_argument("--gpus", type=int, default=8)
    pl.add_argument("--batch", type=int, default=64)
    pl.add_argument("--context", type=int, default=4096)
    pl.add_argument("--gpu-mem-gb", type=float, default=180.0)
    pl.add_argument("--peaks", default=None, help="measured peaks JSON (hbm_gbs)")
    pl.add_argument("--calibrate", action="store_true",
                    help="time two layers of the model on this GPU and use the measured cost")
    pl.add_argument("--launch", action="store_true",
                    help="serve the chosen split under a restart-on-crash supervisor")
    pl.add_argument("--api", default="0.0.0.0:8000")
    pl.add_argument("--max-restarts", type=int, default=3)
    pl.set_defaults(fn=cmd_place)

    args = p.parse_args(argv)
    signal.signal(signal.SIGTERM, lambda *a: sys.exit(0))
    args.fn(args)


if __name__ == "__main__":
    main()
