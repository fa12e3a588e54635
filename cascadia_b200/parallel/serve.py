"""Serving on several GPUs of one box under ``torch.distributed.run``.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m cascadia_b200 run --tp N --model llama-3.1-8b --api 0.0.0.0:8000
    python -m torch.distributed.run --nproc-per-node 2 ... -m cascadia_b200 run --pp 2 ...

Tensor parallelism (``--tp N``, one rank per GPU, every rank holds 1/N of
every layer): the engine is REPLICATED.  Every rank runs the same
:class:`~cascadia_b200.engine.llm.LLMEngine` over its shard; rank 0 also runs
the runner and the OpenAI API.  Before each iteration rank 0 broadcasts the
requests admitted and cancelled since the previous one (a small message on a
gloo group), and every rank then calls ``step()``.  The scheduler is
deterministic, so all ranks admit the same sequences, allocate the same KV
blocks and launch the same kernels (and replay the same CUDA graphs) in the
same order; the collectives inside the forward (fused peer-memory
all-reduce, NCCL for prefill, the vocab-parallel argmax merge) line up by
construction.  Only rank 0 emits chunks.  This replaces the reference's
per-stage TCP relay for ranks of one box (crates/cascadia-cli/src/lib.rs:
1592-2031 ``worker``; crates/cascadia-engine-openvino/src/runtime.rs:774
``send_hidden_frames``).

Pipeline parallelism (``--pp N``): rank 0 owns the scheduler and the first
layers; the other ranks are :class:`~cascadia_b200.parallel.pp.PipelineWorker`
stages that receive the hidden rows and the batch meta over NCCL p2p
(:class:`~cascadia_b200.parallel.pp.NcclChannel`) instead of TCP.

Both (``--pp P --tp T``): P stages of T tensor-parallel ranks each
(:func:`build_pp_tp_stage`).

Failure handling: the device status word that a kernel's bounded wait sets
is combined over the TP ranks (max) before the engine decides to fail a
batch, so every rank drops the same sequences.  A rank that dies makes the
next collective fail within the process group's timeout on the others.
"""
from __future__ import annotations

import datetime
import logging
import os
from typing import List, Optional

import torch
import torch.distributed as dist

from ..engine.base import Engine, StepOutput
from ..types import GenerationTask

log = logging.getLogger("cascadia.serve")

_OP_STEP = "step"
_OP_STOP = "stop"


class DistContext:
    """Ranks of this job: NCCL default group (device collectives) and a gloo
    group for the engine's control messages (host objects)."""

    def __init__(self, rank: int, world: int, local_rank: int, device: torch.device,
                 control) -> None:
        self.rank, self.world, self.local_rank = rank, world, local_rank
        self.device = device
        self.control = control

    @staticmethod
    def from_env(device_type: str = "cuda", timeout_s: float = 300.0) -> "DistContext":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        if device_type == "cuda":
            torch.cuda.set_device(local)
            dev = torch.device("cuda", local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                    device_id=dev)
        else:
            dev = torch.device("cpu")
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
        control = dist.new_group(backend="gloo",
                                 timeout=datetime.timedelta(seconds=timeout_s))
        return DistContext(rank, world, local, dev, control)


class ReplicatedEngine(Engine):
    """Rank 0's engine when every TP rank runs a replica of the scheduler.

    ``submit`` / ``cancel`` apply locally first (a rejected submit is never
    replicated) and queue an event; ``step`` broadcasts the queued events
    and steps the local replica.  The followers (:func:`follower_loop`)
    apply the same events in the same order before the same ``step``."""

    def __init__(self, inner: Engine, control_group) -> None:
        self.inner = inner
        self.group = control_group
        self._events: List[tuple] = []
        self._stopped = False

    def warmup(self) -> None:
        # The warm-up request runs through the replicated path too, so every
        # rank captures the same graphs.
        t = GenerationTask("__warmup__", "warm", max_tokens=2, prompt_ids=[1, 2, 3, 4])
        self.submit(t)
        for _ in range(8):
            out = self.step()
            if any(c.is_final for _, c in out):
                break
        self.cancel("__warmup__")
        self._broadcast()  # the cancel reaches the followers now

    def submit(self, task: GenerationTask) -> None:
        self.inner.submit(task)
        self._events.append(("submit", task.to_dict()))

    def cancel(self, task_id: str) -> None:
        self.inner.cancel(task_id)
        self._events.append(("cancel", task_id))

    def has_work(self) -> bool:
        return self.inner.has_work()

    def _broadcast(self, op: str = _OP_STEP) -> None:
        msg = [(op, self._events)]
        self._events = []
        dist.broadcast_object_list(msg, src=0, group=self.group)

    def step(self) -> StepOutput:
        self._broadcast()
        return self.inner.step()

    def close(self) -> None:
        if not self._stopped:
            self._stopped = True
            try:
                self._broadcast(_OP_STOP)
            except Exception as e:  # noqa: BLE001 - peers may be gone already
                log.warning("stop broadcast failed: %s", e)
        self.inner.close()


def follower_loop(engine: Engine, control_group) -> int:
    """Ranks > 0 of a replicated TP engine: apply rank 0's events and step
    in lockstep until rank 0 says stop.  Returns the number of steps run."""
    steps = 0
    while True:
        msg = [None]
        dist.broadcast_object_list(msg, src=0, group=control_group)
        op, events = msg[0]
        for kind, payload in events:
            if kind == "submit":
                engine.submit(GenerationTask.from_dict(payload))
            else:
                engine.cancel(payload)
        if op == _OP_STOP:
            engine.close()
            return steps
        engine.step()  # outputs are rank 0's to emit
        steps += 1


def build_tp_engine(args, ctx: DistContext):
    """The LLM engine of this TP rank (model shard + fused TP collectives)."""
    from ..engine.llm import LLMBuilder
    from ..models.llama import TPGroup
    from ..types import PeerLayout, ShardSpec

    tp = TPGroup(ctx.rank, ctx.world, dist.group.WORLD)
    from ..models.config import get_config

    name = args.served_model_name or os.path.basename(str(args.model).rstrip("/"))
    builder = LLMBuilder(args.model, device=str(ctx.device), kv_blocks=args.kv_blocks,
                         kv_fraction=args.kv_fraction, max_running=args.max_running,
                         max_model_len=args.max_model_len,
                         prefix_cache_blocks=args.kv_prefix_cache_size,
                         use_graph=not args.no_cuda_graph, seed=args.seed, tp=tp,
                         tokenizer_path=args.tokenizer, spec=args.spec, spec_k=args.spec_k,
                         draft_model=args.draft_model)
    if ctx.device.type == "cuda" and ctx.world > 1:
        from .tp import FusedTP

        cfg = get_config(args.model) if not os.path.isdir(args.model) else None
        hidden = cfg.hidden_size if cfg is not None else None
        if hidden is not None:
            tp.fused = FusedTP(dist.group.WORLD, ctx.rank, ctx.world, ctx.device, hidden,
                               max(64, args.max_running))
    builder.connect(PeerLayout())
    from .. import models  # noqa: F401
    nl = _num_layers(args.model)
    for p in builder.load(ShardSpec(name, 0, nl, nl, str(ctx.device), True, True)):
        log.info("rank %d load: %s", ctx.rank, p.message)
    return builder.build(), name


def build_pp_stage(args, ctx: DistContext):
    """This rank's pipeline stage: (engine, None) on rank 0, (None, worker)
    elsewhere; stages exchange hidden rows over NCCL p2p."""
    from ..engine.llm import LLMBuilder
    from ..models.config import get_config
    from ..types import ShardPlan, ShardSpec
    from .pp import NcclChannel, PipelineHead, PipelineWorker

    name = args.served_model_name or os.path.basename(str(args.model).rstrip("/"))
    nl = _num_layers(args.model)
    st = ShardPlan.uniform(name, nl, 1, 1, 1, ctx.world).stages[ctx.rank]
    first, last = ctx.rank == 0, ctx.rank == ctx.world - 1
    shard = ShardSpec(name, st.layer_start, st.layer_end, nl, str(ctx.device), first, last)
    # The first stage owns the scheduler and the prefix cache.  Every stage
    # addresses the same block ids (tables and slots travel in the batch
    # meta), so a cached prefix's K/V rows stay valid in every stage's pool
    # as long as the first stage keeps the blocks referenced: no
    # cache / restore frames between stages are needed.
    builder = LLMBuilder(args.model, device=str(ctx.device), kv_blocks=args.kv_blocks or 4096,
                         max_running=args.max_running, max_model_len=args.max_model_len,
                         use_graph=False, seed=args.seed, tokenizer_path=args.tokenizer,
                         prefix_cache_blocks=args.kv_prefix_cache_size if first else 0)
    for p in builder.load(shard):
        log.info("rank %d load: %s", ctx.rank, p.message)
    model = builder.model
    # Rows a stage receives: the hidden row, widened by the families that
    # ship more per token (Gemma-4's per-layer inputs and shared K/V rows).
    ch = NcclChannel(ctx.rank, ctx.world, ctx.device, model.payload_in_width)
    if not first:
        return None, PipelineWorker(model, ch, is_last=last), name
    engine = builder.build()
    engine.pipeline = PipelineHead(model, ch)
    return engine, None, name


def build_ep_engine(args, ctx: DistContext):
    """Expert-parallel serving of a sparse-MoE model (``--ep N``): every rank
    holds 1/N of each layer's routed experts (the model no longer needs to
    fit one GPU) and a replica of everything else.  The scheduler is
    replicated as with ``--tp`` (rank 0's events broadcast, every rank steps
    the same batch), so each rank's MoE layers dispatch the same token rows
    to the experts' owners and get back the combined rows.  The expert work
    is not divided (every rank sends every row), the memory is."""
    from ..engine.llm import LLMBuilder
    from ..models.config import get_config
    from ..types import PeerLayout, ShardSpec
    from .ep import ExpertParallel

    cfg = get_config(args.model)
    name = args.served_model_name or os.path.basename(str(args.model).rstrip("/"))
    max_tokens = 2048
    ep = ExpertParallel(dist.group.WORLD, ctx.rank, ctx.world, ctx.device, cfg.num_experts,
                        cfg.hidden_size, cfg.num_experts_per_tok, max_tokens=max_tokens)
    builder = LLMBuilder(args.model, device=str(ctx.device), kv_blocks=args.kv_blocks or 4096,
                         max_running=min(args.max_running, max_tokens),
                         max_model_len=args.max_model_len, use_graph=False, seed=args.seed,
                         tokenizer_path=args.tokenizer, ep=ep, max_prefill_tokens=max_tokens)
    builder.connect(PeerLayout())
    nl = cfg.num_layers
    for p in builder.load(ShardSpec(name, 0, nl, nl, str(ctx.device), True, True)):
        log.info("rank %d load: %s", ctx.rank, p.message)
    return builder.build(), name


def build_pp_tp_stage(args, ctx: DistContext, pp: int, tp: int):
    """Pipeline stages of tensor-parallel groups (``--pp P --tp T``, P * T
    ranks): global rank g is TP rank g % T of stage g // T.  Each stage's T
    ranks hold 1/T of that stage's layers and run their all-reduces in the
    stage's own group; TP rank t of stage s exchanges hidden rows with TP
    rank t of the neighbouring stages (every TP rank of a stage holds the
    full hidden rows after its all-reduce).  The first stage's T ranks run
    replicas of the scheduler (events broadcast on the first stage's gloo
    group, as with ``--tp``); the other stages run relay workers.

    Returns (engine, worker, name, control): the engine on the first
    stage's ranks, the worker elsewhere; `control` is the first stage's
    gloo group (None off the first stage)."""
    from ..engine.llm import LLMBuilder
    from ..models.llama import TPGroup
    from ..types import ShardPlan, ShardSpec
    from .pp import NcclChannel, PipelineHead, PipelineWorker

    stage, t = ctx.rank // tp, ctx.rank % tp
    timeout = datetime.timedelta(seconds=max(60.0, float(getattr(args, "dist_timeout", 300))))
    # Every rank creates every group, in the same order.
    stage_groups = [dist.new_group(ranks=list(range(s * tp, (s + 1) * tp)), timeout=timeout)
                    for s in range(pp)]
    control0 = dist.new_group(ranks=list(range(tp)), backend="gloo", timeout=timeout)
    group = stage_groups[stage]
    name = args.served_model_name or os.path.basename(str(args.model).rstrip("/"))
    nl = _num_layers(args.model)
    st = ShardPlan.uniform(name, nl, 1, 1, 1, pp).stages[stage]
    first, last = stage == 0, stage == pp - 1
    shard = ShardSpec(name, st.layer_start, st.layer_end, nl, str(ctx.device), first, last)
    tpg = TPGroup(t, tp, group)
    # A fixed pool size on every rank: later stages write the blocks the
    # first stage allocates.
    builder = LLMBuilder(args.model, device=str(ctx.device), kv_blocks=args.kv_blocks or 4096,
                         max_running=args.max_running, max_model_len=args.max_model_len,
                         use_graph=False, seed=args.seed, tp=tpg,
                         tokenizer_path=args.tokenizer,
                         prefix_cache_blocks=args.kv_prefix_cache_size if first else 0)
    if ctx.device.type == "cuda":
        from ..models.config import get_config
        from .tp import FusedTP

        if not os.path.isdir(args.model):
            tpg.fused = FusedTP(group, t, tp, ctx.device, get_config(args.model).hidden_size,
                                max(64, args.max_running))
    for p in builder.load(shard):
        log.info("rank %d (stage %d, tp %d) load: %s", ctx.rank, stage, t, p.message)
    model = builder.model
    ch = NcclChannel(ctx.rank, ctx.world, ctx.device, model.payload_in_width)
    ch.prev = ctx.rank - tp if not first else None
    ch.next = ctx.rank + tp if not last else None
    if not first:
        return None, PipelineWorker(model, ch, is_last=last), name, None
    engine = builder.build()
    engine.pipeline = PipelineHead(model, ch)
    return engine, None, name, control0


def _num_layers(model: str) -> int:
    if os.path.isdir(model):
        from ..shard.format import read_pipeline

        return read_pipeline(model)["num_layers"]
    from ..models.config import PRESETS

    return PRESETS[model].num_layers if model in PRESETS else 1
