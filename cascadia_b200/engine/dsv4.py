"""Serving engine for DeepSeek-V4 exports (``models.dsv4``).

The V4 model keeps per-sequence state that does not fit the paged-KV
engine: a raw-latent ring per layer, the compressors' running windows and
the indexer's compressed cache.  This engine therefore runs one sequence
at a time in arrival order (the reference's V4 shell is b = 1 as well,
crates/cascadia-engine-sparse-moe/src/dsv4/model.rs): a step either
prefills the next queued request (emitting its first token) or decodes one
token of the active one.  Greedy decoding; cancellation drops a queued
request or ends the active one; prompts longer than the model's cache
(`max_seq`) fail with an error chunk instead of overrunning it.
"""
from __future__ import annotations

import os
from collections import deque
from typing import Deque, Iterable, List, Optional

import torch

from ..types import Chunk, FinishReason, GenerationTask, LoadProgress, PeerLayout, ShardSpec
from .base import Builder, Engine, NotLoaded, StepOutput


class DSV4Engine(Engine):
    def __init__(self, model, tokenizer=None):
        from ..api.templates import ByteTokenizer

        self.m = model
        cfg = model.cfg
        self.tok = tokenizer or ByteTokenizer(vocab_size=cfg.vocab, eos_id=(cfg.eos_ids or [0])[0])
        self.eos = set(cfg.eos_ids)
        self.queue: Deque[GenerationTask] = deque()
        self.active: Optional[GenerationTask] = None
        self.pos = 0          # tokens of the active sequence in the model state
        self.out: List[int] = []
        self.prompt_len = 0

    def submit(self, task: GenerationTask) -> None:
        self.queue.append(task)

    def has_work(self) -> bool:
        return self.active is not None or bool(self.queue)

    def cancel(self, task_id: str) -> None:
        self.queue = deque(t for t in self.queue if t.task_id != task_id)
        if self.active is not None and self.active.task_id == task_id:
            self.active = None

    def _ids(self, task: GenerationTask) -> List[int]:
        if task.prompt_ids:
            return [int(t) for t in task.prompt_ids]
        v = self.m.cfg.vocab
        return [min(t, v - 1) for t in self.tok.encode(task.prompt)]

    def _emit(self, tok: int) -> StepOutput:
        t = self.active
        self.out.append(tok)
        text = "" if tok in self.eos else self.tok.decode([tok])
        res: StepOutput = []
        finish = None
        if tok in self.eos:
            finish = FinishReason.STOP
        elif len(self.out) >= max(1, t.max_tokens) or self.pos + 1 >= self.m.max_seq:
            finish = FinishReason.LENGTH
        if tok not in self.eos:
            res.append((t.task_id, Chunk.token(t.task_id, tok, text).with_n_tokens(1)))
        if finish is not None:
            res.append((t.task_id, Chunk.final_marker(t.task_id, "").with_finish_reason(finish)
                        .with_prompt_tokens(self.prompt_len)))
            self.active = None
        return res

    def step(self) -> StepOutput:
        with torch.inference_mode():
            if self.active is None:
                if not self.queue:
                    return []
                task = self.queue.popleft()
                ids = self._ids(task)
                if not ids or len(ids) >= self.m.max_seq:
                    return [(task.task_id, Chunk.error_chunk(
                        task.task_id, f"prompt of {len(ids)} tokens does not fit max_seq "
                                      f"{self.m.max_seq}"))]
                self.active, self.out, self.prompt_len = task, [], len(ids)
                logits = self.m.prefill(ids)
                self.pos = len(ids)
                return self._emit(int(torch.argmax(logits)))
            logits = self.m.decode(self.out[-1], self.pos)
            self.pos += 1
            return self._emit(int(torch.argmax(logits)))


class DSV4Builder(Builder):
    """Loads a V4 export directory (manifest.json, embed / head, shells,
    int4_bin experts)."""

    def __init__(self, path: str, device: str = "cuda", max_seq: int = 4096):
        self.path, self.device, self.max_seq = path, device, max_seq
        self.model = None

    def connect(self, peers: PeerLayout) -> None:
        pass

    def load(self, shard: ShardSpec) -> Iterable[LoadProgress]:
        from ..models.dsv4 import DSV4Model

        if not os.path.isfile(os.path.join(self.path, "manifest.json")):
            raise FileNotFoundError(f"no manifest.json in {self.path}")
        yield LoadProgress.msg(f"loading DeepSeek-V4 export {self.path}")
        self.model = DSV4Model(self.path, self.device, max_seq=self.max_seq)
        yield LoadProgress.done()

    def build(self) -> Engine:
        if self.model is None:
            raise NotLoaded()
        return DSV4Engine(self.model)
