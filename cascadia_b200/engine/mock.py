"""Deterministic word-echo engine for tests of the runner, API and CLI.

Behaviour of crates/cascadia-engine-mock/src/lib.rs:13-120: one prompt word
per ``step()``, ``stop`` when the words run out, ``length`` when
``max_tokens`` hits first, ``__engine_error__`` in the prompt yields an error
chunk, and ``fail_next_step`` makes the next step raise.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Tuple

from ..types import Chunk, FinishReason, GenerationTask, LoadProgress, PeerLayout, ShardSpec
from .base import Backend, Builder, Engine, NotLoaded, StepOutput


class MockEngine(Engine):
    def __init__(self):
        self.pending: List[Tuple[GenerationTask, int]] = []
        self._fail_next: Optional[str] = None

    def fail_next_step(self, msg: str) -> None:
        self._fail_next = msg

    def cancel(self, task_id: str) -> None:
        self.pending = [(t, e) for (t, e) in self.pending if t.task_id != task_id]

    def submit(self, task: GenerationTask) -> None:
        if any(t.task_id == task.task_id for t, _ in self.pending):
            return
        self.pending.append((task, 0))

    def has_work(self) -> bool:
        return bool(self.pending)

    def step(self) -> StepOutput:
        if self._fail_next is not None:
            msg, self._fail_next = self._fail_next, None
            raise Backend(msg)
        if not self.pending:
            return []
        task, emitted = self.pending.pop(0)
        if "__engine_error__" in task.prompt:
            return [(task.task_id, Chunk.error_chunk(task.task_id, "mock injected engine failure"))]
        cap = max(task.max_tokens, 1)
        words = task.prompt.split()
        if emitted >= cap or emitted >= len(words):
            reason = FinishReason.STOP if emitted >= len(words) else FinishReason.LENGTH
            return [(task.task_id,
                     Chunk.final_marker(task.task_id, "").with_finish_reason(reason))]
        chunk = Chunk.token(task.task_id, emitted, words[emitted] + " ")
        self.pending.append((task, emitted + 1))
        return [(task.task_id, chunk)]


class MockBuilder(Builder):
    def __init__(self):
        self.connected = False
        self.loaded = False

    def connect(self, peers: PeerLayout) -> None:
        self.connected = True

    def load(self, shard: ShardSpec) -> Iterable[LoadProgress]:
        self.loaded = True
        return [LoadProgress.msg("mock load: starting"), LoadProgress.done()]

    def build(self) -> Engine:
        if not self.loaded:
            raise NotLoaded()
        return MockEngine()
