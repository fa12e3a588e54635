"""Stage runner: builder lifecycle, one engine loop, per-task chunk streams.

Semantics follow crates/cascadia-runner/src/lib.rs:
* ``start`` runs ``configure_listen -> connect -> load -> build -> warmup``
  and records the load / warmup gauges (:381-425);
* ``submit`` registers the task's stream before handing it to the engine; a
  failed submit unregisters it and re-raises (API maps it to a status code);
* ``cancel`` is deferred while the engine is busy and applied before the next
  step; cancelled ids are tombstoned (bounded) so a late submit is dropped
  (:443-510);
* one driver thread steps the engine while any stream or engine work exists
  (the GPU engine batches every active task into one iteration); chunks are
  routed to their task's stream, engine-wide errors fail every stream, a
  task-attributed error fails only that task;
* a bounded no-progress guard ends streams the engine forgot
  (MAX_CONSECUTIVE_EMPTY_STEPS, :30);
* ``run_relay_loop`` (ranks > 0) steps until a connection-fatal error
  (``RelayExit.CONNECTION_FATAL``, supervisor restarts the stage) or close
  (``RelayExit.SLOT_EMPTY``), backing off 200 ms after non-fatal errors (:618-663);
* ``close`` marks teardown first, so in-flight generations end with
  ``finish_reason="teardown"`` rather than counting as client cancels.
"""
from __future__ import annotations

import asyncio
import collections
import enum
import logging
import queue
import threading
import time
from typing import AsyncIterator, Deque, Dict, Iterator, Optional, Set

from .. import metrics
from ..engine.base import Builder, Engine, EngineError, ShutdownRequested, classify_exception
from ..types import Chunk, FinishReason, GenerationTask, PeerLayout, ShardSpec, TaskId

log = logging.getLogger("cascadia.runner")

MAX_CONSECUTIVE_EMPTY_STEPS = 3
RELAY_ERR_BACKOFF_S = 0.2
MAX_TOMBSTONES = 4096
_END = object()


class RelayExit(enum.Enum):
    SLOT_EMPTY = "slot_empty"
    CONNECTION_FATAL = "connection_fatal"


class ChunkStream:
    """Chunks of one task, consumable synchronously or with ``async for``."""

    def __init__(self, runner: "Runner", task: GenerationTask,
                 loop: Optional[asyncio.AbstractEventLoop]):
        self.runner = runner
        self.task_id = task.task_id
        self.submitted = time.monotonic()
        self.first_token_at: Optional[float] = None
        self.last_token_at: Optional[float] = None
        self.done = False
        self.outcome: Optional[str] = None
        self._loop = loop
        self._aq: Optional[asyncio.Queue] = asyncio.Queue() if loop is not None else None
        self._q: "queue.Queue" = queue.Queue()

    # producer side (driver thread)
    def _put(self, item):
        if self._aq is not None:
            try:
                self._loop.call_soon_threadsafe(self._aq.put_nowait, item)
            except RuntimeError:  # loop closed: consumer is gone
                pass
        else:
            self._q.put(item)

    # consumer side
    def _account(self, c: Chunk):
        now = time.monotonic()
        model = self.runner.model_id
        n = c.token_count()
        if n > 0 and c.error is None:
            if self.first_token_at is None:
                self.first_token_at = now
                metrics.TTFT.labels(model=model).observe(now - self.submitted)
            elif self.last_token_at is not None:
                metrics.INTER_TOKEN.labels(model=model).observe(now - self.last_token_at)
            self.last_token_at = now
            metrics.TOKENS_GENERATED.labels(model=model).inc(n)
        if c.prompt_tokens:
            metrics.TOKENS_PROMPT.labels(model=model).inc(c.prompt_tokens)
        if c.is_final:
            if c.error is not None:
                outcome = "teardown" if self.runner.closing else "error"
                if outcome == "error":
                    metrics.TASKS_FAILED.labels(model=model).inc()
            elif c.finish_reason is FinishReason.CANCELLED:
                outcome = "teardown" if self.runner.closing else "cancelled"
                if outcome == "cancelled":
                    metrics.TASKS_CANCELLED.labels(model=model).inc()
            else:
                outcome = (c.finish_reason or FinishReason.STOP).as_openai_str()
            self.outcome = outcome
            metrics.GEN_DURATION.labels(model=model, finish_reason=outcome).observe(
                now - self.submitted)

    def __iter__(self) -> Iterator[Chunk]:
        while True:
            item = self._q.get()
            if item is _END:
                return
            self._account(item)
            yield item
            if item.is_final:
                return

    def __aiter__(self) -> AsyncIterator[Chunk]:
        return self._agen()

    async def _agen(self):
        try:
            while True:
                item = await self._aq.get()
                if item is _END:
                    return
                self._account(item)
                yield item
                if item.is_final:
                    return
        finally:
            if not self.done:
                # Consumer dropped mid-generation (client disconnect).
                self.runner.cancel(self.task_id)

    def collect(self) -> str:
        return "".join(c.text for c in self)


class Runner:
    def __init__(self, builder: Builder, model_id: str = "model", device: str = "cuda"):
        self.builder: Optional[Builder] = builder
        self.engine: Optional[Engine] = None
        self.model_id = model_id
        self.device = device
        self.closing = False
        self._lock = threading.RLock()  # engine lock
        self._cv = threading.Condition()
        self._streams: Dict[TaskId, ChunkStream] = {}
        self._deferred_cancels: Deque[TaskId] = collections.deque()
        self._tombstones: Deque[TaskId] = collections.deque()
        self._tomb_set: Set[TaskId] = set()
        self._driver: Optional[threading.Thread] = None
        self._wake = threading.Event()
        self.load_seconds = 0.0
        self.warmup_seconds = 0.0

    # ----------------------------------------------------------- lifecycle
    def start(self, peers: PeerLayout, shard: ShardSpec, listen: Optional[tuple] = None,
              drive: bool = True) -> None:
        b = self.builder
        if listen is not None:
            b.configure_listen(*listen)
        b.connect(peers)
        t0 = time.monotonic()
        for p in b.load(shard):
            log.info("load: %s", p.message)
        self.engine = b.build()
        self.load_seconds = time.monotonic() - t0
        metrics.LOAD_SECONDS.labels(model=self.model_id, device=self.device).set(self.load_seconds)
        t1 = time.monotonic()
        self.engine.warmup()
        self.warmup_seconds = time.monotonic() - t1
        metrics.WARMUP_SECONDS.labels(model=self.model_id, device=self.device).set(
            self.warmup_seconds)
        if drive:
            self._driver = threading.Thread(target=self._drive, name="engine-driver", daemon=True)
            self._driver.start()

    def start_with_engine(self, engine: Engine, drive: bool = True) -> None:
        self.engine = engine
        if drive:
            self._driver = threading.Thread(target=self._drive, name="engine-driver", daemon=True)
            self._driver.start()

    # ----------------------------------------------------------- requests
    def submit(self, task: GenerationTask,
               loop: Optional[asyncio.AbstractEventLoop] = None) -> ChunkStream:
        if self.closing:
            raise EngineError("runner closing")
        if self.engine is None:
            from ..engine.base import NotLoaded
            raise NotLoaded()
        stream = ChunkStream(self, task, loop)
        with self._cv:
            self._streams[task.task_id] = stream
        try:
            with self._lock:
                self._apply_cancels()
                if task.task_id in self._tomb_set:
                    stream.done = True
                    stream._put(Chunk.final_marker(task.task_id).with_finish_reason(
                        FinishReason.CANCELLED))
                    return stream
                self.engine.submit(task)
        except BaseException:
            with self._cv:
                self._streams.pop(task.task_id, None)
            raise
        metrics.INFLIGHT.inc()
        self._wake.set()
        return stream

    def generate(self, task: GenerationTask) -> ChunkStream:
        return self.submit(task)

    async def generate_async(self, task: GenerationTask) -> ChunkStream:
        loop = asyncio.get_running_loop()
        return await loop.run_in_executor(None, lambda: self.submit(task, loop))

    def cancel(self, task_id: TaskId) -> None:
        if task_id not in self._tomb_set:
            self._tombstones.append(task_id)
            self._tomb_set.add(task_id)
            while len(self._tombstones) > MAX_TOMBSTONES:
                self._tomb_set.discard(self._tombstones.popleft())
        if self._lock.acquire(blocking=False):
            try:
                self._cancel_now(task_id)
            finally:
                self._lock.release()
        else:
            if len(self._deferred_cancels) < MAX_TOMBSTONES:
                self._deferred_cancels.append(task_id)
        self._wake.set()

    def _cancel_now(self, task_id: TaskId):
        if self.engine is not None:
            try:
                self.engine.cancel(task_id)
            except Exception as e:  # cancel must never take the runner down
                log.warning("engine.cancel(%s) failed: %s", task_id, e)
        self._finish(task_id, Chunk.final_marker(task_id).with_finish_reason(
            FinishReason.CANCELLED))

    def _apply_cancels(self):
        while self._deferred_cancels:
            self._cancel_now(self._deferred_cancels.popleft())

    def _finish(self, task_id: TaskId, chunk: Chunk):
        with self._cv:
            s = self._streams.pop(task_id, None)
        if s is not None and not s.done:
            s.done = True
            s._put(chunk)
            metrics.INFLIGHT.dec()

    # ----------------------------------------------------------- driver
    def _route(self, out):
        for task_id, chunk in out:
            with self._cv:
                s = self._streams.get(task_id)
            if s is None:
                continue  # cancelled / unknown: drop
            if chunk.is_final:
                self._finish(task_id, chunk)
            else:
                s._put(chunk)

    def step_once(self) -> int:
        """One engine iteration; returns the number of chunks routed."""
        with self._lock:
            self._apply_cancels()
            try:
                out = self.engine.step()
            except BaseException as e:  # noqa: BLE001
                err = classify_exception(e)
                tid = err.task_id
                if tid is not None:
                    self._finish(tid, Chunk.error_chunk(tid, str(err)))
                else:
                    with self._cv:
                        ids = list(self._streams)
                    for t in ids:
                        self._finish(t, Chunk.error_chunk(t, str(err)))
                raise err
        self._route(out)
        return len(out)

    def _drive(self):
        empty = 0
        while not self.closing:
            with self._cv:
                active = bool(self._streams)
            if not active and not (self.engine and self.engine.has_work()):
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            try:
                n = self.step_once()
            except EngineError as e:
                log.warning("engine step failed: %s", e)
                time.sleep(0.01)
                continue
            if n == 0 and not self.engine.has_work():
                empty += 1
                if empty >= MAX_CONSECUTIVE_EMPTY_STEPS:
                    with self._cv:
                        ids = list(self._streams)
                    for t in ids:
                        self._finish(t, Chunk.error_chunk(t, "engine made no progress"))
                    empty = 0
            else:
                empty = 0

    # ----------------------------------------------------------- relay
    def run_relay_loop(self) -> RelayExit:
        """Worker ranks (> 0): step until a connection-fatal error or close."""
        while not self.closing:
            if self.engine is None:
                return RelayExit.SLOT_EMPTY
            try:
                with self._lock:
                    self.engine.step()
            except ShutdownRequested:
                return RelayExit.SLOT_EMPTY
            except BaseException as e:  # noqa: BLE001
                err = classify_exception(e)
                if err.is_connection_fatal():
                    log.error("relay: connection-fatal: %s", err)
                    return RelayExit.CONNECTION_FATAL
                log.warning("relay: step failed: %s", err)
                time.sleep(RELAY_ERR_BACKOFF_S)
        return RelayExit.SLOT_EMPTY

    def close(self):
        self.closing = True
        self._wake.set()
        if self._driver is not None:
            self._driver.join(timeout=10)
        with self._cv:
            ids = list(self._streams)
        for t in ids:
            self._finish(t, Chunk.error_chunk(t, "server shutting down"))
        with self._lock:
            if self.engine is not None:
                self.engine.close()
                self.engine = None
            if self.builder is not None:
                self.builder.close()
