"""Engine / Builder plugin seam and the engine error taxonomy.

Mirrors the two-trait lifecycle of crates/cascadia-engine/src/lib.rs:186-255:
``Builder.configure_listen -> connect(peers) -> load(shard) -> build()`` and
``Engine.warmup / submit / step / cancel / close``.  ``step()`` advances at
most one scheduler iteration and returns ``(task_id, Chunk)`` pairs.

``EngineError.is_connection_fatal`` restates the classifier of
crates/cascadia-engine/src/lib.rs:131-173: a dead link ends the relay loop,
a per-batch abort never does.
"""
from __future__ import annotations

import abc
import errno
from typing import Iterable, List, Optional, Tuple

from ..types import Chunk, GenerationTask, LoadProgress, PeerLayout, ShardSpec, TaskId


class EngineError(Exception):
    """Base engine error; subclasses mirror the reference's variants."""

    def is_connection_fatal(self) -> bool:
        return False

    @property
    def task_id(self) -> Optional[TaskId]:
        return None

    def for_task(self, task_id: TaskId) -> "EngineError":
        return self if isinstance(self, TaskError) else TaskError(task_id, self)


class InvalidConfig(EngineError):
    def __init__(self, msg: str):
        super().__init__(f"invalid configuration: {msg}")


class NotLoaded(EngineError):
    def __init__(self):
        super().__init__("not yet loaded; call load() before build()")


class NotConnected(EngineError):
    def __init__(self):
        super().__init__("not yet connected; call connect() before build()")

    def is_connection_fatal(self) -> bool:
        return True


class PeerRejected(EngineError):
    def __init__(self, msg: str):
        super().__init__(f"peer layout rejected: {msg}")


class ShardRejected(EngineError):
    def __init__(self, msg: str):
        super().__init__(f"shard rejected: {msg}")


class ModelNotFound(EngineError):
    def __init__(self, path: str):
        super().__init__(f"model not found at {path}")


_FATAL_SUBSTRINGS = ("socket closed", "not connected", "idle ceiling", "connection reset",
                     "broken pipe", "connection aborted", "recv_exact timed out")


class Backend(EngineError):
    def __init__(self, msg: str):
        super().__init__(f"backend error: {msg}")
        self.msg = msg

    def is_connection_fatal(self) -> bool:
        m = self.msg.lower()
        return any(s in m for s in _FATAL_SUBSTRINGS)


class QueueFull(EngineError):
    def __init__(self, queued: int, cap: int):
        super().__init__(f"queue full ({queued} pending, cap {cap})")
        self.queued, self.cap = queued, cap


class PromptTooLong(EngineError):
    def __init__(self, msg: str):
        super().__init__(f"prompt too long: {msg}")


_FATAL_ERRNOS = {errno.ETIMEDOUT, errno.ECONNRESET, errno.EPIPE, errno.ECONNABORTED}


class IoError(EngineError):
    """Structurally-typed I/O failure (kind = errno or 'eof'/'timeout')."""

    def __init__(self, kind, msg: str = ""):
        super().__init__(f"io error: {msg or kind}")
        self.kind = kind

    def is_connection_fatal(self) -> bool:
        return self.kind in _FATAL_ERRNOS or self.kind in ("eof", "timeout")


class BatchAborted(EngineError):
    """The batch is gone, the link is not: never connection-fatal."""

    def __init__(self, msg: str):
        super().__init__(f"batch aborted: {msg}")

    def is_connection_fatal(self) -> bool:
        return False


class DeviceFault(EngineError):
    """A device-side bounded wait expired (status word set by a kernel)."""

    def __init__(self, code: int, msg: str = ""):
        super().__init__(f"device status {code}: {msg}")
        self.code = code


class ShutdownRequested(EngineError):
    """The upstream stage asked this stage to stop (clean relay-loop exit)."""

    def __init__(self):
        super().__init__("pipeline shutdown requested")


class TaskError(EngineError):
    def __init__(self, task_id: TaskId, source: EngineError):
        super().__init__(f"task {task_id}: {source}")
        self._task_id = task_id
        self.source = source

    @property
    def task_id(self) -> Optional[TaskId]:
        return self._task_id

    def is_connection_fatal(self) -> bool:
        return self.source.is_connection_fatal()


def classify_exception(e: BaseException) -> EngineError:
    """Map arbitrary exceptions onto the taxonomy."""
    if isinstance(e, EngineError):
        return e
    if isinstance(e, TimeoutError):
        return IoError("timeout", str(e))
    if isinstance(e, (ConnectionResetError, BrokenPipeError, ConnectionAbortedError)):
        return IoError(e.errno or errno.ECONNRESET, str(e))
    if isinstance(e, EOFError):
        return IoError("eof", str(e))
    if isinstance(e, OSError) and e.errno in _FATAL_ERRNOS:
        return IoError(e.errno, str(e))
    return Backend(str(e))


StepOutput = List[Tuple[TaskId, Chunk]]


class Engine(abc.ABC):
    """One stage's engine.  `step()` is synchronous and advances at most one
    scheduler iteration; all methods are called under the runner's lock."""

    def warmup(self) -> None:
        pass

    @abc.abstractmethod
    def submit(self, task: GenerationTask) -> None:
        ...

    @abc.abstractmethod
    def step(self) -> StepOutput:
        ...

    def cancel(self, task_id: TaskId) -> None:
        pass

    def close(self) -> None:
        pass

    def has_work(self) -> bool:
        return True


class Builder(abc.ABC):
    def configure_listen(self, host: str, port: int) -> None:
        pass

    @abc.abstractmethod
    def connect(self, peers: PeerLayout) -> None:
        ...

    @abc.abstractmethod
    def load(self, shard: ShardSpec) -> Iterable[LoadProgress]:
        ...

    @abc.abstractmethod
    def build(self) -> Engine:
        ...

    def close(self) -> None:
        pass
