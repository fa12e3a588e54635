"""TCP activation transport between pipeline stages (CPU / loopback path).

Python face of the native ``cascadia_b200._runtime`` transport: tensor frames
with the reference's 20-byte big-endian header
(crates/cascadia-transport/src/lib.rs:1-16, send_tensor :183-228), raw
control frames capped at 64 KiB, a per-frame deadline, an idle ceiling for a
frame to start, and a bounded non-fatal "frame start" wait for replies.
Failures are raised as ``EngineError`` subclasses so the runner's
connection-fatal classifier (closed / reset / timeout / idle ceiling ->
fatal; frame-start timeout -> retryable) applies unchanged.
"""
from __future__ import annotations

import time
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from .. import metrics
from ..engine.base import Backend, IoError

try:
    from .. import _runtime as _rt  # type: ignore
except ImportError:  # pragma: no cover - built by setup.py
    _rt = None

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.int8: 2, torch.int32: 3,
               torch.int64: 4, torch.bfloat16: 5}
CODE_DTYPES = {v: k for k, v in DTYPE_CODES.items()}

DEFAULT_TIMEOUT_S = 60.0
DEFAULT_IDLE_CEILING_S = 900.0


class FrameStartTimeout(Backend):
    """No frame started within the bounded wait (not connection-fatal)."""

    def __init__(self, msg: str):
        super().__init__(msg)

    def is_connection_fatal(self) -> bool:
        return False


def _require():
    if _rt is None:
        raise RuntimeError("cascadia_b200._runtime is not built; run setup.py build_ext")
    return _rt


def _translate(e: Exception) -> Exception:
    msg = str(e)
    kind = msg.split(":", 1)[0]
    if kind == "frame_start_timeout":
        return FrameStartTimeout(msg)
    if kind in ("closed", "reset"):
        return Backend(msg)  # message carries "socket closed" / "connection reset"
    if kind == "idle_ceiling":
        return Backend("idle ceiling: " + msg)
    if kind == "timeout":
        return IoError("timeout", msg)
    return Backend(msg)


class TensorLink:
    def __init__(self, link):
        self._l = link

    @staticmethod
    def listen(host: str = "127.0.0.1", port: int = 0):
        return _require().Server(host, port)

    @staticmethod
    def accept(server, timeout_s: float = 30.0, frame_timeout: float = DEFAULT_TIMEOUT_S,
               idle_ceiling: float = DEFAULT_IDLE_CEILING_S) -> "TensorLink":
        try:
            return TensorLink(server.accept(timeout_s, frame_timeout, idle_ceiling))
        except Exception as e:
            raise _translate(e) from e

    @staticmethod
    def connect(host: str, port: int, total_s: float = 30.0,
                frame_timeout: float = DEFAULT_TIMEOUT_S,
                idle_ceiling: float = DEFAULT_IDLE_CEILING_S) -> "TensorLink":
        try:
            return TensorLink(_require().connect(host, port, total_s, frame_timeout, idle_ceiling))
        except Exception as e:
            raise _translate(e) from e

    def send(self, t: torch.Tensor):
        t = t.detach().contiguous().cpu()
        code = DTYPE_CODES[t.dtype]
        shape = list(t.shape) or [1]
        if len(shape) > 3:
            shape = [int(np.prod(shape[:-2])), shape[-2], shape[-1]]
        buf = t.view(torch.uint8).numpy() if t.numel() else np.zeros(0, np.uint8)
        t0 = time.perf_counter()
        try:
            self._l.send_tensor(buf, code, shape)
        except Exception as e:
            raise _translate(e) from e
        metrics.TRANSPORT_SEND_S.observe(time.perf_counter() - t0)
        metrics.TRANSPORT_SENT.labels(kind="tensor").inc(20 + buf.nbytes)

    def recv(self, first_byte_s: float = -1.0) -> torch.Tensor:
        try:
            code, shape, payload = self._l.recv_tensor(first_byte_s)
        except Exception as e:
            raise _translate(e) from e
        dt = CODE_DTYPES.get(code)
        if dt is None:
            raise Backend(f"unknown dtype code {code}")
        metrics.TRANSPORT_RECV.labels(kind="tensor").inc(20 + len(payload))
        if not payload:
            return torch.empty(0, dtype=dt)
        t = torch.frombuffer(bytearray(payload), dtype=torch.uint8).view(dt)
        return t.view(*[int(s) for s in shape])

    def send_raw(self, b: bytes):
        try:
            self._l.send_raw(b)
        except Exception as e:
            raise _translate(e) from e
        metrics.TRANSPORT_SENT.labels(kind="raw").inc(len(b))

    def recv_raw(self, n: int, first_byte_s: float = -1.0) -> bytes:
        try:
            b = self._l.recv_raw(n, first_byte_s)
        except Exception as e:
            raise _translate(e) from e
        metrics.TRANSPORT_RECV.labels(kind="raw").inc(n)
        return b

    def close(self):
        self._l.close()

    @property
    def is_open(self) -> bool:
        return self._l.is_open
