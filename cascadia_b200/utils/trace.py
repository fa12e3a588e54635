"""Tracing helpers: NVTX ranges around engine phases (visible in Nsight
Systems / ncu range filters) that cost nothing when no profiler is attached,
and the per-task phase log line (prefill_ms, decode_tok_s), the same fields
the reference logs at task end (crates/cascadia-engine-openvino/src/runtime.rs:2884-2912)."""
from __future__ import annotations

import contextlib
import logging

import torch

log = logging.getLogger("cascadia.trace")
_NVTX = torch.cuda.is_available()


@contextlib.contextmanager
def span(name: str):
    if _NVTX:
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def task_done(task_id: str, submitted: float, first_token: float, finished: float,
              n_tokens: int, prompt_tokens: int):
    prefill_ms = (first_token - submitted) * 1000 if first_token else 0.0
    dec = (n_tokens - 1) / (finished - first_token) if first_token and n_tokens > 1 and \
        finished > first_token else 0.0
    log.info("task %s done prompt_tokens=%d tokens=%d prefill_ms=%.1f decode_tok_s=%.1f",
             task_id, prompt_tokens, n_tokens, prefill_ms, dec)
    return prefill_ms, dec
