"""Request/response vocabulary shared by every layer.

Field names and JSON shapes match the reference's ``cascadia-types`` crate
(crates/cascadia-types/src/task.rs:10-120, chunk.rs:1-170, shard.rs:12-139,
peer.rs:25-33, stats.rs:13-21) so serialized tasks and chunks are
interchangeable.
"""
from __future__ import annotations

import enum
import threading
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

TaskId = str


@dataclass
class SamplingParams:
    """OpenAI-compatible sampling knobs (task.rs:10-35)."""
    top_p: float = 1.0
    top_k: int = 0
    seed: Optional[int] = None
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    stop: List[str] = field(default_factory=list)

    @staticmethod
    def from_dict(d: Optional[dict]) -> "SamplingParams":
        d = d or {}
        return SamplingParams(top_p=float(d.get("top_p", 1.0)), top_k=int(d.get("top_k", 0)),
                              seed=d.get("seed"),
                              frequency_penalty=float(d.get("frequency_penalty", 0.0)),
                              presence_penalty=float(d.get("presence_penalty", 0.0)),
                              stop=list(d.get("stop", []) or []))


@dataclass
class GenerationTask:
    """One generation request end to end (task.rs:58-120)."""
    task_id: TaskId
    prompt: str
    max_tokens: int = 256
    temperature: float = 0.0
    logprobs: int = 0
    sampling: SamplingParams = field(default_factory=SamplingParams)
    enable_thinking: bool = False
    trust_remote_code: bool = False
    # Tokenizer-free mode: token ids given directly (used by benches/tests).
    prompt_ids: Optional[List[int]] = None

    def to_dict(self) -> dict:
        return asdict(self)

    @staticmethod
    def from_dict(d: dict) -> "GenerationTask":
        d = dict(d)
        d["sampling"] = SamplingParams.from_dict(d.get("sampling"))
        known = set(GenerationTask.__dataclass_fields__)
        return GenerationTask(**{k: v for k, v in d.items() if k in known})


class FinishReason(str, enum.Enum):
    STOP = "stop"
    LENGTH = "length"
    CANCELLED = "cancelled"

    def as_openai_str(self) -> str:
        return "length" if self is FinishReason.LENGTH else "stop"


@dataclass
class TopLogprob:
    token: str
    token_id: int
    logprob: float


@dataclass
class TokenLogprobs:
    token: str
    token_id: int
    logprob: float
    top_logprobs: List[TopLogprob] = field(default_factory=list)


@dataclass
class Chunk:
    """One streamed piece of output (chunk.rs:50-170)."""
    task_id: TaskId
    token_id: int = 0
    text: str = ""
    is_final: bool = False
    logprobs: Optional[TokenLogprobs] = None
    n_tokens: Optional[int] = None
    prompt_tokens: Optional[int] = None
    cached_tokens: Optional[int] = None   # prompt tokens served from the prefix cache
    error: Optional[str] = None
    finish_reason: Optional[FinishReason] = None

    @staticmethod
    def token(task_id: TaskId, token_id: int, text: str) -> "Chunk":
        return Chunk(task_id=task_id, token_id=token_id, text=text)

    @staticmethod
    def final_marker(task_id: TaskId, text: str = "") -> "Chunk":
        return Chunk(task_id=task_id, text=text, is_final=True)

    @staticmethod
    def error_chunk(task_id: TaskId, reason: str) -> "Chunk":
        return Chunk(task_id=task_id, is_final=True, error=reason)

    def with_prompt_tokens(self, n: int) -> "Chunk":
        self.prompt_tokens = n
        return self

    def with_cached_tokens(self, n: int) -> "Chunk":
        self.cached_tokens = n
        return self

    def with_finish_reason(self, r: FinishReason) -> "Chunk":
        self.finish_reason = r
        return self

    def with_n_tokens(self, n: int) -> "Chunk":
        self.n_tokens = n
        return self

    def token_count(self) -> int:
        """Engine `n_tokens` when set, else one per non-empty chunk (chunk.rs:161)."""
        if self.n_tokens is not None:
            return self.n_tokens
        return 0 if not self.text else 1

    def to_dict(self) -> dict:
        d: Dict[str, Any] = {"task_id": self.task_id, "token_id": self.token_id,
                             "text": self.text, "is_final": self.is_final,
                             "logprobs": asdict(self.logprobs) if self.logprobs else None}
        for k in ("n_tokens", "prompt_tokens", "cached_tokens", "error"):
            v = getattr(self, k)
            if v is not None:
                d[k] = v
        if self.finish_reason is not None:
            d["finish_reason"] = self.finish_reason.value
        return d


@dataclass
class ShardSpec:
    """One stage's slice of the model (shard.rs:12-40)."""
    model_id: str
    layer_start: int
    layer_end: int
    total_layers: int
    device: str = "cuda"
    is_first_stage: bool = True
    is_last_stage: bool = True
    tp_size: int = 1
    tp_rank: int = 0

    @property
    def num_layers(self) -> int:
        return self.layer_end - self.layer_start


class ShardError(ValueError):
    pass


@dataclass
class ShardPlan:
    model_id: str
    total_layers: int
    hidden_size: int
    num_attention_heads: int
    vocab_size: int
    stages: List[ShardSpec]

    @property
    def total_stages(self) -> int:
        return len(self.stages)

    @staticmethod
    def uniform(model_id: str, total_layers: int, hidden_size: int, num_attention_heads: int,
                vocab_size: int, num_stages: int, devices: Optional[List[str]] = None,
                tp_size: int = 1) -> "ShardPlan":
        """Even split; trailing layers go to the last stage (shard.rs:79-139)."""
        if num_stages < 1:
            raise ShardError(f"num_stages must be >= 1 (got {num_stages})")
        if num_stages > total_layers:
            raise ShardError(f"num_stages ({num_stages}) exceeds total_layers ({total_layers})")
        devices = devices or ["cuda"] * num_stages
        if len(devices) != num_stages:
            raise ShardError(f"devices ({len(devices)}) must match num_stages ({num_stages})")
        per = total_layers // num_stages
        stages, cur = [], 0
        for i in range(num_stages):
            n = per if i < num_stages - 1 else total_layers - cur
            stages.append(ShardSpec(model_id, cur, cur + n, total_layers, devices[i], i == 0,
                                    i == num_stages - 1, tp_size, 0))
            cur += n
        return ShardPlan(model_id, total_layers, hidden_size, num_attention_heads, vocab_size,
                         stages)


@dataclass
class PeerEndpoint:
    host: str
    port: int

    def __str__(self) -> str:
        return f"{self.host}:{self.port}"

    @staticmethod
    def parse(s: str) -> "PeerEndpoint":
        host, _, port = s.rpartition(":")
        return PeerEndpoint(host or "127.0.0.1", int(port))


@dataclass
class PeerLayout:
    """Adjacent stages of this rank (peer.rs:25-33)."""
    upstream: Optional[PeerEndpoint] = None
    downstream: Optional[PeerEndpoint] = None


@dataclass
class LoadProgress:
    message: str = ""
    fraction: Optional[float] = None
    ready: bool = False

    @staticmethod
    def msg(m: str) -> "LoadProgress":
        return LoadProgress(message=m)

    @staticmethod
    def done() -> "LoadProgress":
        return LoadProgress(message="ready", fraction=1.0, ready=True)


class ApiStats:
    """Live counters shared by the API and the dashboard (stats.rs:13-21)."""

    def __init__(self):
        self._lock = threading.Lock()
        self.requests_total = 0
        self.tokens_total = 0
        self.active_requests = 0

    def begin(self):
        with self._lock:
            self.requests_total += 1
            self.active_requests += 1

    def end(self):
        with self._lock:
            self.active_requests = max(0, self.active_requests - 1)

    def add_tokens(self, n: int):
        with self._lock:
            self.tokens_total += n

    def snapshot(self) -> dict:
        with self._lock:
            return {"requests_total": self.requests_total, "tokens_total": self.tokens_total,
                    "active_requests": self.active_requests}
