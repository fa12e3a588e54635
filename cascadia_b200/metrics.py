"""Prometheus metrics with the reference's names and bucket layouts.

Names / labels / buckets: crates/cascadia-metrics/src/lib.rs:32-291 and
docs/METRICS.md:28-126.  Additions for the GPU engine: device-timed step
latency, KV-block utilisation, speculative acceptance, collective bytes and
an expert-load histogram.
"""
from __future__ import annotations

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest

TTFT_BUCKETS = (0.05, 0.1, 0.25, 0.5, 1, 2, 5, 10, 30, 60)
INTER_TOKEN_BUCKETS = (0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1, 2, 5, 10)
DURATION_BUCKETS = (0.1, 0.5, 1, 5, 10, 30, 60, 120, 300, 600)
TRANSPORT_BUCKETS = (0.0001, 0.001, 0.01, 0.05, 0.1, 0.5, 1)
STEP_BUCKETS = (0.0005, 0.001, 0.002, 0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 1)

REGISTRY = CollectorRegistry()

HTTP_REQUESTS = Counter("cascadia_http_requests_total", "HTTP requests by route and status",
                        ["endpoint", "status"], registry=REGISTRY)
HTTP_DURATION = Histogram("cascadia_http_request_duration_seconds", "HTTP latency (to head)",
                          ["endpoint"], buckets=DURATION_BUCKETS, registry=REGISTRY)
INFLIGHT = Gauge("cascadia_inflight_tasks", "Generations executing", registry=REGISTRY)
API_REJECTED = Counter("cascadia_api_rejected_total", "Rejections before generation",
                       ["reason"], registry=REGISTRY)

TTFT = Histogram("cascadia_generation_ttft_seconds", "Submission to first token chunk",
                 ["model"], buckets=TTFT_BUCKETS, registry=REGISTRY)
INTER_TOKEN = Histogram("cascadia_generation_inter_token_seconds", "Gap between token chunks",
                        ["model"], buckets=INTER_TOKEN_BUCKETS, registry=REGISTRY)
GEN_DURATION = Histogram("cascadia_generation_duration_seconds", "Submission to terminal",
                         ["model", "finish_reason"], buckets=DURATION_BUCKETS, registry=REGISTRY)
TOKENS_GENERATED = Counter("cascadia_tokens_generated_total", "Tokens delivered", ["model"],
                           registry=REGISTRY)
TOKENS_PROMPT = Counter("cascadia_tokens_prompt_total", "Prompt tokens", ["model"],
                        registry=REGISTRY)
TASKS_CANCELLED = Counter("cascadia_tasks_cancelled_total", "Cancelled generations", ["model"],
                          registry=REGISTRY)
TASKS_FAILED = Counter("cascadia_tasks_failed_total", "Failed generations", ["model"],
                       registry=REGISTRY)

LOAD_SECONDS = Gauge("cascadia_engine_model_load_duration_seconds", "Weight load + build",
                     ["model", "device"], registry=REGISTRY)
WARMUP_SECONDS = Gauge("cascadia_engine_warmup_duration_seconds", "Warmup duration",
                       ["model", "device"], registry=REGISTRY)

TRANSPORT_SENT = Counter("cascadia_transport_sent_bytes_total", "Bytes sent", ["kind"],
                         registry=REGISTRY)
TRANSPORT_RECV = Counter("cascadia_transport_recv_bytes_total", "Bytes received", ["kind"],
                         registry=REGISTRY)
TRANSPORT_SEND_S = Histogram("cascadia_transport_send_seconds", "Frame send duration",
                             buckets=TRANSPORT_BUCKETS, registry=REGISTRY)
TRANSPORT_RECV_S = Histogram("cascadia_transport_recv_payload_seconds", "Payload receive",
                             buckets=TRANSPORT_BUCKETS, registry=REGISTRY)

# GPU-engine additions.
STEP_SECONDS = Histogram("cascadia_engine_step_device_seconds",
                         "Device-timed engine iteration (CUDA events, max over ranks)",
                         ["model", "phase"], buckets=STEP_BUCKETS, registry=REGISTRY)
KV_BLOCKS_USED = Gauge("cascadia_kv_blocks_used", "Paged-KV blocks in use", ["model"],
                       registry=REGISTRY)
KV_BLOCKS_TOTAL = Gauge("cascadia_kv_blocks_total", "Paged-KV blocks", ["model"],
                        registry=REGISTRY)
SPEC_ACCEPTED = Counter("cascadia_spec_accepted_tokens_total", "Accepted draft tokens",
                        ["model"], registry=REGISTRY)
SPEC_PROPOSED = Counter("cascadia_spec_proposed_tokens_total", "Proposed draft tokens",
                        ["model"], registry=REGISTRY)
COLLECTIVE_BYTES = Counter("cascadia_collective_bytes_total", "Bytes moved by collectives",
                           ["op"], registry=REGISTRY)
EXPERT_LOAD = Histogram("cascadia_expert_tokens_per_step", "Tokens routed to an expert per step",
                        ["model"], buckets=(0, 1, 2, 4, 8, 16, 32, 64, 128, 256, 1024),
                        registry=REGISTRY)


def encode_text() -> bytes:
    return generate_latest(REGISTRY)


def count_rejected(reason: str) -> None:
    API_REJECTED.labels(reason=reason).inc()
