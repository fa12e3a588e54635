"""OpenAI-compatible HTTP API (FastAPI) on the rank-0 stage.

Routes and limits follow crates/cascadia-api/src/lib.rs:
``/health /metrics /v1/models /v1/chat/completions /v1/completions
/v1/cancel/{task_id}`` (:267-273) plus the dashboard's ``/api/stats`` and
``/api/topology`` (crates/cascadia-dashboard/src/lib.rs:71-81).

* admission: a semaphore of ``max_concurrent`` (16) -> 503 ``capacity``;
  body cap 64 KiB and rendered-prompt cap 32 KiB -> 413 (:30-47, :1805-1828);
* engine errors map to status codes exactly as ``engine_error_response``
  (:2551-2605) and count ``cascadia_api_rejected_total{reason}``;
* streaming is raw SSE ``data: {json}\\n\\n`` ... ``data: [DONE]`` with one
  frame per chunk, an error frame on mid-stream failure and an optional usage
  frame (``stream_options.include_usage``);
* stop sequences are trimmed at the API and end the generation with
  ``finish_reason="stop"``; tool calls are parsed from the output
  (``finish_reason="tool_calls"``);
* ``/health`` latches unhealthy on engine-attributed 5xx responses and
  recovers on the next success.
"""
from __future__ import annotations

import asyncio
import json
import logging
import time
import uuid
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, Response, StreamingResponse

from .. import metrics
from ..engine import base as eb
from ..types import ApiStats, FinishReason, GenerationTask, SamplingParams
from .templates import ChatPromptRenderer
from .toolcalls import parse_tool_calls, tool_call_scan_text

log = logging.getLogger("cascadia.api")

DEFAULT_MAX_BODY_BYTES = 64 * 1024
DEFAULT_MAX_CONCURRENT = 16
DEFAULT_MAX_PROMPT_BYTES = 32 * 1024


@dataclass
class ApiConfig:
    model_name: str = "cascadia-b200"
    max_concurrent_requests: int = DEFAULT_MAX_CONCURRENT
    max_body_bytes: int = DEFAULT_MAX_BODY_BYTES
    max_prompt_bytes: int = DEFAULT_MAX_PROMPT_BYTES
    chat_template: Optional[str] = None


def _now() -> int:
    return int(time.time())


def engine_error_status(err: eb.EngineError) -> (int, str):
    """(HTTP status, rejection reason) for an error raised by submit()."""
    if isinstance(err, eb.QueueFull):
        return 503, "capacity"
    if isinstance(err, eb.PromptTooLong):
        return 413, "prompt_over_window"
    if isinstance(err, (eb.NotLoaded, eb.NotConnected)):
        return 503, "engine_unavailable"
    if isinstance(err, (eb.InvalidConfig, eb.PeerRejected, eb.ShardRejected)):
        return 400, "invalid_request"
    if isinstance(err, eb.ModelNotFound):
        return 404, "invalid_request"
    return 500, "engine_error"


class _Health:
    def __init__(self):
        self.ok = True


def _apply_stop(text: str, stops: List[str]) -> Optional[int]:
    idx = [text.find(s) for s in stops if s]
    idx = [i for i in idx if i >= 0]
    return min(idx) if idx else None


def _hold_back(text: str, stops: List[str]) -> int:
    """Chars at the end that could still be the start of a stop sequence."""
    hold = 0
    for s in stops:
        for k in range(min(len(s) - 1, len(text)), 0, -1):
            if text.endswith(s[:k]):
                hold = max(hold, k)
                break
    return hold


# Self-contained status page: polls the two JSON routes (no assets, no
# graphics API; the reference serves a placeholder page the same way,
# crates/cascadia-dashboard/src/lib.rs:85-93).
DASHBOARD_HTML = """<!doctype html><html><head><meta charset="utf-8">
<title>cascadia-b200</title><style>body{font-family:sans-serif;margin:2em}
table{border-collapse:collapse}td,th{border:1px solid #999;padding:4px 8px}</style></head>
<body><h2>cascadia-b200</h2><div id="stats"></div><h3>Nodes</h3><table id="nodes"></table>
<h3>Links</h3><table id="edges"></table><script>
async function refresh(){
 const s=await (await fetch('/api/stats')).json();
 document.getElementById('stats').textContent=JSON.stringify(s);
 const t=await (await fetch('/api/topology')).json();
 let h='<tr><th>node</th><th>device</th><th>memory MB</th><th>engines</th></tr>';
 for(const n of t.nodes){h+=`<tr><td>${n.node_id}</td><td>${n.device}</td><td>${n.memory_mb}</td><td>${(n.engines||[]).join(',')}</td></tr>`;}
 document.getElementById('nodes').innerHTML=h;
 h='<tr><th>src</th><th>dst</th><th>latency ms</th><th>bandwidth MB/s</th></tr>';
 for(const e of t.edges){h+=`<tr><td>${e.src}</td><td>${e.dst}</td><td>${e.latency_ms.toFixed(4)}</td><td>${e.bandwidth_mbps.toFixed(0)}</td></tr>`;}
 document.getElementById('edges').innerHTML=h;}
refresh();setInterval(refresh,5000);</script></body></html>"""


def make_app(runner, config: Optional[ApiConfig] = None, stats: Optional[ApiStats] = None,
             topology=None) -> FastAPI:
    cfg = config or ApiConfig()
    stats = stats or ApiStats()
    health = _Health()
    sem = asyncio.Semaphore(cfg.max_concurrent_requests)
    renderer = ChatPromptRenderer(cfg.chat_template)
    app = FastAPI(title="cascadia-b200", docs_url=None, redoc_url=None)
    app.state.runner = runner
    app.state.stats = stats

    @app.middleware("http")
    async def limits_and_metrics(request: Request, call_next):
        route = request.url.path
        if route.startswith("/v1/cancel/"):
            route = "/v1/cancel/:task_id"
        t0 = time.monotonic()
        if request.method == "POST":
            cl = request.headers.get("content-length")
            body = await request.body()
            if (cl and int(cl) > cfg.max_body_bytes) or len(body) > cfg.max_body_bytes:
                resp = JSONResponse({"error": "request body too large"}, status_code=413)
                metrics.HTTP_REQUESTS.labels(endpoint=route, status="413").inc()
                return resp
        resp = await call_next(request)
        metrics.HTTP_REQUESTS.labels(endpoint=route, status=str(resp.status_code)).inc()
        metrics.HTTP_DURATION.labels(endpoint=route).observe(time.monotonic() - t0)
        return resp

    @app.get("/health")
    async def health_route():
        if health.ok:
            return {"status": "ok"}
        return JSONResponse({"status": "unhealthy"}, status_code=503)

    @app.get("/metrics")
    async def metrics_route():
        return Response(metrics.encode_text(), media_type="text/plain; version=0.0.4")

    @app.get("/v1/models")
    async def models_route():
        return {"object": "list", "data": [{"id": cfg.model_name, "object": "model",
                                            "created": 0, "owned_by": "cascadia"}]}

    @app.post("/v1/cancel/{task_id}")
    async def cancel_route(task_id: str):
        runner.cancel(task_id)
        return {"cancelled": task_id}

    @app.get("/api/stats")
    async def stats_route():
        return stats.snapshot()

    @app.get("/api/topology")
    async def topology_route():
        return topology.to_json() if topology is not None else {"nodes": [], "edges": []}

    @app.get("/")
    async def dashboard_route():
        from fastapi.responses import HTMLResponse

        return HTMLResponse(DASHBOARD_HTML)

    def _sampling(body: dict) -> (SamplingParams, float):
        stop = body.get("stop")
        if isinstance(stop, str):
            stop = [stop]
        sp = SamplingParams(top_p=float(body.get("top_p") or 1.0),
                            top_k=int(body.get("top_k") or 0), seed=body.get("seed"),
                            frequency_penalty=float(body.get("frequency_penalty") or 0.0),
                            presence_penalty=float(body.get("presence_penalty") or 0.0),
                            stop=list(stop or []))
        return sp, float(body.get("temperature") or 0.0)

    def _logprobs_count(body: dict, chat: bool) -> int:
        """Top-logprobs per position to ask the engine for (0 = off): chat's
        `logprobs` is a bool with `top_logprobs` 1..20 (default 1), legacy
        completions' `logprobs` is the count itself (at most 20), as in
        crates/cascadia-api/src/lib.rs:556-560, 720-724."""
        try:
            if chat:
                if not body.get("logprobs"):
                    return 0
                return max(1, min(20, int(body.get("top_logprobs") or 1)))
            return max(0, min(20, int(body.get("logprobs") or 0)))
        except (TypeError, ValueError):
            return 0

    def _lp_json(lps: list) -> Optional[dict]:
        return {"content": [asdict(lp) for lp in lps]} if lps else None

    def _enable_thinking(body: dict) -> bool:
        kw = body.get("chat_template_kwargs") or {}
        if isinstance(kw, dict) and "enable_thinking" in kw:
            return bool(kw["enable_thinking"])
        if body.get("enable_thinking") is not None:
            return bool(body["enable_thinking"])
        if body.get("reasoning_effort") == "none":
            return False
        return True

    def _reject(status: int, reason: str, msg: str):
        metrics.count_rejected(reason)
        return JSONResponse({"error": msg}, status_code=status)

    async def _admit(task: GenerationTask):
        """Returns (stream, None) or (None, error response)."""
        if sem.locked():
            return None, _reject(503, "capacity", "server at capacity")
        await sem.acquire()
        try:
            stream = await runner.generate_async(task)
        except eb.EngineError as e:
            sem.release()
            status, reason = engine_error_status(e)
            if status >= 500 and reason == "engine_error":
                health.ok = False
            return None, _reject(status, reason, str(e))
        except Exception as e:  # noqa: BLE001
            sem.release()
            health.ok = False
            return None, _reject(500, "engine_error", str(e))
        return stream, None

    async def _run(body: dict, prompt: str, chat: bool, tools: Optional[list]):
        if not prompt or not prompt.strip():
            return _reject(400, "empty_prompt", "empty prompt")
        if len(prompt.encode("utf-8")) > cfg.max_prompt_bytes:
            return _reject(413, "prompt_too_large", "prompt too large")
        sp, temp = _sampling(body)
        prefix = "chatcmpl-" if chat else "cmpl-"
        task = GenerationTask(task_id=prefix + uuid.uuid4().hex, prompt=prompt,
                              max_tokens=int(body.get("max_tokens") or 256), temperature=temp,
                              logprobs=_logprobs_count(body, chat),
                              sampling=sp, enable_thinking=_enable_thinking(body))
        ids = body.get("prompt_token_ids")
        if isinstance(ids, list) and ids:
            task.prompt_ids = [int(t) for t in ids]
        stream, err = await _admit(task)
        if err is not None:
            return err
        stats.begin()
        include_usage = bool((body.get("stream_options") or {}).get("include_usage"))
        tools_active = bool(tools) and body.get("tool_choice") != "none"
        if body.get("stream"):
            return StreamingResponse(_sse(task, stream, chat, include_usage, tools_active),
                                     media_type="text/event-stream",
                                     headers={"Cache-Control": "no-cache",
                                              "x-accel-buffering": "no"})
        done = False
        try:
            text, finish, completion, prompt_toks, error, lps = await _collect(task, stream)
            done = True
        finally:
            sem.release()
            stats.end()
            if not done:
                # The client went away (the handler was cancelled): stop the
                # generation instead of running it to max_tokens.
                runner.cancel(task.task_id)
        if error is not None:
            health.ok = False
            return JSONResponse({"error": error}, status_code=500)
        health.ok = True
        usage = _usage(prompt_toks, completion, getattr(task, "_cached", 0))
        if chat:
            msg: Dict[str, Any] = {"role": "assistant", "content": text}
            calls = parse_tool_calls(tool_call_scan_text(text, task.enable_thinking)) \
                if tools_active else None
            if calls:
                msg = {"role": "assistant", "content": None,
                       "tool_calls": [c.to_openai() for c in calls]}
                finish = "tool_calls"
            choice = {"index": 0, "message": msg, "finish_reason": finish}
            if lps:
                choice["logprobs"] = _lp_json(lps)
            return {"id": task.task_id, "object": "chat.completion", "created": _now(),
                    "model": cfg.model_name, "choices": [choice], "usage": usage}
        return {"id": task.task_id, "object": "text_completion", "created": _now(),
                "model": cfg.model_name,
                "choices": [{"index": 0, "text": text, "finish_reason": finish,
                             "logprobs": _lp_json(lps)}],
                "usage": usage}

    def _usage(prompt_toks: int, completion: int, cached: int) -> dict:
        u = {"prompt_tokens": prompt_toks, "completion_tokens": completion,
             "total_tokens": prompt_toks + completion}
        if cached:
            u["prompt_tokens_details"] = {"cached_tokens": cached}
        return u

    async def _collect(task, stream):
        text, finish, completion, prompt_toks, error = "", "stop", 0, 0, None
        lps = []
        task._cached = 0
        stops = task.sampling.stop
        async for c in stream:
            if c.error is not None:
                error = c.error
                break
            if c.logprobs is not None:
                lps.append(c.logprobs)
            text += c.text
            completion += c.token_count()
            stats.add_tokens(c.token_count())
            if c.prompt_tokens:
                prompt_toks = c.prompt_tokens
            if c.cached_tokens:
                task._cached = c.cached_tokens
            if c.finish_reason is not None:
                finish = c.finish_reason.as_openai_str()
            cut = _apply_stop(text, stops)
            if cut is not None:
                text = text[:cut]
                finish = "stop"
                stream.done = True
                runner.cancel(task.task_id)
                break
        return text, finish, completion, prompt_toks, error, lps

    async def _sse(task, stream, chat: bool, include_usage: bool, tools_active: bool):
        model = cfg.model_name
        obj = "chat.completion.chunk" if chat else "text_completion"
        completion = prompt_toks = cached = 0
        stops = task.sampling.stop
        sent = ""       # text already emitted
        pending = ""    # text held back (possible stop-sequence prefix)
        lp_pending = []  # logprobs of tokens whose text is not emitted yet
        first = True
        finished = False  # False on exit = the client disconnected mid-stream

        def frame(payload) -> bytes:
            return f"data: {json.dumps(payload, ensure_ascii=False)}\n\n".encode()

        def delta_frame(text: str, finish: Optional[str]):
            nonlocal first, lp_pending
            # Logprobs ride on the frame that carries their tokens' text; the
            # finishing frame flushes any whose text was empty or held back.
            lp = _lp_json(lp_pending) if (text or finish is not None) else None
            if text or finish is not None:
                lp_pending = []
            if chat:
                d: Dict[str, Any] = {}
                if first:
                    d["role"] = "assistant"
                if text:
                    d["content"] = text
                first = False
                choice = {"index": 0, "delta": d, "finish_reason": finish}
                if lp is not None:
                    choice["logprobs"] = lp
            else:
                choice = {"index": 0, "text": text, "finish_reason": finish, "logprobs": lp}
            return frame({"id": task.task_id, "object": obj, "created": _now(), "model": model,
                          "choices": [choice]})

        try:
            buf = ""
            finish = "stop"
            async for c in stream:
                if c.error is not None:
                    health.ok = False
                    yield frame({"id": task.task_id, "object": "error",
                                 "error": {"message": c.error, "type": "engine_error"}})
                    finished = True
                    yield b"data: [DONE]\n\n"
                    return
                completion += c.token_count()
                stats.add_tokens(c.token_count())
                if c.logprobs is not None:
                    lp_pending.append(c.logprobs)
                if c.prompt_tokens:
                    prompt_toks = c.prompt_tokens
                if c.cached_tokens:
                    cached = c.cached_tokens
                if c.finish_reason is not None:
                    finish = c.finish_reason.as_openai_str()
                if tools_active:
                    buf += c.text
                    continue
                pending += c.text
                cut = _apply_stop(sent + pending, stops)
                if cut is not None:
                    keep = (sent + pending)[:cut][len(sent):]
                    if keep:
                        yield delta_frame(keep, None)
                    yield delta_frame("", "stop")
                    stream.done = True
                    runner.cancel(task.task_id)
                    finish = None
                    pending = ""
                    break
                hold = _hold_back(pending, stops) if stops else 0
                emit = pending[:len(pending) - hold] if hold else pending
                if emit:
                    yield delta_frame(emit, None)
                    sent += emit
                    pending = pending[len(emit):]
                if c.is_final:
                    break
            if tools_active:
                calls = parse_tool_calls(tool_call_scan_text(buf, task.enable_thinking))
                if calls:
                    yield frame({"id": task.task_id, "object": obj, "created": _now(),
                                 "model": model, "choices": [{"index": 0, "delta": {
                                     "role": "assistant",
                                     "tool_calls": [c.to_openai(i) for i, c in enumerate(calls)]},
                                     "finish_reason": None}]})
                    finish = "tool_calls"
                elif buf:
                    yield delta_frame(buf, None)
            elif pending:
                yield delta_frame(pending, None)
            if finish is not None:
                yield delta_frame("", finish)
            health.ok = True
            if include_usage:
                yield frame({"id": task.task_id, "object": obj, "created": _now(), "model": model,
                             "choices": [], "usage": _usage(prompt_toks, completion, cached)})
            finished = True
            yield b"data: [DONE]\n\n"
        finally:
            sem.release()
            stats.end()
            if not finished:
                runner.cancel(task.task_id)

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        try:
            body = json.loads(await request.body())
        except ValueError:
            return JSONResponse({"error": "invalid JSON"}, status_code=400)
        messages = body.get("messages")
        if not isinstance(messages, list) or not messages:
            return _reject(400, "empty_prompt", "messages must be a non-empty list")
        try:
            prompt = renderer.render(messages, enable_thinking=_enable_thinking(body),
                                     tools=body.get("tools"))
        except Exception as e:  # noqa: BLE001
            return JSONResponse({"error": f"chat template: {e}"}, status_code=500)
        return await _run(body, prompt, True, body.get("tools"))

    @app.post("/v1/completions")
    async def completions(request: Request):
        try:
            body = json.loads(await request.body())
        except ValueError:
            return JSONResponse({"error": "invalid JSON"}, status_code=400)
        prompt = body.get("prompt")
        if isinstance(prompt, list):
            if len(prompt) != 1 or not isinstance(prompt[0], str):
                return _reject(400, "multi_prompt", "exactly one prompt string is supported")
            prompt = prompt[0]
        if not isinstance(prompt, str):
            return _reject(400, "empty_prompt", "prompt must be a string")
        return await _run(body, prompt, False, None)

    return app
