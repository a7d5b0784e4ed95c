"""OpenAI-compatible HTTP server (vLLM API surface the reference serves, ``README.md:213-216``):

  POST /v1/completions           (streaming and non-streaming)
  POST /v1/chat/completions      (streaming; reasoning parser "qwen3", tool parser "qwen3_xml")
  GET  /v1/models, /health, /metrics (Prometheus text, vLLM metric names), /version

One background thread drives ``LLMEngine.step`` and fans results out to per-request queues; with
tensor parallelism only rank 0 serves HTTP and the request stream is broadcast to the other ranks
(``parallel/spmd.py``)."""
from __future__ import annotations

import asyncio
import json
import queue
import threading
import time
import uuid
from typing import Optional

from ..engine.request import SamplingParams
from .parsers import ReasoningParser, ToolParser

try:  # module-level name: endpoint annotations are resolved in module globals
    from fastapi import Request as FReq
except ImportError:   # pragma: no cover
    FReq = None


class EngineLoop:
    """Runs the engine on a dedicated thread; thread-safe submission and per-request queues."""

    def __init__(self, engine, broadcaster=None):
        self.engine = engine
        self.inbox: "queue.Queue" = queue.Queue()
        self.outq: dict = {}
        self.lock = threading.Lock()
        self.broadcaster = broadcaster
        self.running = True
        self.error: Optional[str] = None
        self.kernel_fault = False
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, prompt, params: SamplingParams, request_id: str, loop) -> "asyncio.Queue":
        q: asyncio.Queue = asyncio.Queue()
        with self.lock:
            self.outq[request_id] = (q, loop)
        self.inbox.put(("add", prompt, params, request_id))
        return q

    def abort(self, request_id: str):
        self.inbox.put(("abort", request_id))

    def _loop(self):
        eng = self.engine
        while self.running:
            cmds = []
            try:
                if not eng.has_unfinished_requests():
                    cmds.append(self.inbox.get(timeout=0.05))
                while True:
                    cmds.append(self.inbox.get_nowait())
            except queue.Empty:
                pass
            if self.broadcaster is not None:
                cmds = self.broadcaster.broadcast(cmds)
            for c in cmds:
                try:
                    if c[0] == "add":
                        eng.add_request(c[1], c[2], c[3])
                    elif c[0] == "abort":
                        eng.abort_request(c[1])
                        self._emit(c[1], None)
                except Exception as e:   # bad request: report to its queue
                    self._emit(c[3] if c[0] == "add" else c[1], {"error": str(e)})
            if not eng.has_unfinished_requests():
                continue
            try:
                outs = eng.step()
            except Exception as e:      # engine failure: fail every open request, keep serving
                self.error = repr(e)
                from ..ops.kernels import KernelFaultError
                if isinstance(e, KernelFaultError):
                    self.kernel_fault = True     # device state is suspect: report unhealthy
                with self.lock:
                    ids = list(self.outq)
                for rid in ids:
                    eng.abort_request(rid)
                    self._emit(rid, {"error": f"engine error: {e}"})
                continue
            for o in outs:
                self._emit(o.request_id, o)

    def _emit(self, rid, item):
        with self.lock:
            ent = self.outq.get(rid)
            if ent is not None and (item is None or getattr(item, "finished", True)):
                self.outq.pop(rid, None)
        if ent is not None:
            q, loop = ent
            loop.call_soon_threadsafe(q.put_nowait, item)


def _sampling_from_body(body: dict, default_max: int = 256) -> SamplingParams:
    stop = body.get("stop") or []
    if isinstance(stop, str):
        stop = [stop]
    mt = body.get("max_completion_tokens", body.get("max_tokens")) or default_max
    return SamplingParams(
        temperature=float(body.get("temperature", 1.0)),
        top_p=float(body.get("top_p", 1.0)),
        top_k=int(body.get("top_k", 0) or 0),
        min_p=float(body.get("min_p", 0.0)),
        max_tokens=int(mt),
        seed=body.get("seed"),
        stop=stop,
        stop_token_ids=list(body.get("stop_token_ids") or []),
        ignore_eos=bool(body.get("ignore_eos", False)),
        presence_penalty=float(body.get("presence_penalty", 0.0)),
        frequency_penalty=float(body.get("frequency_penalty", 0.0)),
        repetition_penalty=float(body.get("repetition_penalty", 1.0)),
        min_tokens=int(body.get("min_tokens", 0)))


def build_app(engine, served_model_name: str = "model", reasoning_parser: Optional[str] = None,
              tool_parser: Optional[str] = None, broadcaster=None):
    from fastapi import FastAPI
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI()
    loop_runner = EngineLoop(engine, broadcaster)
    names = [n.strip() for n in served_model_name.split(",") if n.strip()] or ["model"]
    app.state.engine_loop = loop_runner

    def err(msg, code=400):
        return JSONResponse({"error": {"message": msg, "type": "invalid_request_error", "code": code}},
                            status_code=code)

    @app.get("/health")
    async def health():
        if loop_runner.error and not loop_runner.thread.is_alive():
            return PlainTextResponse("engine dead", status_code=503)
        if loop_runner.kernel_fault:
            return PlainTextResponse("kernel fault: " + loop_runner.error, status_code=503)
        return PlainTextResponse("")

    @app.get("/version")
    async def version():
        from .. import __version__
        return {"version": __version__}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": n, "object": "model", "owned_by": "radiance",
                                            "max_model_len": engine.config.max_model_len}
                                           for n in names]}

    @app.get("/metrics")
    async def metrics():
        return PlainTextResponse(engine.metrics.prometheus(names[0]))

    async def _run(prompt, params, rid):
        q = loop_runner.submit(prompt, params, rid, asyncio.get_running_loop())
        while True:
            item = await q.get()
            if item is None:
                return
            yield item
            if isinstance(item, dict) or item.finished:
                return

    @app.post("/v1/completions")
    async def completions(req: FReq):
        body = await req.json()
        if body.get("model") and body["model"] not in names:
            return err(f"model {body['model']!r} not found", 404)
        prompt = body.get("prompt", "")
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], str):
            prompt = prompt[0]
        try:
            params = _sampling_from_body(body, 16)
        except ValueError as e:
            return err(str(e))
        rid = f"cmpl-{uuid.uuid4().hex}"
        created = int(time.time())
        if body.get("stream"):
            async def gen():
                sent = 0
                async for o in _run(prompt, params, rid):
                    if isinstance(o, dict):
                        yield f"data: {json.dumps({'error': o})}\n\n"
                        break
                    text = o.outputs[0].text
                    delta, sent = text[sent:], len(text)
                    chunk = {"id": rid, "object": "text_completion", "created": created,
                             "model": names[0], "choices": [{"index": 0, "text": delta,
                                                             "finish_reason": o.outputs[0].finish_reason}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        last = None
        async for o in _run(prompt, params, rid):
            last = o
        if last is None or isinstance(last, dict):
            return err(str(last), 500)
        out = last.outputs[0]
        n_prompt = len(last.prompt_token_ids)
        return {"id": rid, "object": "text_completion", "created": created, "model": names[0],
                "choices": [{"index": 0, "text": out.text, "finish_reason": out.finish_reason,
                             "token_ids": out.token_ids}],
                "usage": {"prompt_tokens": n_prompt, "completion_tokens": len(out.token_ids),
                          "total_tokens": n_prompt + len(out.token_ids)}}

    @app.post("/v1/chat/completions")
    async def chat(req: FReq):
        body = await req.json()
        if body.get("model") and body["model"] not in names:
            return err(f"model {body['model']!r} not found", 404)
        msgs = body.get("messages") or []
        kw = dict(body.get("chat_template_kwargs") or {})
        if body.get("tools"):
            kw["tools"] = body["tools"]
        try:
            prompt = engine.tokenizer.apply_chat_template(msgs, add_generation_prompt=True, **kw)
            params = _sampling_from_body(body, 256)
        except (ValueError, TypeError) as e:
            return err(str(e))
        rid = f"chatcmpl-{uuid.uuid4().hex}"
        created = int(time.time())
        rp = ReasoningParser(reasoning_parser, thinking=kw.get("enable_thinking", True)) \
            if reasoning_parser else None
        tp = ToolParser(tool_parser) if (tool_parser and body.get("tools")) else None
        if body.get("stream"):
            async def gen():
                sent = 0
                first = True
                async for o in _run(prompt, params, rid):
                    if isinstance(o, dict):
                        yield f"data: {json.dumps({'error': o})}\n\n"
                        break
                    text = o.outputs[0].text
                    delta_text, sent = text[sent:], len(text)
                    delta = {"role": "assistant"} if first else {}
                    first = False
                    if rp is not None:
                        r, c = rp.stream(delta_text)
                        if r:
                            delta["reasoning_content"] = r
                        if c:
                            delta["content"] = c
                    elif delta_text:
                        delta["content"] = delta_text
                    fr = o.outputs[0].finish_reason
                    if fr and tp is not None:
                        calls, _ = tp.parse(rp.content if rp else text)
                        if calls:
                            delta["tool_calls"] = [dict(c, index=i) for i, c in enumerate(calls)]
                            fr = "tool_calls"
                    chunk = {"id": rid, "object": "chat.completion.chunk", "created": created,
                             "model": names[0], "choices": [{"index": 0, "delta": delta,
                                                             "finish_reason": fr}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        last = None
        async for o in _run(prompt, params, rid):
            last = o
        if last is None or isinstance(last, dict):
            return err(str(last), 500)
        out = last.outputs[0]
        msg = {"role": "assistant", "content": out.text}
        fr = out.finish_reason
        if rp is not None:
            reasoning, content = rp.split(out.text)
            msg["content"] = content
            if reasoning is not None:
                msg["reasoning_content"] = reasoning
        if tp is not None:
            calls, rest = tp.parse(msg["content"] or "")
            if calls:
                msg["tool_calls"] = calls
                msg["content"] = rest or None
                fr = "tool_calls"
        n_prompt = len(last.prompt_token_ids)
        return {"id": rid, "object": "chat.completion", "created": created, "model": names[0],
                "choices": [{"index": 0, "message": msg, "finish_reason": fr}],
                "usage": {"prompt_tokens": n_prompt, "completion_tokens": len(out.token_ids),
                          "total_tokens": n_prompt + len(out.token_ids)}}

    return app
