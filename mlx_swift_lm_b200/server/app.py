"""OpenAI-compatible HTTP server wired directly to the continuous-batching engine.

Route manifest (parity: MLXLMServer/Routing/MLXServerRoute.swift:19-34):
  GET  /health /v1/health /metrics /props /v1/models /models
  POST /v1/chat/completions /chat/completions /v1/chat/completions/batch
  POST /v1/completions /completions /completion
  POST /v1/responses /responses ; GET /v1/responses/{id} ; POST /v1/responses/{id}/cancel
  POST /v1/embeddings /embeddings /embedding
  POST /tokenize /detokenize /apply-template
Unlike the reference's server (which serves one request at a time through the
single-request container, MLXServerRunner.swift:29-32), every request here is
submitted to EngineV2 running its step loop on a background thread, so
concurrent HTTP requests are batched together.
SSE framing, logprobs, tool-call deltas and reasoning fields follow the
OpenAI wire format (MLXLMServer/Protocol/*.swift).
"""
from __future__ import annotations

import asyncio
import json
import os
import time
import uuid

from starlette.applications import Starlette
from starlette.requests import Request as HTTPRequest
from starlette.responses import JSONResponse, PlainTextResponse, StreamingResponse
from starlette.routing import Route

from ..api.parsers import make_reasoning_parser, make_tool_parser
from ..engine.types import FinishReason, Request, SamplingParams
from .metrics import ServerMetrics

ROUTES = [
    ("GET", "/health"), ("GET", "/v1/health"), ("GET", "/metrics"), ("GET", "/props"), ("GET", "/v1/models"),
    ("GET", "/models"), ("POST", "/v1/chat/completions"), ("POST", "/chat/completions"),
    ("POST", "/v1/chat/completions/batch"), ("POST", "/v1/completions"), ("POST", "/completions"),
    ("POST", "/completion"), ("POST", "/v1/responses"), ("POST", "/responses"), ("GET", "/v1/responses/{response_id}"),
    ("POST", "/v1/responses/{response_id}/cancel"), ("POST", "/v1/embeddings"), ("POST", "/embeddings"),
    ("POST", "/embedding"), ("POST", "/tokenize"), ("POST", "/detokenize"), ("POST", "/apply-template"),
]


class ValidationError(ValueError):
    pass


def _err(msg, code=400, typ="invalid_request_error"):
    return JSONResponse({"error": {"message": msg, "type": typ, "code": code}}, status_code=code)


def validate_sampling(body: dict) -> SamplingParams:
    """Request validation (Runtime/OpenAIRequestValidation.swift)."""
    t = body.get("temperature", 1.0)
    if t is None:
        t = 1.0
    if not (0.0 <= float(t) <= 2.0):
        raise ValidationError("temperature must be in [0, 2]")
    top_p = float(body.get("top_p", 1.0) if body.get("top_p") is not None else 1.0)
    if not (0.0 < top_p <= 1.0):
        raise ValidationError("top_p must be in (0, 1]")
    n = body.get("n", 1)
    if n not in (None, 1):
        raise ValidationError("only n=1 is supported")
    for k in ("presence_penalty", "frequency_penalty"):
        v = body.get(k)
        if v is not None and not (-2.0 <= float(v) <= 2.0):
            raise ValidationError(f"{k} must be in [-2, 2]")
    top_lp = body.get("top_logprobs") or 0
    if top_lp and not (0 <= int(top_lp) <= 20):
        raise ValidationError("top_logprobs must be in [0, 20]")
    bias = {int(k): float(v) for k, v in (body.get("logit_bias") or {}).items()}
    return SamplingParams(temperature=float(t), top_p=top_p, top_k=int(body.get("top_k") or 0),
                          min_p=float(body.get("min_p") or 0.0),
                          repetition_penalty=float(body.get("repetition_penalty") or 1.0),
                          frequency_penalty=float(body.get("frequency_penalty") or 0.0),
                          presence_penalty=float(body.get("presence_penalty") or 0.0),
                          seed=body.get("seed"), logit_bias=bias, top_logprobs=int(top_lp),
                          logprobs=bool(body.get("logprobs")) or bool(top_lp))


def _decode_image(url: str):
    """A data: URL (base64) or a local file path -> an RGB PIL image. This
    server never fetches remote URLs."""
    import base64
    import io

    from PIL import Image

    if isinstance(url, str) and url.startswith("data:"):
        return Image.open(io.BytesIO(base64.b64decode(url.split(",", 1)[1]))).convert("RGB")
    if isinstance(url, str) and os.path.exists(url):
        return Image.open(url).convert("RGB")
    raise ValidationError("image_url must be a data: URL or a local file path")


class OpenAIService:
    def __init__(self, container, model_name: str = None, tool_parser: str | None = None,
                 reasoning_parser: str | None = None, embedder=None, default_max_tokens: int = 512,
                 constraint_factory=None):
        self.c = container
        self.engine = container.engine
        self.model_name = model_name or getattr(container, "model_id", "local")
        self.tool_parser_name = tool_parser
        self.reasoning_parser_name = reasoning_parser
        self.embedder = embedder
        self.metrics = ServerMetrics()
        self.default_max_tokens = default_max_tokens
        self.response_store: dict[str, dict] = {}
        self.constraint_factory = constraint_factory
        if not self.engine.background:
            self.engine.start()

    # ------------------------------------------------------------------ helpers
    def _max_tokens(self, body, n_prompt):
        mt = body.get("max_completion_tokens") or body.get("max_tokens") or body.get("max_output_tokens")
        mt = int(mt) if mt else self.default_max_tokens
        room = self.engine.cfg.max_model_len - n_prompt
        if room <= 0:
            raise ValidationError(f"prompt of {n_prompt} tokens exceeds the context window")
        return min(mt, room)

    def _constraint(self, body):
        rf = body.get("response_format")
        if not rf or rf.get("type") in (None, "text") or self.constraint_factory is None:
            return None
        return self.constraint_factory(rf)

    def _submit(self, tokens, body, sampling, mm=None):
        stop = body.get("stop") or []
        if isinstance(stop, str):
            stop = [stop]
        req = Request(prompt_tokens=list(tokens), max_tokens=self._max_tokens(body, len(tokens)), sampling=sampling,
                      stop_strings=list(stop), token_constraint=self._constraint(body),
                      cache_salt=body.get("cache_salt"), mm=mm)
        return self.engine.submit(req)

    @staticmethod
    def _split_images(msgs: list) -> tuple[list, list]:
        """OpenAI image parts (``image_url`` with a data: URL or a local path)
        -> ``{"type": "image"}`` parts for the chat template, plus the decoded
        images in order."""
        images, out = [], []
        for m in msgs:
            c = m.get("content")
            if not isinstance(c, list):
                out.append(m)
                continue
            parts = []
            for p in c:
                if isinstance(p, dict) and p.get("type") in ("image_url", "input_image", "image"):
                    url = p.get("image_url")
                    url = url.get("url") if isinstance(url, dict) else url or p.get("url") or p.get("image")
                    images.append(_decode_image(url))
                    parts.append({"type": "image"})
                else:
                    parts.append(p)
            out.append({**m, "content": parts})
        return out, images

    @staticmethod
    def _lp_json(lps, tok):
        if not lps:
            return None
        out = []
        for lp in lps:
            if lp is None:
                continue
            out.append({"token": tok.decode([lp.token]), "logprob": lp.logprob,
                        "top_logprobs": [{"token": tok.decode([i]), "logprob": v} for i, v in lp.top]})
        return out

    # ------------------------------------------------------------------ chat
    async def chat(self, body: dict, stream_override=None):
        self.metrics.inc("requests_total")
        self.metrics.inc("chat_requests_total")
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise ValidationError("messages must be a non-empty list")
        sampling = validate_sampling(body)
        tools = body.get("tools")
        msgs, images = self._split_images(msgs)
        tokens = self.c.apply_chat_template(msgs, tools=tools)
        mm = None
        if images:
            tokens, mm = self.c.prepare_media(tokens, images)
        stream = self._submit(tokens, body, sampling, mm)
        rid = "chatcmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())
        rp = make_reasoning_parser(body.get("reasoning_parser") or self.reasoning_parser_name)
        tp = make_tool_parser(self.tool_parser_name, tools) if tools else None
        want_stream = body.get("stream", False) if stream_override is None else stream_override
        if want_stream:
            return StreamingResponse(self._chat_sse(stream, rid, created, rp, tp, len(tokens), body),
                                     media_type="text/event-stream")
        text, reasoning, finish, usage, lps = [], [], None, None, []
        async for ev in stream:
            t = ev.text
            if rp is not None and t:
                r, t = rp.feed(t)
                reasoning.append(r)
            text.append(t)
            if ev.logprobs:
                lps.extend(ev.logprobs)
            if ev.finished:
                finish, usage = ev.finish_reason, ev.usage
        if rp is not None:
            r, t = rp.flush()
            reasoning.append(r)
            text.append(t)
        content = "".join(text)
        calls = []
        if tp is not None:
            content, calls = tp.parse(content)
        self._count_usage(usage)
        msg = {"role": "assistant", "content": content}
        if any(reasoning):
            msg["reasoning_content"] = "".join(reasoning)
        if calls:
            msg["tool_calls"] = [c.to_openai() for c in calls]
        choice = {"index": 0, "message": msg, "finish_reason": "tool_calls" if calls else _finish(finish)}
        if sampling.logprobs:
            choice["logprobs"] = {"content": self._lp_json(lps, self.c.tokenizer)}
        return JSONResponse({"id": rid, "object": "chat.completion", "created": created, "model": self.model_name,
                             "choices": [choice], "usage": _usage(usage)})

    async def _chat_sse(self, stream, rid, created, rp, tp, n_prompt, body):
        def frame(delta, finish=None, extra=None):
            d = {"id": rid, "object": "chat.completion.chunk", "created": created, "model": self.model_name,
                 "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}
            if extra:
                d.update(extra)
            return f"data: {json.dumps(d)}\n\n"

        yield frame({"role": "assistant", "content": ""})
        usage, finish = None, None
        buffered = []
        async for ev in stream:
            t = ev.text
            if rp is not None and t:
                r, t = rp.feed(t)
                if r:
                    yield frame({"reasoning_content": r})
            if t:
                if tp is not None:
                    c, calls = tp.feed(t)
                    if c:
                        yield frame({"content": c})
                    for i, call in enumerate(calls):
                        yield frame({"tool_calls": [{"index": len(buffered) + i, **call.to_openai()}]})
                    buffered.extend(calls)
                else:
                    yield frame({"content": t})
            if ev.finished:
                finish, usage = ev.finish_reason, ev.usage
        if rp is not None:
            r, t = rp.flush()
            if r:
                yield frame({"reasoning_content": r})
            if t:
                if tp is not None:
                    c, calls = tp.feed(t)
                    if c:
                        yield frame({"content": c})
                    for i, call in enumerate(calls):
                        yield frame({"tool_calls": [{"index": len(buffered) + i, **call.to_openai()}]})
                    buffered.extend(calls)
                else:
                    yield frame({"content": t})
        if tp is not None:  # a frame cut off by end-of-sequence, or content held back at the end
            c, calls = tp.flush()
            if c:
                yield frame({"content": c})
            for i, call in enumerate(calls):
                yield frame({"tool_calls": [{"index": len(buffered) + i, **call.to_openai()}]})
            buffered.extend(calls)
        self._count_usage(usage)
        fin = "tool_calls" if buffered else _finish(finish)
        extra = {"usage": _usage(usage)} if (body.get("stream_options") or {}).get("include_usage") else None
        yield frame({}, fin, extra)
        yield "data: [DONE]\n\n"

    # ------------------------------------------------------------------ completions
    async def completions(self, body: dict):
        self.metrics.inc("requests_total")
        self.metrics.inc("completion_requests_total")
        prompt = body.get("prompt")
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], int):
            tokens = prompt
        elif isinstance(prompt, str):
            tokens = self.c.encode(prompt)
        else:
            raise ValidationError("prompt must be a string or a list of token ids")
        sampling = validate_sampling(body)
        stream = self._submit(tokens, body, sampling)
        rid = "cmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())
        echo = self.c.decode(tokens) if body.get("echo") else ""
        if body.get("stream"):
            async def gen():
                usage = fin = None
                if echo:
                    yield "data: " + json.dumps(_cmpl_chunk(rid, created, self.model_name, echo, None)) + "\n\n"
                async for ev in stream:
                    if ev.text:
                        yield "data: " + json.dumps(_cmpl_chunk(rid, created, self.model_name, ev.text, None)) + "\n\n"
                    if ev.finished:
                        fin, usage = ev.finish_reason, ev.usage
                self._count_usage(usage)
                yield "data: " + json.dumps(_cmpl_chunk(rid, created, self.model_name, "", _finish(fin))) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        text, fin, usage = [echo], None, None
        async for ev in stream:
            text.append(ev.text)
            if ev.finished:
                fin, usage = ev.finish_reason, ev.usage
        self._count_usage(usage)
        return JSONResponse({"id": rid, "object": "text_completion", "created": created, "model": self.model_name,
                             "choices": [{"index": 0, "text": "".join(text), "finish_reason": _finish(fin),
                                          "logprobs": None}], "usage": _usage(usage)})

    # ------------------------------------------------------------------ responses
    async def responses(self, body: dict):
        self.metrics.inc("requests_total")
        self.metrics.inc("response_requests_total")
        inp = body.get("input")
        msgs = []
        if body.get("instructions"):
            msgs.append({"role": "system", "content": body["instructions"]})
        if isinstance(inp, str):
            msgs.append({"role": "user", "content": inp})
        elif isinstance(inp, list):
            for m in inp:
                c = m.get("content")
                if isinstance(c, list):
                    c = "".join(p.get("text", "") for p in c if isinstance(p, dict))
                msgs.append({"role": m.get("role", "user"), "content": c})
        else:
            raise ValidationError("input must be a string or a list of messages")
        prev = body.get("previous_response_id")
        if prev and prev in self.response_store:
            msgs = self.response_store[prev]["_messages"] + msgs
        sampling = validate_sampling(body)
        tokens = self.c.apply_chat_template(msgs)
        stream = self._submit(tokens, body, sampling)
        resp_id = "resp_" + uuid.uuid4().hex[:24]
        rec = {"id": resp_id, "object": "response", "created_at": int(time.time()), "model": self.model_name,
               "status": "in_progress", "output": [], "_messages": msgs, "_stream": stream}
        self.response_store[resp_id] = rec
        text, fin, usage = [], None, None
        async for ev in stream:
            text.append(ev.text)
            if ev.finished:
                fin, usage = ev.finish_reason, ev.usage
        out_text = "".join(text)
        rec["status"] = "cancelled" if fin == FinishReason.CANCELLED else "completed"
        rec["output"] = [{"type": "message", "id": "msg_" + uuid.uuid4().hex[:16], "role": "assistant",
                          "content": [{"type": "output_text", "text": out_text, "annotations": []}]}]
        rec["output_text"] = out_text
        rec["usage"] = {"input_tokens": usage.prompt_tokens if usage else 0,
                        "output_tokens": usage.completion_tokens if usage else 0,
                        "total_tokens": usage.total_tokens if usage else 0}
        rec["_messages"] = msgs + [{"role": "assistant", "content": out_text}]
        self._count_usage(usage)
        return JSONResponse(_public(rec))

    # ------------------------------------------------------------------ embeddings
    async def embeddings(self, body: dict):
        self.metrics.inc("requests_total")
        self.metrics.inc("embedding_requests_total")
        inp = body.get("input")
        texts = [inp] if isinstance(inp, str) else list(inp or [])
        if not texts:
            raise ValidationError("input must be a string or a non-empty list")
        emb = self.embedder or self.c
        vecs = await asyncio.get_running_loop().run_in_executor(None, emb.embed, texts)
        if hasattr(vecs, "tolist"):  # api.embed.Embedder returns one [N, dim] tensor
            vecs = vecs.float().cpu().tolist()
        data = [{"object": "embedding", "index": i, "embedding": v} for i, v in enumerate(vecs)]
        n = sum(len(self.c.encode(t)) if isinstance(t, str) else len(t) for t in texts)
        return JSONResponse({"object": "list", "data": data, "model": self.model_name,
                             "usage": {"prompt_tokens": n, "total_tokens": n}})

    def _count_usage(self, usage):
        if usage is None:
            return
        self.metrics.inc("prompt_tokens_total", usage.prompt_tokens)
        self.metrics.inc("completion_tokens_total", usage.completion_tokens)
        self.metrics.inc("cached_prompt_tokens_total", usage.cached_prompt_tokens)


def _finish(f):
    if f is None:
        return "stop"
    return {"stop": "stop", "length": "length"}.get(f.value, f.value)


def _usage(u):
    if u is None:
        return {"prompt_tokens": 0, "completion_tokens": 0, "total_tokens": 0}
    return {"prompt_tokens": u.prompt_tokens, "completion_tokens": u.completion_tokens,
            "total_tokens": u.total_tokens, "prompt_tokens_details": {"cached_tokens": u.cached_prompt_tokens}}


def _cmpl_chunk(rid, created, model, text, finish):
    return {"id": rid, "object": "text_completion", "created": created, "model": model,
            "choices": [{"index": 0, "text": text, "finish_reason": finish, "logprobs": None}]}


def _public(rec):
    return {k: v for k, v in rec.items() if not k.startswith("_")}


def build_app(service: OpenAIService) -> Starlette:
    s = service

    def wrap(fn):
        async def handler(request: HTTPRequest):
            try:
                body = await request.json() if request.method == "POST" else {}
            except Exception:
                return _err("request body is not valid JSON")
            try:
                return await fn(request, body)
            except ValidationError as e:
                s.metrics.inc("errors_total")
                return _err(str(e))
            except Exception as e:  # pragma: no cover - surfaced as 500
                s.metrics.inc("errors_total")
                return _err(repr(e), 500, "server_error")
        return handler

    async def health(req, body):
        ok = s.engine.healthy
        return JSONResponse({"status": "ok" if ok else "unhealthy"}, status_code=200 if ok else 503)

    async def metrics(req, body):
        return PlainTextResponse(s.metrics.render(s.engine), media_type="text/plain; version=0.0.4")

    async def props(req, body):
        cfg = s.engine.cfg
        return JSONResponse({"model": s.model_name, "max_model_len": cfg.max_model_len,
                             "max_concurrent_requests": cfg.scheduler.max_concurrent_requests,
                             "tool_call_parser": s.tool_parser_name, "reasoning_parser": s.reasoning_parser_name,
                             "routes": [f"{m} {p}" for m, p in ROUTES]})

    async def models(req, body):
        return JSONResponse({"object": "list", "data": [{"id": s.model_name, "object": "model", "owned_by": "local",
                                                         "created": int(s.metrics.start)}]})

    async def chat(req, body):
        return await s.chat(body)

    async def chat_batch(req, body):
        reqs = body.get("requests")
        if not isinstance(reqs, list):
            raise ValidationError("requests must be a list of chat completion requests")
        outs = await asyncio.gather(*[s.chat(r, stream_override=False) for r in reqs])
        return JSONResponse({"object": "list", "data": [json.loads(o.body) for o in outs]})

    async def completions(req, body):
        return await s.completions(body)

    async def responses(req, body):
        return await s.responses(body)

    async def get_response(req, body):
        rec = s.response_store.get(req.path_params["response_id"])
        return JSONResponse(_public(rec)) if rec else _err("response not found", 404, "not_found")

    async def cancel_response(req, body):
        rec = s.response_store.get(req.path_params["response_id"])
        if not rec:
            return _err("response not found", 404, "not_found")
        st = rec.get("_stream")
        if st is not None:
            s.engine.cancel(st.request_id)
        rec["status"] = "cancelled"
        return JSONResponse(_public(rec))

    async def embeddings(req, body):
        return await s.embeddings(body)

    async def tokenize(req, body):
        content = body.get("content", body.get("prompt", ""))
        return JSONResponse({"tokens": s.c.encode(content)})

    async def detokenize(req, body):
        return JSONResponse({"content": s.c.decode(body.get("tokens", []))})

    async def apply_template(req, body):
        msgs = body.get("messages") or []
        prompt = s.c.tokenizer.apply_chat_template(msgs, tools=body.get("tools"), add_generation_prompt=True,
                                                   tokenize=False)
        return JSONResponse({"prompt": prompt})

    table = {"/health": health, "/v1/health": health, "/metrics": metrics, "/props": props, "/v1/models": models,
             "/models": models, "/v1/chat/completions": chat, "/chat/completions": chat,
             "/v1/chat/completions/batch": chat_batch, "/v1/completions": completions, "/completions": completions,
             "/completion": completions, "/v1/responses": responses, "/responses": responses,
             "/v1/responses/{response_id}": get_response, "/v1/responses/{response_id}/cancel": cancel_response,
             "/v1/embeddings": embeddings, "/embeddings": embeddings, "/embedding": embeddings, "/tokenize": tokenize,
             "/detokenize": detokenize, "/apply-template": apply_template}
    routes = [Route(p, wrap(table[p]), methods=[m]) for m, p in ROUTES]
    return Starlette(routes=routes)
