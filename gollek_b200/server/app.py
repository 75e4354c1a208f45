"""HTTP API: OpenAI-compatible routes plus the gollek platform routes.

OpenAI surface (runner/safetensor/gollek-safetensor-api/…/OpenAiCompatibleResource.java:32-462):
  POST /v1/chat/completions (JSON, or SSE ``chat.completion.chunk`` frames + ``[DONE]`` when
  ``stream``), POST /v1/chat/completions/stream, POST /v1/completions, GET /v1/models[/{id}],
  POST /v1/embeddings. Defaults as the reference: temperature 0.7, top_p 0.95, top_k 50,
  max_tokens 2048 (capped by the model length).
gollek surface (inference/gollek-api-rest/…/api/rest/InferenceResource.java:46-266):
  POST /v1/infer/completions → {requestId, content, model, tokensUsed, promptTokens, completionTokens,
  durationMs, timestamp}
  POST /v1/infer/async → {jobId}; GET /v1/infer/async/{jobId}; POST /v1/infer/stream (SSE of
  {index, content, isFinal}); POST /v1/infer/batch; POST /v1/infer/embeddings;
  DELETE /v1/infer/{requestId}. The same routes are served under /v1/inference/* (the path the
  reference SDK calls, sdk/gollek-sdk-java-remote/…/GollekClient.java:96) and POST
  /api/v1/inference (the path its bench script posts to, scripts/bench-multilora-zipf.sh:33).
Operations: GET /health, /q/health[/live|/ready], /metrics (Prometheus), /v1/system, /v1/providers,
optional API-key auth (``Authorization: Bearer`` or ``X-API-Key``; ui/gollek-server-api/…/
SecurityFilter.java), bulkhead / circuit breaker / per-key rate limit / request timeout.
Token counts are real (the reference estimates chars/4, OpenAiCompatibleResource.java:372).
"""
from __future__ import annotations

import asyncio
import contextvars
import json
import re
import os
import time
import uuid
from datetime import datetime, timezone
from typing import Any, Dict, List, Optional, Union

from fastapi import FastAPI, Header, HTTPException, Request
from fastapi.responses import JSONResponse, PlainTextResponse, Response, StreamingResponse
from pydantic import BaseModel, Field

from .. import errors
from ..engine.sequence import SamplingParams
from .async_engine import AsyncEngine, EngineDeadError
from .resilience import Bulkhead, BulkheadFull, CircuitBreaker, CircuitOpen, RateLimited, RateLimiter
from .tools import may_hold_tool_call, messages_for_template, parse_tool_calls, tool_choice_regex


# ----------------------------------------------------------------------------- schemas
class ChatMessage(BaseModel):
    role: str = "user"
    content: Union[str, List[Dict[str, Any]], None] = ""
    name: Optional[str] = None
    tool_calls: Optional[List[Dict[str, Any]]] = None
    tool_call_id: Optional[str] = None


class ChatRequest(BaseModel):
    model: Optional[str] = None
    messages: List[ChatMessage]
    max_tokens: Optional[int] = None
    max_completion_tokens: Optional[int] = None
    temperature: Optional[float] = None
    top_p: Optional[float] = None
    top_k: Optional[int] = None
    min_p: Optional[float] = None
    stop: Union[str, List[str], None] = None
    stream: bool = False
    seed: Optional[int] = None
    presence_penalty: Optional[float] = None
    frequency_penalty: Optional[float] = None
    repetition_penalty: Optional[float] = None
    n: int = 1
    user: Optional[str] = None
    adapter_id: Optional[str] = None
    logprobs: Optional[bool] = None
    top_logprobs: Optional[int] = None
    typical_p: Optional[float] = None
    mirostat: Optional[int] = None
    mirostat_tau: Optional[float] = None
    tools: Optional[List[Dict[str, Any]]] = None
    tool_choice: Union[str, Dict[str, Any], None] = None
    parallel_tool_calls: Optional[bool] = None
    mirostat_eta: Optional[float] = None
    response_format: Optional[Dict[str, Any]] = None
    guided_regex: Optional[str] = None
    rag: Optional[Dict[str, Any]] = None  # {"collection": name, "top_k": 4, "max_context_tokens": 1024}
    mcp: bool = False  # offer the tools of the connected MCP servers (named <server>__<tool>)


class CompletionRequest(BaseModel):
    model: Optional[str] = None
    prompt: Union[str, List[int], List[str], List[List[int]]] = ""
    max_tokens: Optional[int] = 16
    temperature: Optional[float] = None
    top_p: Optional[float] = None
    top_k: Optional[int] = None
    min_p: Optional[float] = None
    stop: Union[str, List[str], None] = None
    stream: bool = False
    seed: Optional[int] = None
    presence_penalty: Optional[float] = None
    frequency_penalty: Optional[float] = None
    repetition_penalty: Optional[float] = None
    ignore_eos: bool = False
    n: int = 1
    adapter_id: Optional[str] = None
    logprobs: Optional[int] = None
    typical_p: Optional[float] = None
    mirostat: Optional[int] = None
    mirostat_tau: Optional[float] = None
    mirostat_eta: Optional[float] = None
    response_format: Optional[Dict[str, Any]] = None
    guided_regex: Optional[str] = None
    use_beam_search: bool = False
    best_of: Optional[int] = None            # beam width (default max(n, 4))
    length_penalty: float = 1.0
    early_stopping: bool = False


class EmbeddingRequest(BaseModel):
    model: Optional[str] = None
    input: Union[str, List[str], List[int], List[List[int]]]


class InferMessage(BaseModel):
    role: str = "user"
    content: Optional[str] = ""


class InferRequest(BaseModel):
    model: Optional[str] = None
    messages: List[InferMessage] = Field(default_factory=list)
    prompt: Optional[str] = None
    parameters: Dict[str, Any] = Field(default_factory=dict)
    timeout: int = 0
    priority: int = 0
    requestId: Optional[str] = None


# ----------------------------------------------------------------------------- helpers
def _now() -> int:
    return int(time.time())


def _param(p: Dict[str, Any], *names, default=None):
    for n in names:
        if n in p and p[n] is not None:
            return p[n]
    return default


_TENANT = contextvars.ContextVar("gollek_tenant", default="")


_ROUTED: contextvars.ContextVar = contextvars.ContextVar("gollek_routed_model", default=None)


class ServerState:
    """Server-wide state. ``ae`` / ``model_name`` are the engine and name serving the current request:
    the model router (``route``) picks one of ``routes`` by the request's ``model`` field, anything
    else goes to the primary engine (the one hot-swap replaces)."""

    def __init__(self, aengine: AsyncEngine, model_name: str, api_keys=None,
                 rate: float = 0.0, burst: float = 0.0, request_timeout: float = 600.0,
                 max_concurrent: int = 1024, max_queue: int = 4096):
        self._ae = aengine
        self._model_name = model_name
        self.routes: Dict[str, AsyncEngine] = {}  # extra served models by name
        # API key -> tenant ("" = no tenant); a list of keys means keys without tenants
        self.api_keys: Dict[str, str] = dict(api_keys) if isinstance(api_keys, dict) else \
            {k: "" for k in (api_keys or [])}
        self.admin_key = os.environ.get("GOLLEK_ADMIN_KEY", "")
        self.bulkhead = Bulkhead(max_concurrent, max_queue)
        self.breaker = CircuitBreaker()
        self.limiter = RateLimiter(rate, burst)
        self.timeout = request_timeout
        self.jobs: Dict[str, Dict[str, Any]] = {}
        self.adapters: Dict[str, int] = {}  # adapter name -> engine LoRA id

    @property
    def ae(self) -> AsyncEngine:
        r = _ROUTED.get()
        return self.routes[r] if (r is not None and r in self.routes) else self._ae

    @ae.setter
    def ae(self, value: AsyncEngine) -> None:
        self._ae = value

    @property
    def model_name(self) -> str:
        r = _ROUTED.get()
        return r if (r is not None and r in self.routes) else self._model_name

    @model_name.setter
    def model_name(self, value: str) -> None:
        self._model_name = value

    def route(self, model: Optional[str]) -> str:
        """Select the engine for this request (by name; unknown or empty names go to the primary)."""
        _ROUTED.set(model if (model and model in self.routes) else None)
        return self.model_name

    @property
    def engine(self):
        return self.ae.engine

    @property
    def tokenizer(self):
        return self.engine.tokenizer

    def max_len(self) -> int:
        return self.engine.cfg.max_model_len

    def lora_id(self, name: Optional[str]) -> int:
        if not name:
            return 0
        lm = getattr(self.engine, "lora_manager", None)
        if lm is None or name not in lm.name_to_id:
            raise HTTPException(404, f"unknown adapter {name!r}")
        return lm.name_to_id[name]


def build_sampling(st: ServerState, d: Dict[str, Any], defaults: Dict[str, Any]) -> SamplingParams:
    stop = _param(d, "stop", default=[]) or []
    if isinstance(stop, str):
        stop = [stop]
    sp = SamplingParams(
        temperature=float(_param(d, "temperature", default=defaults["temperature"])),
        top_p=float(_param(d, "top_p", "topP", default=defaults["top_p"])),
        top_k=int(_param(d, "top_k", "topK", default=defaults["top_k"])),
        min_p=float(_param(d, "min_p", "minP", default=0.0)),
        repetition_penalty=float(_param(d, "repetition_penalty", "repeat_penalty", "repetitionPenalty",
                                        default=defaults.get("repetition_penalty", 1.0))),
        frequency_penalty=float(_param(d, "frequency_penalty", "frequencyPenalty", default=0.0)),
        presence_penalty=float(_param(d, "presence_penalty", "presencePenalty", default=0.0)),
        max_tokens=int(_param(d, "max_tokens", "max_completion_tokens", "maxTokens",
                              default=defaults["max_tokens"])),
        stop=list(stop),
        seed=_param(d, "seed"),
        ignore_eos=bool(_param(d, "ignore_eos", default=False)),
        typical_p=float(_param(d, "typical_p", "typicalP", default=1.0)),
        mirostat=int(_param(d, "mirostat", default=0)),
        mirostat_tau=float(_param(d, "mirostat_tau", default=5.0)),
        mirostat_eta=float(_param(d, "mirostat_eta", default=0.1)),
    )
    rf = _param(d, "response_format") or {}
    if isinstance(rf, dict) and rf.get("type") in ("json_object", "json_schema"):
        sp.guided_json = True  # any JSON object (a json_schema's structure is not enforced)
    if _param(d, "guided_json", "json"):
        sp.guided_json = True
    rx = _param(d, "guided_regex", "regex")
    if rx:
        sp.guided_regex = str(rx)
    lp = _param(d, "logprobs")
    if lp is True:  # chat: logprobs=true + top_logprobs=k
        sp.logprobs = int(_param(d, "top_logprobs", default=0) or 0)
    elif lp is not None and lp is not False:
        sp.logprobs = int(lp)
    try:
        return sp.validate()
    except ValueError as e:
        raise HTTPException(400, str(e))


OPENAI_DEFAULTS = dict(temperature=0.7, top_p=0.95, top_k=50, max_tokens=2048, repetition_penalty=1.0)


class RagDocument(BaseModel):
    id: Optional[str] = None
    content: str


class RagIngestRequest(BaseModel):
    collection: str
    documents: List[RagDocument]
    chunk_size: int = 800          # characters per chunk
    chunk_overlap: int = 100
    embeddingModel: Optional[str] = None


class RagQueryRequest(BaseModel):
    collection: str
    question: str
    topK: Optional[int] = None
    top_k: Optional[int] = None
    maxTokens: Optional[int] = None
    max_tokens: Optional[int] = None
    temperature: Optional[float] = None
    max_context_tokens: int = 1024
    min_similarity: float = -1.0
    llmModel: Optional[str] = None
    embeddingModel: Optional[str] = None


def create_app(aengine: AsyncEngine, model_name: str = "gollek-b200", api_keys: Optional[List[str]] = None,
               rate: float = 0.0, burst: float = 0.0, request_timeout: float = 600.0,
               engine_builder=None, drain_timeout_s: float = 30.0,
               routes: Optional[Dict[str, AsyncEngine]] = None, asr=None, tts=None,
               providers=None) -> FastAPI:
    """``engine_builder(model) -> LLMEngine`` builds the engine of a hot-swap (default: the running
    engine's configuration with ``model`` replaced). ``asr``: a ``WhisperASR`` behind the
    /v1/audio transcription endpoints; ``tts``: a ``SpeechSynth`` behind /v1/audio/speech."""
    st = ServerState(aengine, model_name, api_keys, rate, burst, request_timeout)
    st.routes.update(routes or {})
    from .providers import OpenAIHTTPProvider, ProviderRegistry, ProviderRouter, _ClientError
    st.providers = providers if providers is not None else ProviderRegistry()
    st.provider_router = ProviderRouter(st.providers)
    from .rag import RagStore
    st.rag = RagStore()
    from .plugins import ServerPlugins, UnsafeContent, redact_pii, split_reasoning
    st.plugins = ServerPlugins.from_env()
    from .mcp import MCPError, MCPRegistry, tool_text
    st.mcp = MCPRegistry()
    gollek_defaults = dict(vars(aengine.engine.cfg.sampling))
    app = FastAPI(title="gollek-b200", version="0.1")
    app.state.server = st
    from .converter import register_converter_routes
    st.converter = register_converter_routes(app)
    from .audio import register_audio_routes
    st.asr = register_audio_routes(app, asr, tts)

    def error_response(name: str, message: Optional[str] = None, status: Optional[int] = None) -> JSONResponse:
        code = errors.CODES[name]
        return JSONResponse({"error": errors.payload(code, message)}, status_code=status or code.http)

    @app.exception_handler(HTTPException)
    async def http_error(request: Request, exc: HTTPException):
        code = errors.CODES.get(getattr(exc, "gollek_code", "")) or errors.for_http(exc.status_code)
        body = errors.payload(code, str(exc.detail))
        body["httpStatus"] = exc.status_code
        return JSONResponse({"error": body}, status_code=exc.status_code)

    # -------------------------------------------------------------- middleware
    @app.middleware("http")
    async def auth_and_limits(request: Request, call_next):
        path = request.url.path
        open_paths = ("/health", "/q/health", "/metrics", "/docs", "/openapi.json")
        key = request.headers.get("x-api-key")
        auth = request.headers.get("authorization", "")
        if auth.lower().startswith("bearer "):
            key = auth[7:].strip()
        if path.startswith("/v1/admin"):
            if (st.admin_key or st.api_keys) and key != st.admin_key:
                return error_response("AUTH_FORBIDDEN", "admin routes need GOLLEK_ADMIN_KEY")
        elif st.api_keys and not path.startswith(open_paths):
            if key not in st.api_keys:
                return error_response("AUTH_INVALID_KEY")
        tenant = st.api_keys.get(key, "") if key else ""
        _TENANT.set(tenant or request.headers.get("x-tenant-id", ""))
        try:
            st.limiter.check(key or (request.client.host if request.client else "anon"))
        except RateLimited as e:
            return error_response("RATE_LIMIT_EXCEEDED", str(e))
        return await call_next(request)

    # -------------------------------------------------------------- core runner
    async def run_full(prompt, sp: SamplingParams, rid: Optional[str] = None, lora_id: int = 0,
                       priority: int = 0, timeout: Optional[float] = None, images: Optional[list] = None):
        try:
            st.breaker.before()
        except CircuitOpen as e:
            raise HTTPException(503, str(e))
        try:
            async with st.bulkhead:
                last = None

                async def consume():
                    nonlocal last
                    async for out in st.ae.generate(prompt, sp, request_id=rid, lora_id=lora_id, priority=priority,
                                                    tenant=_TENANT.get(), images=images):
                        last = out

                await asyncio.wait_for(consume(), timeout=timeout or st.timeout)
            st.breaker.record(True)
            return last
        except BulkheadFull as e:
            raise HTTPException(429, str(e))
        except asyncio.TimeoutError:
            st.breaker.record(False)
            raise HTTPException(504, "request timed out")
        except EngineDeadError as e:
            st.breaker.record(False)
            raise HTTPException(503, str(e))
        except ValueError as e:
            raise HTTPException(400, str(e))

    def detok(ids: List[int]) -> str:
        ids = [t for t in list(ids) if t >= 0]  # async scheduling: a token may still be in flight
        return st.tokenizer.decode(ids) if st.tokenizer is not None else " ".join(map(str, ids))

    def chat_prompt(messages, tools: Optional[List[dict]] = None) -> Union[str, List[int]]:
        if st.tokenizer is None:
            raise HTTPException(400, "model has no tokenizer for chat messages")
        msgs = messages_for_template([m if isinstance(m, dict) else m.model_dump(exclude_none=True) for m in messages])
        tmpl = getattr(st.tokenizer, "apply_chat_template", None)
        if tmpl is None:
            return "\n".join(str(m.get("content", "")) for m in msgs)
        return tmpl(msgs, tools=tools) if tools else tmpl(msgs)

    async def sse_stream(prompt, sp, rid, lora_id, frame, final_frame, done_marker=True, tool_frame=None,
                         images=None):
        """Server-sent events of the text deltas. With ``tool_frame``, text from where a tool call may
        begin is held back; at the end it is sent as one tool-call frame if it parses as calls, else
        as text."""
        prev = ""

        async def gen():
            nonlocal prev
            try:
                async for out in st.ae.generate(prompt, sp, request_id=rid, lora_id=lora_id, tenant=_TENANT.get(),
                                                images=images):
                    text = detok(out.output_token_ids)
                    if out.finished and out.text:
                        text = out.text
                    visible = text
                    if tool_frame is not None:
                        if out.finished:
                            content, calls = parse_tool_calls(text)
                            if calls:
                                if content.startswith(prev) and len(content) > len(prev):
                                    yield "data: " + json.dumps(frame(content[len(prev):], None)) + "\n\n"
                                yield "data: " + json.dumps(tool_frame(calls, out)) + "\n\n"
                                yield "data: " + json.dumps(final_frame(out)) + "\n\n"
                                break
                        else:
                            hold = may_hold_tool_call(text)
                            visible = text if hold < 0 else text[:hold]
                    delta = visible[len(prev):] if visible.startswith(prev) else visible
                    prev = visible
                    if delta or out.finished:
                        yield "data: " + json.dumps(frame(delta, out)) + "\n\n"
                    if out.finished:
                        yield "data: " + json.dumps(final_frame(out)) + "\n\n"
                if done_marker:
                    yield "data: [DONE]\n\n"
            except (EngineDeadError, ValueError) as e:
                yield "data: " + json.dumps({"error": {"message": str(e)}}) + "\n\n"

        return StreamingResponse(gen(), media_type="text/event-stream")

    # -------------------------------------------------------------- health / ops
    @app.get("/health")
    @app.get("/q/health")
    @app.get("/q/health/live")
    async def health():
        ok = st.ae.healthy
        return JSONResponse({"status": "UP" if ok else "DOWN", "checks": [{"name": "engine", "status": "UP" if ok else "DOWN"}]},
                            status_code=200 if ok else 503)

    @app.get("/q/health/ready")
    async def ready():
        ok = st.ae.healthy and not st.ae.draining
        return JSONResponse({"status": "UP" if ok else "DOWN"}, status_code=200 if ok else 503)

    # -------------------------------------------------------------- KV eviction (EVICPRESS routes)
    @app.get("/v1/kvcache/stats")
    async def kvcache_stats():
        e = st.engine
        ev = e.evictor
        d = {"kv_total_blocks": e.kv.num_blocks, "kv_free_blocks": e.kv.num_free_blocks(),
             "kv_utilization": e.kv.usage(), "eviction_enabled": ev is not None}
        if ev is not None:
            d.update({"eviction_threshold": ev.threshold, "retention_target": ev.retention_target,
                      **{f"total_{k}": v for k, v in ev.stats.as_dict().items()}})
        return d

    @app.put("/v1/kvcache/retention")
    async def kvcache_retention(target: float):
        ev = st.engine.evictor
        if ev is None:
            raise HTTPException(409, "KV eviction is disabled (kv_eviction=false)")
        if not 0.0 < target <= 1.0:
            raise HTTPException(400, "target must be in (0, 1]")
        old, ev.retention_target = ev.retention_target, target
        return {"previous": old, "current": target}

    @app.post("/v1/kvcache/evict-now")
    async def kvcache_evict_now():
        if st.engine.evictor is None:
            raise HTTPException(409, "KV eviction is disabled (kv_eviction=false)")
        freed = await st.ae.call(lambda eng: eng.evictor.run(eng, force=True))
        return {"blocks_dropped": freed, "utilization": st.engine.kv.usage()}

    @app.get("/metrics")
    async def metrics():
        return PlainTextResponse(st.engine.metrics.prometheus())

    @app.get("/v1/system")
    async def system():
        import torch
        e = st.engine
        info = {"model": st.model_name, "device": str(e.device), "dtype": str(e.dtype),
                "tensor_parallel_size": e.comm.size, "kv_blocks": e.num_blocks, "block_size": e.cfg.block_size,
                "max_model_len": e.cfg.max_model_len, "metrics": e.metrics.snapshot()}
        if torch.cuda.is_available():
            info["gpu"] = torch.cuda.get_device_name(e.device)
        return info

    @app.get("/v1/providers")
    async def providers():
        return {"providers": [{"id": "gollek-b200", "type": "local", "formats": ["safetensors", "gguf"],
                               "healthy": st.ae.healthy, "models": [st.model_name]}]}

    # -------------------------------------------------------------- OpenAI
    @app.get("/v1/models")
    async def models():
        data = [{"id": st.model_name, "object": "model", "created": _now(), "owned_by": "gollek-b200",
                 "max_model_len": st.max_len()}]
        data += [{"id": n, "object": "model", "created": _now(), "owned_by": "gollek-b200",
                  "max_model_len": e.engine.cfg.max_model_len} for n, e in st.routes.items()]
        local = {d["id"] for d in data}
        for p in st.providers.all():
            data += [{"id": m, "object": "model", "created": _now(), "owned_by": p.id}
                     for m in p.models() if m not in local]
        return {"object": "list", "data": data}

    @app.get("/v1/models/{model_id}")
    async def model(model_id: str):
        if model_id != st.model_name:
            raise HTTPException(404, f"model {model_id} not found")
        return {"id": st.model_name, "object": "model", "created": _now(), "owned_by": "gollek-b200"}

    async def beam_completions(req: CompletionRequest, batch, lora: int, cid: str):
        from ..engine.beam import BeamParams, abeam_search
        if req.stream:
            raise HTTPException(400, "beam search does not stream")
        width = req.best_of or max(req.n, 4)
        try:
            bp = BeamParams(beam_width=width, max_tokens=req.max_tokens or 16, length_penalty=req.length_penalty,
                            early_stopping=req.early_stopping, num_return=req.n, ignore_eos=req.ignore_eos)
        except ValueError as e:
            raise HTTPException(400, str(e))

        async def expand(prefix, sp):
            return await run_full(prefix, sp, lora_id=lora)

        choices, pt, ct = [], 0, 0
        for p in batch:
            ids = list(p) if isinstance(p, list) else (st.tokenizer.encode(p) if st.tokenizer is not None else None)
            if ids is None:
                raise HTTPException(400, "model has no tokenizer")
            hyps = await abeam_search(expand, ids, bp, st.engine.eos_token_id)
            for h in hyps:
                choices.append({"index": len(choices), "text": detok(h.tokens), "finish_reason": h.finish_reason,
                                "logprobs": None, "score": h.score(bp.length_penalty)})
                ct += len(h.tokens)
            pt += len(ids)
        return {"id": cid, "object": "text_completion", "created": _now(), "model": st.model_name, "choices": choices,
                "usage": {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct}}

    def _remote(model: Optional[str]) -> bool:
        """A model that no local engine serves but a registered provider does."""
        return bool(model) and model != st._model_name and model not in st.routes and \
            any(p.supports(model) for p in st.providers.all())

    async def _forward(route: str, req):
        body = req.model_dump(exclude_unset=True)
        if body.get("stream"):
            d = st.provider_router.route(body["model"], streaming=True)
            p = st.providers.get(d.provider)
            if not isinstance(p, OpenAIHTTPProvider):
                raise HTTPException(400, f"provider {d.provider} does not stream")
            return StreamingResponse(p.stream(route, body), media_type="text/event-stream")
        try:
            out = await asyncio.to_thread(st.provider_router.execute, route, body)
        except Exception as e:  # every provider failed
            return error_response("RUNTIME_ENGINE_UNAVAILABLE", str(e))
        if isinstance(out, _ClientError):
            return JSONResponse(out.body, status_code=out.status)
        return out

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        if _remote(getattr(req, "model", None)):
            return await _forward("completions", req)
        st.route(getattr(req, "model", None))
        if req.n != 1 and not req.use_beam_search:
            raise HTTPException(400, "n > 1 needs use_beam_search")
        sp = build_sampling(st, req.model_dump(), {**OPENAI_DEFAULTS, "max_tokens": req.max_tokens or 16})
        lora = st.lora_id(req.adapter_id)
        prompts = req.prompt
        if isinstance(prompts, list) and prompts and isinstance(prompts[0], (str, list)):
            batch = prompts
        else:
            batch = [prompts]
        cid = "cmpl-" + uuid.uuid4().hex
        if req.use_beam_search:
            return await beam_completions(req, batch, lora, cid)
        if req.stream:
            if len(batch) != 1:
                raise HTTPException(400, "streaming supports a single prompt")
            frame = lambda d, o: {"id": cid, "object": "text_completion", "created": _now(), "model": st.model_name,  # noqa: E731
                                  "choices": [{"index": 0, "text": d, "finish_reason": o.finish_reason, "logprobs": None}]}
            final = lambda o: {"id": cid, "object": "text_completion", "created": _now(), "model": st.model_name,  # noqa: E731
                               "choices": [], "usage": {"prompt_tokens": len(o.prompt_token_ids),
                                                        "completion_tokens": len(o.output_token_ids),
                                                        "total_tokens": len(o.prompt_token_ids) + len(o.output_token_ids)}}
            return await sse_stream(batch[0], sp, cid, lora, frame, final)
        outs = await asyncio.gather(*[run_full(p, SamplingParams(**vars(sp)), lora_id=lora) for p in batch])
        choices, pt, ct = [], 0, 0
        def tokstr(t):
            return st.tokenizer.decode([t]) if st.tokenizer is not None else str(t)

        for i, o in enumerate(outs):
            lp = None
            if o.logprobs is not None:
                lp = {"tokens": [tokstr(e["token"]) for e in o.logprobs],
                      "token_logprobs": [e["logprob"] for e in o.logprobs],
                      "top_logprobs": [{tokstr(t): v for t, v in e.get("top", {}).items()} for e in o.logprobs]}
            choices.append({"index": i, "text": o.text or detok(o.output_token_ids), "finish_reason": o.finish_reason,
                            "logprobs": lp})
            pt += len(o.prompt_token_ids)
            ct += len(o.output_token_ids)
        return {"id": cid, "object": "text_completion", "created": _now(), "model": st.model_name, "choices": choices,
                "usage": {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct}}

    def chat_logprobs(o):
        if o.logprobs is None:
            return None
        ts = (lambda t: st.tokenizer.decode([t])) if st.tokenizer is not None else str
        return {"content": [{"token": ts(e["token"]), "logprob": e["logprob"],
                             "top_logprobs": [{"token": ts(t), "logprob": v} for t, v in e.get("top", {}).items()]}
                            for e in o.logprobs]}

    async def _chat(req: ChatRequest, force_stream: bool = False):
        if _remote(getattr(req, "model", None)):
            if force_stream:
                req.stream = True
            return await _forward("chat/completions", req)
        st.route(getattr(req, "model", None))
        if req.n != 1:
            raise HTTPException(400, "only n=1 is supported")
        d = req.model_dump()
        d["max_tokens"] = req.max_tokens or req.max_completion_tokens
        sp = build_sampling(st, d, OPENAI_DEFAULTS)
        lora = st.lora_id(req.adapter_id)
        tools = req.tools if (req.tools and req.tool_choice != "none") else None
        if req.mcp and req.tool_choice != "none" and st.mcp.clients:
            tools = (tools or []) + await asyncio.to_thread(st.mcp.openai_tools)
        if tools:
            rx = tool_choice_regex(req.tool_choice)
            if rx and not (sp.guided_json or sp.guided_regex):
                sp.guided_regex = rx  # a forced call: the output is constrained to the call's shape
        rag_sources = None
        pl = st.plugins
        info: Dict[str, Any] = {}
        messages = [m if isinstance(m, dict) else m.model_dump(exclude_none=True) for m in req.messages]
        images = None
        if any(isinstance(m.get("content"), list) for m in messages):  # OpenAI content parts
            from ..models.vlm import flatten_content_parts
            ph = getattr(st.engine, "image_placeholder", None) or "<image>"
            try:
                messages, images = await asyncio.to_thread(flatten_content_parts, messages, ph)
            except Exception as e:  # bad URL / undecodable image / unknown part type
                raise HTTPException(400, f"content parts: {e}")
            if images and getattr(st.engine, "vision", None) is None:
                raise HTTPException(400, "this model takes no images")
        if pl.safety is not None or pl.pii_redaction:  # request plugins: content safety, then PII redaction
            for m in messages:
                c = m.get("content")
                if m.get("role") != "user" or not isinstance(c, str):
                    continue
                if pl.safety is not None:
                    try:
                        pl.safety.check(c)
                    except UnsafeContent as e:
                        raise HTTPException(400, str(e))
                if pl.pii_redaction:
                    m["content"], k = redact_pii(c)
                    info["pii_redactions"] = info.get("pii_redactions", 0) + k
        if req.rag:
            messages, rag_sources = await rag_augment(messages, req.rag)
        prompt = chat_prompt(messages, tools)
        cid = "chatcmpl-" + uuid.uuid4().hex
        cache_key = qvec = None
        if (pl.semantic_cache is not None and not (req.stream or force_stream) and not tools and not images
                and sp.temperature == 0 and not req.logprobs):
            cache_key = json.dumps({"max_tokens": sp.max_tokens, "stop": req.stop, "rf": req.response_format,
                                    "rx": req.guided_regex, "rag": req.rag, "adapter": req.adapter_id},
                                   sort_keys=True, default=str)
            qvec = (await _embed([prompt]))[0]
            hit = pl.semantic_cache.lookup(cache_key, qvec)
            if hit is not None:
                return {**hit["response"], "id": cid, "created": _now(),
                        "gollek": {**info, "semantic_cache": "hit", "similarity": round(hit["similarity"], 6)}}

        def keep_calls(calls):
            return calls[:1] if req.parallel_tool_calls is False else calls

        if req.stream or force_stream:
            first = {"sent": False}

            def frame(delta, o):
                dd = {"content": delta}
                if not first["sent"]:
                    dd["role"] = "assistant"
                    first["sent"] = True
                return {"id": cid, "object": "chat.completion.chunk", "created": _now(), "model": st.model_name,
                        "choices": [{"index": 0, "delta": dd, "finish_reason": o.finish_reason if o else None}]}

            def tool_frame(calls, o):
                dd = {"tool_calls": [{"index": k, **c.openai()} for k, c in enumerate(keep_calls(calls))]}
                if not first["sent"]:
                    dd["role"] = "assistant"
                    first["sent"] = True
                return {"id": cid, "object": "chat.completion.chunk", "created": _now(), "model": st.model_name,
                        "choices": [{"index": 0, "delta": dd, "finish_reason": "tool_calls"}]}

            final = lambda o: {"id": cid, "object": "chat.completion.chunk", "created": _now(), "model": st.model_name,  # noqa: E731
                               "choices": [], "usage": {"prompt_tokens": len(o.prompt_token_ids),
                                                        "completion_tokens": len(o.output_token_ids),
                                                        "total_tokens": len(o.prompt_token_ids) + len(o.output_token_ids)}}
            return await sse_stream(prompt, sp, cid, lora, frame, final, tool_frame=tool_frame if tools else None,
                                    images=images)
        o = await run_full(prompt, sp, lora_id=lora, images=images)
        pt, ct = len(o.prompt_token_ids), len(o.output_token_ids)
        text = o.text or detok(o.output_token_ids)
        message: Dict[str, Any] = {"role": "assistant", "content": text}
        finish = o.finish_reason
        if tools:
            content, calls = parse_tool_calls(text)
            if calls:
                message = {"role": "assistant", "content": content or None,
                           "tool_calls": [c.openai() for c in keep_calls(calls)]}
                finish = "tool_calls"
        resp = {"id": cid, "object": "chat.completion", "created": _now(), "model": st.model_name,
                "choices": [{"index": 0, "message": message, "finish_reason": finish, "logprobs": chat_logprobs(o)}],
                "usage": {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct}}
        if rag_sources is not None:
            resp["rag_sources"] = rag_sources
        if pl.reasoning_split and isinstance(message.get("content"), str):
            reasoning, answer = split_reasoning(message["content"])
            if reasoning is not None:
                message["content"], message["reasoning_content"] = answer, reasoning
        if cache_key is not None:
            pl.semantic_cache.store(cache_key, qvec, {"response": dict(resp)})
            info["semantic_cache"] = "miss"
        if info:
            resp["gollek"] = info
        return resp

    # -------------------------------------------------------------- Model Context Protocol servers
    @app.post("/v1/admin/mcp/servers")
    async def mcp_connect(body: Dict[str, Any]):
        """{"name", "command": [argv]} for a stdio server, or {"name", "url", "transport": "sse" | "http",
        "headers"?} for an HTTP server."""
        name, cmd, url = body.get("name"), body.get("command"), body.get("url")
        if not name or not ((isinstance(cmd, list) and cmd) or isinstance(url, str)):
            raise HTTPException(400, "name and either command (argv list) or url are required")
        transport = str(body.get("transport", "http" if url else "stdio"))
        try:
            info = await asyncio.to_thread(st.mcp.connect, str(name), [str(c) for c in cmd] if cmd else None,
                                           float(body.get("timeout_s", 30.0)), url, transport,
                                           body.get("headers"))
        except (MCPError, OSError, ValueError) as e:
            raise HTTPException(502, f"MCP server {name!r}: {e}")
        return {"name": name, "protocolVersion": info.get("protocolVersion"), "serverInfo": info.get("serverInfo")}

    @app.delete("/v1/admin/mcp/servers/{name}")
    async def mcp_disconnect(name: str):
        if not st.mcp.disconnect(name):
            raise HTTPException(404, f"unknown MCP server {name!r}")
        return Response(status_code=204)

    @app.get("/v1/mcp/tools")
    async def mcp_tools():
        try:
            return {"tools": await asyncio.to_thread(st.mcp.openai_tools)}
        except MCPError as e:
            raise HTTPException(502, str(e))

    @app.post("/v1/mcp/tools/call")
    async def mcp_call(body: Dict[str, Any]):
        try:
            res = await asyncio.to_thread(st.mcp.call, str(body.get("name", "")), body.get("arguments") or {})
        except KeyError as e:
            raise HTTPException(404, str(e))
        except MCPError as e:
            raise HTTPException(502, str(e))
        return {"result": res, "text": tool_text(res), "isError": bool(res.get("isError", False))}

    @app.get("/v1/admin/plugins")
    async def plugins_get():
        return st.plugins.describe()

    @app.post("/v1/admin/plugins")
    async def plugins_set(body: Dict[str, Any]):
        try:
            st.plugins.configure(body)
        except (ValueError, TypeError, re.error) as e:
            raise HTTPException(400, str(e))
        return st.plugins.describe()

    @app.post("/v1/chat/completions")
    async def chat(req: ChatRequest):
        return await _chat(req)

    @app.post("/v1/chat/completions/stream")
    async def chat_stream(req: ChatRequest):
        return await _chat(req, force_stream=True)

    async def _embed(inputs) -> List[List[float]]:
        if isinstance(inputs, str):
            inputs = [inputs]
        elif inputs and isinstance(inputs[0], int):
            inputs = [inputs]
        toks = []
        for x in inputs:
            if isinstance(x, str):
                if st.tokenizer is None:
                    raise HTTPException(400, "model has no tokenizer")
                toks.append(st.tokenizer.encode(x))
            else:
                toks.append(list(x))
        return await st.ae.call(lambda eng: eng.embed(toks))

    @app.post("/v1/embeddings")
    async def embeddings(req: EmbeddingRequest):
        st.route(getattr(req, "model", None))
        vecs = await _embed(req.input)
        n = sum(len(v) for v in vecs)
        return {"object": "list", "model": st.model_name,
                "data": [{"object": "embedding", "index": i, "embedding": v} for i, v in enumerate(vecs)],
                "usage": {"prompt_tokens": n, "total_tokens": n}}

    # -------------------------------------------------------------- retrieval-augmented generation
    def count_tokens(text: str) -> int:
        return len(st.tokenizer.encode(text)) if st.tokenizer is not None else max(1, len(text) // 4)

    async def rag_retrieve(collection: str, question: str, top_k: int, min_similarity: float = -1.0):
        col = st.rag.get(collection)
        if col is None:
            raise HTTPException(404, f"unknown RAG collection {collection!r}")
        qv = (await _embed([question]))[0]
        return col.search(qv, top_k, min_similarity)

    async def rag_augment(messages: List[dict], opts: Dict[str, Any]):
        from .rag import augment_messages, build_context, last_user_text
        hits = await rag_retrieve(str(opts.get("collection", "")), last_user_text(messages),
                                  int(opts.get("top_k", 4)), float(opts.get("min_similarity", -1.0)))
        ctx = build_context(hits, int(opts.get("max_context_tokens", 1024)), count_tokens)
        msgs = augment_messages(messages, ctx) if hits else messages
        return msgs, [h.source() for h in hits]

    @app.post("/v1/rag/ingest")
    async def rag_ingest(req: RagIngestRequest):
        from .rag import chunk_text
        if not req.documents:
            raise HTTPException(400, "documents must be non-empty")
        col = st.rag.get(req.collection, create=True)
        n = 0
        for k, doc in enumerate(req.documents):
            chunks = chunk_text(doc.content, req.chunk_size, req.chunk_overlap)
            if not chunks:
                continue
            vecs = await _embed(chunks)
            col.add(doc.id or f"doc-{len(col)}-{k}", chunks, vecs)
            n += len(chunks)
        return {"collection": req.collection, "chunks": n, "status": "indexed"}

    @app.post("/v1/rag/query")
    async def rag_query(req: RagQueryRequest):
        from .rag import augment_messages, build_context
        top_k = req.topK or req.top_k or 4
        hits = await rag_retrieve(req.collection, req.question, top_k, req.min_similarity)
        msgs = [{"role": "user", "content": req.question}]
        if hits:
            msgs = augment_messages(msgs, build_context(hits, req.max_context_tokens, count_tokens))
        d = {"max_tokens": req.maxTokens or req.max_tokens, "temperature": req.temperature}
        sp = build_sampling(st, d, OPENAI_DEFAULTS)
        o = await run_full(chat_prompt(msgs), sp, lora_id=0)
        return {"answer": o.text or detok(o.output_token_ids), "context_used": bool(hits),
                "sources": [h.source() for h in hits]}

    @app.get("/v1/rag/collections")
    async def rag_collections():
        return {"collections": [{"name": n, "chunks": len(c)} for n, c in list(st.rag.collections.items())]}

    @app.get("/v1/rag/collections/{name}")
    async def rag_collection(name: str):
        c = st.rag.get(name)
        if c is None:
            raise HTTPException(404, f"unknown RAG collection {name!r}")
        return {"name": name, "chunks": len(c)}

    @app.delete("/v1/rag/collections/{name}")
    async def rag_drop(name: str):
        if not st.rag.drop(name):
            raise HTTPException(404, f"unknown RAG collection {name!r}")
        return Response(status_code=204)

    # -------------------------------------------------------------- gollek platform routes
    def infer_prompt(req: InferRequest):
        if req.prompt is not None and not req.messages:
            return req.prompt
        return chat_prompt([m.model_dump() for m in req.messages])

    async def infer_completions(req: InferRequest, x_request_id: Optional[str] = Header(None)):
        st.route(getattr(req, "model", None))
        return await _infer(req, x_request_id)

    async def _infer(req: InferRequest, x_request_id: Optional[str] = None):
        rid = req.requestId or x_request_id or uuid.uuid4().hex
        sp = build_sampling(st, req.parameters, gollek_defaults)
        lora = st.lora_id(_param(req.parameters, "adapter_id", "adapterId", "lora"))
        t0 = time.perf_counter()
        o = await run_full(infer_prompt(req), sp, rid, lora, req.priority, timeout=req.timeout / 1000 if req.timeout else None)
        return {"requestId": rid, "content": o.text or detok(o.output_token_ids), "model": req.model or st.model_name,
                "tokensUsed": len(o.prompt_token_ids) + len(o.output_token_ids),
                "promptTokens": len(o.prompt_token_ids), "completionTokens": len(o.output_token_ids),
                "durationMs": int((time.perf_counter() - t0) * 1e3),
                "timestamp": datetime.now(timezone.utc).isoformat(), "finishReason": o.finish_reason}

    async def infer_async(req: InferRequest):
        st.route(getattr(req, "model", None))
        jid = req.requestId or uuid.uuid4().hex
        st.jobs[jid] = {"jobId": jid, "status": "PENDING", "result": None, "error": None}

        async def run():
            st.jobs[jid]["status"] = "RUNNING"
            try:
                st.jobs[jid]["result"] = await _infer(req)
                st.jobs[jid]["status"] = "COMPLETED"
            except HTTPException as e:
                st.jobs[jid].update(status="FAILED", error=e.detail)
            except Exception as e:  # report, don't crash the server
                st.jobs[jid].update(status="FAILED", error=repr(e))

        asyncio.get_running_loop().create_task(run())
        return JSONResponse({"jobId": jid, "status": "PENDING"}, status_code=202)

    async def infer_async_status(job_id: str):
        if job_id not in st.jobs:
            raise HTTPException(404, "unknown job")
        return st.jobs[job_id]

    async def infer_stream(req: InferRequest):
        st.route(getattr(req, "model", None))
        rid = req.requestId or uuid.uuid4().hex
        sp = build_sampling(st, req.parameters, gollek_defaults)
        lora = st.lora_id(_param(req.parameters, "adapter_id", "adapterId", "lora"))
        counter = {"i": 0}

        def frame(delta, o):
            counter["i"] += 1
            return {"requestId": rid, "index": counter["i"] - 1, "content": delta, "isFinal": bool(o.finished)}

        final = lambda o: {"requestId": rid, "index": counter["i"], "content": "", "isFinal": True,  # noqa: E731
                           "finishReason": o.finish_reason, "tokensUsed": len(o.prompt_token_ids) + len(o.output_token_ids)}
        return await sse_stream(infer_prompt(req), sp, rid, lora, frame, final, done_marker=False)

    async def infer_batch(reqs: List[InferRequest]):
        return await asyncio.gather(*[_infer(r) for r in reqs])

    async def infer_embeddings(req: InferRequest):
        texts = [m.content or "" for m in req.messages] or [req.prompt or ""]
        vecs = await _embed(texts)
        return {"model": req.model or st.model_name, "embeddings": vecs}

    async def infer_cancel(request_id: str):
        await st.ae.abort(request_id)
        return {"requestId": request_id, "status": "CANCELLED"}

    for base in ("/v1/infer", "/v1/inference"):
        app.post(base + "/completions")(infer_completions)
        app.post(base + "/async")(infer_async)
        app.get(base + "/async/{job_id}")(infer_async_status)
        app.post(base + "/stream")(infer_stream)
        app.post(base + "/batch")(infer_batch)
        app.post(base + "/embeddings")(infer_embeddings)
        app.delete(base + "/{request_id}")(infer_cancel)
    app.post("/api/v1/inference")(infer_completions)
    app.post("/v1/inference")(infer_completions)

    # -------------------------------------------------------------- jobs and administration
    @app.get("/v1/jobs")
    async def list_jobs():
        return {"jobs": [{"jobId": j["jobId"], "status": j["status"]} for j in st.jobs.values()]}

    @app.get("/v1/jobs/{job_id}")
    async def get_job(job_id: str):
        if job_id not in st.jobs:
            e = HTTPException(404, "unknown job")
            e.gollek_code = "ROUTING_JOB_NOT_FOUND"
            raise e
        return st.jobs[job_id]

    @app.get("/v1/admin/api-keys")
    async def admin_list_keys():
        return {"keys": [{"key": k[:4] + "…" + k[-2:], "tenant": t} for k, t in st.api_keys.items()]}

    @app.post("/v1/admin/api-keys")
    async def admin_create_key(body: Dict[str, Any] = None):
        import secrets
        key = "gk-" + secrets.token_urlsafe(24)
        st.api_keys[key] = str((body or {}).get("tenant", ""))
        return {"key": key, "tenant": st.api_keys[key]}

    @app.delete("/v1/admin/api-keys/{key}")
    async def admin_revoke_key(key: str):
        if key not in st.api_keys:
            raise HTTPException(404, "unknown key")
        del st.api_keys[key]
        return {"revoked": True}

    # -------------------------------------------------------------- model hot-swap
    from .hotswap import HotSwapManager, default_memory_check

    def _default_builder(model: str):
        import dataclasses
        from ..engine.engine import LLMEngine
        return LLMEngine(dataclasses.replace(st.engine.cfg, model=model))

    swapper = HotSwapManager(st, engine_builder or _default_builder, drain_timeout_s,
                             memory_check=default_memory_check if engine_builder is None else None)
    app.state.hotswap = swapper

    @app.post("/v1/admin/models")
    async def admin_add_model(body: Dict[str, Any]):
        """Serve another model next to the primary one; requests name it in ``model``."""
        name, model = (body or {}).get("name"), (body or {}).get("model")
        if not name or not model or name == st._model_name or name in st.routes:
            raise HTTPException(400, "body needs a new name and a model (preset name or checkpoint path)")
        from .async_engine import AsyncEngine as _AE
        eng = await asyncio.to_thread(engine_builder or _default_builder, str(model))
        st.routes[str(name)] = _AE(eng).start()
        return {"name": name, "model": model, "served": [st._model_name] + list(st.routes)}

    @app.get("/v1/admin/providers")
    async def admin_providers():
        return {"providers": [p.status() for p in st.providers.all()]}

    @app.post("/v1/admin/providers")
    async def admin_add_provider(body: Dict[str, Any]):
        """Register an OpenAI-compatible upstream: {"id", "base_url", "api_key"?, "models"?}."""
        pid, url = (body or {}).get("id"), (body or {}).get("base_url")
        if not pid or not url:
            raise HTTPException(400, "body needs id and base_url")
        st.providers.register(OpenAIHTTPProvider(str(pid), str(url), str(body.get("api_key", "")),
                                                 body.get("models"), float(body.get("timeout", 60.0))))
        return {"registered": pid, "providers": [p.id for p in st.providers.all()]}

    @app.delete("/v1/admin/providers/{pid}")
    async def admin_remove_provider(pid: str):
        if not st.providers.unregister(pid):
            raise HTTPException(404, f"no provider {pid}")
        return {"removed": pid}

    @app.get("/v1/admin/providers/route")
    async def admin_route(model: str, stream: bool = False):
        try:
            d = st.provider_router.route(model, streaming=stream)
        except Exception as e:
            raise HTTPException(404, str(e))
        return {"provider": d.provider, "score": d.score, "fallbacks": d.fallbacks}

    @app.delete("/v1/admin/models/{name}")
    async def admin_remove_model(name: str):
        ae = st.routes.pop(name, None)
        if ae is None:
            raise HTTPException(404, f"unknown routed model {name!r}")
        await asyncio.to_thread(ae.shutdown, True, drain_timeout_s)
        return Response(status_code=204)

    @app.post("/v1/admin/models/swap")
    async def admin_swap(body: Dict[str, Any]):
        model = (body or {}).get("model")
        if not model:
            raise HTTPException(400, "body needs a model (preset name or checkpoint path)")
        try:
            sw = swapper.begin(str(model), body.get("name"))
        except MemoryError as e:
            return error_response("DEVICE_OUT_OF_MEMORY", f"hot-swap refused: {e}")
        except RuntimeError as e:
            raise HTTPException(409, str(e))
        return JSONResponse(sw.as_dict(), status_code=202)

    @app.get("/v1/admin/models/swap")
    async def admin_swap_list():
        act = swapper.active
        return {"active": act.as_dict() if act is not None and not act.done else None,
                "swaps": [s.as_dict() for s in swapper.swaps.values()]}

    @app.get("/v1/admin/models/swap/{swap_id}")
    async def admin_swap_get(swap_id: str):
        sw = swapper.swaps.get(swap_id)
        if sw is None:
            raise HTTPException(404, f"unknown swap {swap_id}")
        return sw.as_dict()

    @app.get("/v1/admin/errors")
    async def admin_error_codes():
        return {"codes": [dict(name=c.name, code=c.code, http=c.http, retryable=c.retryable, message=c.message,
                               category=c.category.value) for c in errors.CODES.values()]}

    @app.get("/v1/admin/tenants")
    async def admin_tenants():
        use = st.engine.scheduler._tenant_usage()
        return {"quotas": st.engine.cfg.tenant_quotas,
                "usage": {t: {"running": u[0], "kv_blocks": u[1]} for t, u in use.items()}}
    return app
