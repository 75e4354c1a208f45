"""Python SDK: local (in-process) and remote (HTTP) clients with one request/response model.

Mirrors the reference SDK surface: ``GenerationRequest(prompt, model, maxTokens=512,
temperature=0.7, topP=1.0, stream, metadata, stop)`` and ``GenerationResponse(text, model,
usage{prompt, completion, total})`` (sdk/gollek-sdk/…/sdk/model/GenerationRequest.java:36-112,
GenerationResponse.java:16-90), the remote ``GollekClient`` (sdk/gollek-sdk-java-remote/…/
client/GollekClient.java:96-706: generate, stream, embeddings, models, health) and the local
in-process SDK (sdk/gollek-sdk-core/…/sdk/core/GollekSdk.java).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Dict, Iterator, List, Optional

from ..engine.sequence import SamplingParams


@dataclass
class Usage:
    prompt_tokens: int = 0
    completion_tokens: int = 0

    @property
    def total_tokens(self) -> int:
        return self.prompt_tokens + self.completion_tokens


@dataclass
class GenerationRequest:
    prompt: str
    model: Optional[str] = None
    max_tokens: int = 512
    temperature: float = 0.7
    top_p: float = 1.0
    top_k: int = 0
    stream: bool = False
    stop: List[str] = field(default_factory=list)
    seed: Optional[int] = None
    adapter_id: Optional[str] = None
    metadata: Dict[str, str] = field(default_factory=dict)

    def sampling(self) -> SamplingParams:
        return SamplingParams(temperature=self.temperature, top_p=self.top_p, top_k=self.top_k,
                              max_tokens=self.max_tokens, stop=list(self.stop), seed=self.seed).validate()

    def parameters(self) -> dict:
        p = {"max_tokens": self.max_tokens, "temperature": self.temperature, "top_p": self.top_p,
             "top_k": self.top_k, "stop": self.stop}
        if self.seed is not None:
            p["seed"] = self.seed
        if self.adapter_id:
            p["adapter_id"] = self.adapter_id
        return p


@dataclass
class GenerationResponse:
    text: str
    model: str
    usage: Usage
    finish_reason: Optional[str] = None
    request_id: Optional[str] = None


class LocalClient:
    """In-process SDK over an ``LLMEngine`` (no server)."""

    def __init__(self, engine, model_name: str = "local"):
        self.engine = engine
        self.model_name = model_name

    def generate(self, req: GenerationRequest) -> GenerationResponse:
        lora = 0
        if req.adapter_id:
            lora = self.engine.lora_manager.name_to_id[req.adapter_id]
        out = self.engine.generate([req.prompt], req.sampling(), lora_ids=[lora])[0]
        text = out.text or (self.engine.tokenizer.decode(out.output_token_ids) if self.engine.tokenizer else "")
        return GenerationResponse(text, req.model or self.model_name,
                                  Usage(len(out.prompt_token_ids), len(out.output_token_ids)),
                                  out.finish_reason, out.request_id)

    def stream(self, req: GenerationRequest) -> Iterator[str]:
        rid = self.engine.add_request(None, req.prompt, req.sampling())
        prev = ""
        while self.engine.has_unfinished():
            for o in self.engine.step():
                if o.request_id != rid:
                    continue
                text = self.engine.tokenizer.decode(o.output_token_ids) if self.engine.tokenizer else ""
                if text.startswith(prev) and len(text) > len(prev):
                    yield text[len(prev):]
                prev = text
                if o.finished:
                    return

    def embed(self, texts: List[str]) -> List[List[float]]:
        return self.engine.embed([self.engine.tokenizer.encode(t) for t in texts])

    def list_models(self) -> List[str]:
        return [self.model_name]


class GollekClient:
    """HTTP client for a gollek-b200 server (``python -m gollek_b200.server``)."""

    def __init__(self, base_url: str = "http://127.0.0.1:8000", api_key: Optional[str] = None,
                 timeout: float = 600.0, session=None):
        import requests
        self.base = base_url.rstrip("/")
        self.timeout = timeout
        self.http = session or requests.Session()
        if api_key:
            self.http.headers["Authorization"] = f"Bearer {api_key}"

    def _post(self, path: str, body: dict, stream: bool = False):
        r = self.http.post(self.base + path, json=body, timeout=self.timeout, stream=stream)
        if r.status_code >= 400:
            raise RuntimeError(f"{path}: HTTP {r.status_code}: {r.text[:500]}")
        return r

    def generate(self, req: GenerationRequest) -> GenerationResponse:
        body = {"model": req.model, "messages": [{"role": "user", "content": req.prompt}],
                "parameters": req.parameters()}
        j = self._post("/v1/inference/completions", body).json()
        usage = (Usage(j["promptTokens"], j["completionTokens"]) if "completionTokens" in j
                 else Usage(0, j.get("tokensUsed", 0)))  # servers that report only the total
        return GenerationResponse(j["content"], j["model"], usage,
                                  j.get("finishReason"), j["requestId"])

    def complete(self, prompt: str, **kw) -> dict:
        return self._post("/v1/completions", {"prompt": prompt, **kw}).json()

    def chat(self, messages: List[dict], **kw) -> dict:
        return self._post("/v1/chat/completions", {"messages": messages, **kw}).json()

    def stream(self, req: GenerationRequest) -> Iterator[str]:
        body = {"model": req.model, "messages": [{"role": "user", "content": req.prompt}],
                "parameters": req.parameters()}
        r = self._post("/v1/inference/stream", body, stream=True)
        for line in r.iter_lines(decode_unicode=True):
            if line and line.startswith("data: "):
                frame = json.loads(line[6:])
                if frame.get("content"):
                    yield frame["content"]
                if frame.get("isFinal"):
                    break

    def embed(self, texts: List[str]) -> List[List[float]]:
        j = self._post("/v1/embeddings", {"input": texts}).json()
        return [d["embedding"] for d in j["data"]]

    def rag_ingest(self, collection: str, documents: List[dict], **kw) -> dict:
        """Chunk, embed and index ``documents`` ([{"id", "content"}]) into ``collection``."""
        return self._post("/v1/rag/ingest", {"collection": collection, "documents": documents, **kw}).json()

    def rag_query(self, collection: str, question: str, **kw) -> dict:
        """Answer ``question`` from the collection's most similar chunks: {answer, context_used, sources}."""
        return self._post("/v1/rag/query", {"collection": collection, "question": question, **kw}).json()

    def list_models(self) -> List[str]:
        r = self.http.get(self.base + "/v1/models", timeout=self.timeout)
        return [m["id"] for m in r.json()["data"]]

    def _get(self, path: str, **params):
        r = self.http.get(self.base + path, params=params or None, timeout=self.timeout)
        if r.status_code >= 400:
            raise RuntimeError(f"{path}: HTTP {r.status_code}: {r.text[:500]}")
        return r.json()

    def submit(self, req: GenerationRequest) -> str:
        """Queue ``req`` as an asynchronous job; returns its job id."""
        body = {"model": req.model, "messages": [{"role": "user", "content": req.prompt}],
                "parameters": req.parameters()}
        return self._post("/v1/infer/async", body).json()["jobId"]

    def job(self, job_id: str) -> dict:
        """{jobId, status (PENDING / RUNNING / COMPLETED / FAILED), result, error}."""
        return self._get(f"/v1/infer/async/{job_id}")

    def wait(self, job_id: str, timeout: float = 600.0, poll: float = 0.05) -> dict:
        import time
        t_end = time.monotonic() + timeout
        while True:
            j = self.job(job_id)
            if j["status"] in ("COMPLETED", "FAILED") or time.monotonic() > t_end:
                return j
            time.sleep(poll)

    def speech(self, text: str, voice: str = "default", response_format: str = "wav") -> bytes:
        """Text to speech (WAV bytes, or raw 16-bit PCM with ``response_format="pcm"``)."""
        return self._post("/v1/audio/speech", {"input": text, "voice": voice,
                                               "response_format": response_format}).content

    def transcribe(self, audio: bytes, filename: str = "audio.wav", translate: bool = False, **fields) -> dict:
        """Speech recognition of an audio file's bytes (``translate`` for English translation)."""
        path = "/v1/audio/translations" if translate else "/v1/audio/transcriptions"
        r = self.http.post(self.base + path, files={"file": (filename, audio)},
                           data={k: str(v) for k, v in fields.items()}, timeout=self.timeout)
        if r.status_code >= 400:
            raise RuntimeError(f"{path}: HTTP {r.status_code}: {r.text[:500]}")
        return r.json()

    def providers(self) -> List[dict]:
        return self._get("/v1/admin/providers")["providers"]

    def add_provider(self, pid: str, base_url: str, api_key: str = "", models: Optional[List[str]] = None) -> dict:
        """Register an OpenAI-compatible upstream that serves models this server does not."""
        body = {"id": pid, "base_url": base_url, "api_key": api_key}
        if models:
            body["models"] = models
        return self._post("/v1/admin/providers", body).json()

    def health(self) -> bool:
        try:
            return self.http.get(self.base + "/health", timeout=5).status_code == 200
        except Exception:
            return False
