"""Provider registry and scored routing with fallback.

A provider serves OpenAI-shaped ``chat/completions`` and ``completions`` bodies for some set of
models. The server's own engines are the local provider; ``OpenAIHTTPProvider`` forwards to any
OpenAI-compatible server (another gollek replica, a vLLM or llama.cpp server). The router mirrors
the reference's selection order (inference/gollek-engine/…/engine/routing/ModelRouterService.java:
323-420 pins a preferred provider, else scores the compatible ones and keeps the runners-up as
fallbacks; :476-515 scores streaming / device / cost; :523 falls back to a GGUF-capable provider when
nothing else is compatible), with its own score: capability matches, then measured health (circuit
breaker state, failure ratio), latency (EWMA of successful calls) and load (calls in flight).
``execute`` tries the winner, then the fallbacks, in order, recording every outcome.
"""
from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterator, List, Optional, Sequence

from .resilience import CircuitBreaker, CircuitOpen


class ProviderError(RuntimeError):
    pass


class NoProvider(ProviderError):
    pass


@dataclass
class Capabilities:
    streaming: bool = True
    formats: Sequence[str] = ("safetensors", "gguf")
    devices: Sequence[str] = ("cuda",)
    adapters: bool = False


class Provider:
    """Base: subclasses implement ``models`` and ``_call``; health / latency bookkeeping is here."""

    def __init__(self, pid: str, caps: Optional[Capabilities] = None, breaker: Optional[CircuitBreaker] = None):
        self.id = pid
        self.caps = caps or Capabilities()
        self.breaker = breaker or CircuitBreaker(volume=4, failure_ratio=0.5, open_seconds=10.0)
        self.latency_ewma = 0.0
        self.inflight = 0
        self.calls = self.failures = 0
        self._lock = threading.Lock()

    def models(self) -> List[str]:
        raise NotImplementedError

    def supports(self, model: str) -> bool:
        return model in self.models()

    def _call(self, route: str, body: dict) -> Any:
        raise NotImplementedError

    def call(self, route: str, body: dict) -> Any:
        self.breaker.before()
        with self._lock:
            self.inflight += 1
            self.calls += 1
        t0 = time.monotonic()
        try:
            out = self._call(route, body)
        except Exception:
            with self._lock:
                self.failures += 1
            self.breaker.record(False)
            raise
        finally:
            with self._lock:
                self.inflight -= 1
        dt = time.monotonic() - t0
        with self._lock:
            self.latency_ewma = dt if self.latency_ewma == 0.0 else 0.8 * self.latency_ewma + 0.2 * dt
        self.breaker.record(True)
        return out

    def status(self) -> dict:
        return {"id": self.id, "models": self.models(), "state": self.breaker.state, "calls": self.calls,
                "failures": self.failures, "inflight": self.inflight,
                "latency_ms": round(self.latency_ewma * 1e3, 3), "streaming": self.caps.streaming,
                "formats": list(self.caps.formats), "devices": list(self.caps.devices)}


class LocalProvider(Provider):
    """In-process engines: ``handler(route, body)`` runs the request (the server passes its own
    handlers); ``model_names()`` lists what is served."""

    def __init__(self, pid: str, model_names: Callable[[], List[str]], handler: Callable[[str, dict], Any],
                 caps: Optional[Capabilities] = None):
        super().__init__(pid, caps or Capabilities(adapters=True))
        self._names, self._handler = model_names, handler

    def models(self) -> List[str]:
        return list(self._names())

    def _call(self, route, body):
        return self._handler(route, body)


class OpenAIHTTPProvider(Provider):
    """An OpenAI-compatible server at ``base_url`` (…/v1). ``models`` is fixed, or read from its
    ``/models`` listing (cached for ``refresh_s``)."""

    def __init__(self, pid: str, base_url: str, api_key: str = "", models: Optional[List[str]] = None,
                 timeout: float = 60.0, caps: Optional[Capabilities] = None, refresh_s: float = 30.0):
        super().__init__(pid, caps)
        self.base = base_url.rstrip("/")
        self.key, self.timeout, self.refresh_s = api_key, timeout, refresh_s
        self._fixed = list(models) if models else None
        self._cached: List[str] = []
        self._cached_at = -1e9

    def _headers(self) -> dict:
        h = {"Content-Type": "application/json"}
        if self.key:
            h["Authorization"] = f"Bearer {self.key}"
        return h

    def models(self) -> List[str]:
        if self._fixed is not None:
            return self._fixed
        if time.monotonic() - self._cached_at > self.refresh_s:
            import requests
            try:
                r = requests.get(self.base + "/models", headers=self._headers(), timeout=min(self.timeout, 5.0))
                r.raise_for_status()
                self._cached = [m["id"] for m in r.json().get("data", [])]
            except Exception:
                self._cached = []
            self._cached_at = time.monotonic()
        return self._cached

    def _call(self, route, body):
        import requests
        r = requests.post(f"{self.base}/{route}", data=json.dumps(body), headers=self._headers(),
                          timeout=self.timeout)
        if r.status_code >= 500:
            raise ProviderError(f"{self.id}: HTTP {r.status_code}")
        if r.status_code >= 400:  # the request itself is bad: no point in failing over
            return _ClientError(r.status_code, r.json() if r.content else {})
        return r.json()

    def stream(self, route: str, body: dict) -> Iterator[bytes]:
        """Server-sent-event lines of a streamed request, passed through unchanged."""
        import requests
        self.breaker.before()
        r = requests.post(f"{self.base}/{route}", data=json.dumps({**body, "stream": True}), headers=self._headers(),
                          timeout=self.timeout, stream=True)
        if r.status_code >= 400:
            self.breaker.record(False)
            raise ProviderError(f"{self.id}: HTTP {r.status_code}")
        self.breaker.record(True)
        for line in r.iter_lines():
            yield line + b"\n"


@dataclass
class _ClientError:
    status: int
    body: dict


@dataclass
class RoutingDecision:
    provider: str
    score: float
    fallbacks: List[str] = field(default_factory=list)


class ProviderRegistry:
    def __init__(self):
        self._p: Dict[str, Provider] = {}
        self._lock = threading.Lock()

    def register(self, p: Provider) -> None:
        with self._lock:
            self._p[p.id] = p

    def unregister(self, pid: str) -> bool:
        with self._lock:
            return self._p.pop(pid, None) is not None

    def get(self, pid: str) -> Optional[Provider]:
        return self._p.get(pid)

    def all(self) -> List[Provider]:
        with self._lock:
            return list(self._p.values())

    def models(self) -> List[str]:
        return sorted({m for p in self.all() for m in p.models()})


class ProviderRouter:
    """Scores providers for a request and executes it with fallback."""

    def __init__(self, registry: ProviderRegistry, max_fallbacks: int = 2):
        self.reg, self.max_fallbacks = registry, max_fallbacks

    def score(self, p: Provider, streaming: bool = False, device: Optional[str] = None,
              cost_sensitive: bool = False) -> float:
        s = 50.0
        if streaming:
            s += 20.0 if p.caps.streaming else -15.0
        if device and device in p.caps.devices:
            s += 30.0
        if cost_sensitive and "cpu" in p.caps.devices:
            s += 10.0
        if p.breaker.state == "open":
            s -= 500.0
        elif p.breaker.state == "half_open":
            s -= 40.0
        if p.calls:
            s -= 40.0 * p.failures / p.calls
        s -= min(30.0, 10.0 * p.latency_ewma)  # seconds of typical latency
        s -= 2.0 * p.inflight
        return s

    def route(self, model: str, streaming: bool = False, preferred: Optional[str] = None,
              device: Optional[str] = None, adapter: bool = False, fmt: Optional[str] = None,
              cost_sensitive: bool = False) -> RoutingDecision:
        provs = self.reg.all()
        if preferred:
            pin = next((p for p in provs if p.id.lower() == preferred.lower() and p.supports(model)), None)
            if pin is not None:
                return RoutingDecision(pin.id, 10_000.0, [])
        cands = [p for p in provs if p.supports(model) and (not adapter or p.caps.adapters)
                 and (fmt is None or fmt in p.caps.formats)]
        if not cands and fmt != "gguf":  # any provider that serves the model from a GGUF file
            cands = [p for p in provs if p.supports(model) and "gguf" in p.caps.formats]
        if not cands:
            raise NoProvider(f"no provider serves model {model!r}")
        ranked = sorted(cands, key=lambda p: -self.score(p, streaming, device, cost_sensitive))
        return RoutingDecision(ranked[0].id, self.score(ranked[0], streaming, device, cost_sensitive),
                               [p.id for p in ranked[1:1 + self.max_fallbacks]])

    def execute(self, route: str, body: dict, **kw) -> Any:
        """Run ``body`` on the routed provider, failing over to the fallbacks on a provider error
        (exception, HTTP 5xx, open circuit); a client error (HTTP 4xx) is returned as is."""
        d = self.route(body.get("model", ""), streaming=bool(body.get("stream")), **kw)
        errors = []
        for pid in [d.provider] + d.fallbacks:
            p = self.reg.get(pid)
            if p is None:
                continue
            try:
                out = p.call(route, body)
            except CircuitOpen:
                errors.append(f"{pid}: circuit open")
                continue
            except Exception as e:  # noqa: BLE001 - any provider failure fails over
                errors.append(f"{pid}: {e}")
                continue
            if isinstance(out, dict):
                out.setdefault("provider", pid)
            return out
        raise ProviderError("all providers failed: " + "; ".join(errors))
