"""Request-level resilience: bulkhead, circuit breaker, per-tenant rate limiting, timeouts.

Same policies the reference applies with resilience4j and MicroProfile Fault Tolerance
(inference/gollek-engine/…/engine/resilience/ResilienceManager.java:52-101; REST annotations
inference/gollek-api-rest/…/InferenceResource.java:78-81 — @Timeout 30 s, @CircuitBreaker
(volume 20, failure ratio 0.5, delay 5 s, 2 successes to close), @Bulkhead(100, queue 50);
tiered rate limiter inference/gollek-runtime-inference/…/ratelimit/RateLimiter.java).
"""
from __future__ import annotations

import asyncio
import threading
import time
from collections import deque
from typing import Deque, Dict


class BulkheadFull(RuntimeError):
    pass


class CircuitOpen(RuntimeError):
    pass


class RateLimited(RuntimeError):
    pass


class Bulkhead:
    """At most ``max_concurrent`` requests in flight plus ``max_queue`` waiting; beyond that reject."""

    def __init__(self, max_concurrent: int = 100, max_queue: int = 50):
        self.sem = asyncio.Semaphore(max_concurrent)
        self.max_concurrent, self.max_queue = max_concurrent, max_queue
        self.waiting = 0

    async def __aenter__(self):
        if self.sem.locked() and self.waiting >= self.max_queue:
            raise BulkheadFull("bulkhead full")
        self.waiting += 1
        try:
            await self.sem.acquire()
        finally:
            self.waiting -= 1
        return self

    async def __aexit__(self, *exc):
        self.sem.release()
        return False


class CircuitBreaker:
    """CLOSED → OPEN when ≥ ``volume`` calls in the window fail at ≥ ``failure_ratio``;
    OPEN rejects for ``open_seconds``; HALF_OPEN closes after ``success_threshold`` successes."""

    def __init__(self, volume: int = 20, failure_ratio: float = 0.5, open_seconds: float = 5.0,
                 success_threshold: int = 2, window: int = 100):
        self.volume, self.ratio, self.open_s, self.succ_needed = volume, failure_ratio, open_seconds, success_threshold
        self.results: Deque[bool] = deque(maxlen=window)
        self.state = "closed"
        self.opened_at = 0.0
        self.half_open_ok = 0
        self.lock = threading.Lock()

    def before(self) -> None:
        with self.lock:
            if self.state == "open":
                if time.monotonic() - self.opened_at >= self.open_s:
                    self.state, self.half_open_ok = "half_open", 0
                else:
                    raise CircuitOpen("circuit open")

    def record(self, ok: bool) -> None:
        with self.lock:
            if self.state == "half_open":
                if ok:
                    self.half_open_ok += 1
                    if self.half_open_ok >= self.succ_needed:
                        self.state = "closed"
                        self.results.clear()
                else:
                    self.state, self.opened_at = "open", time.monotonic()
                return
            self.results.append(ok)
            n = len(self.results)
            if n >= self.volume and self.results.count(False) / n >= self.ratio:
                self.state, self.opened_at = "open", time.monotonic()


class RateLimiter:
    """Token bucket per key: ``rate`` requests/s sustained, ``burst`` capacity (0 rate = unlimited)."""

    def __init__(self, rate: float = 0.0, burst: float = 0.0):
        self.rate, self.burst = rate, burst or max(1.0, rate)
        self.buckets: Dict[str, list] = {}
        self.lock = threading.Lock()

    def check(self, key: str) -> None:
        if self.rate <= 0:
            return
        now = time.monotonic()
        with self.lock:
            tokens, last = self.buckets.get(key, [self.burst, now])
            tokens = min(self.burst, tokens + (now - last) * self.rate)
            if tokens < 1.0:
                self.buckets[key] = [tokens, now]
                raise RateLimited(f"rate limit exceeded for {key}")
            self.buckets[key] = [tokens - 1.0, now]
