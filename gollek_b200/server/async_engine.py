"""Asynchronous front of the engine: one engine thread, many asyncio consumers.

All ``LLMEngine`` calls happen on a single background thread (the engine is not
thread-safe); HTTP handlers submit requests / aborts / callables through a queue and
receive ``RequestOutput`` objects on per-request asyncio queues. While requests are in
flight the thread steps the engine back to back (continuous batching); when idle it blocks
on the submission queue.

This is the serving loop the reference spreads over its coalescer and batch schedulers
(runner/llamacpp/gollek-runner-llamacpp/…/LlamaCppCoalescer.java:80-218; inference/gollek-engine/
…/DefaultBatchScheduler.java:84-195 STATIC/DYNAMIC/CONTINUOUS) — here always continuous.
"""
from __future__ import annotations

import asyncio
import queue
import threading
import traceback
import uuid
from typing import AsyncIterator, Callable, Dict, List, Optional, Union

from ..engine.engine import LLMEngine
from ..engine.sequence import RequestOutput, SamplingParams


class EngineDeadError(RuntimeError):
    pass


class AsyncEngine:
    def __init__(self, engine: LLMEngine):
        self.engine = engine
        self._subs: "queue.Queue" = queue.Queue()
        self._streams: Dict[str, tuple] = {}
        self._lock = threading.Lock()
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()
        self.error: Optional[BaseException] = None
        self.draining = False

    # ------------------------------------------------------------------ lifecycle
    def start(self) -> "AsyncEngine":
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, name="gollek-engine", daemon=True)
            self._thread.start()
        return self

    def shutdown(self, drain: bool = True, timeout: float = 30.0) -> None:
        """Stop accepting work; with ``drain`` let in-flight requests finish first."""
        self.draining = True
        if drain and self._thread is not None:
            self._thread.join(timeout=0)
            deadline = timeout
            import time
            t0 = time.monotonic()
            while self.engine.has_unfinished() and time.monotonic() - t0 < deadline and self.error is None:
                time.sleep(0.01)
        self._stop.set()
        self._subs.put(None)
        if self._thread is not None:
            self._thread.join(timeout=5)
        # checkpoint what a restart can reuse (engine thread has stopped: safe to touch the engine)
        cfg = self.engine.cfg
        if getattr(cfg, "prefix_cache_snapshot", None):
            try:
                self.engine.save_prefix_cache(cfg.prefix_cache_snapshot)
            except Exception as e:  # a failed snapshot must not block shutdown
                self.error = self.error or e
        if getattr(cfg, "request_snapshot", None):
            import json
            with open(cfg.request_snapshot, "w") as f:
                json.dump(self.engine.snapshot_requests(), f)

    @property
    def healthy(self) -> bool:
        return self.error is None and self._thread is not None and self._thread.is_alive()

    # ------------------------------------------------------------------ engine thread
    def _deliver(self, rid: str, item) -> None:
        with self._lock:
            ent = self._streams.get(rid)
        if ent is None:
            return
        loop, q = ent
        loop.call_soon_threadsafe(q.put_nowait, item)

    def _handle(self, sub) -> None:
        kind = sub[0]
        if kind == "add":
            _, rid, prompt, params, lora_id, priority, tenant, images = sub
            try:
                kw = {}
                if tenant:
                    kw["tenant"] = tenant
                if images:
                    kw["images"] = images
                self.engine.add_request(rid, prompt, params, lora_id=lora_id, priority=priority, **kw)
            except Exception as e:  # invalid request: report to that caller only
                self._deliver(rid, e)
        elif kind == "abort":
            self.engine.abort_request(sub[1])
            self._deliver(sub[1], None)
        elif kind == "call":
            _, fn, fut_loop, fut = sub
            try:
                res = fn(self.engine)
                fut_loop.call_soon_threadsafe(fut.set_result, res)
            except Exception as e:
                fut_loop.call_soon_threadsafe(fut.set_exception, e)

    def _loop(self) -> None:
        try:
            while not self._stop.is_set():
                block = not self.engine.has_unfinished()
                try:
                    sub = self._subs.get(block=block, timeout=0.5 if block else None) if block else \
                        self._subs.get_nowait()
                except queue.Empty:
                    sub = "empty"
                while sub != "empty":
                    if sub is None:
                        return
                    self._handle(sub)
                    try:
                        sub = self._subs.get_nowait()
                    except queue.Empty:
                        sub = "empty"
                if self.engine.has_unfinished():
                    for out in self.engine.step():
                        self._deliver(out.request_id, out)
        except BaseException as e:  # the engine died: fail every waiter loudly
            self.error = e
            traceback.print_exc()
            with self._lock:
                rids = list(self._streams)
            for rid in rids:
                self._deliver(rid, EngineDeadError(f"engine failed: {e!r}"))

    # ------------------------------------------------------------------ client API
    async def generate(self, prompt: Union[str, List[int]], params: SamplingParams,
                       request_id: Optional[str] = None, lora_id: int = 0,
                       priority: int = 0, tenant: str = "", images: Optional[list] = None
                       ) -> AsyncIterator[RequestOutput]:
        if self.error is not None:
            raise EngineDeadError(str(self.error))
        if self.draining:
            raise EngineDeadError("server is draining")
        rid = request_id or uuid.uuid4().hex
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        with self._lock:
            if rid in self._streams:
                raise ValueError(f"duplicate request id {rid}")
            self._streams[rid] = (loop, q)
        self._subs.put(("add", rid, prompt, params, lora_id, priority, tenant, images))
        finished = False
        try:
            while True:
                item = await q.get()
                if item is None:
                    return
                if isinstance(item, BaseException):
                    raise item
                yield item
                if item.finished:
                    finished = True
                    return
        finally:
            with self._lock:
                self._streams.pop(rid, None)
            if not finished:
                self._subs.put(("abort", rid))

    async def abort(self, request_id: str) -> None:
        self._subs.put(("abort", request_id))

    async def call(self, fn: Callable[[LLMEngine], object]):
        """Run ``fn(engine)`` on the engine thread (between steps) and await its result."""
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self._subs.put(("call", fn, loop, fut))
        return await fut
