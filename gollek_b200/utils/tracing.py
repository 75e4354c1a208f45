"""Tracing and profiling hooks.

* NVTX ranges (``GOLLEK_NVTX=1`` or ``set_nvtx(True)``): engine step phases (schedule, launch,
  read-back), every decoder layer and its attention / FFN / collective phases, so an Nsight
  timeline shows where a step's time goes. Disabled, a range costs one flag test.
* ``profile_steps``: a ``torch.profiler`` trace (CPU + CUDA activity) of N engine steps, written
  as a Chrome trace.
* Request lifecycle spans (arrival → admission → first token → finish, with per-token times) are
  kept on every ``Sequence`` and exported by ``request_spans`` as OpenTelemetry-shaped dicts; when
  the ``opentelemetry`` API is installed they are also emitted as real spans.

Replaces the reference's OTel tracer/meter and per-request InferenceTrace
(core/gollek-observability/…/observability/ObservabilityManager.java:19-26,82;
inference/gollek-runtime-inference/…/observability/InferenceTrace.java), which have no GPU view.
"""
from __future__ import annotations

import contextlib
import json
import os
import time
from typing import Iterator, List, Optional

import torch

_NVTX = os.environ.get("GOLLEK_NVTX", "0") not in ("", "0", "false", "False")


def set_nvtx(on: bool) -> None:
    global _NVTX
    _NVTX = bool(on)


def nvtx_enabled() -> bool:
    return _NVTX


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if not _NVTX or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx_push(name: str) -> None:
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)


def nvtx_pop() -> None:
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_pop()


def profile_steps(engine, steps: int, path: str, record_shapes: bool = False) -> str:
    """Run ``steps`` engine steps under torch.profiler; writes a Chrome trace to ``path``."""
    from torch.profiler import ProfilerActivity, profile
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    with profile(activities=acts, record_shapes=record_shapes) as prof:
        for _ in range(steps):
            if not engine.has_unfinished():
                break
            engine.step()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    prof.export_chrome_trace(path)
    return path


def _otel_tracer():
    try:
        from opentelemetry import trace  # optional dependency
        return trace.get_tracer("gollek_b200")
    except Exception:
        return None


def request_spans(seqs) -> List[dict]:
    """OpenTelemetry-shaped spans of finished or running sequences (times in ns since epoch)."""
    off = time.time() - time.perf_counter()  # perf_counter -> wall clock
    ns = lambda t: int((t + off) * 1e9) if t is not None else None  # noqa: E731
    out = []
    tracer = _otel_tracer()
    for s in seqs:
        end = s.finish_time if s.finish_time is not None else (s.token_times[-1] if s.token_times else None)
        span = {
            "name": "gollek.request", "trace_id": s.request_id, "start_time_unix_nano": ns(s.arrival_time),
            "end_time_unix_nano": ns(end),
            "attributes": {"gollek.prompt_tokens": s.num_prompt_tokens,
                           "gollek.output_tokens": sum(1 for t in s.output_token_ids if t >= 0),
                           "gollek.lora_id": s.lora_id, "gollek.preemptions": s.num_preemptions,
                           "gollek.status": s.status.value},
            "events": [e for e in (
                {"name": "admitted", "time_unix_nano": ns(s.scheduled_time)} if s.scheduled_time else None,
                {"name": "first_token", "time_unix_nano": ns(s.first_token_time)} if s.first_token_time else None,
            ) if e],
        }
        if s.first_token_time is not None:
            span["attributes"]["gollek.ttft_ms"] = (s.first_token_time - s.arrival_time) * 1e3
        if len(s.token_times) > 1:
            span["attributes"]["gollek.tpot_ms"] = (s.token_times[-1] - s.token_times[0]) / (len(s.token_times) - 1) * 1e3
        out.append(span)
        if tracer is not None and span["start_time_unix_nano"] is not None:
            sp = tracer.start_span("gollek.request", start_time=span["start_time_unix_nano"],
                                   attributes=span["attributes"])
            sp.end(end_time=span["end_time_unix_nano"])
    return out


def write_spans(spans: List[dict], path: str) -> None:
    with open(path, "a") as f:
        for sp in spans:
            f.write(json.dumps(sp) + "\n")
